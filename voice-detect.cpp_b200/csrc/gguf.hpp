// Standalone GGUF (v2/v3) reader: the KV store and the tensor table, with f32 /
// f16 / bf16 / q8_0 payloads widened to f32. It replaces the ggml gguf loader the
// reference's ModelLoader::load uses (src/model_loader.cpp:114-215), which lives in
// the absent ggml submodule. Every size and offset is checked against the file
// length, so a truncated or corrupt file fails with a message instead of reading
// out of bounds.
#pragma once
#include <cstdint>
#include <map>
#include <string>
#include <vector>

namespace vdb {

enum GgufType : uint32_t {
    GGUF_U8 = 0, GGUF_I8 = 1, GGUF_U16 = 2, GGUF_I16 = 3, GGUF_U32 = 4, GGUF_I32 = 5,
    GGUF_F32 = 6, GGUF_BOOL = 7, GGUF_STR = 8, GGUF_ARR = 9, GGUF_U64 = 10, GGUF_I64 = 11,
    GGUF_F64 = 12,
};

// ggml tensor types this reader can widen.
enum GgmlType : uint32_t { GGML_F32 = 0, GGML_F16 = 1, GGML_Q8_0 = 8, GGML_BF16 = 30 };

struct GgufValue {
    uint32_t type = 0;
    uint32_t arr_type = 0;
    double num = 0.0;          // numeric scalar (ints, floats, bool)
    std::string str;           // string scalar
    std::vector<double> nums;  // numeric array
    std::vector<std::string> strs;  // string array
};

struct GgufTensor {
    std::string name;
    std::vector<int64_t> ne;  // ggml order, fastest first
    uint32_t type = 0;
    uint64_t offset = 0;      // relative to the data section
    const uint8_t* data = nullptr;
    size_t nbytes = 0;
    int64_t nelements() const {
        int64_t n = 1;
        for (int64_t v : ne) n *= v;
        return n;
    }
};

class Gguf {
public:
    Gguf() = default;
    ~Gguf();
    Gguf(const Gguf&) = delete;
    Gguf& operator=(const Gguf&) = delete;
    // Returns false (and sets err) on a missing, truncated or malformed file. The file
    // is memory-mapped read-only (tensor data is read in place, never copied whole);
    // where mapping fails it is read into memory instead.
    bool load(const std::string& path, std::string& err);

    bool has(const std::string& key) const { return kv_.count(key) != 0; }
    uint32_t u32(const std::string& key, uint32_t def = 0) const;
    float f32(const std::string& key, float def = 0.0f) const;
    bool boolean(const std::string& key, bool def = false) const;
    std::string str(const std::string& key, const std::string& def = "") const;
    std::vector<std::string> str_arr(const std::string& key) const;
    std::vector<int32_t> i32_arr(const std::string& key) const;

    const GgufTensor* tensor(const std::string& name) const;
    // Widen a tensor to f32 in its stored element order. False on unknown type.
    bool to_f32(const GgufTensor& t, std::vector<float>& out, std::string& err) const;

    uint32_t version() const { return version_; }
    size_t n_tensors() const { return tensors_.size(); }

private:
    std::vector<uint8_t> buf_;      // the file, when it could not be mapped
    void* map_ = nullptr;           // the read-only mapping, or null
    size_t map_len_ = 0;
    const uint8_t* data_ = nullptr;  // file bytes (mapping or buf_)
    size_t size_ = 0;
    uint32_t version_ = 0;
    std::map<std::string, GgufValue> kv_;
    std::map<std::string, GgufTensor> tensors_;
};

float half_to_float(uint16_t h);

}  // namespace vdb
