#include "gguf.hpp"

#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <cstdio>
#include <cstring>

namespace vdb {

float half_to_float(uint16_t h) {
    const uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
    uint32_t exp = (h >> 10) & 0x1Fu;
    uint32_t man = h & 0x3FFu;
    uint32_t bits;
    if (exp == 0) {
        if (man == 0) {
            bits = sign;
        } else {  // subnormal: normalise
            exp = 127 - 15 + 1;
            while ((man & 0x400u) == 0) {
                man <<= 1;
                --exp;
            }
            man &= 0x3FFu;
            bits = sign | (exp << 23) | (man << 13);
        }
    } else if (exp == 0x1F) {
        bits = sign | 0x7F800000u | (man << 13);
    } else {
        bits = sign | ((exp + 127 - 15) << 23) | (man << 13);
    }
    float f;
    std::memcpy(&f, &bits, 4);
    return f;
}

namespace {

struct Cursor {
    const uint8_t* p;
    const uint8_t* end;
    bool ok = true;
    template <typename T>
    T get() {
        T v{};
        if (!ok || (size_t)(end - p) < sizeof(T)) {
            ok = false;
            return v;
        }
        std::memcpy(&v, p, sizeof(T));
        p += sizeof(T);
        return v;
    }
    std::string str() {
        const uint64_t n = get<uint64_t>();
        if (!ok || n > (uint64_t)(end - p)) {
            ok = false;
            return {};
        }
        std::string s(reinterpret_cast<const char*>(p), (size_t)n);
        p += n;
        return s;
    }
};

size_t scalar_size(uint32_t t) {
    switch (t) {
        case GGUF_U8: case GGUF_I8: case GGUF_BOOL: return 1;
        case GGUF_U16: case GGUF_I16: return 2;
        case GGUF_U32: case GGUF_I32: case GGUF_F32: return 4;
        case GGUF_U64: case GGUF_I64: case GGUF_F64: return 8;
        default: return 0;
    }
}

double read_num(Cursor& c, uint32_t t) {
    switch (t) {
        case GGUF_U8: return c.get<uint8_t>();
        case GGUF_I8: return c.get<int8_t>();
        case GGUF_BOOL: return c.get<uint8_t>() ? 1.0 : 0.0;
        case GGUF_U16: return c.get<uint16_t>();
        case GGUF_I16: return c.get<int16_t>();
        case GGUF_U32: return c.get<uint32_t>();
        case GGUF_I32: return c.get<int32_t>();
        case GGUF_F32: return c.get<float>();
        case GGUF_U64: return (double)c.get<uint64_t>();
        case GGUF_I64: return (double)c.get<int64_t>();
        case GGUF_F64: return c.get<double>();
        default: c.ok = false; return 0.0;
    }
}

bool ggml_row_bytes(uint32_t type, int64_t n0, size_t& bytes) {
    switch (type) {
        case GGML_F32: bytes = (size_t)n0 * 4; return true;
        case GGML_F16: case GGML_BF16: bytes = (size_t)n0 * 2; return true;
        case GGML_Q8_0:
            if (n0 % 32 != 0) return false;
            bytes = (size_t)(n0 / 32) * 34;
            return true;
        default: return false;
    }
}

}  // namespace

Gguf::~Gguf() {
    if (map_) munmap(map_, map_len_);
}

bool Gguf::load(const std::string& path, std::string& err) {
    const int fd = ::open(path.c_str(), O_RDONLY);
    if (fd < 0) {
        err = "cannot open GGUF: " + path;
        return false;
    }
    struct stat st {};
    if (fstat(fd, &st) != 0 || st.st_size < 24) {
        ::close(fd);
        err = "GGUF too small: " + path;
        return false;
    }
    const size_t sz = (size_t)st.st_size;
    void* m = mmap(nullptr, sz, PROT_READ, MAP_PRIVATE, fd, 0);
    if (m != MAP_FAILED) {
        map_ = m;
        map_len_ = sz;
        data_ = static_cast<const uint8_t*>(m);
    } else {
        buf_.resize(sz);
        size_t got = 0;
        while (got < sz) {
            const ssize_t r = ::read(fd, buf_.data() + got, sz - got);
            if (r <= 0) break;
            got += (size_t)r;
        }
        if (got != sz) {
            ::close(fd);
            err = "short read: " + path;
            return false;
        }
        data_ = buf_.data();
    }
    ::close(fd);
    size_ = sz;
    Cursor c{data_, data_ + size_};
    const uint32_t magic = c.get<uint32_t>();
    if (magic != 0x46554747u) {  // "GGUF"
        err = "not a GGUF file (bad magic): " + path;
        return false;
    }
    version_ = c.get<uint32_t>();
    if (version_ < 2 || version_ > 3) {
        err = "unsupported GGUF version " + std::to_string(version_);
        return false;
    }
    const uint64_t n_tensors = c.get<uint64_t>();
    const uint64_t n_kv = c.get<uint64_t>();
    if (!c.ok || n_tensors > (1u << 24) || n_kv > (1u << 24)) {
        err = "corrupt GGUF header";
        return false;
    }
    for (uint64_t i = 0; i < n_kv && c.ok; ++i) {
        std::string key = c.str();
        GgufValue v;
        v.type = c.get<uint32_t>();
        if (v.type == GGUF_STR) {
            v.str = c.str();
        } else if (v.type == GGUF_ARR) {
            v.arr_type = c.get<uint32_t>();
            const uint64_t n = c.get<uint64_t>();
            if (!c.ok) break;
            if (v.arr_type == GGUF_STR) {
                if (n > (uint64_t)(c.end - c.p) / 8) { c.ok = false; break; }
                v.strs.reserve((size_t)n);
                for (uint64_t j = 0; j < n && c.ok; ++j) v.strs.push_back(c.str());
            } else {
                const size_t es = scalar_size(v.arr_type);
                if (es == 0 || n > (uint64_t)(c.end - c.p) / es) { c.ok = false; break; }
                v.nums.reserve((size_t)n);
                for (uint64_t j = 0; j < n && c.ok; ++j) v.nums.push_back(read_num(c, v.arr_type));
            }
        } else {
            v.num = read_num(c, v.type);
        }
        kv_[key] = std::move(v);
    }
    if (!c.ok) {
        err = "corrupt GGUF metadata";
        return false;
    }
    std::vector<GgufTensor> infos;
    infos.reserve((size_t)n_tensors);
    for (uint64_t i = 0; i < n_tensors && c.ok; ++i) {
        GgufTensor t;
        t.name = c.str();
        const uint32_t nd = c.get<uint32_t>();
        if (nd == 0 || nd > 4) { c.ok = false; break; }
        for (uint32_t d = 0; d < nd; ++d) t.ne.push_back((int64_t)c.get<uint64_t>());
        t.type = c.get<uint32_t>();
        t.offset = c.get<uint64_t>();
        infos.push_back(std::move(t));
    }
    if (!c.ok) {
        err = "corrupt GGUF tensor table";
        return false;
    }
    uint64_t align = 32;
    auto it = kv_.find("general.alignment");
    if (it != kv_.end() && it->second.num > 0) align = (uint64_t)it->second.num;
    const uint64_t pos = (uint64_t)(c.p - data_);
    const uint64_t data0 = (pos + align - 1) / align * align;
    for (GgufTensor& t : infos) {
        size_t row = 0;
        for (int64_t v : t.ne)
            if (v <= 0) {
                err = "tensor '" + t.name + "' has a non-positive dimension";
                return false;
            }
        // A tensor must fit in the file, so no dimension, element count or byte count
        // can exceed the file size: checking that before every multiply keeps a crafted
        // header from wrapping the product to a small value that passes the bounds check.
        const uint64_t limit = (uint64_t)size_;
        uint64_t elems = 1;
        for (int64_t v : t.ne) {
            if ((uint64_t)v > limit || elems > limit / (uint64_t)v) {
                err = "tensor '" + t.name + "' is larger than the file (corrupt dimensions)";
                return false;
            }
            elems *= (uint64_t)v;
        }
        if (!ggml_row_bytes(t.type, t.ne[0], row)) {
            err = "tensor '" + t.name + "' has unsupported type " + std::to_string(t.type);
            return false;
        }
        uint64_t nb = row;
        for (size_t d = 1; d < t.ne.size(); ++d) {
            if (nb > limit / (uint64_t)t.ne[d]) {
                err = "tensor '" + t.name + "' is larger than the file (corrupt dimensions)";
                return false;
            }
            nb *= (uint64_t)t.ne[d];
        }
        t.nbytes = (size_t)nb;
        if (t.offset > limit || data0 > limit - t.offset || nb > limit - (data0 + t.offset)) {
            err = "tensor '" + t.name + "' extends past the end of the file (truncated GGUF?)";
            return false;
        }
        t.data = data_ + data0 + t.offset;
        tensors_[t.name] = t;
    }
    return true;
}

uint32_t Gguf::u32(const std::string& key, uint32_t def) const {
    auto it = kv_.find(key);
    if (it == kv_.end() || it->second.type == GGUF_STR || it->second.type == GGUF_ARR) return def;
    return (uint32_t)it->second.num;
}

float Gguf::f32(const std::string& key, float def) const {
    auto it = kv_.find(key);
    if (it == kv_.end() || it->second.type == GGUF_STR || it->second.type == GGUF_ARR) return def;
    return (float)it->second.num;
}

bool Gguf::boolean(const std::string& key, bool def) const {
    auto it = kv_.find(key);
    if (it == kv_.end() || it->second.type == GGUF_STR || it->second.type == GGUF_ARR) return def;
    return it->second.num != 0.0;
}

std::string Gguf::str(const std::string& key, const std::string& def) const {
    auto it = kv_.find(key);
    if (it == kv_.end() || it->second.type != GGUF_STR) return def;
    return it->second.str;
}

std::vector<std::string> Gguf::str_arr(const std::string& key) const {
    auto it = kv_.find(key);
    if (it == kv_.end() || it->second.type != GGUF_ARR || it->second.arr_type != GGUF_STR)
        return {};
    return it->second.strs;
}

std::vector<int32_t> Gguf::i32_arr(const std::string& key) const {
    auto it = kv_.find(key);
    std::vector<int32_t> out;
    if (it == kv_.end() || it->second.type != GGUF_ARR || it->second.arr_type == GGUF_STR)
        return out;
    for (double v : it->second.nums) out.push_back((int32_t)v);
    return out;
}

const GgufTensor* Gguf::tensor(const std::string& name) const {
    auto it = tensors_.find(name);
    return it == tensors_.end() ? nullptr : &it->second;
}

bool Gguf::to_f32(const GgufTensor& t, std::vector<float>& out, std::string& err) const {
    const int64_t n = t.nelements();
    out.resize((size_t)n);
    switch (t.type) {
        case GGML_F32:
            std::memcpy(out.data(), t.data, (size_t)n * 4);
            return true;
        case GGML_F16: {
            const uint16_t* h = reinterpret_cast<const uint16_t*>(t.data);
            for (int64_t i = 0; i < n; ++i) {
                uint16_t v;
                std::memcpy(&v, h + i, 2);
                out[(size_t)i] = half_to_float(v);
            }
            return true;
        }
        case GGML_BF16: {
            for (int64_t i = 0; i < n; ++i) {
                uint16_t v;
                std::memcpy(&v, t.data + 2 * i, 2);
                const uint32_t bits = (uint32_t)v << 16;
                std::memcpy(&out[(size_t)i], &bits, 4);
            }
            return true;
        }
        case GGML_Q8_0: {
            // blocks of 32: f16 scale d, then 32 int8 q; value = d * q
            const int64_t nb = n / 32;
            for (int64_t b = 0; b < nb; ++b) {
                const uint8_t* blk = t.data + b * 34;
                uint16_t dh;
                std::memcpy(&dh, blk, 2);
                const float d = half_to_float(dh);
                const int8_t* q = reinterpret_cast<const int8_t*>(blk + 2);
                for (int i = 0; i < 32; ++i) out[(size_t)(b * 32 + i)] = d * (float)q[i];
            }
            return true;
        }
        default:
            err = "tensor '" + t.name + "': unsupported type";
            return false;
    }
}

}  // namespace vdb
