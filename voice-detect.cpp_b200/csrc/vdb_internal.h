// Host-side helpers shared by the engine's .cu/.cpp files (not part of the ABI).
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>

#include <string>

namespace vdb {

// Thread-local last error for the op-level C ABI (vdb_last_error).
void set_error(const std::string& msg);
const std::string& get_error();

// cuTensorMapEncodeTiled resolved through the runtime's driver entry point
// (no link-time dependency on libcuda).
using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                   const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                   const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion,
                                   CUtensorMapFloatOOBfill);
EncodeTiledFn encode_tiled_fn();

int num_sms();

// Pooling + FC + L2 launcher with an optional output-row map (row b of the batch
// is written to out_rows[b]); vdb_pool_embed is the public wrapper. `scratch`
// holds pool_embed_scratch_floats(...) floats of device working memory (the
// pooled vectors and the split-K FC partials).
int pool_fc_splits(int batch, int P, int emb_dim);
size_t pool_embed_scratch_floats(int batch, int f, int c, int emb_dim);
int pool_embed_launch(const void* x, const int* tvalid, int batch, int t, int f, int c,
                      const float* seg_w, const float* seg_b, const float* mean_vec, int emb_dim,
                      float var_eps, int l2, const int* out_rows, float* emb_out,
                      float* prenorm_out, float* scratch, cudaStream_t stream);

}  // namespace vdb

#define VDB_CHECK_CUDA(expr)                                                        \
    do {                                                                            \
        cudaError_t _e = (expr);                                                    \
        if (_e != cudaSuccess) {                                                    \
            ::vdb::set_error(std::string(#expr) + ": " + cudaGetErrorString(_e));   \
            return 1;                                                               \
        }                                                                           \
    } while (0)
