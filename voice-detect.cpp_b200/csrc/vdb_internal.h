// Host-side helpers shared by the engine's .cu/.cpp files (not part of the ABI).
#pragma once
#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <string>

namespace vdb {

// Thread-local last error for the op-level C ABI (vdb_last_error).
void set_error(const std::string& msg);
const std::string& get_error();

// Kernels the calling thread's last vdb_conv / vdb_conv1d call launched (the conv, plus
// one per q8_0 weight segment it expanded into the scratch).
int last_conv_launches();

// cuTensorMapEncodeTiled resolved through the runtime's driver entry point
// (no link-time dependency on libcuda).
using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                   const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                   const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion,
                                   CUtensorMapFloatOOBfill);
EncodeTiledFn encode_tiled_fn();

int num_sms();

// Keeps memory freed by cudaFreeAsync cached in the current device's default pool
// (once per device), so repeated calls with stream-ordered workspace do not pay a
// fresh allocation each time.
void keep_async_pool();

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
// The embedding FC + bias - mean_vec + L2 of pool_embed_launch on pooled vectors
// already in device memory (f32 [batch][P]); `part` holds
// pool_fc_splits(batch, P, emb_dim) * batch * emb_dim floats.
int fc_embed_launch(const float* pooled, int batch, int P, const float* seg_w,
                    const float* seg_b, const float* mean_vec, int emb_dim, int l2,
                    const int* out_rows, float* emb_out, float* prenorm_out, float* part,
                    cudaStream_t stream);

// CMN + stem of vdb_cmn_stem with the output in GRID (fphase 0), FPHASE (fphase 1,
// for a frequency-stride-2 consumer: CAM++'s FCM) or QPACK (fphase 2, oc 32: the
// ResNet stage-1 convs) layout.
int cmn_stem_launch(const float* feats, const int* frames, int batch, int t_max, int n_mels,
                    int cmn, const float* stem_w, const float* stem_b, int oc,
                    float* mean_scratch, void* y, int fphase, cudaStream_t stream);

// ECAPA-TDNN glue kernels on the SEQ layout (ecapa.cu). tv: device int32 [batch]
// valid frames; T and pad describe the SEQ tensors; ld* are row pitches.
int ecapa_cmn_pack(const float* feats, const int* frames, int batch, int t_max, int n_mels,
                   int cmn, int pad, __half* x, cudaStream_t st);
int ecapa_seq_mean(const __half* x, int ldx, const int* tv, int batch, int T, int pad, int C,
                   float* out, cudaStream_t st);
// out[b][n] = act(bias[n] + W[n] . in[b]) for f32 in [batch][K], W [N][K], out [batch][N]
// (dense); act 0 none, 1 ReLU, 2 sigmoid. A tiled split-K GEMM (the embedding FC's
// kernel) plus a finish pass; `part` holds small_gemm_scratch_floats(batch, K, N).
size_t small_gemm_scratch_floats(int batch, int K, int N);
int small_gemm_launch(const float* in, int batch, int K, const float* W, int N, const float* bias,
                      int act, float* out, float* part, cudaStream_t stream);
int ecapa_se_apply(const __half* h, int ldh, const float* gate, const __half* res, int ldr,
                   const int* tv, int batch, int T, int pad, int C, __half* y, int ldy,
                   cudaStream_t st);
int ecapa_meanstd(const __half* x, int ldx, const int* tv, int batch, int T, int pad, int C,
                  float eps, float* stats, cudaStream_t st);
// stats: [batch][2C] global mean | std of x (ecapa_meanstd), the shift of the moments
int ecapa_asp_pool(const float* logits, int ldl, const __half* x, int ldx, const float* stats,
                   const int* tv, int batch, int T, int pad, int C, float eps, float* pooled,
                   cudaStream_t st);

// CAM++ (campplus.cu): mean / std pooling with the unbiased variance and no floor
// (ecapa.cu's kernel) and the CAM gate [batch][nseg_max][G] =
// sigmoid(w2 . ReLU(w1 . ctx + b1) + b2) per 100-frame segment, with the weights
// transposed: w1t f32 [C][M], w2t f32 [M][G].
int seq_meanstd_unbiased(const __half* x, int ldx, const int* tv, int batch, int T, int pad,
                         int C, float* stats, cudaStream_t st);
size_t campp_gate_smem(int C, int M, int G, int nseg_max);
int campp_cam_gate(const __half* cc, int ldc, const int* tv, int batch, int T, int pad, int C,
                   int seg, int nseg_max, const float* w1t, const float* b1, int M,
                   const float* w2t, const float* b2, int G, float* gate, cudaStream_t st);

}  // namespace vdb

#define VDB_CHECK_CUDA(expr)                                                        \
    do {                                                                            \
        cudaError_t _e = (expr);                                                    \
        if (_e != cudaSuccess) {                                                    \
            ::vdb::set_error(std::string(#expr) + ": " + cudaGetErrorString(_e));   \
            return 1;                                                               \
        }                                                                           \
    } while (0)
