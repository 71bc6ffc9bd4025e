// Front and tail of the encoder around the tensor-core conv stack:
//   * CMN + stem: per-utterance cepstral mean normalisation (src/fbank.cpp:194-201)
//     fused into the IC=1 stem conv3x3 + bias + ReLU (src/encoder_resnet.cpp:116-117,
//     reference kernel src/directconv.cpp:463-521). With K = 9 the stem does not
//     fit a tensor-core tile; it is a CUDA-core kernel, one thread per output
//     pixel writing all its channels, memory-bound on the f16 GRID output.
//   * TSTP + FC + L2: temporal statistics pooling (mean and unbiased std over the
//     valid frames, src/encoder_resnet.cpp:143-157), the embedding layer
//     (:162-170) and the L2 normalisation the reference does on the host
//     (:177-183), fused in one kernel with one CTA per clip.
#include <cuda_fp16.h>

#include <cmath>
#include <algorithm>
#include <cstdint>
#include <mutex>
#include <string>

#include "vdb_internal.h"
#include "vdb_ops.h"

namespace vdb {
namespace {

// mean[b][m] = (float)(sum_{t < T_b} feats[b][t][m] / T_b), summed in f64.
__global__ void cmn_mean_kernel(const float* __restrict__ feats, const int* __restrict__ frames,
                                int t_max, int n_mels, float* __restrict__ mean) {
    __shared__ double part[4][128];
    const int b = blockIdx.x;
    const int m = threadIdx.x;
    const int ty = threadIdx.y;
    const int T = min(frames[b], t_max);
    double s = 0.0;
    if (m < n_mels)
        for (int t = ty; t < T; t += 4) s += (double)feats[((long long)b * t_max + t) * n_mels + m];
    part[ty][m] = s;
    __syncthreads();
    if (ty == 0 && m < n_mels) {
        const double tot = part[0][m] + part[1][m] + part[2][m] + part[3][m];
        mean[b * n_mels + m] = T > 0 ? (float)(tot / T) : 0.0f;
    }
}

template <int OC>
__global__ void __launch_bounds__(256)
stem_kernel(const float* __restrict__ feats, const int* __restrict__ frames,
            const float* __restrict__ mean, int batch, int t_max, int n_mels, int cmn,
            const float* __restrict__ w, const float* __restrict__ bias, __half* __restrict__ y) {
    __shared__ float sw[OC * 9];
    __shared__ float sb[OC];
    for (int i = threadIdx.x; i < OC * 9; i += blockDim.x) sw[i] = w[i];
    for (int i = threadIdx.x; i < OC; i += blockDim.x) sb[i] = bias[i];
    __syncthreads();
    const int Wp = n_mels + 2, Hp = t_max + 2;
    const long long rows = (long long)batch * Hp * Wp;
    const long long r = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (r >= rows) return;
    const int b = (int)(r / ((long long)Hp * Wp));
    const int rr = (int)(r - (long long)b * Hp * Wp);
    const int tp = rr / Wp, fp = rr - tp * Wp;
    const int T = min(frames[b], t_max);
    float acc[OC];
#pragma unroll
    for (int o = 0; o < OC; ++o) acc[o] = 0.0f;
    const bool valid = tp >= 1 && tp <= T && fp >= 1 && fp <= n_mels;
    if (valid) {
        const int t = tp - 1, f = fp - 1;
        const float* fb = feats + (long long)b * t_max * n_mels;
        const float* mb = mean + (long long)b * n_mels;
        // accumulate in the reference's kh (freq) -> kw (time) order
#pragma unroll
        for (int kf = 0; kf < 3; ++kf) {
            const int ff = f + kf - 1;
#pragma unroll
            for (int kt = 0; kt < 3; ++kt) {
                const int tt = t + kt - 1;
                float xin = 0.0f;
                if (ff >= 0 && ff < n_mels && tt >= 0 && tt < T) {
                    xin = __ldg(fb + (long long)tt * n_mels + ff);
                    if (cmn) xin = __fsub_rn(xin, __ldg(mb + ff));
                }
#pragma unroll
                for (int o = 0; o < OC; ++o) acc[o] = fmaf(sw[o * 9 + kt * 3 + kf], xin, acc[o]);
            }
        }
#pragma unroll
        for (int o = 0; o < OC; ++o) acc[o] = fmaxf(acc[o] + sb[o], 0.0f);
    }
    uint4* yp = reinterpret_cast<uint4*>(y + r * OC);
#pragma unroll
    for (int j = 0; j < OC / 8; ++j) {
        uint4 q;
        __half2 h0 = __floats2half2_rn(acc[j * 8 + 0], acc[j * 8 + 1]);
        __half2 h1 = __floats2half2_rn(acc[j * 8 + 2], acc[j * 8 + 3]);
        __half2 h2 = __floats2half2_rn(acc[j * 8 + 4], acc[j * 8 + 5]);
        __half2 h3 = __floats2half2_rn(acc[j * 8 + 6], acc[j * 8 + 7]);
        q.x = *reinterpret_cast<uint32_t*>(&h0);
        q.y = *reinterpret_cast<uint32_t*>(&h1);
        q.z = *reinterpret_cast<uint32_t*>(&h2);
        q.w = *reinterpret_cast<uint32_t*>(&h3);
        yp[j] = q;
    }
}

__device__ __forceinline__ double block_sum_d(double v, double* red) {
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    __syncthreads();
    if (lane == 0) red[warp] = v;
    __syncthreads();
    double t = 0.0;
    for (int i = 0; i < (int)(blockDim.x >> 5); ++i) t += red[i];
    return t;
}

// One CTA per clip. Dynamic smem: pooled [2*c*f] + emb [emb_dim] floats.
__global__ void __launch_bounds__(256)
pool_embed_kernel(const __half* __restrict__ x, const int* __restrict__ tvalid, int T, int F,
                  int C, const float* __restrict__ seg_w, const float* __restrict__ seg_b,
                  const float* __restrict__ mean_vec, int D, float eps, int l2,
                  const int* __restrict__ out_rows, float* __restrict__ emb_out,
                  float* __restrict__ prenorm_out) {
    extern __shared__ float sm[];
    __shared__ double red[32];
    const int b = blockIdx.x;
    const int HC = C * F;
    float* pooled = sm;
    float* emb = sm + 2 * HC;
    const int N = min(tvalid[b], T);
    const long long img_row0 = (long long)b * (T + 2) * (F + 2);
    for (int p = threadIdx.x; p < HC; p += blockDim.x) {
        const int c = p % C, f = p / C;
        const __half* col = x + (img_row0 + (F + 2) + f + 1) * C + c;  // (t=0, f)
        const long long tstride = (long long)(F + 2) * C;
        double s = 0.0;
        for (int t = 0; t < N; ++t) s += (double)__half2float(col[t * tstride]);
        const float mean = N > 0 ? (float)(s / N) : 0.0f;
        double s2 = 0.0;
        for (int t = 0; t < N; ++t) {
            const float d = __half2float(col[t * tstride]) - mean;
            s2 += (double)(d * d);
        }
        float var = N > 0 ? (float)(s2 / N) : 0.0f;
        if (N > 1) var = var * ((float)N / (float)(N - 1));
        pooled[c * F + f] = mean;
        pooled[HC + c * F + f] = sqrtf(var + eps);
    }
    __syncthreads();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
    const int P = 2 * HC;
    for (int j = warp; j < D; j += nw) {
        const float* wr = seg_w + (long long)j * P;
        float a = 0.0f;
        for (int i = lane; i < P; i += 32) a = fmaf(__ldg(wr + i), pooled[i], a);
#pragma unroll
        for (int o = 16; o >= 1; o >>= 1) a += __shfl_xor_sync(0xffffffffu, a, o);
        if (lane == 0) {
            float v = a + seg_b[j];
            if (mean_vec) v -= mean_vec[j];
            emb[j] = v;
        }
    }
    __syncthreads();
    double n2 = 0.0;
    for (int j = threadIdx.x; j < D; j += blockDim.x) n2 += (double)emb[j] * (double)emb[j];
    n2 = block_sum_d(n2, red);
    const double nrm = sqrt(n2);
    const long long orow = out_rows ? out_rows[b] : b;
    for (int j = threadIdx.x; j < D; j += blockDim.x) {
        const float v = emb[j];
        if (prenorm_out) prenorm_out[orow * D + j] = v;
        emb_out[orow * D + j] = (l2 && nrm > 0.0) ? (float)((double)v / nrm) : v;
    }
}

}  // namespace

int pool_embed_launch(const void* x, const int* tvalid, int batch, int t, int f, int c,
                      const float* seg_w, const float* seg_b, const float* mean_vec, int emb_dim,
                      float var_eps, int l2, const int* out_rows, float* emb_out,
                      float* prenorm_out, cudaStream_t stream) {
    const size_t smem = sizeof(float) * ((size_t)2 * c * f + emb_dim);
    if (smem > 200 * 1024) {
        set_error("vdb_pool_embed: pooled vector too large");
        return 1;
    }
    static bool attr = false;
    if (!attr) {
        VDB_CHECK_CUDA(cudaFuncSetAttribute(pool_embed_kernel,
                                            cudaFuncAttributeMaxDynamicSharedMemorySize,
                                            200 * 1024));
        attr = true;
    }
    pool_embed_kernel<<<batch, 256, smem, stream>>>(static_cast<const __half*>(x), tvalid, t, f,
                                                    c, seg_w, seg_b, mean_vec, emb_dim, var_eps,
                                                    l2, out_rows, emb_out, prenorm_out);
    VDB_CHECK_CUDA(cudaGetLastError());
    return 0;
}

}  // namespace vdb

using namespace vdb;

extern "C" int vdb_cmn_stem(const float* feats, const int* frames, int batch, int t_max,
                            int n_mels, int cmn, const float* stem_w, const float* stem_b,
                            int oc, float* mean_scratch, void* y, void* stream) {
    if (!feats || !frames || !stem_w || !stem_b || !y || (cmn && !mean_scratch)) {
        set_error("vdb_cmn_stem: NULL argument");
        return 1;
    }
    if (batch <= 0 || t_max <= 0 || n_mels <= 0 || n_mels > 128) {
        set_error("vdb_cmn_stem: bad shape");
        return 1;
    }
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    if (cmn) {
        cmn_mean_kernel<<<batch, dim3(128, 4), 0, st>>>(feats, frames, t_max, n_mels,
                                                       mean_scratch);
        VDB_CHECK_CUDA(cudaGetLastError());
    }
    const long long rows = vdb_grid_rows(batch, t_max, n_mels);
    const int threads = 256;
    const unsigned blocks = (unsigned)((rows + threads - 1) / threads);
    __half* yh = static_cast<__half*>(y);
    switch (oc) {
        case 16:
            stem_kernel<16><<<blocks, threads, 0, st>>>(feats, frames, mean_scratch, batch, t_max,
                                                        n_mels, cmn, stem_w, stem_b, yh);
            break;
        case 32:
            stem_kernel<32><<<blocks, threads, 0, st>>>(feats, frames, mean_scratch, batch, t_max,
                                                        n_mels, cmn, stem_w, stem_b, yh);
            break;
        case 64:
            stem_kernel<64><<<blocks, threads, 0, st>>>(feats, frames, mean_scratch, batch, t_max,
                                                        n_mels, cmn, stem_w, stem_b, yh);
            break;
        default:
            set_error("vdb_cmn_stem: stem channels must be 16, 32 or 64");
            return 1;
    }
    VDB_CHECK_CUDA(cudaGetLastError());
    return 0;
}

namespace vdb {
namespace {
__global__ void add_slices_kernel(const uint4* __restrict__ a, int lda8, const uint4* __restrict__ b,
                                  int ldb8, uint4* __restrict__ y, int ldy8, long long rows,
                                  int c8) {
    const long long n = rows * c8;
    for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n;
         i += (long long)gridDim.x * blockDim.x) {
        const long long r = i / c8;
        const int c = (int)(i - r * c8);
        const uint4 va = a[r * lda8 + c], vb = b[r * ldb8 + c];
        uint4 o;
        const __half2* ha = reinterpret_cast<const __half2*>(&va);
        const __half2* hb = reinterpret_cast<const __half2*>(&vb);
        __half2* ho = reinterpret_cast<__half2*>(&o);
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            const float2 fa = __half22float2(ha[k]), fb = __half22float2(hb[k]);
            ho[k] = __floats2half2_rn(fa.x + fb.x, fa.y + fb.y);
        }
        y[r * ldy8 + c] = o;
    }
}
}  // namespace
}  // namespace vdb

extern "C" int vdb_add(const void* a, int lda, const void* b, int ldb, void* y, int ldy,
                       long long rows, int C, void* stream) {
    auto mis = [](const void* q) { return (reinterpret_cast<uintptr_t>(q) & 15u) != 0; };
    if (!a || !b || !y || rows <= 0 || C <= 0 || C % 8 || lda % 8 || ldb % 8 || ldy % 8 ||
        lda < C || ldb < C || ldy < C || mis(a) || mis(b) || mis(y)) {
        set_error("vdb_add: bad arguments (NULL, pitch < C, or not multiples of 8 / 16 B)");
        return 1;
    }
    const long long n = rows * (C / 8);
    const int threads = 256;
    const int blocks = (int)std::min<long long>((n + threads - 1) / threads, 148LL * 16);
    add_slices_kernel<<<blocks, threads, 0, static_cast<cudaStream_t>(stream)>>>(
        static_cast<const uint4*>(a), lda / 8, static_cast<const uint4*>(b), ldb / 8,
        static_cast<uint4*>(y), ldy / 8, rows, C / 8);
    VDB_CHECK_CUDA(cudaGetLastError());
    return 0;
}

// ---- CMN + stem without any allocation ---------------------------------------
// vdb_cmn_stem needs working memory for the per-clip CMN means and asks the caller
// for it. Some callers cannot provide or allocate it: a streaming audio callback
// must not call cudaMalloc/cudaFree (they can synchronise the whole device and
// take unbounded time), and a host that owns all device memory through its own
// pool does not allow a library to allocate behind its back. For them the means
// live in this fixed array, compiled into the library, which every GPU that loads
// the library holds until the process exits.
namespace {
constexpr int kNoAllocMaxMeans = 65536;  // batch * n_mels (256 KB of f32)
static __device__ __align__(256) float g_cmn_means[kNoAllocMaxMeans];
constexpr int kMaxDevices = 64;
std::once_flag g_means_once[kMaxDevices];
float* g_means_addr[kMaxDevices] = {};
cudaError_t g_means_status[kMaxDevices] = {};
}  // namespace

extern "C" int vdb_cmn_stem_noalloc(const float* feats, const int* frames, int batch, int t_max,
                                    int n_mels, int cmn, const float* stem_w,
                                    const float* stem_b, int oc, void* y, void* stream) {
    if (!feats || !frames || !stem_w || !stem_b || !y) {
        set_error("vdb_cmn_stem_noalloc: NULL argument");
        return 1;
    }
    if (batch <= 0 || t_max <= 0 || n_mels <= 0 || n_mels > 128) {
        set_error("vdb_cmn_stem_noalloc: bad shape");
        return 1;
    }
    if ((long long)batch * n_mels > kNoAllocMaxMeans) {
        set_error("vdb_cmn_stem_noalloc: batch * n_mels = " +
                  std::to_string((long long)batch * n_mels) +
                  " exceeds the built-in limit of 65536 (use vdb_cmn_stem with caller memory)");
        return 1;
    }
    if (!(oc == 16 || oc == 32 || oc == 64)) {
        set_error("vdb_cmn_stem_noalloc: stem channels must be 16, 32 or 64");
        return 1;
    }
    int dev = 0;
    VDB_CHECK_CUDA(cudaGetDevice(&dev));
    if (dev < 0 || dev >= kMaxDevices) {
        set_error("vdb_cmn_stem_noalloc: device ordinal out of range");
        return 1;
    }
    // First call on this device (with it current): look up the array's device
    // address. A host-side reference to g_cmn_means is not a device address.
    std::call_once(g_means_once[dev], [dev] {
        void* p = nullptr;
        g_means_status[dev] = cudaGetSymbolAddress(&p, g_cmn_means);
        g_means_addr[dev] = static_cast<float*>(p);
    });
    if (g_means_status[dev] != cudaSuccess || !g_means_addr[dev]) {
        set_error(std::string("vdb_cmn_stem_noalloc: cudaGetSymbolAddress failed: ") +
                  cudaGetErrorString(g_means_status[dev]));
        return 1;
    }
    float* means = g_means_addr[dev];
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    // The mean kernel writes every entry the stem kernel reads, so the array's
    // previous contents never leak into a result.
    if (cmn) {
        cmn_mean_kernel<<<batch, dim3(128, 4), 0, st>>>(feats, frames, t_max, n_mels, means);
        VDB_CHECK_CUDA(cudaGetLastError());
    }
    const long long rows = vdb_grid_rows(batch, t_max, n_mels);
    const int threads = 256;
    const unsigned blocks = (unsigned)((rows + threads - 1) / threads);
    __half* yh = static_cast<__half*>(y);
    if (oc == 16)
        stem_kernel<16><<<blocks, threads, 0, st>>>(feats, frames, means, batch, t_max, n_mels,
                                                    cmn, stem_w, stem_b, yh);
    else if (oc == 32)
        stem_kernel<32><<<blocks, threads, 0, st>>>(feats, frames, means, batch, t_max, n_mels,
                                                    cmn, stem_w, stem_b, yh);
    else
        stem_kernel<64><<<blocks, threads, 0, st>>>(feats, frames, means, batch, t_max, n_mels,
                                                    cmn, stem_w, stem_b, yh);
    VDB_CHECK_CUDA(cudaGetLastError());
    return 0;
}

extern "C" int vdb_pool_embed(const void* x, const int* tvalid, int batch, int t, int f, int c,
                              const float* seg_w, const float* seg_b, const float* mean_vec,
                              int emb_dim, float var_eps, int l2, float* emb_out,
                              float* prenorm_out, void* stream) {
    if (!x || !tvalid || !seg_w || !seg_b || !emb_out) {
        set_error("vdb_pool_embed: NULL argument");
        return 1;
    }
    if (batch <= 0 || t <= 0 || f <= 0 || c <= 0 || emb_dim <= 0) {
        set_error("vdb_pool_embed: bad shape");
        return 1;
    }
    return pool_embed_launch(x, tvalid, batch, t, f, c, seg_w, seg_b, mean_vec, emb_dim, var_eps,
                             l2, nullptr, emb_out, prenorm_out, static_cast<cudaStream_t>(stream));
}
