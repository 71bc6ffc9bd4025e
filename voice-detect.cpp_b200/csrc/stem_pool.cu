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

// The stem, one block per (image, run of kStemRows padded time rows). The block
// first stages the CMN'd features its rows read — kStemRows + 2 feature rows,
// zero outside the clip and at the frequency borders — in shared memory (a warp per
// row), so the nine taps need no bounds checks and CMN is applied once per input.
// Then each thread computes 8 channels of one padded pixel per step (weights in
// registers) and a warp stores 512 contiguous bytes; the block's output rows are
// contiguous. 64 rows per block: with two blocks per SM (125 registers a thread) the
// staging phase's load latency and the per-thread weight loads are paid once per
// block (16 rows: 810 us for the 131 x 20 s bucket, 64 rows with two pixels per
// thread: 728 us, bit-identical output).
constexpr int kStemRows = 64;

template <int OC>
__global__ void __launch_bounds__(256, 2)
stem_kernel(const float* __restrict__ feats, const int* __restrict__ frames,
            const float* __restrict__ mean, int batch, int t_max, int n_mels, int cmn,
            const float* __restrict__ w, const float* __restrict__ bias, __half* __restrict__ y,
            int fphase) {
    constexpr int G = OC / 8;
    constexpr int PPB = 256 / G;  // pixel pairs per block step
    __shared__ float sx[(kStemRows + 2) * 130];
    const int g = (int)threadIdx.x % G;
    const int pl = (int)threadIdx.x / G;
    const int Wp = n_mels + 2, Hp = t_max + 2;
    const int b = blockIdx.y;
    const int tp0 = blockIdx.x * kStemRows;
    const int T = min(frames[b], t_max);
    const float* fb = feats + (long long)b * t_max * n_mels;
    const float* mb = mean + (long long)b * n_mels;
    // sx[i][j] = feature(row tp0 - 2 + i, mel j - 1) - mean, 0 outside the clip
    {
        const int warp = (int)threadIdx.x >> 5, lane = (int)threadIdx.x & 31;
        for (int i = warp; i < kStemRows + 2; i += (int)blockDim.x >> 5) {
            const int tt = tp0 - 2 + i;
            const bool row_in = tt >= 0 && tt < T;
            for (int j = lane; j < Wp; j += 32) {
                const int ff = j - 1;
                float v = 0.0f;
                if (row_in && ff >= 0 && ff < n_mels) {
                    v = __ldg(fb + (long long)tt * n_mels + ff);
                    if (cmn) v = __fsub_rn(v, __ldg(mb + ff));
                }
                sx[i * Wp + j] = v;
            }
        }
    }
    // weights of channel pairs (2i, 2i+1) packed for the f32x2 fused multiply-add:
    // each lane rounds exactly like fmaf, with half the instructions (the stem is
    // issue bound)
    float2 wr[4][9];
    float br[8];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
#pragma unroll
        for (int k = 0; k < 9; ++k)
            wr[i][k] = make_float2(__ldg(w + (g * 8 + 2 * i) * 9 + k),
                                   __ldg(w + (g * 8 + 2 * i + 1) * 9 + k));
    }
#pragma unroll
    for (int o = 0; o < 8; ++o) br[o] = __ldg(bias + g * 8 + o);
    __syncthreads();
    // QPACK (fphase 2) rows carry 4 * Wq pixels: the ones past the padded grid are 0
    const int Wq4 = 4 * ((n_mels + 2 + 3) / 4);
    const int Wx = fphase == 2 ? Wq4 : Wp;  // pixels stored per time row
    uint4* yb = reinterpret_cast<uint4*>(y) + ((long long)b * Hp + tp0) * Wp * G;
    auto store_px = [&](int r, int fp, const float* acc) {
        const int tp = tp0 + r;
        uint4 v;
        __half2 h0 = __floats2half2_rn(acc[0], acc[1]);
        __half2 h1 = __floats2half2_rn(acc[2], acc[3]);
        __half2 h2 = __floats2half2_rn(acc[4], acc[5]);
        __half2 h3 = __floats2half2_rn(acc[6], acc[7]);
        v.x = *reinterpret_cast<uint32_t*>(&h0);
        v.y = *reinterpret_cast<uint32_t*>(&h1);
        v.z = *reinterpret_cast<uint32_t*>(&h2);
        v.w = *reinterpret_cast<uint32_t*>(&h3);
        if (fphase == 2) {
            // QPACK output (vdb_ops.h): pixel fp of time row tp is channels
            // (fp & 3) * OC .. of QPACK row (b * Hp + tp) * Wq + fp / 4
            const long long row = ((long long)b * Hp + tp) * (Wq4 / 4) + (fp >> 2);
            reinterpret_cast<uint4*>(y)[(row * 4 + (fp & 3)) * G + g] = v;
        } else if (fphase) {
            // FPHASE output for a frequency-stride-2 consumer (vdb_ops.h)
            const int Wq = (n_mels - 1) / 2 + 1 + 2;
            const long long dst = (long long)(fp & 1) * batch * Hp * Wq +
                                  ((long long)b * Hp + tp) * Wq + (fp >> 1) + 1;
            reinterpret_cast<uint4*>(y)[dst * G + g] = v;
        } else {
            yb[((long long)r * Wx + fp) * G + g] = v;
        }
    };
    // Each step a thread computes 8 channels of two neighbouring padded pixels (fp,
    // fp + 1) of one time row: the pair shares two of its three tap columns and the
    // weights in registers, so a pixel costs two thirds of the shared-memory loads and
    // half the index, predicate and store work of one pixel per step, with twice the
    // independent accumulation chains. Each pixel's sums run in the same order.
    const int Wx2 = (Wx + 1) / 2;  // pixel pairs per time row
    const int npairs = min(kStemRows, Hp - tp0) * Wx2;
    // pair q = r * Wx2 + fp / 2, stepped without a division
    int r = pl / Wx2, fp = 2 * (pl - (pl / Wx2) * Wx2);
    for (int q = pl; q < npairs; q += PPB) {
        if (q != pl) {
            fp += 2 * PPB;
            while (fp >= 2 * Wx2) {
                fp -= 2 * Wx2;
                ++r;
            }
        }
        const int tp = tp0 + r;
        const bool row_in = tp >= 1 && tp <= T;
        const bool va = row_in && fp >= 1 && fp <= n_mels;
        const bool vb = row_in && fp + 1 <= n_mels;
        float acc[2][8];
#pragma unroll
        for (int o = 0; o < 8; ++o) acc[0][o] = acc[1][o] = 0.0f;
        if (va || vb) {
            // tap columns fp - 1 .. fp + 2 of staged rows r .. r + 2; a valid pixel's
            // columns lie in [0, Wp); the clamp only touches a discarded pixel's
            float xs[3][4];
#pragma unroll
            for (int kt = 0; kt < 3; ++kt)
#pragma unroll
                for (int c = 0; c < 4; ++c)
                    xs[kt][c] = sx[(r + kt) * Wp + min(max(fp - 1 + c, 0), Wp - 1)];
            float2 aa[4], ab[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) aa[i] = ab[i] = make_float2(0.f, 0.f);
            // accumulate in the reference's kh (freq) -> kw (time) order
#pragma unroll
            for (int kf = 0; kf < 3; ++kf) {
#pragma unroll
                for (int kt = 0; kt < 3; ++kt) {
                    const float2 xa = make_float2(xs[kt][kf], xs[kt][kf]);
                    const float2 xb = make_float2(xs[kt][kf + 1], xs[kt][kf + 1]);
#pragma unroll
                    for (int i = 0; i < 4; ++i) {
                        aa[i] = __ffma2_rn(wr[i][kt * 3 + kf], xa, aa[i]);
                        ab[i] = __ffma2_rn(wr[i][kt * 3 + kf], xb, ab[i]);
                    }
                }
            }
            if (va)
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    acc[0][2 * i] = fmaxf(aa[i].x + br[2 * i], 0.0f);
                    acc[0][2 * i + 1] = fmaxf(aa[i].y + br[2 * i + 1], 0.0f);
                }
            if (vb)
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    acc[1][2 * i] = fmaxf(ab[i].x + br[2 * i], 0.0f);
                    acc[1][2 * i + 1] = fmaxf(ab[i].y + br[2 * i + 1], 0.0f);
                }
        }
        store_px(r, fp, acc[0]);
        if (fp + 1 < Wx) store_px(r, fp + 1, acc[1]);
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

// TSTP, one CTA per clip: pooled[b][c*F + f] = mean, pooled[b][C*F + c*F + f] = std
// over the clip's valid frames (two passes in f64, unbiased variance, eps inside
// the sqrt), in the reference's C-outer / F-inner flattening. Thread u owns 8
// channels of one mel column (u = f * C/8 + c/8): a warp reads 512 contiguous bytes
// per frame, and each channel's sums run over the frames in order, as before.
__global__ void __launch_bounds__(1024)
tstp_kernel(const __half* __restrict__ x, const int* __restrict__ tvalid, int T, int F, int C,
            float eps, float* __restrict__ pooled) {
    const int b = blockIdx.x;
    const int HC = C * F;
    const int C8 = C / 8;
    const int N = min(tvalid[b], T);
    const long long img_row0 = (long long)b * (T + 2) * (F + 2);
    float* out = pooled + (long long)b * 2 * HC;
    const long long tstride = (long long)(F + 2) * C8;  // in 16-byte units
    for (int u = threadIdx.x; u < F * C8; u += blockDim.x) {
        const int f = u / C8, c0 = (u - f * C8) * 8;
        const uint4* col = reinterpret_cast<const uint4*>(x + (img_row0 + (F + 2) + f + 1) * C + c0);
        double s[8];
#pragma unroll
        for (int k = 0; k < 8; ++k) s[k] = 0.0;
#pragma unroll 4
        for (int t = 0; t < N; ++t) {
            const uint4 v = __ldg(col + t * tstride);
            const __half2* h = reinterpret_cast<const __half2*>(&v);
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                const float2 p = __half22float2(h[k]);
                s[2 * k] += (double)p.x;
                s[2 * k + 1] += (double)p.y;
            }
        }
        float mean[8];
#pragma unroll
        for (int k = 0; k < 8; ++k) mean[k] = N > 0 ? (float)(s[k] / N) : 0.0f;
        double s2[8];
#pragma unroll
        for (int k = 0; k < 8; ++k) s2[k] = 0.0;
#pragma unroll 4
        for (int t = 0; t < N; ++t) {
            const uint4 v = __ldg(col + t * tstride);
            const __half2* h = reinterpret_cast<const __half2*>(&v);
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                const float2 p = __half22float2(h[k]);
                const float d0 = p.x - mean[2 * k], d1 = p.y - mean[2 * k + 1];
                s2[2 * k] += (double)(d0 * d0);
                s2[2 * k + 1] += (double)(d1 * d1);
            }
        }
#pragma unroll
        for (int k = 0; k < 8; ++k) {
            float var = N > 0 ? (float)(s2[k] / N) : 0.0f;
            if (N > 1) var = var * ((float)N / (float)(N - 1));
            out[(c0 + k) * F + f] = mean[k];
            out[HC + (c0 + k) * F + f] = sqrtf(var + eps);
        }
    }
}

// Embedding FC over a bucket as a split-K f32 GEMM: part[s][b][j] = sum over the
// s-th K range of pooled[b][k] * W[j][k]. 64 clips x 64 outputs per CTA, K tiles
// of 16 staged k-major in shared memory with float4 global loads, 4 x 4 outputs per
// thread read as two float4s per k (16 FMAs per 2 shared loads). Each weight tile
// is read once per 64 clips instead of once per clip. K must be a multiple of 4
// (16-byte rows); k_per_split a multiple of kFcBK.
constexpr int kFcBM = 64, kFcBN = 64, kFcBK = 16;

__global__ void __launch_bounds__(256)
fc_partial_kernel(const float* __restrict__ pooled, const float* __restrict__ W, int B, int D,
                  int P, int k_per_split, float* __restrict__ part) {
    __shared__ __align__(16) float As[kFcBK][kFcBM + 4];
    __shared__ __align__(16) float Ws[kFcBK][kFcBN + 4];
    const int b0 = blockIdx.x * kFcBM, j0 = blockIdx.y * kFcBN;
    const int k_lo = blockIdx.z * k_per_split, k_hi = min(P, k_lo + k_per_split);
    const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;  // 16 x 16 threads
    const int lr = threadIdx.x >> 2, lk = (threadIdx.x & 3) * 4;  // loader: row, k quad
    float acc[4][4];
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = 0.0f;
    for (int k0 = k_lo; k0 < k_hi; k0 += kFcBK) {
        const int kk = k0 + lk;  // k_hi - k0 is a multiple of 4, so a quad is all in or out
        float4 a = make_float4(0.f, 0.f, 0.f, 0.f), w = a;
        if (b0 + lr < B && kk < k_hi)
            a = __ldg(reinterpret_cast<const float4*>(pooled + (long long)(b0 + lr) * P + kk));
        if (j0 + lr < D && kk < k_hi)
            w = __ldg(reinterpret_cast<const float4*>(W + (long long)(j0 + lr) * P + kk));
        As[lk][lr] = a.x;
        As[lk + 1][lr] = a.y;
        As[lk + 2][lr] = a.z;
        As[lk + 3][lr] = a.w;
        Ws[lk][lr] = w.x;
        Ws[lk + 1][lr] = w.y;
        Ws[lk + 2][lr] = w.z;
        Ws[lk + 3][lr] = w.w;
        __syncthreads();
#pragma unroll
        for (int k = 0; k < kFcBK; ++k) {
            const float4 av = *reinterpret_cast<const float4*>(&As[k][ty * 4]);
            const float4 wv = *reinterpret_cast<const float4*>(&Ws[k][tx * 4]);
            const float a4[4] = {av.x, av.y, av.z, av.w};
            const float w4[4] = {wv.x, wv.y, wv.z, wv.w};
#pragma unroll
            for (int i = 0; i < 4; ++i)
#pragma unroll
                for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(a4[i], w4[j], acc[i][j]);
        }
        __syncthreads();
    }
    float* out = part + (long long)blockIdx.z * B * D;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const int bb = b0 + ty * 4 + i;
        if (bb >= B) continue;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const int jj = j0 + tx * 4 + j;
            if (jj < D) out[(long long)bb * D + jj] = acc[i][j];
        }
    }
}

// Sum the split-K partials in a fixed order, + bias - mean_vec, then the L2
// normalisation the reference does on the host in double. One CTA per clip.
__global__ void __launch_bounds__(256)
fc_finish_kernel(const float* __restrict__ part, int n_split, int B, int D,
                 const float* __restrict__ seg_b, const float* __restrict__ mean_vec, int l2,
                 const int* __restrict__ out_rows, float* __restrict__ emb_out,
                 float* __restrict__ prenorm_out) {
    extern __shared__ float emb[];
    __shared__ double red[32];
    const int b = blockIdx.x;
    for (int j = threadIdx.x; j < D; j += blockDim.x) {
        float v = 0.0f;
        for (int sp = 0; sp < n_split; ++sp) v += part[((long long)sp * B + b) * D + j];
        v += seg_b[j];
        if (mean_vec) v -= mean_vec[j];
        emb[j] = v;
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

size_t pool_embed_scratch_floats(int batch, int f, int c, int emb_dim) {
    const int P = 2 * c * f;
    const int n_split = pool_fc_splits(batch, P, emb_dim);
    return (size_t)batch * P + (size_t)n_split * batch * emb_dim;
}

int pool_fc_splits(int batch, int P, int emb_dim) {
    // enough CTAs to cover the SMs about twice, K ranges of at least 8 tiles
    const int tiles = ((batch + kFcBM - 1) / kFcBM) * ((emb_dim + kFcBN - 1) / kFcBN);
    int n = std::max(1, (2 * num_sms() + tiles - 1) / tiles);
    n = std::min(n, std::max(1, P / (8 * kFcBK)));
    return n;
}

namespace {
bool fc_shape_ok(int K) {
    if (K % 4 != 0) {
        set_error("FC: the input length must be a multiple of 4");
        return false;
    }
    return true;
}
}  // namespace

int fc_embed_launch(const float* pooled, int batch, int P, const float* seg_w,
                    const float* seg_b, const float* mean_vec, int emb_dim, int l2,
                    const int* out_rows, float* emb_out, float* prenorm_out, float* part,
                    cudaStream_t stream) {
    if ((size_t)emb_dim * sizeof(float) > 48 * 1024) {
        set_error("vdb_pool_embed: embedding too large");
        return 1;
    }
    if (!fc_shape_ok(P)) return 1;
    const int n_split = pool_fc_splits(batch, P, emb_dim);
    const int k_per = ((P + n_split - 1) / n_split + kFcBK - 1) / kFcBK * kFcBK;
    const dim3 grid((batch + kFcBM - 1) / kFcBM, (emb_dim + kFcBN - 1) / kFcBN,
                    (P + k_per - 1) / k_per);
    fc_partial_kernel<<<grid, 256, 0, stream>>>(pooled, seg_w, batch, emb_dim, P, k_per, part);
    VDB_CHECK_CUDA(cudaGetLastError());
    fc_finish_kernel<<<batch, 256, emb_dim * sizeof(float), stream>>>(
        part, (int)grid.z, batch, emb_dim, seg_b, mean_vec, l2, out_rows, emb_out, prenorm_out);
    VDB_CHECK_CUDA(cudaGetLastError());
    return 0;
}

namespace {

// out[i] = act(sum of the split-K partials + bias[i % N]); act 0 none, 1 ReLU, 2 sigmoid.
__global__ void bias_act_finish_kernel(const float* __restrict__ part, int n_split, long long BN,
                                       int N, const float* __restrict__ bias, int act,
                                       float* __restrict__ out) {
    const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= BN) return;
    float v = 0.0f;
    for (int sp = 0; sp < n_split; ++sp) v += part[(long long)sp * BN + i];
    if (bias) v += bias[i % N];
    if (act == 1) v = fmaxf(v, 0.0f);
    else if (act == 2) v = 1.0f / (1.0f + expf(-v));
    out[i] = v;
}

}  // namespace

size_t small_gemm_scratch_floats(int batch, int K, int N) {
    return (size_t)pool_fc_splits(batch, K, N) * batch * N;
}

int small_gemm_launch(const float* in, int batch, int K, const float* W, int N, const float* bias,
                      int act, float* out, float* part, cudaStream_t stream) {
    if (!fc_shape_ok(K)) return 1;
    const int n_split = pool_fc_splits(batch, K, N);
    const int k_per = ((K + n_split - 1) / n_split + kFcBK - 1) / kFcBK * kFcBK;
    const dim3 grid((batch + kFcBM - 1) / kFcBM, (N + kFcBN - 1) / kFcBN, (K + k_per - 1) / k_per);
    fc_partial_kernel<<<grid, 256, 0, stream>>>(in, W, batch, N, K, k_per, part);
    VDB_CHECK_CUDA(cudaGetLastError());
    const long long BN = (long long)batch * N;
    bias_act_finish_kernel<<<(unsigned)((BN + 255) / 256), 256, 0, stream>>>(part, (int)grid.z, BN, N,
                                                                             bias, act, out);
    VDB_CHECK_CUDA(cudaGetLastError());
    return 0;
}

int pool_embed_launch(const void* x, const int* tvalid, int batch, int t, int f, int c,
                      const float* seg_w, const float* seg_b, const float* mean_vec, int emb_dim,
                      float var_eps, int l2, const int* out_rows, float* emb_out,
                      float* prenorm_out, float* scratch, cudaStream_t stream) {
    const int P = 2 * c * f;
    float* pooled = scratch;
    float* part = scratch + (size_t)batch * P;
    if (c % 8 != 0) {
        set_error("vdb_pool_embed: channels must be a multiple of 8");
        return 1;
    }
    const int units = f * (c / 8);
    const int tthreads = std::min(1024, (units + 31) / 32 * 32);
    tstp_kernel<<<batch, tthreads, 0, stream>>>(static_cast<const __half*>(x), tvalid, t, f, c,
                                                var_eps, pooled);
    VDB_CHECK_CUDA(cudaGetLastError());
    return fc_embed_launch(pooled, batch, P, seg_w, seg_b, mean_vec, emb_dim, l2, out_rows,
                           emb_out, prenorm_out, part, stream);
}

}  // namespace vdb

using namespace vdb;

extern "C" int vdb_cmn_stem(const float* feats, const int* frames, int batch, int t_max,
                            int n_mels, int cmn, const float* stem_w, const float* stem_b,
                            int oc, float* mean_scratch, void* y, void* stream) {
    return vdb::cmn_stem_launch(feats, frames, batch, t_max, n_mels, cmn, stem_w, stem_b, oc,
                                mean_scratch, y, 0, static_cast<cudaStream_t>(stream));
}

extern "C" int vdb_cmn_stem_qpack(const float* feats, const int* frames, int batch, int t_max,
                                  int n_mels, int cmn, const float* stem_w, const float* stem_b,
                                  float* mean_scratch, void* y, void* stream) {
    return vdb::cmn_stem_launch(feats, frames, batch, t_max, n_mels, cmn, stem_w, stem_b, 32,
                                mean_scratch, y, 2, static_cast<cudaStream_t>(stream));
}

int vdb::cmn_stem_launch(const float* feats, const int* frames, int batch, int t_max,
                         int n_mels, int cmn, const float* stem_w, const float* stem_b, int oc,
                         float* mean_scratch, void* y, int fphase, cudaStream_t stream) {
    if (!feats || !frames || !stem_w || !stem_b || !y || (cmn && !mean_scratch)) {
        set_error("vdb_cmn_stem: NULL argument");
        return 1;
    }
    if (fphase == 2 && oc != 32) {
        set_error("vdb_cmn_stem: the QPACK output needs 32 stem channels");
        return 1;
    }
    if (batch <= 0 || batch > 65535 || t_max <= 0 || t_max > (1 << 22) || n_mels <= 0 ||
        n_mels > 128) {
        set_error("vdb_cmn_stem: bad shape");
        return 1;
    }
    cudaStream_t st = stream;
    if (cmn) {
        cmn_mean_kernel<<<batch, dim3(128, 4), 0, st>>>(feats, frames, t_max, n_mels,
                                                       mean_scratch);
        VDB_CHECK_CUDA(cudaGetLastError());
    }
    const int threads = 256;
    const dim3 blocks((unsigned)((t_max + 2 + kStemRows - 1) / kStemRows), (unsigned)batch);
    __half* yh = static_cast<__half*>(y);
    switch (oc) {
        case 16:
            stem_kernel<16><<<blocks, threads, 0, st>>>(feats, frames, mean_scratch, batch, t_max,
                                                        n_mels, cmn, stem_w, stem_b, yh, fphase);
            break;
        case 32:
            stem_kernel<32><<<blocks, threads, 0, st>>>(feats, frames, mean_scratch, batch, t_max,
                                                        n_mels, cmn, stem_w, stem_b, yh, fphase);
            break;
        case 64:
            stem_kernel<64><<<blocks, threads, 0, st>>>(feats, frames, mean_scratch, batch, t_max,
                                                        n_mels, cmn, stem_w, stem_b, yh, fphase);
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
// Per device: the array's device address once a lookup has succeeded (null until
// then), guarded by that device's mutex. Only a success is kept, so a lookup that
// failed (made during a stream capture, or a transient error) is tried again on the
// next call instead of leaving the entry point unusable on that device.
std::mutex g_means_mu[kMaxDevices];
float* g_means_addr[kMaxDevices] = {};

// The device address of g_cmn_means on device `dev` (current), or null with the
// error in `status`.
float* means_address(int dev, cudaError_t& status) {
    std::lock_guard<std::mutex> lk(g_means_mu[dev]);
    status = cudaSuccess;
    if (!g_means_addr[dev]) {
        void* addr = nullptr;
        status = cudaGetSymbolAddress(&addr, g_cmn_means);
        if (status == cudaSuccess && addr) g_means_addr[dev] = static_cast<float*>(addr);
        else cudaGetLastError();  // do not leave the failure as the sticky last error
    }
    return g_means_addr[dev];
}
}  // namespace

extern "C" int vdb_cmn_stem_noalloc(const float* feats, const int* frames, int batch, int t_max,
                                    int n_mels, int cmn, const float* stem_w,
                                    const float* stem_b, int oc, void* y, void* stream) {
    if (!feats || !frames || !stem_w || !stem_b || !y) {
        set_error("vdb_cmn_stem_noalloc: NULL argument");
        return 1;
    }
    if (batch <= 0 || batch > 65535 || t_max <= 0 || t_max > (1 << 22) || n_mels <= 0 ||
        n_mels > 128) {
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
    // First successful call on this device (with it current) looks up the array's
    // device address. A host-side reference to g_cmn_means is not a device address.
    cudaError_t status = cudaSuccess;
    float* means = means_address(dev, status);
    if (!means) {
        set_error(std::string("vdb_cmn_stem_noalloc: cudaGetSymbolAddress failed (retried on "
                              "the next call): ") +
                  cudaGetErrorString(status));
        return 1;
    }
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    // The mean kernel writes every entry the stem kernel reads, so the array's
    // previous contents never leak into a result.
    if (cmn) {
        cmn_mean_kernel<<<batch, dim3(128, 4), 0, st>>>(feats, frames, t_max, n_mels, means);
        VDB_CHECK_CUDA(cudaGetLastError());
    }
    const int threads = 256;
    const dim3 blocks((unsigned)((t_max + 2 + kStemRows - 1) / kStemRows), (unsigned)batch);
    __half* yh = static_cast<__half*>(y);
    if (oc == 16)
        stem_kernel<16><<<blocks, threads, 0, st>>>(feats, frames, means, batch, t_max, n_mels,
                                                    cmn, stem_w, stem_b, yh, 0);
    else if (oc == 32)
        stem_kernel<32><<<blocks, threads, 0, st>>>(feats, frames, means, batch, t_max, n_mels,
                                                    cmn, stem_w, stem_b, yh, 0);
    else
        stem_kernel<64><<<blocks, threads, 0, st>>>(feats, frames, means, batch, t_max, n_mels,
                                                    cmn, stem_w, stem_b, yh, 0);
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
    // stream-ordered working memory for the pooled vectors and the FC partials
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    float* scratch = nullptr;
    keep_async_pool();
    VDB_CHECK_CUDA(cudaMallocAsync(&scratch,
                                   sizeof(float) * pool_embed_scratch_floats(batch, f, c, emb_dim),
                                   st));
    const int rc = pool_embed_launch(x, tvalid, batch, t, f, c, seg_w, seg_b, mean_vec, emb_dim,
                                     var_eps, l2, nullptr, emb_out, prenorm_out, scratch, st);
    cudaFreeAsync(scratch, st);
    return rc;
}
