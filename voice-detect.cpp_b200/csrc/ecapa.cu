// ECAPA-TDNN glue on the SEQ layout (vdb_ops.h): everything of the reference's
// EcapaEncoder (src/encoder.cpp:157-340) that is not a conv. The convs themselves
// (stem, TDNN 1x1s, dilated Res2Net convs, MFA, attention) run on the tensor cores
// through vdb_conv1d with their ReLU -> BatchNorm (-> tanh) epilogues.
//
//   cmn_pack_seq_kernel   FBank CMN (src/fbank.cpp:194-201) + f16 pack into the
//                         SEQ layout with the reflect padding the k=5 stem reads
//                         (src/encoder.cpp:32-50)
//   seq_mean_kernel       SE squeeze: per-clip mean over time (src/encoder.cpp:200)
//   se_apply_kernel       x * gate + block input (:208, :229)
//   seq_meanstd_kernel    ASP global statistics mean / sqrt(clamp(var, eps)) (:261-264);
//                         with `unbiased`, CAM++'s statistics pooling (mean, std with
//                         the T/(T-1) correction, no floor: src/encoder_campplus.cpp:283-292)
//   asp_pool_kernel       softmax over time + attention-weighted mean / std (:280-285)
//
// Every kernel reads only a clip's valid frames (t < tvalid[b]); rows outside them
// are never used, so length-bucketed batches are exact.
//
// ASP note. The reference concatenates [x; mean; std] (3C channels) and runs the
// attention TDNN's 1x1 conv over it (src/encoder.cpp:268-275). The mean / std
// blocks are constant over time, so W * [x; m; s] = W_x * x + (W_m * m + W_s * s):
// the second term is one [B, 2C] x [2C, att] product per clip (small_gemm_launch),
// added as a per-clip bias in the tensor-core conv's epilogue before its ReLU.
#include <cuda_fp16.h>

#include <algorithm>
#include <cmath>

#include "vdb_internal.h"
#include "vdb_ops.h"

namespace vdb {
namespace {

__device__ __forceinline__ void unpack8(const uint4& v, float (&f)[8]) {
    const __half2* h = reinterpret_cast<const __half2*>(&v);
#pragma unroll
    for (int q = 0; q < 4; ++q) {
        const float2 t = __half22float2(h[q]);
        f[2 * q] = t.x;
        f[2 * q + 1] = t.y;
    }
}

// One block per clip, blockDim (128, 4): thread x = mel bin (n_mels <= 128).
// Writes frames -pad .. T+pad-1 of the clip (reflected at both ends).
__global__ void cmn_pack_seq_kernel(const float* __restrict__ feats,
                                    const int* __restrict__ frames, int t_max, int n_mels,
                                    int cmn, int pad, __half* __restrict__ x) {
    __shared__ double part[4][128];
    __shared__ float mu[128];
    const int b = blockIdx.x;
    const int m = threadIdx.x, ty = threadIdx.y;
    const int T = min(frames[b], t_max);
    const float* fb = feats + (long long)b * t_max * n_mels;
    double s = 0.0;
    if (cmn && m < n_mels)
        for (int t = ty; t < T; t += 4) s += (double)fb[(long long)t * n_mels + m];
    part[ty][m] = s;
    __syncthreads();
    if (ty == 0 && m < n_mels)
        mu[m] = (cmn && T > 0) ? (float)((part[0][m] + part[1][m] + part[2][m] + part[3][m]) / T)
                               : 0.0f;
    __syncthreads();
    if (T <= 0 || m >= n_mels) return;
    const long long row0 = (long long)b * (t_max + 2 * pad);
    for (int tp = ty; tp < T + 2 * pad; tp += 4) {
        int u = tp - pad;
        if (u < 0) u = -u;
        if (u >= T) u = 2 * (T - 1) - u;
        u = min(max(u, 0), T - 1);  // clips shorter than pad + 1 frames are refused by the host
        x[(row0 + tp) * n_mels + m] = __float2half_rn(fb[(long long)u * n_mels + m] - mu[m]);
    }
}

// out[b][c] = mean over the valid frames of x (f32 sums). Block (b, 512 channels):
// 64 channel groups of 8 x 4 time lanes.
__global__ void seq_mean_kernel(const __half* __restrict__ x, int ldx,
                                const int* __restrict__ tv, int T, int pad, int C,
                                float* __restrict__ out) {
    __shared__ float red[4][512];
    const int b = blockIdx.x;
    const int g = threadIdx.x & 63, ty = threadIdx.x >> 6;
    const int c = blockIdx.y * 512 + g * 8;
    const int tvb = min(tv[b], T);
    float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    if (c < C) {
        const __half* xb = x + ((long long)b * (T + 2 * pad) + pad) * ldx + c;
        for (int t = ty; t < tvb; t += 4) {
            float f[8];
            unpack8(__ldg(reinterpret_cast<const uint4*>(xb + (long long)t * ldx)), f);
#pragma unroll
            for (int i = 0; i < 8; ++i) acc[i] += f[i];
        }
    }
#pragma unroll
    for (int i = 0; i < 8; ++i) red[ty][g * 8 + i] = acc[i];
    __syncthreads();
    const int j = threadIdx.x;  // 256 threads, 512 sums: two each
    for (int k = j; k < 512; k += 256) {
        const int cc = blockIdx.y * 512 + k;
        if (cc < C && tvb > 0)
            out[(long long)b * C + cc] = (red[0][k] + red[1][k] + red[2][k] + red[3][k]) / tvb;
    }
}

// y = h * gate[b] + res at the valid frames (8 channels per thread).
__global__ void se_apply_kernel(const __half* __restrict__ h, int ldh,
                                const float* __restrict__ gate, const __half* __restrict__ res,
                                int ldr, const int* __restrict__ tv, int T, int pad, int C,
                                long long rows, __half* __restrict__ y, int ldy) {
    const int groups = C / 8;
    const long long u = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (u >= rows * groups) return;
    const long long r = u / groups;
    const int c = (int)(u - r * groups) * 8;
    const int Hp = T + 2 * pad;
    const int b = (int)(r / Hp);
    const int t = (int)(r - (long long)b * Hp) - pad;
    if (t < 0 || t >= tv[b]) return;
    float fh[8], fr[8];
    unpack8(__ldg(reinterpret_cast<const uint4*>(h + r * ldh + c)), fh);
    unpack8(__ldg(reinterpret_cast<const uint4*>(res + r * ldr + c)), fr);
    const float4 g0 = __ldg(reinterpret_cast<const float4*>(gate + (long long)b * C + c));
    const float4 g1 = __ldg(reinterpret_cast<const float4*>(gate + (long long)b * C + c + 4));
    const float gv[8] = {g0.x, g0.y, g0.z, g0.w, g1.x, g1.y, g1.z, g1.w};
    uint4 o;
    __half2* oh = reinterpret_cast<__half2*>(&o);
#pragma unroll
    for (int q = 0; q < 4; ++q)
        oh[q] = __floats2half2_rn(fh[2 * q] * gv[2 * q] + fr[2 * q],
                                  fh[2 * q + 1] * gv[2 * q + 1] + fr[2 * q + 1]);
    *reinterpret_cast<uint4*>(y + r * ldy + c) = o;
}

// stats[b][c] = mean, stats[b][C + c] = sqrt(max(mean((x - mean)^2), eps)) over the
// valid frames: two passes, like the reference's mean -> sub -> sqr -> mean.
__global__ void seq_meanstd_kernel(const __half* __restrict__ x, int ldx,
                                   const int* __restrict__ tv, int T, int pad, int C, float eps,
                                   int unbiased, float* __restrict__ stats) {
    __shared__ float red[4][512];
    __shared__ float mean_s[512];
    const int b = blockIdx.x;
    const int g = threadIdx.x & 63, ty = threadIdx.x >> 6;
    const int c = blockIdx.y * 512 + g * 8;
    const int tvb = min(tv[b], T);
    const __half* xb = x + ((long long)b * (T + 2 * pad) + pad) * ldx + c;
    float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    if (c < C)
        for (int t = ty; t < tvb; t += 4) {
            float f[8];
            unpack8(__ldg(reinterpret_cast<const uint4*>(xb + (long long)t * ldx)), f);
#pragma unroll
            for (int i = 0; i < 8; ++i) acc[i] += f[i];
        }
#pragma unroll
    for (int i = 0; i < 8; ++i) red[ty][g * 8 + i] = acc[i];
    __syncthreads();
    for (int k = threadIdx.x; k < 512; k += 256)
        mean_s[k] = tvb > 0 ? (red[0][k] + red[1][k] + red[2][k] + red[3][k]) / tvb : 0.0f;
    __syncthreads();
    float mv[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        mv[i] = mean_s[g * 8 + i];
        acc[i] = 0.0f;
    }
    if (c < C)
        for (int t = ty; t < tvb; t += 4) {
            float f[8];
            unpack8(__ldg(reinterpret_cast<const uint4*>(xb + (long long)t * ldx)), f);
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                const float d = f[i] - mv[i];
                acc[i] += d * d;
            }
        }
    __syncthreads();
#pragma unroll
    for (int i = 0; i < 8; ++i) red[ty][g * 8 + i] = acc[i];
    __syncthreads();
    for (int k = threadIdx.x; k < 512; k += 256) {
        const int cc = blockIdx.y * 512 + k;
        if (cc >= C || tvb <= 0) continue;
        float var = (red[0][k] + red[1][k] + red[2][k] + red[3][k]) / tvb;
        if (unbiased && tvb > 1) var *= (float)tvb / (float)(tvb - 1);
        stats[(long long)b * 2 * C + cc] = mean_s[k];
        stats[(long long)b * 2 * C + C + cc] = sqrtf(fmaxf(var, eps));
    }
}

// Attentive statistics pooling of one clip's channels: a = softmax over the valid
// frames of the logits, mu = sum a*x, sd = sqrt(max(sum a*(x - mu)^2, eps)).
// One pass: each thread keeps, for its channels, the running maximum m of the
// logits and S = sum w, A = sum w*d, Q = sum w*d^2 with w = exp(l - m) and
// d = x - g, g the channel's global mean (the shift keeps Q/S - (A/S)^2 well
// conditioned); a new maximum rescales S, A, Q by exp(m_old - m_new). Then
// mu = g + A/S, var = Q/S - (A/S)^2. The four time lanes of a channel are merged
// the same way. Block (b, 128 channels): 64 channel pairs x 4 time lanes.
struct AspAcc {
    float m, s, a, q;
};

__device__ __forceinline__ void asp_update(AspAcc& st, float l, float d) {
    if (l > st.m) {
        const float r = __expf(st.m - l);  // 0 for the first frame (m = -inf)
        st.s *= r;
        st.a *= r;
        st.q *= r;
        st.m = l;
    }
    const float w = __expf(l - st.m);
    st.s += w;
    st.a = fmaf(w, d, st.a);
    st.q = fmaf(w * d, d, st.q);
}

__global__ void __launch_bounds__(256)
asp_pool_kernel(const float* __restrict__ logits, int ldl, const __half* __restrict__ x, int ldx,
                const float* __restrict__ stats, const int* __restrict__ tv, int T, int pad,
                int C, float eps, float* __restrict__ pooled) {
    __shared__ AspAcc sm[4][128];
    const int b = blockIdx.x;
    const int cp = threadIdx.x & 63, ty = threadIdx.x >> 6;
    const int c = blockIdx.y * 128 + 2 * cp;
    const int tvb = min(tv[b], T);
    AspAcc u{-INFINITY, 0.0f, 0.0f, 0.0f}, v{-INFINITY, 0.0f, 0.0f, 0.0f};
    if (c < C) {
        const float g0 = stats[(long long)b * 2 * C + c], g1 = stats[(long long)b * 2 * C + c + 1];
        const long long row0 = (long long)b * (T + 2 * pad) + pad;
#pragma unroll 4
        for (int t = ty; t < tvb; t += 4) {
            const float2 l = __ldg(reinterpret_cast<const float2*>(logits + (row0 + t) * ldl + c));
            const float2 xv = __half22float2(
                *reinterpret_cast<const __half2*>(x + (row0 + t) * ldx + c));
            asp_update(u, l.x, xv.x - g0);
            asp_update(v, l.y, xv.y - g1);
        }
    }
    sm[ty][2 * cp] = u;
    sm[ty][2 * cp + 1] = v;
    __syncthreads();
    if (threadIdx.x >= 128) return;
    const int cl = threadIdx.x, cc = blockIdx.y * 128 + cl;
    if (cc >= C) return;
    float m = -INFINITY;
    for (int k = 0; k < 4; ++k)
        if (sm[k][cl].s > 0.0f) m = fmaxf(m, sm[k][cl].m);
    float S = 0.0f, A = 0.0f, Q = 0.0f;
    for (int k = 0; k < 4; ++k) {
        const AspAcc& e = sm[k][cl];
        if (e.s <= 0.0f) continue;
        const float r = __expf(e.m - m);
        S += e.s * r;
        A += e.a * r;
        Q += e.q * r;
    }
    const float g = stats[(long long)b * 2 * C + cc];
    const float mean_d = S > 0.0f ? A / S : 0.0f;
    const float var = S > 0.0f ? fmaxf(Q / S - mean_d * mean_d, 0.0f) : 0.0f;
    pooled[(long long)b * 2 * C + cc] = g + mean_d;
    pooled[(long long)b * 2 * C + C + cc] = sqrtf(fmaxf(var, eps));
}

}  // namespace

int ecapa_cmn_pack(const float* feats, const int* frames, int batch, int t_max, int n_mels,
                   int cmn, int pad, __half* x, cudaStream_t st) {
    if (n_mels > 128) {
        set_error("ecapa: n_mels must be <= 128");
        return 1;
    }
    cmn_pack_seq_kernel<<<batch, dim3(128, 4), 0, st>>>(feats, frames, t_max, n_mels, cmn, pad, x);
    VDB_CHECK_CUDA(cudaGetLastError());
    return 0;
}

int ecapa_seq_mean(const __half* x, int ldx, const int* tv, int batch, int T, int pad, int C,
                   float* out, cudaStream_t st) {
    const dim3 grid((unsigned)batch, (unsigned)((C + 511) / 512));
    seq_mean_kernel<<<grid, 256, 0, st>>>(x, ldx, tv, T, pad, C, out);
    VDB_CHECK_CUDA(cudaGetLastError());
    return 0;
}

int ecapa_se_apply(const __half* h, int ldh, const float* gate, const __half* res, int ldr,
                   const int* tv, int batch, int T, int pad, int C, __half* y, int ldy,
                   cudaStream_t st) {
    const long long rows = vdb_seq_rows(batch, T, pad);
    const long long units = rows * (C / 8);
    se_apply_kernel<<<(unsigned)((units + 255) / 256), 256, 0, st>>>(h, ldh, gate, res, ldr, tv, T,
                                                                    pad, C, rows, y, ldy);
    VDB_CHECK_CUDA(cudaGetLastError());
    return 0;
}

int ecapa_meanstd(const __half* x, int ldx, const int* tv, int batch, int T, int pad, int C,
                  float eps, float* stats, cudaStream_t st) {
    const dim3 grid((unsigned)batch, (unsigned)((C + 511) / 512));
    seq_meanstd_kernel<<<grid, 256, 0, st>>>(x, ldx, tv, T, pad, C, eps, 0, stats);
    VDB_CHECK_CUDA(cudaGetLastError());
    return 0;
}

int seq_meanstd_unbiased(const __half* x, int ldx, const int* tv, int batch, int T, int pad,
                         int C, float* stats, cudaStream_t st) {
    const dim3 grid((unsigned)batch, (unsigned)((C + 511) / 512));
    seq_meanstd_kernel<<<grid, 256, 0, st>>>(x, ldx, tv, T, pad, C, 0.0f, 1, stats);
    VDB_CHECK_CUDA(cudaGetLastError());
    return 0;
}

int ecapa_asp_pool(const float* logits, int ldl, const __half* x, int ldx, const float* stats,
                   const int* tv, int batch, int T, int pad, int C, float eps, float* pooled,
                   cudaStream_t st) {
    if (C % 2 != 0 || ldl % 2 != 0 || ldx % 2 != 0) {
        set_error("ecapa: attentive pooling needs an even channel count and pitches");
        return 1;
    }
    const dim3 grid((unsigned)batch, (unsigned)((C + 127) / 128));
    asp_pool_kernel<<<grid, 256, 0, st>>>(logits, ldl, x, ldx, stats, tv, T, pad, C, eps, pooled);
    VDB_CHECK_CUDA(cudaGetLastError());
    return 0;
}

}  // namespace vdb
