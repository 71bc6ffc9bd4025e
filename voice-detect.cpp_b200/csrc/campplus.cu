// CAM++ glue kernels on the SEQ layout (the dense TDNN backbone of the reference's
// CamPPlusEncoder, src/encoder_campplus.cpp:243-281):
//   seg_sum_kernel,  the CAM layer's context attention (:262-268): per clip the
//   gate_mlp_kernel  channel means over all valid frames and over each 100-frame
//                    segment, context = mean + segment mean, then
//                    sigmoid(linear2(ReLU(linear1(context)))) per segment. The conv
//                    epilogue multiplies linear_local's output by it (act 5), so
//                    the per-frame context is never materialised.
// The BatchNorm + ReLU in front of each bottleneck / transit 1x1 conv has no kernel
// of its own: the conv applies it to its A tiles in shared memory (conv_tc.cu).
// Every kernel reads only a clip's valid frames (t < tvalid[b]).
#include <cuda_fp16.h>

#include <algorithm>
#include <cmath>
#include <string>

#include "vdb_internal.h"
#include "vdb_ops.h"

namespace vdb {
namespace {

// Segment sums, one block (256 threads) per (segment, clip): seg[b][s][c] = sum of
// channel c over frames [s*seg_len, min((s+1)*seg_len, tvalid[b])) (0 past the clip).
// Thread (g, l) sums 8 channels (16 bytes) of every lanes-th frame, its loads issued
// 8 at a time (the input was just written by the bottleneck conv and sits in L2: the
// kernel is latency-bound), then the lanes are added in a fixed order (no atomics:
// graph replays are bitwise stable).
__global__ void __launch_bounds__(256)
seg_sum_kernel(const __half* __restrict__ cc, int ldc, const int* __restrict__ tv, int T,
               int pad, int C, int seg, int nseg_max, float* __restrict__ out) {
    __shared__ float red[2048];
    const int b = blockIdx.y, s = blockIdx.x;
    const int tvb = min(tv[b], T);
    const int groups = C / 8, lanes = 256 / groups;
    const int g = threadIdx.x % groups, ln = threadIdx.x / groups;
    const int t1 = min((s + 1) * seg, tvb);
    const __half* xb = cc + ((long long)b * (T + 2 * pad) + pad) * ldc + g * 8;
    float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    if (ln < lanes)
        for (int t0 = s * seg + ln; t0 < t1; t0 += 8 * lanes) {
            uint4 v[8];
#pragma unroll
            for (int u = 0; u < 8; ++u) {
                const int t = t0 + u * lanes;
                v[u] = t < t1 ? __ldg(reinterpret_cast<const uint4*>(xb + (long long)t * ldc))
                              : make_uint4(0u, 0u, 0u, 0u);
            }
#pragma unroll
            for (int u = 0; u < 8; ++u) {
                const __half2* hv = reinterpret_cast<const __half2*>(&v[u]);
#pragma unroll
                for (int q = 0; q < 4; ++q) {
                    const float2 x = __half22float2(hv[q]);
                    acc[2 * q] += x.x;
                    acc[2 * q + 1] += x.y;
                }
            }
        }
    if (ln < lanes)
#pragma unroll
        for (int q = 0; q < 8; ++q) red[ln * C + g * 8 + q] = acc[q];
    __syncthreads();
    for (int c = threadIdx.x; c < C; c += blockDim.x) {
        float v = 0.0f;
        for (int l = 0; l < lanes; ++l) v += red[l * C + c];
        out[((long long)b * nseg_max + s) * C + c] = v;
    }
}

// The gate MLP, one block (256 threads) per `cpb` clips (rows r = (clip, segment)):
// context[r] = mean over the clip's valid frames (its segment sums added in order /
// tvalid) + seg[r] / seg_len, hidden = ReLU(w1 . context + b1), gate = sigmoid(w2 .
// hidden + b2). Both weights are staged transposed in shared memory once per block
// (a warp reads 32 consecutive outputs' weights of one input: conflict-free; the
// context / hidden value is a broadcast), shared by the block's rows.
// Shared memory: w1t [C][M], w2t [M][G], ctx [rows][C], hid [rows][M].
__global__ void __launch_bounds__(256)
gate_mlp_kernel(const float* __restrict__ segsum, const int* __restrict__ tv, int batch, int T,
                int C, int seg, int nseg_max, int cpb, const float* __restrict__ w1,
                const float* __restrict__ b1, int M, const float* __restrict__ w2,
                const float* __restrict__ b2, int G, float* __restrict__ gate) {
    extern __shared__ float sm[];
    const int rows = cpb * nseg_max;
    float* w1t = sm;
    float* w2t = w1t + C * M;
    float* ctx = w2t + M * G;
    float* hid = ctx + (size_t)rows * C;
    const int tid = threadIdx.x;
    const int b0 = blockIdx.x * cpb;
#pragma unroll 8
    for (int i = tid; i < M * C; i += 256) {
        const int j = i / C, c = i - j * C;
        w1t[c * M + j] = __ldg(w1 + i);
    }
#pragma unroll 8
    for (int i = tid; i < G * M; i += 256) {
        const int k = i / M, j = i - k * M;
        w2t[j * G + k] = __ldg(w2 + i);
    }
    for (int u = tid; u < cpb * C; u += 256) {
        const int i = u / C, c = u - i * C;
        if (b0 + i >= batch) continue;
        const int tvb = min(tv[b0 + i], T);
        const int nseg = (tvb + seg - 1) / seg;
        const float* sb = segsum + (long long)(b0 + i) * nseg_max * C + c;
        float* x = ctx + (size_t)i * nseg_max * C + c;
        float v = 0.0f;
        for (int s = 0; s < nseg; ++s) {
            const float q = __ldg(sb + (long long)s * C);
            x[s * C] = q;
            v += q;
        }
        const float mean = tvb > 0 ? v / (float)tvb : 0.0f;
        for (int s = 0; s < nseg_max; ++s) x[s * C] = s < nseg ? mean + x[s * C] / (float)seg : 0.0f;
    }
    __syncthreads();
    for (int u = tid; u < rows * M; u += 256) {
        const int r = u / M, j = u - r * M;
        const float* x = ctx + r * C;
        float v = 0.0f;
#pragma unroll 8
        for (int c = 0; c < C; ++c) v = fmaf(w1t[c * M + j], x[c], v);
        hid[u] = fmaxf(v + __ldg(b1 + j), 0.0f);
    }
    __syncthreads();
    for (int u = tid; u < rows * G; u += 256) {
        const int r = u / G, k = u - r * G;
        const int i = r / nseg_max, s = r - i * nseg_max;
        if (b0 + i >= batch) continue;
        const float* x = hid + r * M;
        float v = 0.0f;
#pragma unroll 8
        for (int j = 0; j < M; ++j) v = fmaf(w2t[j * G + k], x[j], v);
        gate[((long long)(b0 + i) * nseg_max + s) * G + k] =
            1.0f / (1.0f + expf(-(v + __ldg(b2 + k))));
    }
}

// clips per gate-MLP block: amortise the weight staging, at most 32 rows
int gate_cpb(int nseg_max) { return std::max(1, std::min(8, 32 / std::max(nseg_max, 1))); }

}  // namespace

size_t campp_gate_smem(int C, int M, int G, int nseg_max) {
    const int rows = gate_cpb(nseg_max) * nseg_max;
    return ((size_t)C * M + (size_t)M * G + (size_t)rows * (C + M)) * sizeof(float);
}

int campp_cam_gate(const __half* cc, int ldc, const int* tv, int batch, int T, int pad, int C,
                   int seg, int nseg_max, const float* w1, const float* b1, int M,
                   const float* w2, const float* b2, int G, float* segsum, float* gate,
                   cudaStream_t st) {
    if (C % 8 != 0 || C > 2048 || 256 % (C / 8) != 0 || ldc % 8 != 0 || seg < 1 ||
        (long long)nseg_max * seg < T || nseg_max > 65535) {
        set_error("campplus: CAM context needs C a multiple of 8 dividing 2048 and "
                  "nseg_max * seg >= T");
        return 1;
    }
    const size_t smem = campp_gate_smem(C, M, G, nseg_max);
    if (smem > 200 * 1024) {
        set_error("campplus: clip too long or layer too wide for the CAM gate kernel (" +
                  std::to_string(nseg_max) + " context segments)");
        return 1;
    }
    seg_sum_kernel<<<dim3((unsigned)nseg_max, (unsigned)batch), 256, 0, st>>>(
        cc, ldc, tv, T, pad, C, seg, nseg_max, segsum);
    VDB_CHECK_CUDA(cudaGetLastError());
    cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
    VDB_CHECK_CUDA(cudaStreamIsCapturing(st, &cs));
    if (cs == cudaStreamCaptureStatusNone)
        VDB_CHECK_CUDA(cudaFuncSetAttribute(gate_mlp_kernel,
                                            cudaFuncAttributeMaxDynamicSharedMemorySize,
                                            200 * 1024));
    const int cpb = gate_cpb(nseg_max);
    gate_mlp_kernel<<<(batch + cpb - 1) / cpb, 256, smem, st>>>(
        segsum, tv, batch, T, C, seg, nseg_max, cpb, w1, b1, M, w2, b2, G, gate);
    VDB_CHECK_CUDA(cudaGetLastError());
    return 0;
}

}  // namespace vdb
