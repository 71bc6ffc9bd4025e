// CAM++ glue kernels on the SEQ layout (the dense TDNN backbone of the reference's
// CamPPlusEncoder, src/encoder_campplus.cpp:243-281):
//   cam_gate_kernel  the CAM layer's context attention (:262-268): per clip the
//                    channel means over all valid frames and over each 100-frame
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

#include "sm100_ptx.cuh"
#include "vdb_internal.h"
#include "vdb_ops.h"

namespace vdb {
namespace {

// The CAM gate of one layer, one block (256 threads) per clip:
// 1. segment sums: thread (g, l) sums 8 channels (16 bytes) of every lanes-th frame of
//    a segment, its loads issued 8 at a time (the input was just written by the
//    bottleneck conv and sits in L2: the kernel is latency-bound), then the lanes are
//    added in a fixed order (no atomics: graph replays are bitwise stable);
// 2. context[s] = mean over the valid frames (the segment sums added in order /
//    tvalid) + sum[s] / seg_len;
// 3. hidden = ReLU(w1 . context + b1), gate = sigmoid(w2 . hidden + b2) per segment,
//    one thread per output with the weights stored transposed (w1t [C][M], w2t
//    [M][G]) and copied to shared memory first with 16-byte loads all in flight at
//    once (the block's chain of dependent memory round trips is what bounds it): a
//    warp's 32 outputs then read consecutive banks per input, the input a broadcast.
// Shared memory: w1t [C][M], w2t [M][G], ctx [nseg_max][C], hid [nseg_max][M],
// red [2048].
__global__ void __launch_bounds__(256)
cam_gate_kernel(const __half* __restrict__ cc, int ldc, const int* __restrict__ tv, int T,
                int pad, int C, int seg, int nseg_max, const float* __restrict__ w1t_g,
                const float* __restrict__ b1, int M, const float* __restrict__ w2t_g,
                const float* __restrict__ b2, int G, float* __restrict__ gate) {
    extern __shared__ float sm[];
    // launched with programmatic stream serialization: the gate conv that follows may
    // start its prologue now; every read below waits for the bottleneck conv
    if (threadIdx.x == 0) pdl_launch_dependents();
    pdl_wait();
    const int b = blockIdx.x;
    const int tvb = min(tv[b], T);
    const int nseg = (tvb + seg - 1) / seg;
    float* w1t = sm;
    float* w2t = w1t + C * M;
    float* ctx = w2t + M * G;
    float* hid = ctx + (size_t)nseg_max * C;
    float* red = hid + (size_t)nseg_max * M;
    const int tid = threadIdx.x;
    {
        const float4* a = reinterpret_cast<const float4*>(w1t_g);
        float4* d = reinterpret_cast<float4*>(w1t);
#pragma unroll 8
        for (int i = tid; i < C * M / 4; i += 256) d[i] = __ldg(a + i);
        const float4* a2 = reinterpret_cast<const float4*>(w2t_g);
        float4* d2 = reinterpret_cast<float4*>(w2t);
#pragma unroll 4
        for (int i = tid; i < M * G / 4; i += 256) d2[i] = __ldg(a2 + i);
    }
    const int groups = C / 8, lanes = 256 / groups;
    const int g = tid % groups, ln = tid / groups;
    const __half* xb = cc + ((long long)b * (T + 2 * pad) + pad) * ldc + g * 8;
    for (int s = 0; s < nseg; ++s) {
        float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
        const int t1 = min((s + 1) * seg, tvb);
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
        for (int c = tid; c < C; c += blockDim.x) {
            float v = 0.0f;
            for (int l = 0; l < lanes; ++l) v += red[l * C + c];
            ctx[s * C + c] = v;
        }
        __syncthreads();
    }
    for (int c = tid; c < C; c += blockDim.x) {
        float v = 0.0f;
        for (int s = 0; s < nseg; ++s) v += ctx[s * C + c];
        const float mean = tvb > 0 ? v / (float)tvb : 0.0f;
        for (int s = 0; s < nseg; ++s) ctx[s * C + c] = mean + ctx[s * C + c] / (float)seg;
    }
    __syncthreads();
    for (int u = tid; u < nseg * M; u += blockDim.x) {
        const int r = u / M, j = u - r * M;
        const float* x = ctx + r * C;
        float v = 0.0f;
#pragma unroll 16
        for (int c = 0; c < C; ++c) v = fmaf(w1t[c * M + j], x[c], v);
        hid[u] = fmaxf(v + __ldg(b1 + j), 0.0f);
    }
    __syncthreads();
    for (int u = tid; u < nseg * G; u += blockDim.x) {
        const int r = u / G, k = u - r * G;
        const float* x = hid + r * M;
        float v = 0.0f;
#pragma unroll 16
        for (int j = 0; j < M; ++j) v = fmaf(w2t[j * G + k], x[j], v);
        gate[((long long)b * nseg_max + r) * G + k] = 1.0f / (1.0f + expf(-(v + __ldg(b2 + k))));
    }
}

}  // namespace

size_t campp_gate_smem(int C, int M, int G, int nseg_max) {
    return ((size_t)C * M + (size_t)M * G + (size_t)nseg_max * (C + M) + 2048) * sizeof(float);
}

int campp_cam_gate(const __half* cc, int ldc, const int* tv, int batch, int T, int pad, int C,
                   int seg, int nseg_max, const float* w1t, const float* b1, int M,
                   const float* w2t, const float* b2, int G, float* gate, cudaStream_t st) {
    if (C % 8 != 0 || C > 2048 || 256 % (C / 8) != 0 || ldc % 8 != 0 || seg < 1 ||
        (long long)nseg_max * seg < T || (C * M) % 4 != 0 || (M * G) % 4 != 0) {
        set_error("campplus: CAM context needs C a multiple of 8 dividing 2048 and "
                  "nseg_max * seg >= T");
        return 1;
    }
    const size_t smem = campp_gate_smem(C, M, G, nseg_max);
    if (smem > 200 * 1024) {
        set_error("campplus: clip too long for the CAM gate kernel (" +
                  std::to_string(nseg_max) + " context segments)");
        return 1;
    }
    cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
    VDB_CHECK_CUDA(cudaStreamIsCapturing(st, &cs));
    if (cs == cudaStreamCaptureStatusNone)
        VDB_CHECK_CUDA(cudaFuncSetAttribute(cam_gate_kernel,
                                            cudaFuncAttributeMaxDynamicSharedMemorySize,
                                            200 * 1024));
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3((unsigned)batch);
    cfg.blockDim = dim3(256);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    VDB_CHECK_CUDA(cudaLaunchKernelEx(&cfg, cam_gate_kernel, cc, ldc, tv, T, pad, C, seg, nseg_max,
                                      w1t, b1, M, w2t, b2, G, gate));
    return 0;
}

}  // namespace vdb
