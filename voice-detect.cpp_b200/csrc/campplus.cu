// CAM++ glue kernels on the SEQ layout (the dense TDNN backbone of the reference's
// CamPPlusEncoder, src/encoder_campplus.cpp:243-281):
//   bn_relu_kernel   a = ReLU(BN(h)) over the first C channels of the dense block's
//                    concatenated features (nonlinear1 / transit nonlinear, :252-253,
//                    :275-276), the input of the 1x1 conv that follows
//   cam_gate_kernel  the CAM layer's context attention (:262-268): per clip the
//                    channel means over all valid frames and over each 100-frame
//                    segment, context = mean + segment mean, then
//                    sigmoid(linear2(ReLU(linear1(context)))) per segment. The conv
//                    epilogue multiplies linear_local's output by it (act 5), so
//                    the per-frame context is never materialised.
// Every kernel reads only a clip's valid frames (t < tvalid[b]).
#include <cuda_fp16.h>

#include <algorithm>
#include <cmath>

#include "vdb_internal.h"
#include "vdb_ops.h"

namespace vdb {
namespace {

// One thread per 8 channels of a row; every row of the slots (padding included).
__global__ void bn_relu_kernel(const __half* __restrict__ h, int ldh, int C,
                               const float* __restrict__ scale, const float* __restrict__ shift,
                               long long rows, __half* __restrict__ a, int lda) {
    const int c8 = C / 8;
    const long long n = rows * c8;
    for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n;
         i += (long long)gridDim.x * blockDim.x) {
        const long long r = i / c8;
        const int c = (int)(i - r * c8) * 8;
        const uint4 v = __ldg(reinterpret_cast<const uint4*>(h + r * ldh + c));
        const float4 s0 = __ldg(reinterpret_cast<const float4*>(scale + c));
        const float4 s1 = __ldg(reinterpret_cast<const float4*>(scale + c + 4));
        const float4 t0 = __ldg(reinterpret_cast<const float4*>(shift + c));
        const float4 t1 = __ldg(reinterpret_cast<const float4*>(shift + c + 4));
        const float sc[8] = {s0.x, s0.y, s0.z, s0.w, s1.x, s1.y, s1.z, s1.w};
        const float sh[8] = {t0.x, t0.y, t0.z, t0.w, t1.x, t1.y, t1.z, t1.w};
        const __half2* hv = reinterpret_cast<const __half2*>(&v);
        uint4 o;
        __half2* ho = reinterpret_cast<__half2*>(&o);
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            const float2 x = __half22float2(hv[q]);
            ho[q] = __floats2half2_rn(fmaxf(fmaf(x.x, sc[2 * q], sh[2 * q]), 0.0f),
                                      fmaxf(fmaf(x.y, sc[2 * q + 1], sh[2 * q + 1]), 0.0f));
        }
        *reinterpret_cast<uint4*>(a + r * lda + c) = o;
    }
}

// One block (256 threads) per clip. Shared memory: segment sums [nseg][C], then
// the reduction rows, the context and the hidden layer.
__global__ void __launch_bounds__(256)
cam_gate_kernel(const __half* __restrict__ cc, int ldc, const int* __restrict__ tv, int T,
                int pad, int C, int seg, int nseg_max, const float* __restrict__ w1,
                const float* __restrict__ b1, int M, const float* __restrict__ w2,
                const float* __restrict__ b2, int G, float* __restrict__ gate) {
    extern __shared__ float sm[];
    float* segsum = sm;                          // [nseg_max][C]
    float* red = segsum + (size_t)nseg_max * C;  // [256 * 8 / C][C] = 2048
    float* ctx = red + 2048;                     // [C]
    float* hid = ctx + C;                        // [M]
    const int b = blockIdx.x;
    const int tvb = min(tv[b], T);
    const int nseg = (tvb + seg - 1) / seg;
    const int groups = C / 8;                    // 8-channel groups
    const int lanes = 256 / groups;              // time lanes
    const int g = threadIdx.x % groups, ln = threadIdx.x / groups;
    const __half* xb = cc + ((long long)b * (T + 2 * pad) + pad) * ldc + g * 8;
    for (int s = 0; s < nseg; ++s) {
        float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
        const int t1 = min((s + 1) * seg, tvb);
        if (ln < lanes)
            for (int t = s * seg + ln; t < t1; t += lanes) {
                const uint4 v = __ldg(reinterpret_cast<const uint4*>(xb + (long long)t * ldc));
                const __half2* hv = reinterpret_cast<const __half2*>(&v);
#pragma unroll
                for (int q = 0; q < 4; ++q) {
                    const float2 x = __half22float2(hv[q]);
                    acc[2 * q] += x.x;
                    acc[2 * q + 1] += x.y;
                }
            }
        if (ln < lanes)
#pragma unroll
            for (int i = 0; i < 8; ++i) red[ln * C + g * 8 + i] = acc[i];
        __syncthreads();
        for (int c = threadIdx.x; c < C; c += blockDim.x) {
            float v = 0.0f;
            for (int l = 0; l < lanes; ++l) v += red[l * C + c];
            segsum[s * C + c] = v;
        }
        __syncthreads();
    }
    // global mean over the valid frames (from the segment sums)
    for (int c = threadIdx.x; c < C; c += blockDim.x) {
        float v = 0.0f;
        for (int s = 0; s < nseg; ++s) v += segsum[s * C + c];
        red[c] = tvb > 0 ? v / (float)tvb : 0.0f;
    }
    __syncthreads();
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    for (int s = 0; s < nseg; ++s) {
        for (int c = threadIdx.x; c < C; c += blockDim.x)
            ctx[c] = red[c] + segsum[s * C + c] / (float)seg;
        __syncthreads();
        // linear1 + ReLU: one warp per output, lanes over the channels
        for (int j = warp; j < M; j += 8) {
            float v = 0.0f;
            for (int c = lane; c < C; c += 32) v = fmaf(__ldg(w1 + (size_t)j * C + c), ctx[c], v);
#pragma unroll
            for (int o = 16; o >= 1; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
            if (lane == 0) hid[j] = fmaxf(v + b1[j], 0.0f);
        }
        __syncthreads();
        // linear2 + sigmoid
        for (int k = warp; k < G; k += 8) {
            float v = 0.0f;
            for (int j = lane; j < M; j += 32) v = fmaf(__ldg(w2 + (size_t)k * M + j), hid[j], v);
#pragma unroll
            for (int o = 16; o >= 1; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
            if (lane == 0)
                gate[((long long)b * nseg_max + s) * G + k] = 1.0f / (1.0f + expf(-(v + b2[k])));
        }
        __syncthreads();
    }
}

}  // namespace

int campp_bn_relu(const __half* h, int ldh, int C, const float* scale, const float* shift,
                  long long rows, __half* a, int lda, cudaStream_t st) {
    if (C % 8 != 0 || ldh % 8 != 0 || lda % 8 != 0) {
        set_error("campplus: BN + ReLU needs channel counts and pitches that are multiples of 8");
        return 1;
    }
    const long long n = rows * (C / 8);
    const int blocks = (int)std::min<long long>((n + 255) / 256, (long long)num_sms() * 16);
    bn_relu_kernel<<<std::max(blocks, 1), 256, 0, st>>>(h, ldh, C, scale, shift, rows, a, lda);
    VDB_CHECK_CUDA(cudaGetLastError());
    return 0;
}

size_t campp_gate_smem(int C, int M, int nseg_max) {
    return ((size_t)nseg_max * C + 2048 + C + M) * sizeof(float);
}

int campp_cam_gate(const __half* cc, int ldc, const int* tv, int batch, int T, int pad, int C,
                   int seg, int nseg_max, const float* w1, const float* b1, int M,
                   const float* w2, const float* b2, int G, float* gate, cudaStream_t st) {
    if (C % 8 != 0 || C > 2048 || 256 % (C / 8) != 0 || ldc % 8 != 0 || seg < 1 ||
        (long long)nseg_max * seg < T) {
        set_error("campplus: CAM context needs C a multiple of 8 dividing 2048 and "
                  "nseg_max * seg >= T");
        return 1;
    }
    const size_t smem = campp_gate_smem(C, M, nseg_max);
    if (smem > 200 * 1024) {
        set_error("campplus: clip too long for the CAM context kernel (" +
                  std::to_string(nseg_max) + " segments)");
        return 1;
    }
    cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
    VDB_CHECK_CUDA(cudaStreamIsCapturing(st, &cs));
    if (cs == cudaStreamCaptureStatusNone)
        VDB_CHECK_CUDA(cudaFuncSetAttribute(cam_gate_kernel,
                                            cudaFuncAttributeMaxDynamicSharedMemorySize,
                                            200 * 1024));
    cam_gate_kernel<<<batch, 256, smem, st>>>(cc, ldc, tv, T, pad, C, seg, nseg_max, w1, b1, M,
                                              w2, b2, G, gate);
    VDB_CHECK_CUDA(cudaGetLastError());
    return 0;
}

}  // namespace vdb
