// Device-side audio ingest: int16 or f32 mono PCM at any sample rate -> the f32
// 16 kHz samples FBank reads, for a whole bucket in one launch. The reference does
// this on the host per clip: drwav's s16 -> f32 scaling by 2^-15 and
// vd::resample_linear (src/audio_io.cpp:9-23). The arithmetic here is the same,
// step for step (positions and the blend in double, the difference of neighbours in
// float), so the device result is bitwise the host one.
#include <cuda_fp16.h>
#include <cstdint>

#include <algorithm>
#include <cmath>

#include "vdb_internal.h"
#include "vdb_ops.h"

namespace vdb {
namespace {

template <int TYPE>
__device__ __forceinline__ float pcm_sample(const void* in, long long k) {
    if constexpr (TYPE == 1)
        return (float)static_cast<const int16_t*>(in)[k] * (1.0f / 32768.0f);
    else
        return static_cast<const float*>(in)[k];
}

// blockIdx.y = clip; thread i of the grid's x extent produces output sample i.
template <int TYPE>
__global__ void __launch_bounds__(256)
pcm_ingest_kernel(const void* __restrict__ in, const long long* __restrict__ in_off,
                  const int* __restrict__ n_in, const long long* __restrict__ out_off,
                  const int* __restrict__ n_out, int in_sr, int out_sr, float* __restrict__ out) {
    const int b = blockIdx.y;
    const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n_out[b]) return;
    const long long io = in_off[b];
    float v;
    if (in_sr == out_sr) {
        v = pcm_sample<TYPE>(in, io + i);
    } else {
        // src/audio_io.cpp:11-20: src = i / ratio, i0 = floor, frac = src - i0,
        // out = a + (b - a) * frac with b the next sample (or a at the end)
        // (explicit round-to-nearest operations: no multiply-add contraction, so each
        // step rounds exactly as the C++ source's separate operations do)
        const double ratio = __ddiv_rn((double)out_sr, (double)in_sr);
        const double src = __ddiv_rn((double)i, ratio);
        const long long i0 = (long long)src;
        const double frac = __dsub_rn(src, (double)i0);
        const float a = pcm_sample<TYPE>(in, io + i0);
        const float c = (i0 + 1 < (long long)n_in[b]) ? pcm_sample<TYPE>(in, io + i0 + 1) : a;
        v = (float)__dadd_rn((double)a, __dmul_rn((double)__fsub_rn(c, a), frac));
    }
    out[out_off[b] + i] = v;
}

}  // namespace
}  // namespace vdb

using namespace vdb;

extern "C" long long vdb_resampled_length(long long n_in, int in_sr, int out_sr) {
    if (n_in <= 0 || in_sr <= 0 || out_sr <= 0) return 0;
    if (in_sr == out_sr) return n_in;
    const double ratio = (double)out_sr / (double)in_sr;
    return (long long)std::floor((double)n_in * ratio);
}

extern "C" int vdb_pcm_ingest(const void* in, int in_type, const long long* in_off,
                              const int* n_in, int batch, int in_sr, int out_sr,
                              const long long* out_off, const int* n_out, int max_out, float* out,
                              void* stream) {
    if (!in || !in_off || !n_in || !out_off || !n_out || !out) {
        set_error("vdb_pcm_ingest: NULL buffer");
        return 1;
    }
    if (batch <= 0 || batch > 65535 || in_sr <= 0 || out_sr <= 0 || max_out < 0) {
        set_error("vdb_pcm_ingest: batch must be in [1, 65535] and the rates positive");
        return 1;
    }
    if (in_type != 0 && in_type != 1) {
        set_error("vdb_pcm_ingest: in_type must be 0 (f32) or 1 (int16)");
        return 1;
    }
    if (max_out == 0) return 0;
    const dim3 grid((unsigned)((max_out + 255) / 256), (unsigned)batch);
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    if (in_type == 1)
        pcm_ingest_kernel<1><<<grid, 256, 0, st>>>(in, in_off, n_in, out_off, n_out, in_sr, out_sr,
                                                    out);
    else
        pcm_ingest_kernel<0><<<grid, 256, 0, st>>>(in, in_off, n_in, out_off, n_out, in_sr, out_sr,
                                                    out);
    VDB_CHECK_CUDA(cudaGetLastError());
    return 0;
}
