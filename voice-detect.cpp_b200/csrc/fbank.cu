// Kaldi-compatible log-mel FBank on the GPU: the B200 replacement for the host
// loop in the reference's FBank::compute (src/fbank.cpp:121-191; CMN, :194-201,
// is fused into the stem kernel in stem.cu).
//
// One warp per frame. The 512 real FFT inputs are packed as 256 complex values
// z[n] = v[2n] + i v[2n+1] (the standard real-input trick), held 8 per lane at
// n = lane + 32*j. The 256-point DFT is split as 256 = 8 x 32 (n = n1 + 32*n2,
// k = k2 + 8*k1):
//   1. 8-point DFT over each lane's registers (radix-2 DIF, unrolled);
//   2. twiddle by W256^(lane*k2);
//   3. 32-point DFT across the lanes of each register slot (radix-2 DIF with
//      __shfl_xor_sync, 5 stages).
// Z goes through shared memory, where each lane forms its bins of the real DFT,
// X[k] = (Z[k] + conj Z[256-k])/2 + W512^k (Z[k] - conj Z[256-k])/2i, and the power
// spectrum; the mel stage then reads bins 0..256 (one lane per filter), then
// log(max(e, FLT_EPSILON)).
//
// Per-frame steps before the FFT follow the reference exactly, including its
// float/double mix: f64 frame mean, f32 DC subtraction, f32 pre-emphasis
// y[i] = x[i] - 0.97*x[i-1] with y[0] = x[0] - 0.97*x[0] (:169-178), and the
// Povey window multiply in f64 rounded to f32 (:181-182). The FFT and the mel
// sums run in f32 with twiddles and filter weights computed on the host in f64.
#include <cuda_fp16.h>

#include <algorithm>
#include <cfloat>
#include <cmath>
#include <string>
#include <vector>

#include "vdb_internal.h"
#include "vdb_ops.h"

struct vdb_fbank_plan {
    int sample_rate, n_mels, n_fft, win, hop, n_weights;
    float preemph;
    double* d_window;    // [win] Povey window (f64)
    float2* d_twiddle;   // [512] W512^m = (cos, -sin)(2*pi*m/512)
    int* d_kstart;       // [n_mels] first FFT bin with nonzero weight
    int* d_klen;         // [n_mels] number of bins
    int* d_woff;         // [n_mels] offset into d_weights
    float* d_weights;    // flattened triangle weights
};

namespace vdb {
namespace {

constexpr int kFFT = 512;
constexpr int kFramesPerBlock = 8;
constexpr int kMaxMels = 128;
constexpr int kMaxWeights = 4096;  // filter weights kept in shared memory

__device__ __forceinline__ void cmul(float& re, float& im, float2 w) {
    const float r = re * w.x - im * w.y;
    const float i = re * w.y + im * w.x;
    re = r;
    im = i;
}

__device__ __forceinline__ int bitrev5(int x) { return __brev(x) >> 27; }

__global__ void __launch_bounds__(32 * kFramesPerBlock)
fbank_kernel(const float* __restrict__ pcm, const long long* __restrict__ offsets,
             const int* __restrict__ nsamp, int batch, int t_max, int win, int hop,
             float preemph, int n_mels, const double* __restrict__ window,
             const float2* __restrict__ twiddle, const int* __restrict__ kstart,
             const int* __restrict__ klen, const int* __restrict__ woff,
             const float* __restrict__ weights, int n_weights, float* __restrict__ feats) {
    // Persistent blocks: the tables are staged in shared memory once per block,
    // then each warp walks frames (b, t) of the flattened batch x t_max range.
    __shared__ float2 s_tw[kFFT];
    __shared__ double s_win[kFFT];
    // per warp: the 256 complex Z[k] (2 KB), then the 257-bin power spectrum
    __shared__ __align__(16) float s_ps[kFramesPerBlock][kFFT];
    __shared__ float s_w[kMaxWeights];
    __shared__ int s_ks[kMaxMels], s_kl[kMaxMels], s_wo[kMaxMels];
    for (int i = threadIdx.x; i < kFFT; i += blockDim.x) {
        s_tw[i] = twiddle[i];
        s_win[i] = i < win ? window[i] : 0.0;
    }
    for (int i = threadIdx.x; i < n_weights; i += blockDim.x) s_w[i] = weights[i];
    for (int i = threadIdx.x; i < n_mels; i += blockDim.x) {
        s_ks[i] = kstart[i];
        s_kl[i] = klen[i];
        s_wo[i] = woff[i];
    }
    __syncthreads();

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const long long n_frames = (long long)batch * t_max;
    for (long long id = (long long)blockIdx.x * kFramesPerBlock + warp; id < n_frames;
         id += (long long)gridDim.x * kFramesPerBlock) {
    const int b = (int)(id / t_max);
    const int t = (int)(id - (long long)b * t_max);
    const int n = nsamp[b];
    const int T = n >= win ? 1 + (n - win) / hop : 0;
    if (t >= T) continue;
    const float* x = pcm + offsets[b] + (long long)t * hop;

    // The 512 real inputs are packed as 256 complex z[n] = v[2n] + i v[2n+1]; lane l
    // holds n = l + 32j (j = 0..7), i.e. samples 2l + 64j and 2l + 1 + 64j.
    float ev[8], od[8];
    double s = 0.0;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
        const int i0 = 2 * lane + 64 * j;
        ev[j] = i0 < win ? __ldg(x + i0) : 0.0f;
        od[j] = i0 + 1 < win ? __ldg(x + i0 + 1) : 0.0f;
        s += (double)ev[j] + (double)od[j];
    }
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    const float mean_f = (float)(s / win);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
        const int i0 = 2 * lane + 64 * j;
        if (i0 < win) ev[j] = __fsub_rn(ev[j], mean_f);
        if (i0 + 1 < win) od[j] = __fsub_rn(od[j], mean_f);
    }
    // Pre-emphasis on the DC-removed frame. The odd sample's predecessor is the even
    // sample in the same register; the even sample's is the odd sample of n - 1:
    // lane - 1 in the same slot, or lane 31 of slot j - 1 for lane 0 (sample 0 uses
    // itself, the reference's replicate rule).
    float re[8], im[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
        const float up = __shfl_up_sync(0xffffffffu, od[j], 1);
        const float wrap = __shfl_sync(0xffffffffu, j > 0 ? od[j - 1] : 0.0f, 31);
        const float prev = lane > 0 ? up : (j > 0 ? wrap : ev[0]);
        const int i0 = 2 * lane + 64 * j;
        float ye = 0.0f, yo = 0.0f;
        if (i0 < win) ye = (float)((double)__fsub_rn(ev[j], __fmul_rn(preemph, prev)) * s_win[i0]);
        if (i0 + 1 < win)
            yo = (float)((double)__fsub_rn(od[j], __fmul_rn(preemph, ev[j])) * s_win[i0 + 1]);
        re[j] = ye;
        im[j] = yo;
    }

    // 256-point DFT of z, 256 = 8 x 32 (n = n1 + 32 n2, k = k2 + 8 k1):
    // 1. 8-point DIF over the register slots (output slot r holds k2 = bitrev3(r)).
#pragma unroll
    for (int h = 4; h >= 1; h >>= 1) {
#pragma unroll
        for (int s0 = 0; s0 < 8; s0 += 2 * h) {
#pragma unroll
            for (int i = 0; i < h; ++i) {
                const int a = s0 + i, c = s0 + i + h;
                const float ur = re[a], ui = im[a], vr = re[c], vi = im[c];
                re[a] = ur + vr;
                im[a] = ui + vi;
                float dr = ur - vr, di = ui - vi;
                if (i != 0) cmul(dr, di, s_tw[i * (4 / h) * 64]);  // W8^(i*4/h)
                re[c] = dr;
                im[c] = di;
            }
        }
    }
    // 2. twiddle W256^(lane * k2) = W512^(2 * lane * k2).
#pragma unroll
    for (int r = 0; r < 8; ++r) {
        const int k2 = ((r & 1) << 2) | (r & 2) | ((r & 4) >> 2);
        if (k2 != 0 && lane != 0) cmul(re[r], im[r], s_tw[(2 * lane * k2) & (kFFT - 1)]);
    }
    // 3. 32-point DIF across lanes for every slot (lane l ends with k1 = bitrev5(l)).
#pragma unroll
    for (int h = 16; h >= 1; h >>= 1) {
        const bool upper = (lane & h) != 0;
        const float2 tw = s_tw[(lane & (h - 1)) * (256 / h)];  // W_{2h}^(lane mod h)
#pragma unroll
        for (int r = 0; r < 8; ++r) {
            const float pr = __shfl_xor_sync(0xffffffffu, re[r], h);
            const float pi = __shfl_xor_sync(0xffffffffu, im[r], h);
            if (!upper) {
                re[r] += pr;
                im[r] += pi;
            } else {
                float dr = pr - re[r], di = pi - im[r];
                cmul(dr, di, tw);
                re[r] = dr;
                im[r] = di;
            }
        }
    }
    // Z[k] to shared memory, then the real-input split
    // X[k] = A + W512^k B, A = (Z[k] + conj Z[256-k]) / 2, B = (Z[k] - conj Z[256-k]) / 2i,
    // and the power spectrum |X[k]|^2 for k = 0..256.
    float2* zs = reinterpret_cast<float2*>(s_ps[warp]);
    {
        const int k1 = bitrev5(lane);
#pragma unroll
        for (int r = 0; r < 8; ++r) {
            const int k2 = ((r & 1) << 2) | (r & 2) | ((r & 4) >> 2);
            zs[k2 + 8 * k1] = make_float2(re[r], im[r]);
        }
    }
    __syncwarp();
    float pw[8];
#pragma unroll
    for (int m = 0; m < 8; ++m) {
        const int k = lane + 32 * m;
        const float2 zk = zs[k], zc = zs[(256 - k) & 255];
        const float ar = 0.5f * (zk.x + zc.x), ai = 0.5f * (zk.y - zc.y);
        const float br = 0.5f * (zk.y + zc.y), bi = -0.5f * (zk.x - zc.x);
        const float2 w = s_tw[k];
        const float xr = ar + (w.x * br - w.y * bi);
        const float xi = ai + (w.x * bi + w.y * br);
        pw[m] = xr * xr + xi * xi;
    }
    const float2 z0 = zs[0];
    __syncwarp();  // all Z reads done before the power spectrum overwrites the buffer
    float* ps = s_ps[warp];
#pragma unroll
    for (int m = 0; m < 8; ++m) ps[lane + 32 * m] = pw[m];
    if (lane == 0) {
        const float xn = z0.x - z0.y;  // X[256] = Re Z[0] - Im Z[0]
        ps[256] = xn * xn;
    }
    __syncwarp();
    float* out = feats + ((long long)b * t_max + t) * n_mels;
    for (int m = lane; m < n_mels; m += 32) {
        const int k0 = s_ks[m], kl = s_kl[m], wo = s_wo[m];
        float e = 0.0f;
        for (int i = 0; i < kl; ++i) e = fmaf(s_w[wo + i], ps[k0 + i], e);
        out[m] = logf(fmaxf(e, FLT_EPSILON));
    }
    __syncwarp();  // ps is rewritten by this warp's next frame
    }
}

double mel_of(double f) { return 1127.0 * std::log(1.0 + f / 700.0); }

}  // namespace
}  // namespace vdb

using namespace vdb;

extern "C" vdb_fbank_plan* vdb_fbank_plan_create(int sample_rate, int n_mels, int n_fft, int win,
                                                 int hop, float preemph, float low_freq,
                                                 float high_freq) {
    if (n_fft != kFFT) {
        set_error("vdb_fbank_plan_create: only n_fft = 512 is supported");
        return nullptr;
    }
    if (win <= 1 || win > n_fft || hop <= 0 || n_mels <= 0 || n_mels > kMaxMels ||
        sample_rate <= 0) {
        set_error("vdb_fbank_plan_create: invalid FBank configuration");
        return nullptr;
    }
    const double kPI = 3.14159265358979323846;
    std::vector<double> window(win);
    for (int i = 0; i < win; ++i)
        window[i] = std::pow(0.5 - 0.5 * std::cos(2.0 * kPI * i / (win - 1)), 0.85);
    std::vector<float2> tw(kFFT);
    for (int m = 0; m < kFFT; ++m) {
        const double a = 2.0 * kPI * m / kFFT;
        tw[m] = make_float2((float)std::cos(a), (float)-std::sin(a));
    }
    // Triangular mel filters, same construction as src/fbank.cpp:140-158.
    const int half = n_fft / 2;
    const double lo = low_freq;
    const double hi = high_freq > 0.0f ? (double)high_freq : sample_rate / 2.0;
    const double mlo = mel_of(lo), mhi = mel_of(hi);
    const double mstep = (mhi - mlo) / (n_mels + 1);
    std::vector<int> ks(n_mels), kl(n_mels), wo(n_mels);
    std::vector<float> wts;
    for (int m = 0; m < n_mels; ++m) {
        const double l = mlo + m * mstep, c = mlo + (m + 1) * mstep, r = mlo + (m + 2) * mstep;
        int first = -1, last = -1;
        std::vector<double> row(half + 1, 0.0);
        for (int k = 0; k <= half; ++k) {
            const double mf = mel_of((double)k * sample_rate / n_fft);
            double w = 0.0;
            if (mf > l && mf <= c) w = (mf - l) / (c - l);
            else if (mf > c && mf < r) w = (r - mf) / (r - c);
            row[k] = w;
            if (w != 0.0) {
                if (first < 0) first = k;
                last = k;
            }
        }
        if (first < 0) first = last = 0;
        ks[m] = first;
        kl[m] = last - first + 1;
        wo[m] = (int)wts.size();
        for (int k = first; k <= last; ++k) wts.push_back((float)row[k]);
    }
    vdb_fbank_plan* p = new vdb_fbank_plan{};
    p->sample_rate = sample_rate;
    p->n_mels = n_mels;
    p->n_fft = n_fft;
    p->win = win;
    p->hop = hop;
    p->preemph = preemph;
    p->n_weights = (int)wts.size();
    if (p->n_weights > kMaxWeights) {
        set_error("vdb_fbank_plan_create: mel filter bank too large");
        delete p;
        return nullptr;
    }
    bool ok = cudaMalloc(&p->d_window, sizeof(double) * win) == cudaSuccess &&
              cudaMalloc(&p->d_twiddle, sizeof(float2) * kFFT) == cudaSuccess &&
              cudaMalloc(&p->d_kstart, sizeof(int) * n_mels) == cudaSuccess &&
              cudaMalloc(&p->d_klen, sizeof(int) * n_mels) == cudaSuccess &&
              cudaMalloc(&p->d_woff, sizeof(int) * n_mels) == cudaSuccess &&
              cudaMalloc(&p->d_weights, sizeof(float) * wts.size()) == cudaSuccess;
    ok = ok &&
         cudaMemcpy(p->d_window, window.data(), sizeof(double) * win,
                    cudaMemcpyHostToDevice) == cudaSuccess &&
         cudaMemcpy(p->d_twiddle, tw.data(), sizeof(float2) * kFFT, cudaMemcpyHostToDevice) ==
             cudaSuccess &&
         cudaMemcpy(p->d_kstart, ks.data(), sizeof(int) * n_mels, cudaMemcpyHostToDevice) ==
             cudaSuccess &&
         cudaMemcpy(p->d_klen, kl.data(), sizeof(int) * n_mels, cudaMemcpyHostToDevice) ==
             cudaSuccess &&
         cudaMemcpy(p->d_woff, wo.data(), sizeof(int) * n_mels, cudaMemcpyHostToDevice) ==
             cudaSuccess &&
         cudaMemcpy(p->d_weights, wts.data(), sizeof(float) * wts.size(),
                    cudaMemcpyHostToDevice) == cudaSuccess;
    if (!ok) {
        set_error("vdb_fbank_plan_create: device allocation/upload failed");
        vdb_fbank_plan_destroy(p);
        return nullptr;
    }
    return p;
}

extern "C" void vdb_fbank_plan_destroy(vdb_fbank_plan* p) {
    if (!p) return;
    cudaFree(p->d_window);
    cudaFree(p->d_twiddle);
    cudaFree(p->d_kstart);
    cudaFree(p->d_klen);
    cudaFree(p->d_woff);
    cudaFree(p->d_weights);
    delete p;
}

extern "C" int vdb_fbank_plan_n_mels(const vdb_fbank_plan* p) { return p ? p->n_mels : 0; }

extern "C" int vdb_fbank(const vdb_fbank_plan* p, const float* pcm, const long long* offsets,
                         const int* n_samples, int batch, int t_max, float* feats,
                         void* stream) {
    if (!p || !pcm || !offsets || !n_samples || !feats) {
        set_error("vdb_fbank: NULL argument");
        return 1;
    }
    if (batch <= 0 || t_max <= 0) {
        set_error("vdb_fbank: empty batch");
        return 1;
    }
    const long long frames = (long long)batch * t_max;
    const int grid = (int)std::min<long long>((frames + kFramesPerBlock - 1) / kFramesPerBlock,
                                              (long long)num_sms() * 6);
    fbank_kernel<<<grid, 32 * kFramesPerBlock, 0, static_cast<cudaStream_t>(stream)>>>(
        pcm, offsets, n_samples, batch, t_max, p->win, p->hop, p->preemph, p->n_mels,
        p->d_window, p->d_twiddle, p->d_kstart, p->d_klen, p->d_woff, p->d_weights,
        p->n_weights, feats);
    VDB_CHECK_CUDA(cudaGetLastError());
    return 0;
}
