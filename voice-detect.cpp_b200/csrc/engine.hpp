// The B200 embedding engine behind the C ABI: the counterpart of the reference's
// vd::Model (src/model.hpp:18-56) + ResNet34Encoder (src/encoder_resnet.cpp) +
// ModelLoader (src/model_loader.cpp), re-designed for batched GPU execution.
//
// A loaded Engine owns its weights on one device (packed once at load: conv
// weights f16 [OC][taps][IC], stem and FC f32), an FBank plan, a CUDA stream and
// a grow-only workspace. embed_* calls sort clips by length, cut them into
// buckets (at most max_clips clips and max_frames padded frames each) and run
// each bucket as one batched pass: FBank -> CMN+stem -> 32 tensor-core convs ->
// TSTP+FC+L2. Ragged clips inside a bucket are exact: every conv masks rows past
// each clip's valid length (see conv_tc.cu).
#pragma once
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <memory>
#include <string>
#include <vector>

#include "vdb_ops.h"

namespace vdb {

class Gguf;

struct EngineConfig {
    std::string arch;
    int emb_dim = 0;
    bool l2 = true;
    int sample_rate = 16000, n_mels = 80, n_fft = 512, win = 400, hop = 160;
    float preemph = 0.97f, low_freq = 20.0f, high_freq = 0.0f;
    bool cmn = true;
};

// Conv weights are f16, or (q8_0 GGUF tensors) int8 values in the same layout with an
// f16 scale per 32 input channels of a tap (the `...s` pointers, null for f16); the
// conv kernel expands q8_0 to f16 in shared memory.
struct ResBlockDev {
    int ic = 0, oc = 0, stride = 1;
    void* w1 = nullptr;          // [oc][9][ic]
    const void* w1s = nullptr;   // q8_0 scales [oc][9][ic / 32]
    float* b1 = nullptr;
    void* w2 = nullptr;          // [oc][9][oc]
    const void* w2s = nullptr;
    float* b2 = nullptr;    // conv2 bias (+ downsample bias when fused)
    void* wd = nullptr;     // [oc][ic], or the f16 [oc][oc] identity for an identity shortcut
    const void* wds = nullptr;
    bool identity = false;
    // stage-1 blocks run over the QPACK layout: conv1 / conv2 weights packed for it
    // (vdb_qpack_pack_weights, [3][384][32]; q8_0: one scale per packed row)
    void* w1q = nullptr;
    const void* w1qs = nullptr;
    void* w2q = nullptr;
    const void* w2qs = nullptr;
};

// ERes2Net runs from a plan compiled once at load from the conv manifest
// (src/encoder_eres2net.cpp:147-226 replayed with a running conv index): a flat
// list of conv / add steps over named activation buffers. An operand is a
// buffer plus a channel offset, so the Res2Net split and concat are views.
struct EOperand {
    int buf = -1;
    int c0 = 0;
};

struct EStep {
    int kind = 0;    // 0: vdb_conv, 1: vdb_add (y = x0 + x1 over oc channels)
    int level = 0;   // resolution level of the output
    int oc = 0, k0 = 1, stride0 = 1, ic0 = 0, ic1 = 0, stride1 = 1;
    EOperand x0, x1, res, res2, y, y2, ysum, addend;
    const __half* w0 = nullptr;
    const __half* w1 = nullptr;
    const float* bias = nullptr;
    int relu = 0, act = 0, y_phase = 0;
    float clamp_hi = 0.0f;
    double flops_px = 0.0;   // algorithmic FLOPs per valid output pixel
};

// ECAPA-TDNN (src/encoder.cpp). One TDNN conv: f16 weights [oc][k][ic], the conv
// bias, and the eval BatchNorm after its ReLU folded to scale / shift (or none).
struct TdnnDev {
    int ic = 0, oc = 0, k = 1, dil = 1;
    __half* w = nullptr;
    float* b = nullptr;
    float* scale = nullptr;
    float* shift = nullptr;
};

struct EcapaBlockDev {
    int dil = 1;                     // dilation of the Res2Net convs (block index + 1)
    TdnnDev tdnn1, tdnn2;            // tdnn2.w: the columns reading group 0 ([C][C/scale])
    __half* tdnn2_w_rest = nullptr;  // the columns reading groups 1.. ([C][C - C/scale])
    std::vector<TdnnDev> groups;     // scale - 1 dilated convs, C/scale -> C/scale
    int se = 0;                      // SE bottleneck
    float* se_w1 = nullptr;          // [se][C]
    float* se_b1 = nullptr;
    float* se_w2 = nullptr;          // [C][se]
    float* se_b2 = nullptr;
};

struct EcapaDev {
    int C = 0, Cm = 0, att = 0, scale = 0, pad = 0;
    TdnnDev stem, mfa, asp_tdnn, asp_conv;  // asp_tdnn.w: the columns reading x ([att][Cm])
    float* asp_ctx_w = nullptr;             // [att][2*Cm]: the columns reading mean / std
    std::vector<EcapaBlockDev> blocks;
    float* fc_w = nullptr;                  // [emb][2*Cm], asp_bn folded in
    float* fc_b = nullptr;
};

// CAM++ (src/encoder_campplus.cpp). FCM 2-D convs: f16 [oc][kt*k + kf][ic] + bias
// (BN folded; the stride-2 block's conv2 bias includes its shortcut's).
struct Fcm2dDev {
    int ic = 0, oc = 0, k = 3;
    __half* w = nullptr;
    float* b = nullptr;
};

struct CamppStageDev {
    Fcm2dDev c1, c2, c3, c4;    // stride-2 block conv1 / conv2, stride-1 block conv1 / conv2
    __half* sc_w = nullptr;     // stride-2 block 1x1 shortcut [oc][ic]
};

struct CamppLayerDev {
    int c_in = 0;
    float* bn_scale = nullptr;  // nonlinear1 BN over c_in channels
    float* bn_shift = nullptr;
    TdnnDev lin1;               // 1x1 c_in -> bnc, bias, ReLU
    TdnnDev local;              // k=3 dilated bnc -> growth, no bias, * CAM gate
    float* cam_w1 = nullptr;    // transposed: [bnc][cam_m]
    float* cam_b1 = nullptr;
    float* cam_w2 = nullptr;    // transposed: [cam_m][growth]
    float* cam_b2 = nullptr;
};

struct CamppBlockDev {
    int dil = 1, c0 = 0, cmax = 0;
    std::vector<CamppLayerDev> layers;
    float* tr_scale = nullptr;  // transit BN over cmax
    float* tr_shift = nullptr;
    TdnnDev transit;            // 1x1 cmax -> cmax/2
};

struct CamppDev {
    int M = 0, f_out = 0, bnc = 0, growth = 0, cam_m = 0, c_out = 0;
    int pad = 2;                // SEQ padding rows at the TDNN rate (>= the widest dilation)
    float* stem_w = nullptr;    // [M][9], tap kt*3 + kf
    float* stem_b = nullptr;
    CamppStageDev stages[2];
    Fcm2dDev fcm_out;           // FCM conv2 (freq stride 2)
    TdnnDev tdnn;               // k=5 time stride 2, columns f*M + c
    std::vector<CamppBlockDev> blocks;
    float* fc_w = nullptr;      // [emb][2*c_out], output BN folded
    float* fc_b = nullptr;
};

struct EBuf {
    int level = 0, c = 0;
    bool phase = false;      // P layout (for a stride-2 consumer) instead of G
    void* p = nullptr;
    size_t bytes = 0;
};

class Engine {
public:
    // Loads a GGUF on the current CUDA device. Returns nullptr and sets err on failure.
    static std::unique_ptr<Engine> load(const std::string& path, std::string& err);
    ~Engine();

    const EngineConfig& config() const { return cfg_; }
    int emb_dim() const { return cfg_.emb_dim; }
    bool supported(std::string& err) const;

    // Embeds n clips of 16 kHz f32 PCM already in device memory (clip i at
    // d_pcm + offsets[i], nsamp[i] samples; offsets/nsamp are host arrays). Writes
    // L2-normalised embeddings to d_out[i*emb_dim ...] (device). Asynchronous on
    // `stream` (nullptr = the engine's stream). Returns 0 or sets err.
    int embed_device(const float* d_pcm, const long long* offsets, const int* nsamp, int n,
                     float* d_out, cudaStream_t stream, std::string& err);

    // Host PCM in, host embeddings out (synchronous). pcm[i] has nsamp[i] samples.
    int embed_host(const float* const* pcm, const int* nsamp, int n, float* out,
                   std::string& err);
    // Host mono PCM of element type `type` (0 f32, 1 int16 scaled by 2^-15) at
    // `sample_rate`: the raw samples are copied to the device and converted /
    // linearly resampled to f32 16 kHz there (vdb_pcm_ingest) before the buckets run.
    int embed_host_raw(const void* const* pcm, int type, const int* nsamp, int n,
                       int sample_rate, float* out, std::string& err);

    // Reads and clears the device error word (kernel timeouts). Synchronises.
    int check_device_error(std::string& err);

    // Synchronises, then drops every captured CUDA graph and frees the workspace
    // (activations, staging and ring buffers); weights stay resident. The next embed
    // call re-allocates and re-captures, producing identical results.
    int release_cache(std::string& err);

    // Bucketing policy.
    int max_clips = 512;
    long long max_frames = 262144;

    // Number of GPU kernels launched by the last embed call (for benchmarks).
    long long last_launches = 0;
    // Device bytes of the ResNet block conv weights (values, q8_0 scales, QPACK copies).
    long long conv_weight_bytes = 0;

    // Conv-kernel profiling: when enabled, every tensor-core conv launch is
    // bracketed by CUDA events on its stream and its algorithmic FLOPs
    // (2*OC*IC*k*k*F_out*sum of valid output frames) are accumulated.
    void set_profiling(bool on);
    // Synchronises, then returns totals since the last read and resets them.
    int read_profile(double& conv_ms, double& conv_flops, long long& conv_launches,
                     std::string& err);

    cudaStream_t stream() const { return stream_; }
    int device() const { return device_; }

private:
    Engine() = default;
    int run_bucket(const float* d_pcm, const long long* h_off, const int* h_ns,
                   const int* h_outrow, int B, cudaStream_t st, float* d_out, std::string& err);
    // Length-sorted buckets: clip indices longest first in `order`; bucket k is
    // order[bk[k] .. bk[k+1]).
    void plan_buckets(const int* nsamp, int n, long long frame_cap, std::vector<int>& order,
                      std::vector<size_t>& bk) const;
    // Every kernel launch of one bucket (metadata already on the device).
    int launch_bucket(const float* d_pcm, int B, int t_max, const std::vector<long long>& tv_sum,
                      cudaStream_t st, float* d_out, long long& launches, std::string& err);
    void clear_graphs();
    int run_eres2net(int B, int t_max, const std::vector<long long>& tv_sum, cudaStream_t st,
                     float* d_out, long long& launches, std::string& err);
    int ensure_workspace(int B, int t_max, std::string& err);
    void free_workspace();
    bool load_eres2net(const Gguf& g, std::string& err);
    bool load_ecapa(const Gguf& g, std::string& err);
    int run_ecapa(int B, int t_max, const std::vector<long long>& tv_sum, cudaStream_t st,
                  float* d_out, long long& launches, std::string& err);
    size_t ecapa_ws_bytes(int B, int t_max) const;
    size_t ecapa_gemm_scratch(int B) const;
    bool load_campplus(const Gguf& g, std::string& err);
    int run_campplus(int B, int t_max, const std::vector<long long>& tv_sum, cudaStream_t st,
                     float* d_out, long long& launches, std::string& err);
    size_t campp_ws_bytes(int B, int t_max) const;
    bool upload_f32(const std::vector<float>& v, float** dst, std::string& err);
    bool upload_f16(const std::vector<float>& v, __half** dst, std::string& err);
    bool upload_bytes(const void* src, size_t n, void** dst, std::string& err);
    // f16 identity [c][c]: an identity shortcut added on the tensor cores as a 1x1
    // input segment of the conv that ends the block (x * 1.0 is exact, and the sum
    // is accumulated in f32 like the epilogue add it replaces). One per width.
    const __half* identity(int c, std::string& err);
    std::vector<std::pair<int, __half*>> identities_;

    EngineConfig cfg_;
    int device_ = 0;
    cudaStream_t stream_ = nullptr;
    vdb_fbank_plan* plan_ = nullptr;
    // weights
    int stem_oc_ = 0;
    // ResNet stage 1 (every block before the first stride-2 one: 32 -> 32 with identity
    // shortcuts, 32 stem channels) runs over QPACK rows: the stem writes QPACK, its convs
    // take the (time tap, pixel shift) schedule and the last one writes the PHASE input
    // of the first stride-2 block.
    bool qpack_ = false;
    float* stem_w_ = nullptr;   // [oc][9], tap kt*3 + kf
    float* stem_b_ = nullptr;
    std::vector<ResBlockDev> blocks_;
    float* seg_w_ = nullptr;    // [D][P]
    float* seg_b_ = nullptr;
    float* mean_vec_ = nullptr;
    int pooled_ = 0;
    float var_eps_ = 1e-8f;
    std::vector<void*> weight_allocs_;
    // f16 expansion target of the q8_0 weights a conv streams (one conv at a time on the
    // engine's stream): sized at load for the largest block conv
    void* wscratch_ = nullptr;
    long long wscratch_bytes_ = 0;
    // CUDA graphs of a bucket's launch sequence, keyed by everything its kernel
    // arguments depend on (the per-clip metadata lives in device buffers that are
    // refreshed before each launch). A shape is captured the second time it is seen;
    // any workspace growth drops them all.
    struct GraphEntry {
        int B, t_max;
        const float* d_pcm;
        float* d_out;
        cudaStream_t st;
        int seen;
        cudaGraphExec_t exec;
        long long launches;
    };
    std::vector<GraphEntry> graphs_;
    bool graphs_enabled_ = true;
    // ECAPA-TDNN / CAM++ weights; their workspace (ecapa_ws_) is carved per bucket shape
    CamppDev campp_;
    EcapaDev ecapa_;
    void* ecapa_ws_ = nullptr;
    size_t ecapa_ws_bytes_ = 0;
    // ERes2Net plan
    std::vector<EBuf> ebufs_;
    std::vector<EStep> esteps_;
    int e_stem_buf_ = -1, e_out_buf_ = -1, e_out_level_ = 0;
    // workspace (grow-only)
    struct Level {
        int c = 0;
        size_t g_bytes = 0, p_bytes = 0;
        void* g[3] = {nullptr, nullptr, nullptr};
        void* p = nullptr;
    };
    std::vector<Level> levels_;
    float* feats_ = nullptr;
    size_t feats_bytes_ = 0;
    float* mean_ = nullptr;
    size_t mean_bytes_ = 0;
    float* pool_scratch_ = nullptr;   // pooled vectors + FC partials of one bucket
    size_t pool_scratch_bytes_ = 0;
    int* meta_ = nullptr;         // device int32: frames, tvalid per level, out rows
    long long* offs_ = nullptr;   // device int64 offsets
    int* nsamp_ = nullptr;
    int meta_cap_ = 0;
    int* errword_ = nullptr;
    // pinned, mapped staging for small per-bucket host->device metadata, which a kernel
    // reads through d_stage_ (the same memory's device address)
    void* h_stage_ = nullptr;
    void* d_stage_ = nullptr;
    size_t h_stage_bytes_ = 0;   // bytes per slot (two slots)
    int stage_slot_ = 0;
    bool stage_used_[2] = {false, false};
    cudaEvent_t stage_ev_[2] = {nullptr, nullptr};
    // Host PCM path: a two-slot ring of pinned host + device PCM buffers, each
    // holding one bucket. The host gathers bucket k+1 into its pinned slot while
    // the GPU runs bucket k; the H2D copy runs on copy_stream_ and overlaps compute.
    // A bucket whose clips all lie in page-locked caller memory skips the host slot:
    // one DMA per clip into the device slot.
    cudaStream_t copy_stream_ = nullptr;
    void* h_ring_[2] = {nullptr, nullptr};   // raw PCM of one bucket (f32 or int16)
    void* d_ring_[2] = {nullptr, nullptr};
    size_t ring_bytes_ = 0;
    // device conversion of raw PCM (int16 / other rates): f32 16 kHz output per slot
    // and the per-clip offsets / lengths the ingest kernel reads
    float* d_conv_[2] = {nullptr, nullptr};
    size_t conv_bytes_ = 0;
    void* h_imeta_[2] = {nullptr, nullptr};
    void* d_imeta_[2] = {nullptr, nullptr};
    int imeta_cap_ = 0;
    bool ring_used_[2] = {false, false};
    cudaEvent_t h2d_ev_[2] = {nullptr, nullptr};    // slot's H2D copy finished
    cudaEvent_t comp_ev_[2] = {nullptr, nullptr};   // slot's bucket compute finished
    float* h_out_ = nullptr;
    float* d_out_ = nullptr;
    size_t out_bytes_ = 0;
    // profiling
    bool profiling_ = false;
    std::vector<cudaEvent_t> prof_ev_;  // pairs (start, stop)
    size_t prof_used_ = 0;              // events in use
    double prof_flops_ = 0.0;
    // Event pairs are tagged with a stage: 0 conv, 1 FBank, 2 pooling (TSTP + FC +
    // L2), 3 other (element-wise adds), 4 CMN + stem.
    int prof_begin(cudaStream_t st, int stage = 0);  // returns event-pair index or -1
    void prof_end(int idx, cudaStream_t st, double flops, const vdb_conv_args* conv = nullptr);
    std::vector<int> prof_stage_;
public:
    // One profiled conv launch: its duration, algorithmic FLOPs and shape.
    struct ConvRecord {
        double ms, flops;
        int ic, oc, k, stride, f_out, t_out, batch, ic1, res, qpack;  // ic1 0: one segment
    };
    // Per-stage summed launch durations (ms) of the last read_profile call.
    double stage_ms[5] = {0, 0, 0, 0, 0};
    // The conv launches of the last read_profile call, in launch order.
    std::vector<ConvRecord> conv_records;
private:
    std::vector<ConvRecord> prof_conv_;  // per event pair (stage 0 only meaningful)
private:
};

// Linear resampling, src/audio_io.cpp:9-23.
std::vector<float> resample_linear(const std::vector<float>& in, int in_sr, int out_sr);
// WAV decode to mono f32 (channels averaged) at the file's rate; false on error.
bool read_wav_mono(const std::string& path, std::vector<float>& out, int& sample_rate,
                   std::string& err);

}  // namespace vdb
