// Engine implementation: GGUF -> device weights, bucketing, and the per-bucket
// launch sequence. See engine.hpp for the overview.
#include "engine.hpp"

#include <algorithm>
#include <climits>
#include <cmath>
#include <cstdlib>
#include <cstring>

#include "host_copy.h"
#include <numeric>
#include <thread>

#include "gguf.hpp"
#include "vdb_internal.h"

namespace vdb {
namespace {

__global__ void f32_to_f16_kernel(const float* __restrict__ in, __half* __restrict__ out,
                                  long long n) {
    const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) out[i] = __float2half_rn(in[i]);
}

// Copies one bucket's metadata from its pinned staging slot, read through the slot's
// mapped device address, into the device buffers the bucket's kernels read: n_meta ints
// (valid lengths per level, output rows), then B offsets and B sample counts. A kernel
// rather than cudaMemcpyAsync: a host-to-device copy on the compute stream waits on the
// copy engine behind whatever transfer holds it, and in the host-PCM path that is the
// next bucket's PCM (160+ MB, ~3 ms), which held every bucket's compute back as long.
__global__ void stage_meta_kernel(const int* __restrict__ hm, int n_meta,
                                  const long long* __restrict__ ho, const int* __restrict__ hn,
                                  int B, int* __restrict__ meta, long long* __restrict__ offs,
                                  int* __restrict__ nsamp) {
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n_meta + B;
         i += gridDim.x * blockDim.x) {
        if (i < n_meta) {
            meta[i] = hm[i];
        } else {
            const int b = i - n_meta;
            offs[b] = ho[b];
            nsamp[b] = hn[b];
        }
    }
}

struct Loader {
    const Gguf& g;
    std::string& err;

    bool is_q8(const std::string& name) const {
        const GgufTensor* t = g.tensor(name);
        return t && t->type == GGML_Q8_0;
    }

    // A q8_0 conv tensor as stored (OHWI, ne = [IC, KW, KH, OC], 32-element blocks
    // along IC), split into its int8 values in the packed tap layout of pack_taps,
    // [oc][kw*k + kh][ic] (tap = time tap * k + frequency tap), and its f16 scale bits
    // block-major, [(kw*k + kh) * ic / 32 + block][oc] (the conv's w_scale layout).
    bool conv_q8(const std::string& name, std::vector<int8_t>& q, std::vector<uint16_t>& d,
                 int& oc, int& ic, int& k) {
        const GgufTensor* t = g.tensor(name);
        if (!t || t->type != GGML_Q8_0) {
            err = "tensor '" + name + "' is not q8_0";
            return false;
        }
        std::vector<int64_t> ne = t->ne;
        while (ne.size() < 4) ne.push_back(1);
        ic = (int)ne[0];
        k = (int)ne[1];
        oc = (int)ne[3];
        const int64_t n = t->nelements();
        if (ne[2] != ne[1] || ic % 32 != 0 || (size_t)(n / 32) * 34 > t->nbytes) {
            err = "tensor '" + name + "': q8_0 conv weight must be [IC, K, K, OC], IC % 32 == 0";
            return false;
        }
        q.resize((size_t)n);
        d.resize((size_t)(n / 32));
        const int nbk = ic / 32;  // blocks per (oc, kh, kw)
        for (int o = 0; o < oc; ++o)
            for (int kh = 0; kh < k; ++kh)
                for (int kw = 0; kw < k; ++kw)
                    for (int c = 0; c < nbk; ++c) {
                        const int64_t src = (((int64_t)o * k + kh) * k + kw) * nbk + c;
                        const int64_t kblk = ((int64_t)kw * k + kh) * nbk + c;  // K block
                        const int64_t dst = (int64_t)o * k * k * nbk + kblk;
                        const uint8_t* blk = t->data + src * 34;
                        std::memcpy(&d[(size_t)(kblk * oc + o)], blk, 2);
                        std::memcpy(&q[(size_t)dst * 32], blk + 2, 32);
                    }
        return true;
    }

    // Conv weight as torch-order f32 [OC][IC][K][K]. f32/f16 tensors use the
    // reference's ggml layout ne = [KW, KH, IC, OC] (src/encoder_resnet.cpp:16-20);
    // q8_0 conv tensors (a new format: the reference never quantises 4-D weights)
    // are stored OHWI, ne = [IC, KW, KH, OC], so the 32-element blocks run along IC.
    bool conv(const std::string& name, std::vector<float>& w, int& oc, int& ic, int& k) {
        const GgufTensor* t = g.tensor(name);
        if (!t) {
            err = "missing tensor '" + name + "'";
            return false;
        }
        std::vector<float> raw;
        if (!g.to_f32(*t, raw, err)) return false;
        std::vector<int64_t> ne = t->ne;
        while (ne.size() < 4) ne.push_back(1);
        if (t->type == GGML_Q8_0) {
            ic = (int)ne[0];
            k = (int)ne[1];
            oc = (int)ne[3];
            if (ne[2] != ne[1]) {
                err = "tensor '" + name + "': q8_0 conv weight must be [IC, K, K, OC]";
                return false;
            }
            w.assign((size_t)oc * ic * k * k, 0.0f);
            for (int o = 0; o < oc; ++o)
                for (int kh = 0; kh < k; ++kh)
                    for (int kw = 0; kw < k; ++kw)
                        for (int i = 0; i < ic; ++i)
                            w[(((size_t)o * ic + i) * k + kh) * k + kw] =
                                raw[(((size_t)o * k + kh) * k + kw) * ic + i];
        } else {
            k = (int)ne[0];
            ic = (int)ne[2];
            oc = (int)ne[3];
            if (ne[1] != ne[0]) {
                err = "tensor '" + name + "': conv weight must be square [K, K, IC, OC]";
                return false;
            }
            w = std::move(raw);
        }
        return true;
    }

    bool vec(const std::string& name, std::vector<float>& v, int expect) {
        const GgufTensor* t = g.tensor(name);
        if (!t) {
            err = "missing tensor '" + name + "'";
            return false;
        }
        if (!g.to_f32(*t, v, err)) return false;
        if (expect >= 0 && (int)v.size() != expect) {
            err = "tensor '" + name + "' has " + std::to_string(v.size()) + " elements, expected " +
                  std::to_string(expect);
            return false;
        }
        return true;
    }
};

// torch [OC][IC][K][K] -> [OC][kt*K + kf][IC] with kt = kw (time), kf = kh (freq).
std::vector<float> pack_taps(const std::vector<float>& w, int oc, int ic, int k) {
    std::vector<float> out((size_t)oc * k * k * ic);
    for (int o = 0; o < oc; ++o)
        for (int kh = 0; kh < k; ++kh)
            for (int kw = 0; kw < k; ++kw)
                for (int i = 0; i < ic; ++i)
                    out[((size_t)o * k * k + (size_t)kw * k + kh) * ic + i] =
                        w[(((size_t)o * ic + i) * k + kh) * k + kw];
    return out;
}

// The QPACK weight of a stage-1 conv from its packed taps ([32][9][32], tap kt*3 + kf):
// for time tap kt and input pixel shift u = -1..4, the rows (j, oc) of the output pixel
// phases j with 0 <= u - j + 1 <= 2 (blocks of 32 / 64 / 96 / 96 / 64 / 32 rows, 384
// per kt) hold W[oc][kt*3 + u - j + 1][:] (the layout vdb_qpack_pack_weights writes).
std::vector<float> pack_qpack(const std::vector<float>& taps) {
    std::vector<float> out((size_t)1152 * 32, 0.0f);
    for (int kt = 0; kt < 3; ++kt) {
        int row = kt * 384;
        for (int u = -1; u <= 4; ++u) {
            const int jmin = std::max(0, u - 1), jmax = std::min(3, u + 1);
            for (int j = jmin; j <= jmax; ++j)
                for (int oc = 0; oc < 32; ++oc, ++row)
                    for (int ic = 0; ic < 32; ++ic)
                        out[(size_t)row * 32 + ic] =
                            taps[((size_t)oc * 9 + kt * 3 + (u - j + 1)) * 32 + ic];
        }
    }
    return out;
}

// The same packing of q8_0 weights: rows of 32 int8 values (one q8_0 block) and their
// scales (one per packed row), from the [oc][9][32] tap layout and its block-major
// scales [tap][oc].
void pack_qpack_q8(const std::vector<int8_t>& q, const std::vector<uint16_t>& d,
                   std::vector<int8_t>& pq, std::vector<uint16_t>& pd) {
    pq.assign((size_t)1152 * 32, 0);
    pd.assign(1152, 0);
    for (int kt = 0; kt < 3; ++kt) {
        int row = kt * 384;
        for (int u = -1; u <= 4; ++u) {
            const int jmin = std::max(0, u - 1), jmax = std::min(3, u + 1);
            for (int j = jmin; j <= jmax; ++j)
                for (int oc = 0; oc < 32; ++oc, ++row) {
                    const size_t tap = (size_t)kt * 3 + (u - j + 1);
                    std::memcpy(&pq[(size_t)row * 32], &q[((size_t)oc * 9 + tap) * 32], 32);
                    pd[(size_t)row] = d[tap * 32 + oc];
                }
        }
    }
}

inline int frames_of(int n, int win, int hop) { return n >= win ? 1 + (n - win) / hop : 0; }
inline int half_extent(int n) { return (n - 1) / 2 + 1; }

}  // namespace

Engine::~Engine() {
    if (device_ >= 0) cudaSetDevice(device_);
    if (stream_) cudaStreamSynchronize(stream_);
    clear_graphs();
    free_workspace();
    for (void* p : weight_allocs_) cudaFree(p);
    if (plan_) vdb_fbank_plan_destroy(plan_);
    if (errword_) cudaFree(errword_);
    for (cudaEvent_t& ev : stage_ev_)
        if (ev) cudaEventDestroy(ev);
    for (cudaEvent_t ev : prof_ev_) cudaEventDestroy(ev);
    for (int s = 0; s < 2; ++s) {
        if (h2d_ev_[s]) cudaEventDestroy(h2d_ev_[s]);
        if (comp_ev_[s]) cudaEventDestroy(comp_ev_[s]);
    }
    if (copy_stream_) {
        cudaStreamSynchronize(copy_stream_);
        cudaStreamDestroy(copy_stream_);
    }
    if (stream_) cudaStreamDestroy(stream_);
}

void Engine::free_workspace() {
    for (Level& L : levels_) {
        for (void*& p : L.g) {
            cudaFree(p);
            p = nullptr;
        }
        cudaFree(L.p);
        L.p = nullptr;
        L.g_bytes = L.p_bytes = 0;
    }
    for (EBuf& eb : ebufs_) {
        cudaFree(eb.p);
        eb.p = nullptr;
        eb.bytes = 0;
    }
    cudaFree(feats_);
    feats_ = nullptr;
    feats_bytes_ = 0;
    cudaFree(mean_);
    mean_ = nullptr;
    mean_bytes_ = 0;
    cudaFree(pool_scratch_);
    pool_scratch_ = nullptr;
    pool_scratch_bytes_ = 0;
    cudaFree(ecapa_ws_);
    ecapa_ws_ = nullptr;
    ecapa_ws_bytes_ = 0;
    cudaFree(meta_);
    meta_ = nullptr;
    cudaFree(offs_);
    offs_ = nullptr;
    cudaFree(nsamp_);
    nsamp_ = nullptr;
    meta_cap_ = 0;
    cudaFreeHost(h_stage_);
    h_stage_ = nullptr;
    d_stage_ = nullptr;
    h_stage_bytes_ = 0;
    for (int s = 0; s < 2; ++s) {
        cudaFreeHost(h_ring_[s]);
        cudaFree(d_ring_[s]);
        h_ring_[s] = nullptr;
        d_ring_[s] = nullptr;
        ring_used_[s] = false;
    }
    ring_bytes_ = 0;
    for (int s = 0; s < 2; ++s) {
        cudaFree(d_conv_[s]);
        cudaFreeHost(h_imeta_[s]);
        cudaFree(d_imeta_[s]);
        d_conv_[s] = nullptr;
        h_imeta_[s] = nullptr;
        d_imeta_[s] = nullptr;
    }
    conv_bytes_ = 0;
    imeta_cap_ = 0;
    cudaFreeHost(h_out_);
    h_out_ = nullptr;
    cudaFree(d_out_);
    d_out_ = nullptr;
    out_bytes_ = 0;
}

std::unique_ptr<Engine> Engine::load(const std::string& path, std::string& err) {
    Gguf g;
    if (!g.load(path, err)) return nullptr;
    std::unique_ptr<Engine> e(new Engine());
    EngineConfig& c = e->cfg_;
    // KV schema of src/model_loader.cpp:120-136 (same keys and defaults).
    c.arch = g.str("voicedetect.arch");
    c.emb_dim = (int)g.u32("voicedetect.embedding_dim");
    c.l2 = g.boolean("voicedetect.l2_normalize", true);
    c.sample_rate = (int)g.u32("voicedetect.fbank.sample_rate", 16000);
    c.n_mels = (int)g.u32("voicedetect.fbank.n_mels", 80);
    c.n_fft = (int)g.u32("voicedetect.fbank.n_fft", 512);
    c.win = (int)g.u32("voicedetect.fbank.win_length", 400);
    c.hop = (int)g.u32("voicedetect.fbank.hop_length", 160);
    c.preemph = g.f32("voicedetect.fbank.preemph", 0.97f);
    c.low_freq = g.f32("voicedetect.fbank.low_freq", 20.0f);
    c.high_freq = g.f32("voicedetect.fbank.high_freq", 0.0f);
    c.cmn = g.boolean("voicedetect.fbank.cmn", true);
    if (c.emb_dim <= 0) {  // the reference's load() fails the same way (:213-214)
        err = "GGUF has no voicedetect.embedding_dim";
        return nullptr;
    }
    if (cudaGetDevice(&e->device_) != cudaSuccess) {
        err = "no CUDA device";
        return nullptr;
    }
    if (cudaStreamCreateWithFlags(&e->stream_, cudaStreamNonBlocking) != cudaSuccess ||
        cudaEventCreateWithFlags(&e->stage_ev_[0], cudaEventDisableTiming) != cudaSuccess ||
        cudaEventCreateWithFlags(&e->stage_ev_[1], cudaEventDisableTiming) != cudaSuccess ||
        cudaStreamCreateWithFlags(&e->copy_stream_, cudaStreamNonBlocking) != cudaSuccess ||
        cudaEventCreateWithFlags(&e->h2d_ev_[0], cudaEventDisableTiming) != cudaSuccess ||
        cudaEventCreateWithFlags(&e->h2d_ev_[1], cudaEventDisableTiming) != cudaSuccess ||
        cudaEventCreateWithFlags(&e->comp_ev_[0], cudaEventDisableTiming) != cudaSuccess ||
        cudaEventCreateWithFlags(&e->comp_ev_[1], cudaEventDisableTiming) != cudaSuccess ||
        cudaMalloc(&e->errword_, sizeof(int)) != cudaSuccess ||
        cudaMemset(e->errword_, 0, sizeof(int)) != cudaSuccess) {
        err = "CUDA stream/alloc failed";
        return nullptr;
    }
    // load succeeds for other archs; embed then reports the arch as not implemented
    if (c.arch != "wespeaker_resnet34" && c.arch != "eres2net" && c.arch != "ecapa_tdnn" &&
        c.arch != "campplus")
        return e;

    e->plan_ = vdb_fbank_plan_create(c.sample_rate, c.n_mels, c.n_fft, c.win, c.hop, c.preemph,
                                     c.low_freq, c.high_freq);
    if (!e->plan_) {
        err = vdb_last_error();
        return nullptr;
    }
    if (c.arch == "eres2net") {
        if (!e->load_eres2net(g, err)) return nullptr;
        return e;
    }
    if (c.arch == "ecapa_tdnn") {
        if (!e->load_ecapa(g, err)) return nullptr;
        return e;
    }
    if (c.arch == "campplus") {
        if (!e->load_campplus(g, err) || !e->identity(e->campp_.M, err)) return nullptr;
        return e;
    }
    Loader L{g, err};
    auto upload = [&](const std::vector<float>& v, float** dst) -> bool {
        return e->upload_f32(v, dst, err);
    };
    auto upload_h = [&](const std::vector<float>& v, void** dst) -> bool {
        __half* h = nullptr;
        if (!e->upload_f16(v, &h, err)) return false;
        *dst = h;
        e->conv_weight_bytes += (long long)v.size() * 2;
        return true;
    };
    // q8_0 conv tensors stay q8_0 on the device (int8 values + f16 scales, expanded in
    // the conv kernel's shared memory) unless VDB_Q8_WIDEN=1 asks for f16 weights
    // widened on the host (the same f16 values either way)
    const char* widen = std::getenv("VDB_Q8_WIDEN");
    const bool q8_dev = !(widen && widen[0] == '1');
    auto upload_q8 = [&](const std::vector<int8_t>& q, const std::vector<uint16_t>& d, void** dq,
                         const void** dd) -> bool {
        void* ps = nullptr;
        if (!e->upload_bytes(q.data(), q.size(), dq, err) ||
            !e->upload_bytes(d.data(), d.size() * 2, &ps, err))
            return false;
        *dd = ps;
        e->conv_weight_bytes += (long long)q.size() + (long long)d.size() * 2;
        return true;
    };

    // ResNet manifest, src/model_loader.cpp:138-152.
    const std::string pre = "voicedetect.resnet.";
    const auto c1w = g.str_arr(pre + "conv1_weight"), c1b = g.str_arr(pre + "conv1_bias");
    const auto c2w = g.str_arr(pre + "conv2_weight"), c2b = g.str_arr(pre + "conv2_bias");
    const auto dw = g.str_arr(pre + "down_weight"), db = g.str_arr(pre + "down_bias");
    const auto strides = g.i32_arr(pre + "stride");
    const size_t nb = c1w.size();
    if (nb == 0 || c1b.size() != nb || c2w.size() != nb || c2b.size() != nb ||
        dw.size() != nb || db.size() != nb || strides.size() != nb) {
        err = "inconsistent voicedetect.resnet.* block manifest";
        return nullptr;
    }
    // stem
    {
        std::vector<float> w, b;
        int oc, ic, k;
        if (!L.conv(g.str(pre + "stem_weight"), w, oc, ic, k)) return nullptr;
        if (ic != 1 || k != 3 || !(oc == 16 || oc == 32 || oc == 64)) {
            err = "stem must be a 3x3 conv from 1 channel to 16/32/64";
            return nullptr;
        }
        if (!L.vec(g.str(pre + "stem_bias"), b, oc)) return nullptr;
        std::vector<float> sw((size_t)oc * 9);
        for (int o = 0; o < oc; ++o)
            for (int kh = 0; kh < 3; ++kh)
                for (int kw = 0; kw < 3; ++kw) sw[(size_t)o * 9 + kw * 3 + kh] = w[(size_t)o * 9 + kh * 3 + kw];
        e->stem_oc_ = oc;
        if (!upload(sw, &e->stem_w_) || !upload(b, &e->stem_b_)) return nullptr;
    }
    int cin = e->stem_oc_;
    int F = c.n_mels;
    for (size_t i = 0; i < nb; ++i) {
        ResBlockDev blk;
        blk.stride = strides[i];
        if (blk.stride != 1 && blk.stride != 2) {
            err = "block stride must be 1 or 2";
            return nullptr;
        }
        std::vector<float> w1, w2, b1, b2;
        int oc, ic, k, oc2, ic2, k2;
        if (!L.conv(c1w[i], w1, oc, ic, k) || !L.conv(c2w[i], w2, oc2, ic2, k2)) return nullptr;
        if (k != 3 || k2 != 3 || ic != cin || ic2 != oc || oc2 != oc) {
            err = "block " + std::to_string(i) + ": unexpected conv shapes";
            return nullptr;
        }
        if (!L.vec(c1b[i], b1, oc) || !L.vec(c2b[i], b2, oc)) return nullptr;
        blk.ic = ic;
        blk.oc = oc;
        if (!dw[i].empty()) {
            std::vector<float> wd, bd;
            int ocd, icd, kd;
            if (!L.conv(dw[i], wd, ocd, icd, kd) || !L.vec(db[i], bd, oc)) return nullptr;
            if (kd != 1 || ocd != oc || icd != ic) {
                err = "block " + std::to_string(i) + ": bad downsample shape";
                return nullptr;
            }
            for (int o = 0; o < oc; ++o) b2[o] += bd[o];  // both biases land in one epilogue
            if (q8_dev && L.is_q8(dw[i]) && ic % 32 == 0) {
                std::vector<int8_t> q;
                std::vector<uint16_t> d;
                int o2, i2, k2d;
                if (!L.conv_q8(dw[i], q, d, o2, i2, k2d) || !upload_q8(q, d, &blk.wd, &blk.wds))
                    return nullptr;
            } else if (!upload_h(wd, &blk.wd)) {
                return nullptr;
            }
        } else if (ic != oc || blk.stride != 1) {
            err = "block " + std::to_string(i) + ": identity shortcut needs equal shapes";
            return nullptr;
        } else {
            const __half* eye = e->identity(oc, err);
            if (!eye) return nullptr;
            blk.wd = const_cast<__half*>(eye);  // f16 (wds stays null)
            blk.identity = true;
        }
        if (ic % 16 != 0 || oc % 16 != 0) {
            err = "block channels must be multiples of 16";
            return nullptr;
        }
        const bool qp_blk = ic == 32 && oc == 32 && blk.stride == 1 && blk.identity;
        if (!upload(b1, &blk.b1) || !upload(b2, &blk.b2)) return nullptr;
        if (q8_dev && L.is_q8(c1w[i]) && L.is_q8(c2w[i]) && ic % 32 == 0 && oc % 32 == 0) {
            std::vector<int8_t> q1, q2;
            std::vector<uint16_t> d1, d2;
            int o_, i_, k_;
            if (!L.conv_q8(c1w[i], q1, d1, o_, i_, k_) || !L.conv_q8(c2w[i], q2, d2, o_, i_, k_) ||
                !upload_q8(q1, d1, &blk.w1, &blk.w1s) || !upload_q8(q2, d2, &blk.w2, &blk.w2s))
                return nullptr;
            if (qp_blk) {
                std::vector<int8_t> pq;
                std::vector<uint16_t> pd;
                pack_qpack_q8(q1, d1, pq, pd);
                if (!upload_q8(pq, pd, &blk.w1q, &blk.w1qs)) return nullptr;
                pack_qpack_q8(q2, d2, pq, pd);
                if (!upload_q8(pq, pd, &blk.w2q, &blk.w2qs)) return nullptr;
            }
        } else {
            const std::vector<float> t1 = pack_taps(w1, oc, ic, 3), t2 = pack_taps(w2, oc, oc, 3);
            if (!upload_h(t1, &blk.w1) || !upload_h(t2, &blk.w2)) return nullptr;
            if (qp_blk)
                if (!upload_h(pack_qpack(t1), &blk.w1q) || !upload_h(pack_qpack(t2), &blk.w2q))
                    return nullptr;
        }
        e->blocks_.push_back(blk);
        if (blk.stride == 2) F = half_extent(F);
        cin = oc;
    }
    // scratch for the f16 expansion of streamed q8_0 weights (both segments of the
    // largest block conv)
    for (const ResBlockDev& b : e->blocks_) {
        if (!b.w1s && !b.w2s) continue;
        const long long need = 2LL * b.oc * 9 * std::max(b.ic, b.oc) + 256 + 2LL * b.oc * b.ic + 256;
        e->wscratch_bytes_ = std::max(e->wscratch_bytes_, need);
    }
    if (e->wscratch_bytes_ > 0 &&
        !e->upload_bytes(std::vector<uint8_t>((size_t)e->wscratch_bytes_).data(),
                         (size_t)e->wscratch_bytes_, &e->wscratch_, err))
        return nullptr;
    for (size_t i = 0; i < nb; ++i)
        if (e->blocks_[i].stride == 2 && i == 0) {
            err = "the first block may not be strided";
            return nullptr;
        }
    // embedding head
    {
        std::vector<float> sw, sb, mv;
        const GgufTensor* t = g.tensor(g.str(pre + "seg_weight"));
        if (!t || t->ne.size() < 2) {
            err = "missing or malformed seg_weight";
            return nullptr;
        }
        const int P = (int)t->ne[0], D = (int)t->ne[1];
        if (D != c.emb_dim || P != 2 * cin * F) {
            err = "seg_weight shape does not match the backbone (" + std::to_string(P) + " vs " +
                  std::to_string(2 * cin * F) + ")";
            return nullptr;
        }
        if (!g.to_f32(*t, sw, err)) return nullptr;
        if (!L.vec(g.str(pre + "seg_bias"), sb, D)) return nullptr;
        e->pooled_ = P;
        if (!upload(sw, &e->seg_w_) || !upload(sb, &e->seg_b_)) return nullptr;
        const std::string mvn = g.str(pre + "mean_vec");
        if (!mvn.empty()) {
            if (!L.vec(mvn, mv, D) || !upload(mv, &e->mean_vec_)) return nullptr;
        }
        e->var_eps_ = g.f32(pre + "var_eps", 1e-8f);
    }
    // QPACK stage 1: every block before the first stride-2 one packed (32 -> 32,
    // identity), 32 stem channels, and a stride-2 block after them
    {
        size_t i = 0;
        bool ok = e->stem_oc_ == 32;
        for (; i < e->blocks_.size() && e->blocks_[i].stride == 1; ++i)
            ok = ok && e->blocks_[i].w1q != nullptr;
        e->qpack_ = ok && i > 0 && i < e->blocks_.size();
    }
    // workspace levels: channels of the activation kept at each resolution level
    e->levels_.clear();
    e->levels_.push_back(Level{});
    e->levels_[0].c = e->stem_oc_;
    for (const ResBlockDev& b : e->blocks_) {
        if (b.stride == 2) e->levels_.push_back(Level{});
        e->levels_.back().c = std::max(e->levels_.back().c, b.oc);
    }
    return e;
}

const __half* Engine::identity(int c, std::string& err) {
    for (const auto& id : identities_)
        if (id.first == c) return id.second;
    std::vector<float> eye((size_t)c * c, 0.0f);
    for (int i = 0; i < c; ++i) eye[(size_t)i * c + i] = 1.0f;
    __half* p = nullptr;
    if (!upload_f16(eye, &p, err)) return nullptr;
    identities_.emplace_back(c, p);
    return p;
}

bool Engine::upload_f32(const std::vector<float>& v, float** dst, std::string& err) {
    void* p = nullptr;
    if (cudaMalloc(&p, v.size() * sizeof(float)) != cudaSuccess ||
        cudaMemcpy(p, v.data(), v.size() * sizeof(float), cudaMemcpyHostToDevice) != cudaSuccess) {
        if (p) cudaFree(p);
        err = "weight upload failed";
        return false;
    }
    weight_allocs_.push_back(p);
    *dst = static_cast<float*>(p);
    return true;
}

bool Engine::upload_f16(const std::vector<float>& v, __half** dst, std::string& err) {
    float* tmp = nullptr;
    if (cudaMalloc(&tmp, v.size() * sizeof(float)) != cudaSuccess) {
        err = "weight upload failed";
        return false;
    }
    void* p = nullptr;
    bool ok = cudaMalloc(&p, v.size() * sizeof(__half)) == cudaSuccess &&
              cudaMemcpy(tmp, v.data(), v.size() * sizeof(float), cudaMemcpyHostToDevice) ==
                  cudaSuccess;
    if (ok) {
        const long long n = (long long)v.size();
        f32_to_f16_kernel<<<(unsigned)((n + 255) / 256), 256>>>(tmp, (__half*)p, n);
        ok = cudaDeviceSynchronize() == cudaSuccess;
    }
    cudaFree(tmp);
    if (!ok) {
        err = "weight conversion failed";
        if (p) cudaFree(p);
        return false;
    }
    weight_allocs_.push_back(p);
    *dst = static_cast<__half*>(p);
    return true;
}

bool Engine::upload_bytes(const void* src, size_t n, void** dst, std::string& err) {
    void* p = nullptr;
    if (cudaMalloc(&p, n) != cudaSuccess ||
        cudaMemcpy(p, src, n, cudaMemcpyHostToDevice) != cudaSuccess) {
        err = "weight upload failed";
        if (p) cudaFree(p);
        return false;
    }
    weight_allocs_.push_back(p);
    *dst = p;
    return true;
}

// ERes2Net manifest (src/model_loader.cpp:153-165) compiled into a step plan by
// replaying the reference forward with a running conv index:
//   stem 3x3 + ReLU                                   (encoder_eres2net.cpp:196)
//   layer1..4 of Res2Net blocks                       (:111-145, :200-218)
//   cross-stage downsample + AFF after layers 2, 3, 4 (:206-218)
// Layouts: a tensor read by a stride-2 conv is written in the PHASE layout (the
// last block of layers 1-3 and the fused features f12 / f123); o2 and o3 are read
// both ways and get both (y + y2). AFF's channel concat becomes the two input
// segments of the local_att conv1 (x with W[:, :C], ds with W[:, C:]); the
// Res2Net split / concat are channel offsets into the conv1 and accumulator
// buffers.
bool Engine::load_eres2net(const Gguf& g, std::string& err) {
    const std::string pre = "voicedetect.eres2net.";
    const auto wn = g.str_arr(pre + "conv_weight"), bn = g.str_arr(pre + "conv_bias");
    const auto sn = g.i32_arr(pre + "conv_stride"), nb = g.i32_arr(pre + "num_blocks");
    const int M = (int)g.u32(pre + "m_channels");
    const int S = (int)g.u32(pre + "scale", 2);
    const float hi = g.f32(pre + "relu_clamp", 20.0f);
    var_eps_ = g.f32(pre + "var_eps", 1e-8f);
    if (wn.empty() || bn.size() != wn.size() || sn.size() != wn.size() || nb.size() != 4 ||
        M <= 0 || S < 1) {
        err = "inconsistent voicedetect.eres2net.* manifest";
        return false;
    }
    for (int v : nb)
        if (v < 1) {
            err = "eres2net: every layer needs at least one block";
            return false;
        }
    Loader L{g, err};
    struct MC {
        std::vector<float> w, b;
        int oc = 0, ic = 0, k = 0;
    };
    size_t idx = 0;
    auto take = [&](MC& m, int k, int ic, int stride) -> bool {
        if (idx >= wn.size()) {
            err = "eres2net manifest has fewer convs than the topology needs";
            return false;
        }
        const size_t i = idx++;
        if (!L.conv(wn[i], m.w, m.oc, m.ic, m.k)) return false;
        if (m.k != k || m.ic != ic || sn[i] != stride) {
            err = "eres2net conv " + std::to_string(i) + " ('" + wn[i] + "'): expected " +
                  std::to_string(k) + "x" + std::to_string(k) + " stride " +
                  std::to_string(stride) + " from " + std::to_string(ic) + " channels, got " +
                  std::to_string(m.k) + "x" + std::to_string(m.k) + " stride " +
                  std::to_string(sn[i]) + " from " + std::to_string(m.ic);
            return false;
        }
        if (ic > 1) {  // every conv but the IC = 1 stem runs on the tensor-core kernel
            if (m.oc % 16 || m.ic % 16) {
                err = "eres2net conv " + std::to_string(i) + ": channels must be multiples of 16";
                return false;
            }
        }
        m.b.clear();
        if (!bn[i].empty() && !L.vec(bn[i], m.b, m.oc)) return false;
        return true;
    };
    auto dev_w = [&](const MC& m, const __half** out) -> bool {
        __half* p = nullptr;
        if (!upload_f16(pack_taps(m.w, m.oc, m.ic, m.k), &p, err)) return false;
        *out = p;
        return true;
    };
    // bias of one conv, or the sum of two (both segments land in one epilogue)
    auto dev_b = [&](const std::vector<float>& b0, const std::vector<float>& b1, int oc,
                     const float** out) -> bool {
        *out = nullptr;
        if (b0.empty() && b1.empty()) return true;
        std::vector<float> s((size_t)oc, 0.0f);
        for (size_t i = 0; i < b0.size(); ++i) s[i] += b0[i];
        for (size_t i = 0; i < b1.size(); ++i) s[i] += b1[i];
        float* p = nullptr;
        if (!upload_f32(s, &p, err)) return false;
        *out = p;
        return true;
    };
    enum Role { R_STEM, R_XA, R_XB, R_A, R_ACC, R_TM, R_Z, R_POUT, R_PF, R_GD, R_GF };
    std::vector<std::pair<int, int>> keys;  // (level, role) of each buffer
    auto buf = [&](int level, int role, int c, bool phase) -> int {
        for (size_t i = 0; i < keys.size(); ++i)
            if (keys[i].first == level && keys[i].second == role) {
                ebufs_[i].c = std::max(ebufs_[i].c, c);
                return (int)i;
            }
        EBuf b;
        b.level = level;
        b.c = c;
        b.phase = phase;
        ebufs_.push_back(b);
        keys.emplace_back(level, role);
        return (int)ebufs_.size() - 1;
    };
    auto conv_step = [&](int level, int oc, int k0, int stride0, int ic0, EOperand x0,
                         const __half* w0) {
        EStep st;
        st.kind = 0;
        st.level = level;
        st.oc = oc;
        st.k0 = k0;
        st.stride0 = stride0;
        st.ic0 = ic0;
        st.x0 = x0;
        st.w0 = w0;
        st.flops_px = 2.0 * oc * ic0 * k0 * k0;
        return st;
    };

    // stem: 3x3, 1 -> M, bias + plain ReLU
    {
        MC st;
        if (!take(st, 3, 1, 1)) return false;
        if (st.oc != M || !(M == 16 || M == 32 || M == 64)) {
            err = "eres2net stem must be a 3x3 conv from 1 channel to m_channels (16/32/64)";
            return false;
        }
        if (st.b.empty()) st.b.assign((size_t)M, 0.0f);
        std::vector<float> sw((size_t)M * 9);
        for (int o = 0; o < M; ++o)
            for (int kh = 0; kh < 3; ++kh)
                for (int kw = 0; kw < 3; ++kw)
                    sw[(size_t)o * 9 + kw * 3 + kh] = st.w[(size_t)o * 9 + kh * 3 + kw];
        stem_oc_ = M;
        if (!upload_f32(sw, &stem_w_, err) || !upload_f32(st.b, &stem_b_, err)) return false;
        e_stem_buf_ = buf(0, R_STEM, M, false);
    }

    // AFF(x, ds) over C channels at `level` -> out (src/encoder_eres2net.cpp:91-101)
    auto emit_aff = [&](int level, EOperand x, EOperand ds, int C, EOperand out,
                        bool out_phase) -> bool {
        MC la1, la2;
        if (!take(la1, 1, 2 * C, 1)) return false;
        const int Cq = la1.oc;
        if (!take(la2, 1, Cq, 1)) return false;
        if (la2.oc != C) {
            err = "eres2net AFF: local_att conv2 must map back to " + std::to_string(C);
            return false;
        }
        std::vector<float> wa((size_t)Cq * C), wb((size_t)Cq * C);
        for (int o = 0; o < Cq; ++o)
            for (int i = 0; i < C; ++i) {
                wa[(size_t)o * C + i] = la1.w[(size_t)o * 2 * C + i];
                wb[(size_t)o * C + i] = la1.w[(size_t)o * 2 * C + C + i];
            }
        const int z = buf(level, R_Z, Cq, false);
        __half *pa = nullptr, *pb = nullptr;
        if (!upload_f16(wa, &pa, err) || !upload_f16(wb, &pb, err)) return false;
        EStep s1 = conv_step(level, Cq, 1, 1, C, x, pa);
        s1.ic1 = C;
        s1.x1 = ds;
        s1.stride1 = 1;
        s1.w1 = pb;
        s1.flops_px = 2.0 * Cq * 2 * C;
        s1.act = 1;  // SiLU
        s1.y = EOperand{z, 0};
        if (!dev_b(la1.b, {}, Cq, &s1.bias)) return false;
        esteps_.push_back(s1);
        const __half* w2 = nullptr;
        if (!dev_w(la2, &w2)) return false;
        EStep s2 = conv_step(level, C, 1, 1, Cq, EOperand{z, 0}, w2);
        if (!dev_b(la2.b, {}, C, &s2.bias)) return false;
        s2.act = 2;  // (x + ds) + tanh(.) * (x - ds)
        s2.res = x;
        s2.res2 = ds;
        s2.y = out;
        s2.y_phase = out_phase ? 1 : 0;
        esteps_.push_back(s2);
        return true;
    };

    int in_planes = M;
    // Res2Net block (src/encoder_eres2net.cpp:111-137). x: G (stride 1) or P (stride 2)
    // at level lo - (s == 2); outputs: yg (G, may be absent) and / or yp (P).
    auto emit_block = [&](EOperand x, int s, int lo, int planes, bool is_aff, EOperand yg,
                          EOperand yp) -> bool {
        MC c1;
        if (!take(c1, 1, in_planes, s)) return false;
        if (c1.oc % S || (c1.oc / S) % 16) {
            err = "eres2net: conv1 width must split into scale chunks of a multiple of 16";
            return false;
        }
        const int w = c1.oc / S;
        const int A = buf(lo, R_A, c1.oc, false), Acc = buf(lo, R_ACC, c1.oc, false);
        const int Tm = buf(lo, R_TM, w, false);
        const __half* pw = nullptr;
        if (!dev_w(c1, &pw)) return false;
        EStep st = conv_step(lo, c1.oc, 1, s, in_planes, x, pw);
        if (!dev_b(c1.b, {}, c1.oc, &st.bias)) return false;
        st.relu = 1;
        st.clamp_hi = hi;
        st.y = EOperand{A, 0};
        esteps_.push_back(st);
        for (int i = 0; i < S; ++i) {
            const EOperand chunk{A, i * w};
            EOperand cur = chunk;
            if (i > 0) {
                const EOperand sp{Acc, (i - 1) * w};
                if (is_aff) {
                    if (!emit_aff(lo, sp, chunk, w, EOperand{Tm, 0}, false)) return false;
                } else {
                    // A separate element-wise add: folding it into the previous chunk
                    // conv's epilogue (the conv's ysum output) measured slower, since
                    // the epilogue, not memory, bounds these convs.
                    EStep ad;
                    ad.kind = 1;
                    ad.level = lo;
                    ad.oc = w;
                    ad.x0 = sp;
                    ad.x1 = chunk;
                    ad.y = EOperand{Tm, 0};
                    esteps_.push_back(ad);
                }
                cur = EOperand{Tm, 0};
            }
            MC cv;
            if (!take(cv, 3, w, 1)) return false;
            if (cv.oc != w) {
                err = "eres2net: chunk conv must keep the width";
                return false;
            }
            if (!dev_w(cv, &pw)) return false;
            EStep sc = conv_step(lo, w, 3, 1, w, cur, pw);
            if (!dev_b(cv.b, {}, w, &sc.bias)) return false;
            sc.relu = 1;
            sc.clamp_hi = hi;
            sc.y = EOperand{Acc, i * w};
            esteps_.push_back(sc);
        }
        MC c3;
        if (!take(c3, 1, c1.oc, 1)) return false;
        if (c3.oc != 2 * planes) {
            err = "eres2net: conv3 must produce 2 * planes channels";
            return false;
        }
        if (!dev_w(c3, &pw)) return false;
        EStep s3 = conv_step(lo, c3.oc, 1, 1, c1.oc, EOperand{Acc, 0}, pw);
        std::vector<float> sb;
        if (s != 1 || in_planes != 2 * planes) {  // 1x1 shortcut, fused as input segment 1
            MC sh;
            if (!take(sh, 1, in_planes, s)) return false;
            if (sh.oc != 2 * planes) {
                err = "eres2net: shortcut must produce 2 * planes channels";
                return false;
            }
            __half* p1 = nullptr;
            if (!upload_f16(sh.w, &p1, err)) return false;
            s3.x1 = x;
            s3.ic1 = in_planes;
            s3.stride1 = s;
            s3.w1 = p1;
            s3.flops_px += 2.0 * c3.oc * in_planes;
            sb = sh.b;
        } else {  // identity shortcut on the tensor cores (exact; see identity())
            const __half* eye = identity(in_planes, err);
            if (!eye) return false;
            s3.x1 = x;
            s3.ic1 = in_planes;
            s3.stride1 = 1;
            s3.w1 = eye;
        }
        if (!dev_b(c3.b, sb, c3.oc, &s3.bias)) return false;
        s3.relu = 1;
        s3.clamp_hi = hi;
        if (yg.buf >= 0) {
            s3.y = yg;
            s3.y2 = yp;
        } else {
            s3.y = yp;
            s3.y_phase = 1;
        }
        esteps_.push_back(s3);
        in_planes = 2 * planes;
        return true;
    };

    // body (src/encoder_eres2net.cpp:200-218)
    EOperand x{e_stem_buf_, 0};
    EOperand lay_g[4], lay_p[4], fused_p;
    int lev = 0;
    for (int l = 0; l < 4; ++l) {
        const int planes = M << l;
        if (l > 0) x = lay_p[l - 1];
        for (int b = 0; b < nb[l]; ++b) {
            const int s = (b == 0 && l > 0) ? 2 : 1;
            const int lo = lev + (s == 2 ? 1 : 0);
            const bool last = b == nb[l] - 1;
            EOperand yg, yp;
            if (!last || l > 0) {
                // ping-pong: never the buffer holding x
                const int ra = buf(lo, R_XA, 2 * planes, false);
                const int rb = buf(lo, R_XB, 2 * planes, false);
                yg = EOperand{x.buf == ra ? rb : ra, 0};
            }
            if (last && l < 3) yp = EOperand{buf(lo, R_POUT, 2 * planes, true), 0};
            if (!emit_block(x, s, lo, planes, l >= 2, yg, yp)) return false;
            x = yg;
            lev = lo;
        }
        lay_p[l] = (l < 3) ? EOperand{buf(lev, R_POUT, 2 * planes, true), 0} : EOperand{};
        lay_g[l] = x;
        if (l >= 1) {
            // previous-scale feature: o1 (P) for layer 2, then the fused f12 / f123 (P)
            const EOperand src = (l == 1) ? lay_p[0] : fused_p;
            MC d;
            if (!take(d, 3, planes, 2)) return false;
            if (d.oc != 2 * planes) {
                err = "eres2net: cross-stage downsample must produce 2 * planes channels";
                return false;
            }
            const __half* pd = nullptr;
            if (!dev_w(d, &pd)) return false;
            const int gd = buf(lev, R_GD, 2 * planes, false);
            EStep sd = conv_step(lev, d.oc, 3, 2, planes, src, pd);
            if (!dev_b(d.b, {}, d.oc, &sd.bias)) return false;
            sd.y = EOperand{gd, 0};
            esteps_.push_back(sd);
            const bool final_stage = (l == 3);
            const EOperand out = final_stage ? EOperand{buf(lev, R_GF, 2 * planes, false), 0}
                                             : EOperand{buf(lev, R_PF, 2 * planes, true), 0};
            if (!emit_aff(lev, lay_g[l], EOperand{gd, 0}, 2 * planes, out, !final_stage))
                return false;
            fused_p = out;
            if (final_stage) {
                e_out_buf_ = out.buf;
                e_out_level_ = lev;
            }
        }
    }
    if (idx != wn.size()) {
        err = "eres2net manifest has " + std::to_string(wn.size()) + " convs, the topology uses " +
              std::to_string(idx);
        return false;
    }
    // embedding head (src/encoder_eres2net.cpp:228-250)
    int F = cfg_.n_mels;
    for (int l = 0; l < e_out_level_; ++l) F = half_extent(F);
    const int cl = ebufs_[e_out_buf_].c;
    const GgufTensor* t = g.tensor(g.str(pre + "seg_weight"));
    if (!t || t->ne.size() < 2) {
        err = "missing or malformed eres2net seg_weight";
        return false;
    }
    const int P = (int)t->ne[0], D = (int)t->ne[1];
    if (D != cfg_.emb_dim || P != 2 * cl * F) {
        err = "eres2net seg_weight shape does not match the backbone (" + std::to_string(P) +
              " vs " + std::to_string(2 * cl * F) + ")";
        return false;
    }
    std::vector<float> sw, sb;
    if (!g.to_f32(*t, sw, err)) return false;
    if (!L.vec(g.str(pre + "seg_bias"), sb, D)) return false;
    pooled_ = P;
    if (!upload_f32(sw, &seg_w_, err) || !upload_f32(sb, &seg_b_, err)) return false;
    // metadata levels (valid lengths per resolution); activations live in ebufs_
    levels_.assign((size_t)e_out_level_ + 1, Level{});
    return true;
}

bool Engine::supported(std::string& err) const {
    if (cfg_.arch != "wespeaker_resnet34" && cfg_.arch != "eres2net" &&
        cfg_.arch != "ecapa_tdnn" && cfg_.arch != "campplus") {
        err = "voicedetect: arch '" + cfg_.arch + "' is not implemented by the B200 engine";
        return false;
    }
    return true;
}

int Engine::ensure_workspace(int B, int t_max, std::string& err) {
    auto grow = [&](void** p, size_t& have, size_t need) -> bool {
        if (need <= have) return true;
        cudaDeviceSynchronize();  // the old buffer may still be read by queued work
        clear_graphs();           // captured launches point at the old buffers
        cudaFree(*p);
        *p = nullptr;
        have = 0;
        if (cudaMalloc(p, need) != cudaSuccess) {
            err = "device out of memory (workspace)";
            return false;
        }
        have = need;
        return true;
    };
    int T = t_max, F = cfg_.n_mels;
    for (size_t li = 0; li < levels_.size(); ++li) {
        Level& L = levels_[li];
        size_t g = (size_t)vdb_grid_rows(B, T, F) * L.c * sizeof(__half);
        if (li == 0 && qpack_)  // QPACK rows of 4 pixels x 32 channels
            g = std::max(g, (size_t)vdb_qpack_rows(B, T, F) * 128 * sizeof(__half));
        size_t have = L.g_bytes;
        for (int k = 0; k < 3; ++k) {
            size_t h = have;
            if (!grow(&L.g[k], h, g)) return 1;
        }
        L.g_bytes = std::max(L.g_bytes, g);
        if (li + 1 < levels_.size()) {
            const size_t pb = (size_t)vdb_phase_rows(B, T, F) * L.c * sizeof(__half);
            if (!grow(&L.p, L.p_bytes, pb)) return 1;
        }
        T = half_extent(T);
        F = half_extent(F);
    }
    std::vector<int> lt(1, t_max), lf(1, cfg_.n_mels);
    for (size_t l = 1; l < std::max<size_t>(levels_.size(), 1); ++l) {
        lt.push_back(half_extent(lt.back()));
        lf.push_back(half_extent(lf.back()));
    }
    for (EBuf& eb : ebufs_) {
        const long long rows = eb.phase ? vdb_phase_rows(B, lt[eb.level], lf[eb.level])
                                        : vdb_grid_rows(B, lt[eb.level], lf[eb.level]);
        if (!grow(&eb.p, eb.bytes, (size_t)rows * eb.c * sizeof(__half))) return 1;
    }
    if (!grow((void**)&feats_, feats_bytes_, (size_t)B * t_max * cfg_.n_mels * sizeof(float)))
        return 1;
    if (!grow((void**)&mean_, mean_bytes_, (size_t)B * cfg_.n_mels * sizeof(float))) return 1;
    if (cfg_.arch == "ecapa_tdnn") {
        if (!grow(&ecapa_ws_, ecapa_ws_bytes_, ecapa_ws_bytes(B, t_max))) return 1;
    } else if (cfg_.arch == "campplus") {
        if (!grow(&ecapa_ws_, ecapa_ws_bytes_, campp_ws_bytes(B, t_max))) return 1;
    } else {
        // pooling input: the last level's frequency extent and channels
        const int lev = cfg_.arch == "eres2net" ? e_out_level_ : (int)levels_.size() - 1;
        const int pc = cfg_.arch == "eres2net" ? ebufs_[e_out_buf_].c : levels_.back().c;
        const size_t n = pool_embed_scratch_floats(B, lf[lev], pc, cfg_.emb_dim);
        if (!grow((void**)&pool_scratch_, pool_scratch_bytes_, n * sizeof(float))) return 1;
    }
    if (B > meta_cap_) {
        cudaDeviceSynchronize();
        clear_graphs();
        stage_used_[0] = stage_used_[1] = false;
        cudaFree(meta_);
        cudaFree(offs_);
        cudaFree(nsamp_);
        cudaFreeHost(h_stage_);
        meta_ = nullptr;
        offs_ = nullptr;
        nsamp_ = nullptr;
        h_stage_ = nullptr;
        d_stage_ = nullptr;
        const int cap = std::max(B, 64);
        const size_t nlev = levels_.size();
        // two staging slots so the host can fill bucket k+1 while bucket k copies; a
        // slot's size is a multiple of 256 bytes so that both slots, and the int64
        // offsets inside each, are 8-byte aligned for the staging kernel's loads
        h_stage_bytes_ =
            ((size_t)cap * (sizeof(long long) + sizeof(int) * (nlev + 3)) + 64 + 255) & ~(size_t)255;
        if (cudaMalloc(&meta_, sizeof(int) * cap * (nlev + 2)) != cudaSuccess ||
            cudaMalloc(&offs_, sizeof(long long) * cap) != cudaSuccess ||
            cudaMalloc(&nsamp_, sizeof(int) * cap) != cudaSuccess ||
            cudaHostAlloc(&h_stage_, 2 * h_stage_bytes_, cudaHostAllocMapped) != cudaSuccess ||
            cudaHostGetDevicePointer(&d_stage_, h_stage_, 0) != cudaSuccess) {
            err = "device out of memory (metadata)";
            return 1;
        }
        meta_cap_ = cap;
    }
    return 0;
}

// One bucket of B clips: h_off/h_ns are device-pointer offsets and sample counts,
// h_outrow the output row of each clip.
int Engine::run_bucket(const float* d_pcm, const long long* h_off, const int* h_ns,
                       const int* h_outrow, int B, cudaStream_t st, float* d_out,
                       std::string& err) {
    const size_t nlev = levels_.size();
    int t_max = 0;
    for (int b = 0; b < B; ++b) t_max = std::max(t_max, frames_of(h_ns[b], cfg_.win, cfg_.hop));
    if (cfg_.arch == "ecapa_tdnn") {
        // reflect padding needs more frames than the widest conv reaches on either side
        // (torch's reflect pad has the same precondition; the reference's index list
        // would read outside the clip, src/encoder.cpp:36-44)
        for (int b = 0; b < B; ++b)
            if (frames_of(h_ns[b], cfg_.win, cfg_.hop) < ecapa_.pad + 1) {
                err = "voicedetect: ECAPA-TDNN needs at least " + std::to_string(ecapa_.pad + 1) +
                      " FBank frames per clip (" +
                      std::to_string(cfg_.win + ecapa_.pad * cfg_.hop) + " samples at 16 kHz)";
                return 1;
            }
    }
    if (ensure_workspace(B, t_max, err)) return 1;
    // Per-bucket metadata: [tvalid level 0..nlev-1][B], [outrow][B], then offsets, nsamp.
    // A staging slot is only rewritten after the kernel that last read it finished.
    const int slot = stage_slot_;
    stage_slot_ ^= 1;
    if (stage_used_[slot]) VDB_CHECK_CUDA(cudaEventSynchronize(stage_ev_[slot]));
    int* hm = reinterpret_cast<int*>(static_cast<char*>(h_stage_) + slot * h_stage_bytes_);
    std::vector<long long> tv_sum(nlev, 0);
    for (int b = 0; b < B; ++b) {
        int tv = frames_of(h_ns[b], cfg_.win, cfg_.hop);
        for (size_t l = 0; l < nlev; ++l) {
            hm[l * B + b] = tv;
            tv_sum[l] += tv;
            tv = half_extent(tv);
        }
        hm[nlev * B + b] = h_outrow[b];
    }
    long long* ho = reinterpret_cast<long long*>(hm + (nlev + 1) * B + ((nlev + 1) * B) % 2);
    int* hn = reinterpret_cast<int*>(ho + B);
    std::memcpy(ho, h_off, sizeof(long long) * B);
    std::memcpy(hn, h_ns, sizeof(int) * B);
    {
        // the same slot through its mapped device address
        const ptrdiff_t d = static_cast<char*>(d_stage_) - static_cast<char*>(h_stage_);
        const int n_meta = (int)((nlev + 1) * B);
        stage_meta_kernel<<<(n_meta + B + 255) / 256, 256, 0, st>>>(
            reinterpret_cast<const int*>(reinterpret_cast<const char*>(hm) + d), n_meta,
            reinterpret_cast<const long long*>(reinterpret_cast<const char*>(ho) + d),
            reinterpret_cast<const int*>(reinterpret_cast<const char*>(hn) + d), B, meta_, offs_,
            nsamp_);
        VDB_CHECK_CUDA(cudaGetLastError());
        ++last_launches;
    }
    VDB_CHECK_CUDA(cudaEventRecord(stage_ev_[slot], st));
    stage_used_[slot] = true;
    long long launches = 0;
    if (!graphs_enabled_ || profiling_) {
        if (launch_bucket(d_pcm, B, t_max, tv_sum, st, d_out, launches, err)) return 1;
        last_launches += launches;
        return 0;
    }
    GraphEntry* ge = nullptr;
    for (GraphEntry& g : graphs_)
        if (g.B == B && g.t_max == t_max && g.d_pcm == d_pcm && g.d_out == d_out && g.st == st)
            ge = &g;
    if (!ge) {
        graphs_.push_back(GraphEntry{B, t_max, d_pcm, d_out, st, 0, nullptr, 0});
        ge = &graphs_.back();
    }
    if (!ge->exec && ge->seen++ == 0) {
        // first sight: plain launches (they also set every kernel attribute)
        if (launch_bucket(d_pcm, B, t_max, tv_sum, st, d_out, launches, err)) return 1;
        last_launches += launches;
        return 0;
    }
    if (!ge->exec) {
        cudaGraph_t graph = nullptr;
        long long n = 0;
        int rc = 1;
        if (cudaStreamBeginCapture(st, cudaStreamCaptureModeThreadLocal) == cudaSuccess) {
            rc = launch_bucket(d_pcm, B, t_max, tv_sum, st, d_out, n, err);
            const cudaError_t ce = cudaStreamEndCapture(st, &graph);
            if (ce != cudaSuccess) rc = rc ? rc : 2;
        }
        cudaGraphExec_t exec = nullptr;
        if (rc == 0 && cudaGraphInstantiate(&exec, graph, 0) != cudaSuccess) rc = 2;
        if (graph) cudaGraphDestroy(graph);
        if (rc != 0) {
            // capture not possible here: run plainly from now on
            cudaGetLastError();
            graphs_enabled_ = false;
            clear_graphs();
            if (launch_bucket(d_pcm, B, t_max, tv_sum, st, d_out, launches, err)) return 1;
            last_launches += launches;
            return 0;
        }
        ge->exec = exec;
        ge->launches = n;
    }
    VDB_CHECK_CUDA(cudaGraphLaunch(ge->exec, st));
    last_launches += ge->launches;
    return 0;
}

int Engine::release_cache(std::string& err) {
    if (cudaStreamSynchronize(stream_) != cudaSuccess || cudaDeviceSynchronize() != cudaSuccess) {
        err = std::string("CUDA error: ") + cudaGetErrorString(cudaGetLastError());
        return 1;
    }
    clear_graphs();
    free_workspace();
    return 0;
}

void Engine::clear_graphs() {
    for (GraphEntry& g : graphs_)
        if (g.exec) cudaGraphExecDestroy(g.exec);
    graphs_.clear();
}

int Engine::launch_bucket(const float* d_pcm, int B, int t_max,
                          const std::vector<long long>& tv_sum, cudaStream_t st, float* d_out,
                          long long& launches, std::string& err) {
    const size_t nlev = levels_.size();
    // FBank -> CMN + stem
    const int pf = prof_begin(st, 1);
    if (vdb_fbank(plan_, d_pcm, offs_, nsamp_, B, t_max, feats_, st)) {
        err = vdb_last_error();
        return 1;
    }
    prof_end(pf, st, 0.0);
    if (cfg_.arch == "ecapa_tdnn") return run_ecapa(B, t_max, tv_sum, st, d_out, launches, err);
    if (cfg_.arch == "campplus") return run_campplus(B, t_max, tv_sum, st, d_out, launches, err);
    const int ps = prof_begin(st, 4);
    const bool eres = cfg_.arch == "eres2net";
    if (cmn_stem_launch(feats_, meta_, B, t_max, cfg_.n_mels, cfg_.cmn ? 1 : 0, stem_w_, stem_b_,
                        stem_oc_, mean_, eres ? ebufs_[e_stem_buf_].p : levels_[0].g[0],
                        (!eres && qpack_) ? 2 : 0, st)) {
        err = vdb_last_error();
        return 1;
    }
    prof_end(ps, st, 0.0);
    launches += cfg_.cmn ? 3 : 2;
    if (eres) return run_eres2net(B, t_max, tv_sum, st, d_out, launches, err);
    // Backbone.
    int lev = 0, T = t_max, F = cfg_.n_mels;
    int cur = 0;            // index of the G buffer holding the block input
    bool cur_phase = false;  // block input is the level's PHASE buffer
    for (size_t i = 0; i < blocks_.size(); ++i) {
        const ResBlockDev& blk = blocks_[i];
        const bool next_s2 = (i + 1 < blocks_.size()) && blocks_[i + 1].stride == 2;
        Level& Lin = levels_[lev];
        const void* x = cur_phase ? Lin.p : Lin.g[cur];
        int To = T, Fo = F, lev_out = lev;
        if (blk.stride == 2) {
            To = half_extent(T);
            Fo = half_extent(F);
            lev_out = lev + 1;
        }
        Level& Lo = levels_[lev_out];
        const int* tv_out = meta_ + (size_t)lev_out * B;
        const int h_slot = (lev_out == lev) ? (cur + 1) % 3 : 0;
        const int o_slot = (lev_out == lev) ? (cur + 2) % 3 : 1;
        // stage-1 blocks over QPACK rows (lev 0, identity shortcut as the epilogue residual)
        const bool qp = qpack_ && lev == 0 && blk.stride == 1;
        vdb_conv_args a{};
        a.batch = B;
        a.t_out = To;
        a.f_out = Fo;
        a.oc = blk.oc;
        a.k0 = 3;
        a.stride0 = blk.stride;
        a.ic0 = blk.ic;
        a.x0 = x;
        a.w0 = qp ? blk.w1q : blk.w1;
        a.w0_scale = qp ? blk.w1qs : blk.w1s;
        a.w_scratch = wscratch_;
        a.w_scratch_bytes = wscratch_bytes_;
        a.bias = blk.b1;
        a.relu = 1;
        a.tvalid = tv_out;
        a.y = Lo.g[h_slot];
        a.err = errword_;
        a.qpack = qp ? 1 : 0;
        // algorithmic FLOPs over valid output frames only (padding excluded)
        const double valid_px = (double)Fo * (double)tv_sum[lev_out];
        int pe = prof_begin(st);
        if (vdb_conv(&a, st)) {
            err = vdb_last_error();
            return 1;
        }
        launches += last_conv_launches();
        prof_end(pe, st, 2.0 * blk.oc * blk.ic * 9 * valid_px, &a);
        vdb_conv_args c2{};
        c2.batch = B;
        c2.t_out = To;
        c2.f_out = Fo;
        c2.oc = blk.oc;
        c2.k0 = 3;
        c2.stride0 = 1;
        c2.ic0 = blk.oc;
        c2.x0 = Lo.g[h_slot];
        c2.w0 = qp ? blk.w2q : blk.w2;
        c2.w0_scale = qp ? blk.w2qs : blk.w2s;
        c2.w_scratch = wscratch_;
        c2.w_scratch_bytes = wscratch_bytes_;
        c2.bias = blk.b2;
        c2.relu = 1;
        c2.tvalid = tv_out;
        c2.err = errword_;
        if (qp) {
            // QPACK: the identity shortcut is the epilogue residual (the block input's
            // QPACK row is contiguous with the output row)
            c2.qpack = 1;
            c2.residual = x;
        } else if (blk.identity && blk.oc >= 128) {
            // identity shortcut of a 128 / 256-channel block as the epilogue residual:
            // 3.5-4.7 % faster than the identity MMA segment at batch 512 (at 64
            // channels the segment is the faster one)
            c2.residual = x;
        } else {
            // 1x1 downsample, or the identity shortcut, as input segment 1
            c2.x1 = x;
            c2.w1 = blk.wd;
            c2.w1_scale = blk.wds;
            c2.ic1 = blk.ic;
            c2.stride1 = blk.stride;
        }
        c2.y_phase = next_s2 ? 1 : 0;
        c2.y = next_s2 ? Lo.p : Lo.g[o_slot];
        pe = prof_begin(st);
        if (vdb_conv(&c2, st)) {
            err = vdb_last_error();
            return 1;
        }
        launches += last_conv_launches();
        prof_end(pe, st,
                 2.0 * blk.oc * blk.oc * 9 * valid_px +
                     (blk.identity ? 0.0 : 2.0 * blk.oc * blk.ic * valid_px),
                 &c2);
        lev = lev_out;
        T = To;
        F = Fo;
        cur = o_slot;
        cur_phase = next_s2;
    }
    const Level& Lf = levels_[lev];
    const int pp = prof_begin(st, 2);
    if (pool_embed_launch(Lf.g[cur], meta_ + (size_t)lev * B, B, T, F, Lf.c, seg_w_, seg_b_,
                          mean_vec_, cfg_.emb_dim, var_eps_, cfg_.l2 ? 1 : 0,
                          meta_ + nlev * B, d_out, nullptr, pool_scratch_, st)) {
        err = vdb_last_error();
        return 1;
    }
    prof_end(pp, st, 0.0);
    launches += 3;
    return 0;
}

int Engine::run_eres2net(int B, int t_max, const std::vector<long long>& tv_sum, cudaStream_t st,
                         float* d_out, long long& launches, std::string& err) {
    const size_t nlev = levels_.size();
    std::vector<int> lt(1, t_max), lf(1, cfg_.n_mels);
    for (size_t l = 1; l < nlev; ++l) {
        lt.push_back(half_extent(lt.back()));
        lf.push_back(half_extent(lf.back()));
    }
    auto ptr = [&](const EOperand& o) -> void* {
        if (o.buf < 0) return nullptr;
        return static_cast<__half*>(ebufs_[o.buf].p) + o.c0;
    };
    auto ld = [&](const EOperand& o) -> int { return o.buf < 0 ? 0 : ebufs_[o.buf].c; };
    for (const EStep& s : esteps_) {
        const int To = lt[s.level], Fo = lf[s.level];
        if (s.kind == 1) {
            const int pa = prof_begin(st, 3);
            if (vdb_add(ptr(s.x0), ld(s.x0), ptr(s.x1), ld(s.x1), ptr(s.y), ld(s.y),
                        vdb_grid_rows(B, To, Fo), s.oc, st)) {
                err = vdb_last_error();
                return 1;
            }
            prof_end(pa, st, 0.0);
            ++launches;
            continue;
        }
        if (s.y2.buf >= 0 && ebufs_[s.y2.buf].c != s.oc) {
            err = "eres2net plan: second output must be a dense tensor";
            return 1;
        }
        vdb_conv_args a{};
        a.batch = B;
        a.t_out = To;
        a.f_out = Fo;
        a.oc = s.oc;
        a.k0 = s.k0;
        a.stride0 = s.stride0;
        a.ic0 = s.ic0;
        a.x0 = ptr(s.x0);
        a.ldx0 = ld(s.x0);
        a.w0 = s.w0;
        if (s.x1.buf >= 0) {
            a.x1 = ptr(s.x1);
            a.ldx1 = ld(s.x1);
            a.ic1 = s.ic1;
            a.stride1 = s.stride1;
            a.w1 = s.w1;
        }
        a.bias = s.bias;
        a.residual = ptr(s.res);
        a.ldr = ld(s.res);
        a.residual2 = ptr(s.res2);
        a.ldr2 = ld(s.res2);
        a.relu = s.relu;
        a.clamp_hi = s.clamp_hi;
        a.act = s.act;
        a.tvalid = meta_ + (size_t)s.level * B;
        a.y = ptr(s.y);
        a.ldy = ld(s.y);
        a.y_phase = s.y_phase;
        a.y2 = ptr(s.y2);
        a.ysum = ptr(s.ysum);
        a.ldsum = ld(s.ysum);
        a.addend = ptr(s.addend);
        a.ldaddend = ld(s.addend);
        a.err = errword_;
        const int pe = prof_begin(st);
        if (vdb_conv(&a, st)) {
            err = vdb_last_error();
            return 1;
        }
        prof_end(pe, st, s.flops_px * (double)Fo * (double)tv_sum[s.level], &a);
        launches += last_conv_launches();
    }
    const int lev = e_out_level_;
    const int pp = prof_begin(st, 2);
    if (pool_embed_launch(ebufs_[e_out_buf_].p, meta_ + (size_t)lev * B, B, lt[lev], lf[lev],
                          ebufs_[e_out_buf_].c, seg_w_, seg_b_, nullptr, cfg_.emb_dim, var_eps_,
                          cfg_.l2 ? 1 : 0, meta_ + nlev * B, d_out, nullptr, pool_scratch_, st)) {
        err = vdb_last_error();
        return 1;
    }
    prof_end(pp, st, 0.0);
    launches += 3;
    return 0;
}

int Engine::embed_device(const float* d_pcm, const long long* offsets, const int* nsamp, int n,
                         float* d_out, cudaStream_t stream, std::string& err) {
    if (!supported(err)) return 1;
    if (n <= 0) {
        err = "no clips";
        return 1;
    }
    if (cudaSetDevice(device_) != cudaSuccess) {
        err = "cudaSetDevice failed";
        return 1;
    }
    cudaStream_t st = stream ? stream : stream_;
    for (int i = 0; i < n; ++i)
        if (frames_of(nsamp[i], cfg_.win, cfg_.hop) <= 0) {
            // src/model.cpp:26-29
            err = "voicedetect: FBank produced no frames (clip " + std::to_string(i) + ")";
            return 1;
        }
    std::vector<int> order;
    std::vector<size_t> bk;
    plan_buckets(nsamp, n, max_frames, order, bk);
    last_launches = 0;
    std::vector<long long> bo;
    std::vector<int> bn;
    for (size_t k = 0; k + 1 < bk.size(); ++k) {
        bo.clear();
        bn.clear();
        for (size_t j = bk[k]; j < bk[k + 1]; ++j) {
            bo.push_back(offsets[order[j]]);
            bn.push_back(nsamp[order[j]]);
        }
        if (run_bucket(d_pcm, bo.data(), bn.data(), order.data() + bk[k], (int)bo.size(), st,
                       d_out, err))
            return 1;
    }
    return 0;
}

void Engine::plan_buckets(const int* nsamp, int n, long long frame_cap, std::vector<int>& order,
                          std::vector<size_t>& bk) const {
    // Longest first; consecutive clips of similar length share a bucket.
    order.resize((size_t)n);
    std::iota(order.begin(), order.end(), 0);
    std::stable_sort(order.begin(), order.end(),
                     [&](int a, int b) { return nsamp[a] > nsamp[b]; });
    bk.assign(1, 0);
    size_t i = 0;
    while (i < order.size()) {
        const int t0 = frames_of(nsamp[order[i]], cfg_.win, cfg_.hop);  // bucket's t_max
        size_t j = i;
        while (j < order.size() && (long long)(j - i) < max_clips &&
               (long long)(j - i + 1) * t0 <= std::max<long long>(frame_cap, t0))
            ++j;
        bk.push_back(j);
        i = j;
    }
}

// Copies clips into one pinned buffer, splitting the bytes over threads (one per
// 4 MB, at most 16 and the host's cores): one core's memcpy moves ~5 GB/s, and with
// 8 MB per thread the gather of a 128-clip bucket of 4 s clips took longer than its
// compute, which bounded the host-PCM path at half the device rate. The buffer is
// written with streaming stores (host_copy.h): only the copy engine reads it.
// Gather `count` clips (elements of `esz` bytes; clip idx[k] has nsamp[idx[k]]
// elements at pcm[idx[k]]) back to back into dst.
static void gather_clips(char* dst, const void* const* pcm, const int* nsamp, size_t esz,
                         const int* idx, int count) {
    std::vector<size_t> off((size_t)count + 1, 0);
    for (int k = 0; k < count; ++k) off[k + 1] = off[k] + (size_t)nsamp[idx[k]] * esz;
    const size_t total = off[count];
    const unsigned hw = std::max(1u, std::thread::hardware_concurrency());
    const int nt = (int)std::min<size_t>(std::min(16u, hw), 1 + total / (4u << 20));
    auto work = [&](int t) {
        // thread t copies the byte range [t*total/nt, (t+1)*total/nt)
        const size_t lo = total * t / nt, hi = total * (t + 1) / nt;
        int k = (int)(std::upper_bound(off.begin(), off.end(), lo) - off.begin()) - 1;
        for (size_t pos = lo; pos < hi && k < count; ++k) {
            const size_t a = std::max(pos, off[k]), b = std::min(hi, off[k + 1]);
            if (b > a)
                vdb_stream_copy(dst + a, static_cast<const char*>(pcm[idx[k]]) + (a - off[k]),
                                b - a);
            pos = b;
        }
        vdb_stream_fence();  // visible before the caller issues the DMA
    };
    if (nt <= 1) {
        work(0);
        return;
    }
    std::vector<std::thread> th;
    for (int t = 1; t < nt; ++t) th.emplace_back(work, t);
    work(0);
    for (std::thread& x : th) x.join();
}

// True when the `bytes` at p lie in page-locked host memory (cudaHostAlloc /
// cudaMallocHost / cudaHostRegister): the copy engine can then read them directly.
// Pageable, managed or device memory answers false. Both ends of the range are
// checked, so a clip that runs past a registered region is gathered instead.
static bool host_pinned(const void* p, size_t bytes) {
    if (!p || bytes == 0) return false;
    for (const void* q : {p, static_cast<const void*>(static_cast<const char*>(p) + bytes - 1)}) {
        cudaPointerAttributes a{};
        if (cudaPointerGetAttributes(&a, q) != cudaSuccess) {
            cudaGetLastError();
            return false;
        }
        if (a.type != cudaMemoryTypeHost) return false;
    }
    return true;
}

int Engine::embed_host(const float* const* pcm, const int* nsamp, int n, float* out,
                       std::string& err) {
    return embed_host_raw(reinterpret_cast<const void* const*>(pcm), 0, nsamp, n, 16000, out,
                          err);
}

int Engine::embed_host_raw(const void* const* pcm, int type, const int* n_in, int n,
                           int sample_rate, float* out, std::string& err) {
    if (!supported(err)) return 1;
    if (n <= 0) {
        err = "no clips";
        return 1;
    }
    if ((type != 0 && type != 1) || sample_rate <= 0) {
        err = "invalid PCM type or sample rate";
        return 1;
    }
    if (cudaSetDevice(device_) != cudaSuccess) {
        err = "cudaSetDevice failed";
        return 1;
    }
    const size_t esz = type == 1 ? sizeof(int16_t) : sizeof(float);
    // int16 or a rate other than 16 kHz: the raw samples cross PCIe and a kernel
    // converts / resamples them on the device (src/audio_io.cpp:9-23 semantics)
    const bool convert = type != 0 || sample_rate != 16000;
    std::vector<int> ns((size_t)n);
    for (int i = 0; i < n; ++i) {
        if (n_in[i] < 0) {
            err = "negative sample count";
            return 1;
        }
        const long long n16 = convert ? vdb_resampled_length(n_in[i], sample_rate, 16000) : n_in[i];
        if (n16 > INT32_MAX) {
            err = "clip too long";
            return 1;
        }
        ns[i] = (int)n16;
        if (frames_of(ns[i], cfg_.win, cfg_.hop) <= 0) {  // src/model.cpp:26-29
            err = "voicedetect: FBank produced no frames (clip " + std::to_string(i) + ")";
            return 1;
        }
    }
    // At least 2 buckets when the call is large enough, so that the host gather and
    // the H2D copy of one bucket hide behind the compute of the other. Not more: a
    // bucket too small to fill the GPU costs more device time than the overlap saves
    // (CAM++, 512 x 4 s clips: one 128-clip bucket 3.5 ms of device time against 8.9 ms
    // for all 512 at once, so four of them made the call slower than no split).
    long long frames_total = 0;
    for (int i = 0; i < n; ++i) frames_total += frames_of(ns[i], cfg_.win, cfg_.hop);
    const long long cap = std::min<long long>(max_frames, std::max<long long>(frames_total / 2, 16384));
    std::vector<int> order;
    std::vector<size_t> bk;
    plan_buckets(ns.data(), n, cap, order, bk);
    // ring slots hold the largest bucket the policy allows (and this call's largest)
    size_t need = convert ? 0 : ((size_t)max_frames * cfg_.hop + (size_t)max_clips * cfg_.win) * sizeof(float);
    size_t need_conv = 0;
    int max_cnt = 0;
    for (size_t k = 0; k + 1 < bk.size(); ++k) {
        size_t b = 0, c = 0;
        for (size_t j = bk[k]; j < bk[k + 1]; ++j) {
            b += (size_t)n_in[order[j]] * esz;
            c += (size_t)ns[order[j]] * sizeof(float);
        }
        need = std::max(need, b);
        need_conv = std::max(need_conv, c);
        max_cnt = std::max(max_cnt, (int)(bk[k + 1] - bk[k]));
    }
    need = std::max<size_t>(need, 16);
    if (need > ring_bytes_) {
        VDB_CHECK_CUDA(cudaDeviceSynchronize());
        clear_graphs();
        for (int s = 0; s < 2; ++s) {
            cudaFreeHost(h_ring_[s]);
            cudaFree(d_ring_[s]);
            h_ring_[s] = nullptr;
            d_ring_[s] = nullptr;
            ring_used_[s] = false;
        }
        ring_bytes_ = 0;
        for (int s = 0; s < 2; ++s)
            if (cudaMallocHost(&h_ring_[s], need) != cudaSuccess ||
                cudaMalloc(&d_ring_[s], need) != cudaSuccess) {
                err = "out of memory (PCM staging)";
                return 1;
            }
        ring_bytes_ = need;
    }
    if (convert && (need_conv > conv_bytes_ || max_cnt > imeta_cap_)) {
        VDB_CHECK_CUDA(cudaDeviceSynchronize());
        clear_graphs();  // captured buckets read the old converted-PCM buffers
        for (int s = 0; s < 2; ++s) {
            cudaFree(d_conv_[s]);
            cudaFreeHost(h_imeta_[s]);
            cudaFree(d_imeta_[s]);
            d_conv_[s] = nullptr;
            h_imeta_[s] = nullptr;
            d_imeta_[s] = nullptr;
            ring_used_[s] = false;
        }
        conv_bytes_ = 0;
        imeta_cap_ = 0;
        const int cap_c = std::max(max_cnt, max_clips);
        const size_t mb = (size_t)cap_c * (2 * sizeof(long long) + 2 * sizeof(int));
        for (int s = 0; s < 2; ++s)
            if (cudaMalloc(&d_conv_[s], std::max(need_conv, conv_bytes_)) != cudaSuccess ||
                cudaMallocHost(&h_imeta_[s], mb) != cudaSuccess ||
                cudaMalloc(&d_imeta_[s], mb) != cudaSuccess) {
                err = "out of memory (PCM conversion)";
                return 1;
            }
        conv_bytes_ = need_conv;
        imeta_cap_ = cap_c;
    }
    const size_t ob = (size_t)n * cfg_.emb_dim * sizeof(float);
    if (ob > out_bytes_) {
        VDB_CHECK_CUDA(cudaDeviceSynchronize());
        clear_graphs();
        cudaFreeHost(h_out_);
        cudaFree(d_out_);
        h_out_ = nullptr;
        d_out_ = nullptr;
        out_bytes_ = 0;
        if (cudaMallocHost(&h_out_, ob) != cudaSuccess || cudaMalloc(&d_out_, ob) != cudaSuccess) {
            err = "out of memory (output staging)";
            return 1;
        }
        out_bytes_ = ob;
    }
    last_launches = 0;
    std::vector<long long> bo, bi;
    std::vector<int> bn;
    // Clips in page-locked memory go to the device by one DMA each, straight from the
    // caller's buffers; a bucket with any pageable clip is gathered into the pinned
    // ring and copied in one piece. The gather costs the host three passes over its
    // DRAM per input byte (read the caller's array, write the ring, DMA out of it)
    // against one for the direct copy, and with eight ranks per host that memory
    // bandwidth, not PCIe, bounded the f32 call.
    // Buckets run shortest clips first: the first bucket's host gather and copy are
    // the only ones nothing overlaps, so it should be the smallest.
    const size_t nbk = bk.size() - 1;
    for (size_t step = 0; step < nbk; ++step) {
        const size_t k = nbk - 1 - step;
        const int s = (int)(step & 1);
        const int cnt = (int)(bk[k + 1] - bk[k]);
        const int* idx = order.data() + bk[k];
        // checked bucket by bucket, so that all but the first bucket's checks overlap
        // the previous bucket's compute
        bool direct = true;
        for (int j = 0; j < cnt && direct; ++j)
            direct = host_pinned(pcm[idx[j]], (size_t)n_in[idx[j]] * esz);
        // the pinned slots (PCM ring, conversion metadata) are free once their
        // previous H2D copies finished
        if (ring_used_[s]) VDB_CHECK_CUDA(cudaEventSynchronize(h2d_ev_[s]));
        if (!direct) gather_clips(reinterpret_cast<char*>(h_ring_[s]), pcm, n_in, esz, idx, cnt);
        bo.assign((size_t)cnt, 0);
        bi.assign((size_t)cnt, 0);
        bn.assign((size_t)cnt, 0);
        long long tot = 0, tot_in = 0;
        int max_out = 0;
        // conversion metadata: [in_off][out_off] (int64), [n_in][n_out] (int32)
        long long* mi = convert ? static_cast<long long*>(h_imeta_[s]) : nullptr;
        for (int j = 0; j < cnt; ++j) {
            bo[j] = tot;
            bi[j] = tot_in;
            bn[j] = ns[idx[j]];
            if (convert) {
                mi[j] = tot_in;
                mi[imeta_cap_ + j] = tot;
                int* mn = reinterpret_cast<int*>(mi + 2 * imeta_cap_);
                mn[j] = n_in[idx[j]];
                mn[imeta_cap_ + j] = bn[j];
            }
            tot += bn[j];
            tot_in += n_in[idx[j]];
            max_out = std::max(max_out, bn[j]);
        }
        // the device slot is free once the bucket that last read it finished
        if (ring_used_[s]) VDB_CHECK_CUDA(cudaStreamWaitEvent(copy_stream_, comp_ev_[s], 0));
        if (direct) {
            // the same packed layout the gather writes: clip j at input offset bi[j];
            // clips that also follow one another in the caller's memory go as one copy
            for (int j = 0; j < cnt;) {
                const char* src = static_cast<const char*>(pcm[idx[j]]);
                size_t bytes = (size_t)n_in[idx[j]] * esz;
                int e = j + 1;
                while (e < cnt && static_cast<const char*>(pcm[idx[e]]) == src + bytes) {
                    bytes += (size_t)n_in[idx[e]] * esz;
                    ++e;
                }
                VDB_CHECK_CUDA(cudaMemcpyAsync(static_cast<char*>(d_ring_[s]) + (size_t)bi[j] * esz,
                                               src, bytes, cudaMemcpyHostToDevice, copy_stream_));
                j = e;
            }
        } else {
            VDB_CHECK_CUDA(cudaMemcpyAsync(d_ring_[s], h_ring_[s], (size_t)tot_in * esz,
                                           cudaMemcpyHostToDevice, copy_stream_));
        }
        if (convert)
            VDB_CHECK_CUDA(cudaMemcpyAsync(d_imeta_[s], h_imeta_[s],
                                           (size_t)imeta_cap_ * (2 * sizeof(long long) + 2 * sizeof(int)),
                                           cudaMemcpyHostToDevice, copy_stream_));
        VDB_CHECK_CUDA(cudaEventRecord(h2d_ev_[s], copy_stream_));
        VDB_CHECK_CUDA(cudaStreamWaitEvent(stream_, h2d_ev_[s], 0));
        ring_used_[s] = true;
        const float* d_pcm = reinterpret_cast<const float*>(d_ring_[s]);
        if (convert) {
            long long* dm = static_cast<long long*>(d_imeta_[s]);
            const int* dn = reinterpret_cast<const int*>(dm + 2 * imeta_cap_);
            if (vdb_pcm_ingest(d_ring_[s], type, dm, dn, cnt, sample_rate, 16000, dm + imeta_cap_,
                               dn + imeta_cap_, max_out, d_conv_[s], stream_)) {
                err = vdb_last_error();
                cudaStreamSynchronize(stream_);
                return 1;
            }
            ++last_launches;
            d_pcm = d_conv_[s];
        }
        if (run_bucket(d_pcm, bo.data(), bn.data(), idx, cnt, stream_, d_out_, err)) {
            cudaStreamSynchronize(stream_);
            return 1;
        }
        VDB_CHECK_CUDA(cudaEventRecord(comp_ev_[s], stream_));
    }
    VDB_CHECK_CUDA(cudaMemcpyAsync(h_out_, d_out_, ob, cudaMemcpyDeviceToHost, stream_));
    VDB_CHECK_CUDA(cudaStreamSynchronize(stream_));
    if (check_device_error(err)) return 1;
    std::memcpy(out, h_out_, ob);
    return 0;
}

int Engine::check_device_error(std::string& err) {
    int h = 0;
    if (cudaMemcpy(&h, errword_, sizeof(int), cudaMemcpyDeviceToHost) != cudaSuccess) {
        err = std::string("CUDA error: ") + cudaGetErrorString(cudaGetLastError());
        return 1;
    }
    if (h != 0) {
        cudaMemset(errword_, 0, sizeof(int));
        char buf[96];
        std::snprintf(buf, sizeof(buf), "GPU kernel wait timed out (code 0x%x)", h);
        err = buf;
        return 1;
    }
    return 0;
}

void Engine::set_profiling(bool on) { profiling_ = on; }

int Engine::prof_begin(cudaStream_t st, int stage) {
    if (!profiling_) return -1;
    if (prof_used_ + 2 > prof_ev_.size()) {
        for (int i = 0; i < 64; ++i) {
            cudaEvent_t ev;
            if (cudaEventCreate(&ev) != cudaSuccess) return -1;
            prof_ev_.push_back(ev);
        }
    }
    const int idx = (int)prof_used_;
    prof_used_ += 2;
    prof_stage_.resize(prof_used_ / 2);
    prof_stage_[idx / 2] = stage;
    prof_conv_.resize(prof_used_ / 2);
    prof_conv_[idx / 2] = ConvRecord{0.0, 0.0, 0, 0, 0, 0, 0, 0, 0, 0, 0, 0};
    cudaEventRecord(prof_ev_[idx], st);
    return idx;
}

void Engine::prof_end(int idx, cudaStream_t st, double flops, const vdb_conv_args* conv) {
    if (idx < 0) return;
    cudaEventRecord(prof_ev_[idx + 1], st);
    if (prof_stage_[idx / 2] == 0) prof_flops_ += flops;
    ConvRecord& r = prof_conv_[idx / 2];
    r.flops = flops;
    if (conv) {
        r.ic = conv->ic0;
        r.oc = conv->oc;
        r.k = conv->k0;
        r.stride = conv->stride0;
        r.f_out = conv->f_out;
        r.t_out = conv->t_out;
        r.batch = conv->batch;
        r.ic1 = conv->x1 ? conv->ic1 : 0;
        r.res = conv->residual ? 1 : 0;
        r.qpack = conv->qpack;
    }
}

int Engine::read_profile(double& conv_ms, double& conv_flops, long long& conv_launches,
                         std::string& err) {
    conv_ms = 0.0;
    conv_flops = prof_flops_;
    conv_launches = 0;
    for (double& v : stage_ms) v = 0.0;
    conv_records.clear();
    for (size_t i = 0; i + 1 < prof_used_; i += 2) {
        if (cudaEventSynchronize(prof_ev_[i + 1]) != cudaSuccess) {
            err = "profile event failed";
            return 1;
        }
        float ms = 0.0f;
        if (cudaEventElapsedTime(&ms, prof_ev_[i], prof_ev_[i + 1]) != cudaSuccess) {
            cudaGetLastError();  // do not leave the error for an unrelated later check
            err = "profile event pair " + std::to_string(i / 2) + " was not recorded";
            prof_used_ = 0;
            prof_flops_ = 0.0;
            return 1;
        }
        const int stg = prof_stage_[i / 2];
        stage_ms[stg] += ms;
        if (stg == 0) {
            conv_ms += ms;
            ++conv_launches;
            conv_records.push_back(prof_conv_[i / 2]);
            conv_records.back().ms = ms;
        }
    }
    prof_used_ = 0;
    prof_flops_ = 0.0;
    return 0;
}

std::vector<float> resample_linear(const std::vector<float>& in, int in_sr, int out_sr) {
    if (in_sr == out_sr || in.empty()) return in;
    const double ratio = (double)out_sr / (double)in_sr;
    const size_t n_out = (size_t)std::floor(in.size() * ratio);
    std::vector<float> out(n_out);
    for (size_t i = 0; i < n_out; ++i) {
        const double src = i / ratio;
        const size_t i0 = (size_t)src;
        const double frac = src - i0;
        const float a = in[i0];
        const float b = (i0 + 1 < in.size()) ? in[i0 + 1] : a;
        out[i] = (float)(a + (b - a) * frac);
    }
    return out;
}

}  // namespace vdb
