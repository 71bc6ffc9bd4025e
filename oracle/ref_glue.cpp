// extern "C" glue around the reference's OWN kernel sources, compiled unmodified
// from the reference checkout against oracle/ggml_shim/ggml.h. Built by
// oracle/Makefile into oracle/_ref/libvdref.so.
//
// TEST INFRASTRUCTURE ONLY: used by tests/ (to pin the C restatement in
// oracle/vd_oracle.c and to check the CUDA path) and by bench.py's CPU-baseline
// leg. The product library never links or loads it.
//
// What runs here is the reference's code:
//   vd::FBank::compute                          src/fbank.cpp:121-205
//   vd::directconv_conv3x3 (NCHW stem conv)     src/directconv.cpp:1449-1458
//   vd::blocked_reorder_in/out                  src/directconv.cpp:1481-1494
//   vd::blocked_conv3x3 / blocked_conv1x1       src/directconv.cpp:1496-1522
//   vd::blocked_add_relu                        src/directconv.cpp:1542-1546
//   vd::winograd_conv3x3                        src/winograd.cpp:638-648
// and the ResNet34 graph glue below restates src/encoder_resnet.cpp:94-185 op for
// op (the ggml graph ops it uses - add, relu, mean, sub, sqr, scale, sqrt,
// mul_mat - live in the absent ggml submodule and are restated as plain loops).
#include "ggml.h"
#include "directconv.hpp"
#include "winograd.hpp"
#include "fbank.hpp"
#include "model_loader.hpp"
#include "vd_oracle.h"

#include <omp.h>
#include <cmath>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <vector>

namespace {

// The reference caches packed weights keyed on the weight's data pointer
// (src/directconv.cpp:1375-1445, src/winograd.cpp:595-634). Every weight handed
// to a reference op therefore lives in a buffer that is never freed, so no later
// allocation can reuse its address with different contents.
float* stable_copy(const float* src, size_t n) {
    static std::mutex mu;
    std::lock_guard<std::mutex> lk(mu);
    void* p = nullptr;
    if (posix_memalign(&p, 64, (n ? n : 1) * sizeof(float)) != 0) std::abort();
    if (n) std::memcpy(p, src, n * sizeof(float));
    return (float*)p;  // intentionally never freed
}

struct Ctx {
    ggml_context* c = shim_ctx_new();
    ~Ctx() { shim_ctx_free(c); }
};

void add_bias_relu_nchw(float* y, int W, int H, int C, const float* b, bool relu) {
    const size_t HW = (size_t)W * H;
    for (int c = 0; c < C; ++c) {
        float* yc = y + (size_t)c * HW;
        const float bc = b ? b[c] : 0.0f;
        for (size_t p = 0; p < HW; ++p) {
            float v = yc[p] + bc;                 // ggml_add (src/encoder_resnet.cpp:26-29)
            if (relu) v = v > 0.0f ? v : 0.0f;    // ggml_relu (:117)
            yc[p] = v;
        }
    }
}

}  // namespace

extern "C" {

void vdref_set_threads(int n) {
    omp_set_dynamic(0);
    shim_set_threads(n);
}

int vdref_get_threads(void) { return shim_get_threads(); }

// vd::FBank::compute on 16 kHz mono PCM. Writes feat-major [n_mels, T] into `out`
// when out != NULL and out_cap >= n_mels*T. Returns 0 on success, 1 when FBank
// produced no frames (the reference's "FBank produced no frames" condition,
// src/model.cpp:26-29), 2 when out_cap is too small.
int vdref_fbank(const float* pcm, int n, int sample_rate, int n_mels, int n_fft, int win,
                int hop, float preemph, float low_freq, float high_freq, int cmn,
                float* out, long out_cap, int* out_T) {
    vd::VoiceDetectConfig cfg;
    cfg.sample_rate = (uint32_t)sample_rate;
    cfg.n_mels = (uint32_t)n_mels;
    cfg.n_fft = (uint32_t)n_fft;
    cfg.win_length = (uint32_t)win;
    cfg.hop_length = (uint32_t)hop;
    cfg.preemph = preemph;
    cfg.fbank_low_freq = low_freq;
    cfg.fbank_high_freq = high_freq;
    cfg.fbank_cmn = cmn != 0;
    std::vector<float> pcm16k(pcm, pcm + (n > 0 ? n : 0));
    vd::FBank fb(cfg);
    int T = 0;
    std::vector<float> feats = fb.compute(pcm16k, T);
    if (out_T) *out_T = T;
    if (feats.empty() || T == 0) return 1;
    if (!out) return 0;
    if ((long)feats.size() > out_cap) return 2;
    std::memcpy(out, feats.data(), feats.size() * sizeof(float));
    return 0;
}

// Blocked (nChw16c) 3x3 conv, reference path of test_blocked.cpp:94-103:
// reorder_in -> blocked_conv3x3(pad 1, stride, optional fused bias/ReLU) ->
// reorder_out. x NCHW [W,H,IC] (ggml ne order), w ggml [3,3,IC,OC] (= torch
// (OC,IC,3,3)), y [Wout,Hout,OC].
void vdref_conv3x3_blocked(const float* x, int W, int H, int IC, const float* w, int OC,
                           const float* bias, int relu, int stride, float* y) {
    Ctx ctx;
    float* ws = stable_copy(w, (size_t)9 * IC * OC);
    float* bs = bias ? stable_copy(bias, (size_t)OC) : nullptr;
    ggml_tensor* xt = shim_wrap_f32(ctx.c, const_cast<float*>(x), W, H, IC, 1);
    ggml_tensor* wt = shim_wrap_f32(ctx.c, ws, 3, 3, IC, OC);
    ggml_tensor* bt = bs ? shim_wrap_f32(ctx.c, bs, OC, 1, 1, 1) : nullptr;
    ggml_tensor* xb = vd::blocked_reorder_in(ctx.c, xt);
    ggml_tensor* yb = vd::blocked_conv3x3(ctx.c, wt, xb, 1, stride, bt, relu != 0);
    ggml_tensor* yt = vd::blocked_reorder_out(ctx.c, yb, OC);
    std::memcpy(y, yt->data, (size_t)ggml_nelements(yt) * sizeof(float));
}

// Blocked 1x1 strided conv (the BasicBlock downsample), test_blocked.cpp:157-166.
void vdref_conv1x1_blocked(const float* x, int W, int H, int IC, const float* w, int OC,
                           const float* bias, int relu, int stride, float* y) {
    Ctx ctx;
    float* ws = stable_copy(w, (size_t)IC * OC);
    float* bs = bias ? stable_copy(bias, (size_t)OC) : nullptr;
    ggml_tensor* xt = shim_wrap_f32(ctx.c, const_cast<float*>(x), W, H, IC, 1);
    ggml_tensor* wt = shim_wrap_f32(ctx.c, ws, 1, 1, IC, OC);
    ggml_tensor* bt = bs ? shim_wrap_f32(ctx.c, bs, OC, 1, 1, 1) : nullptr;
    ggml_tensor* xb = vd::blocked_reorder_in(ctx.c, xt);
    ggml_tensor* yb = vd::blocked_conv1x1(ctx.c, wt, xb, stride, bt, relu != 0);
    ggml_tensor* yt = vd::blocked_reorder_out(ctx.c, yb, OC);
    std::memcpy(y, yt->data, (size_t)ggml_nelements(yt) * sizeof(float));
}

// NCHW direct 3x3 stride-1 conv (the stem path), no bias.
void vdref_directconv3x3(const float* x, int W, int H, int IC, const float* w, int OC,
                         float* y) {
    Ctx ctx;
    float* ws = stable_copy(w, (size_t)9 * IC * OC);
    ggml_tensor* xt = shim_wrap_f32(ctx.c, const_cast<float*>(x), W, H, IC, 1);
    ggml_tensor* wt = shim_wrap_f32(ctx.c, ws, 3, 3, IC, OC);
    ggml_tensor* yt = vd::directconv_conv3x3(ctx.c, wt, xt, 1);
    std::memcpy(y, yt->data, (size_t)ggml_nelements(yt) * sizeof(float));
}

// Winograd 3x3 stride-1 pad-1 conv (mode from VOICEDETECT_WINO, default f2b).
void vdref_winograd3x3(const float* x, int W, int H, int IC, const float* w, int OC,
                       float* y) {
    Ctx ctx;
    float* ws = stable_copy(w, (size_t)9 * IC * OC);
    ggml_tensor* xt = shim_wrap_f32(ctx.c, const_cast<float*>(x), W, H, IC, 1);
    ggml_tensor* wt = shim_wrap_f32(ctx.c, ws, 3, 3, IC, OC);
    ggml_tensor* yt = vd::winograd_conv3x3(ctx.c, wt, xt, 1);
    std::memcpy(y, yt->data, (size_t)ggml_nelements(yt) * sizeof(float));
}

// ---------------------------------------------------------------------------
// ResNet34 (WeSpeaker) forward on the reference kernels.
// ---------------------------------------------------------------------------
typedef vd_resnet_desc vdref_resnet_desc;

struct RefResNet {
    int nb = 0, c0 = 0, emb = 0, pooled = 0, l2 = 1;
    float eps = 1e-8f;
    float *stem_w = nullptr, *stem_b = nullptr;
    std::vector<float*> c1w, c1b, c2w, c2b, dw, db;
    std::vector<int> ic, oc, st;
    float *seg_w = nullptr, *seg_b = nullptr, *mean_vec = nullptr;
};

void* vdref_resnet34_new(const vdref_resnet_desc* d) {
    RefResNet* m = new RefResNet();
    m->nb = d->n_blocks;
    m->c0 = d->stem_oc;
    m->emb = d->emb_dim;
    m->pooled = d->pooled_dim;
    m->eps = d->var_eps;
    m->l2 = d->l2_normalize;
    m->stem_w = stable_copy(d->stem_w, (size_t)9 * d->stem_oc);
    m->stem_b = stable_copy(d->stem_b, (size_t)d->stem_oc);
    for (int i = 0; i < d->n_blocks; ++i) {
        const int ic = d->in_ch[i], oc = d->out_ch[i];
        m->ic.push_back(ic);
        m->oc.push_back(oc);
        m->st.push_back(d->stride[i]);
        m->c1w.push_back(stable_copy(d->conv1_w[i], (size_t)9 * ic * oc));
        m->c1b.push_back(stable_copy(d->conv1_b[i], (size_t)oc));
        m->c2w.push_back(stable_copy(d->conv2_w[i], (size_t)9 * oc * oc));
        m->c2b.push_back(stable_copy(d->conv2_b[i], (size_t)oc));
        if (d->down_w[i]) {
            m->dw.push_back(stable_copy(d->down_w[i], (size_t)ic * oc));
            m->db.push_back(stable_copy(d->down_b[i], (size_t)oc));
        } else {
            m->dw.push_back(nullptr);
            m->db.push_back(nullptr);
        }
    }
    m->seg_w = stable_copy(d->seg_w, (size_t)d->pooled_dim * d->emb_dim);
    m->seg_b = stable_copy(d->seg_b, (size_t)d->emb_dim);
    if (d->mean_vec) m->mean_vec = stable_copy(d->mean_vec, (size_t)d->emb_dim);
    return m;
}

// Embed one utterance: feats feat-major [n_mels, T] (post-CMN FBank). Writes the
// pre-norm embedding to `prenorm` (if non-NULL) and the L2-normalised embedding to
// `emb`. Follows src/encoder_resnet.cpp:94-185 with the blocked island covering
// every block (the default on an AVX-512 host, :83-92).
int vdref_resnet34_forward(void* handle, const float* feats, int T, int n_mels, float* emb,
                           float* prenorm) {
    RefResNet* m = (RefResNet*)handle;
    Ctx ctx;
    ggml_tensor* x = shim_wrap_f32(ctx.c, const_cast<float*>(feats), T, n_mels, 1, 1);
    // Stem: directconv 3x3 s1 p1 -> + bias -> ReLU (:116-117).
    ggml_tensor* sw = shim_wrap_f32(ctx.c, m->stem_w, 3, 3, 1, m->c0);
    ggml_tensor* h = vd::directconv_conv3x3(ctx.c, sw, x, 1);
    add_bias_relu_nchw((float*)h->data, T, n_mels, m->c0, m->stem_b, true);
    // Blocked island over all blocks (:127-136, basic_block_blocked :54-73).
    ggml_tensor* xb = vd::blocked_reorder_in(ctx.c, h);
    for (int i = 0; i < m->nb; ++i) {
        const int ic = m->ic[i], oc = m->oc[i], s = m->st[i];
        ggml_tensor* w1 = shim_wrap_f32(ctx.c, m->c1w[i], 3, 3, ic, oc);
        ggml_tensor* b1 = shim_wrap_f32(ctx.c, m->c1b[i], oc, 1, 1, 1);
        ggml_tensor* hb = vd::blocked_conv3x3(ctx.c, w1, xb, 1, s, b1, true);
        ggml_tensor* w2 = shim_wrap_f32(ctx.c, m->c2w[i], 3, 3, oc, oc);
        ggml_tensor* b2 = shim_wrap_f32(ctx.c, m->c2b[i], oc, 1, 1, 1);
        hb = vd::blocked_conv3x3(ctx.c, w2, hb, 1, 1, b2, false);
        ggml_tensor* sc = xb;
        if (m->dw[i]) {
            ggml_tensor* dw = shim_wrap_f32(ctx.c, m->dw[i], 1, 1, ic, oc);
            ggml_tensor* db = shim_wrap_f32(ctx.c, m->db[i], oc, 1, 1, 1);
            sc = vd::blocked_conv1x1(ctx.c, dw, xb, s, db, false);
        }
        xb = vd::blocked_add_relu(ctx.c, hb, sc);
    }
    const int C = m->oc[m->nb - 1];
    ggml_tensor* ho = vd::blocked_reorder_out(ctx.c, xb, C);
    const int Wp = (int)ho->ne[0], Hp = (int)ho->ne[1];
    const float* a = (const float*)ho->data;
    // TSTP (:143-157): per (c, h) over time w. mean -> sub -> sqr -> mean ->
    // scale N/(N-1) -> + eps -> sqrt. Flatten C-outer/H-inner, concat [mean; std].
    const int HC = Hp * C;
    if (2 * HC != m->pooled) return 3;
    std::vector<float> pooled((size_t)2 * HC);
    for (int c = 0; c < C; ++c)
        for (int hh = 0; hh < Hp; ++hh) {
            const float* row = a + ((size_t)c * Hp + hh) * Wp;
            double s = 0.0;
            for (int w = 0; w < Wp; ++w) s += row[w];
            const float mean = (float)(s / Wp);
            double s2 = 0.0;
            for (int w = 0; w < Wp; ++w) {
                const float dv = row[w] - mean;
                s2 += (double)(dv * dv);
            }
            float var = (float)(s2 / Wp);
            if (Wp > 1) var = var * ((float)Wp / (float)(Wp - 1));
            const float sd = std::sqrt(var + m->eps);
            pooled[(size_t)c * Hp + hh] = mean;
            pooled[(size_t)HC + (size_t)c * Hp + hh] = sd;
        }
    // FC (:162-170): emb[j] = sum_i W[j*pooled + i] * pooled[i] + b[j] - mean_vec[j].
    std::vector<float> out((size_t)m->emb);
    for (int j = 0; j < m->emb; ++j) {
        const float* wr = m->seg_w + (size_t)j * m->pooled;
        double acc = 0.0;
        for (int i = 0; i < m->pooled; ++i) acc += (double)wr[i] * (double)pooled[i];
        float v = (float)acc + m->seg_b[j];
        if (m->mean_vec) v -= m->mean_vec[j];
        out[j] = v;
    }
    if (prenorm) std::memcpy(prenorm, out.data(), out.size() * sizeof(float));
    // Host L2 normalise in double (:177-183).
    if (m->l2) {
        double n2 = 0.0;
        for (float v : out) n2 += (double)v * (double)v;
        const double nrm = std::sqrt(n2);
        if (nrm > 0.0)
            for (float& v : out) v = (float)((double)v / nrm);
    }
    std::memcpy(emb, out.data(), out.size() * sizeof(float));
    return 0;
}

}  // extern "C"

// ---------------------------------------------------------------------------
// ERes2Net forward on the reference kernels: the stem through directconv_conv3x3
// + bias + ReLU, every body conv through the blocked island ops
// (blocked_conv1x1 / blocked_conv3x3 with fused bias, src/encoder_eres2net.cpp:44-50).
// The elementwise glue (clamp, split, concat, add, SiLU, tanh, AFF mix) and the
// tail are restated from src/encoder_eres2net.cpp:60-264.
// ---------------------------------------------------------------------------
struct RefERes2Net {
    vd_eres2net_desc d{};
    std::vector<float*> w, b;
    std::vector<int> ic, oc, k, st;
    float* seg_w = nullptr;
    float* seg_b = nullptr;
};

struct RAct {
    std::vector<float> v;
    int C = 0, H = 0, W = 0;
    size_t hw() const { return (size_t)H * W; }
};

struct REnc {
    RefERes2Net* m;
    int idx = 0;

    RAct conv(const RAct& x) {
        const int i = idx++;
        const int k = m->k[i], s = m->st[i], OC = m->oc[i];
        Ctx ctx;
        ggml_tensor* xt = shim_wrap_f32(ctx.c, const_cast<float*>(x.v.data()), x.W, x.H, x.C, 1);
        ggml_tensor* wt = shim_wrap_f32(ctx.c, m->w[i], k, k, x.C, OC);
        ggml_tensor* bt = m->b[i] ? shim_wrap_f32(ctx.c, m->b[i], OC, 1, 1, 1) : nullptr;
        ggml_tensor* xb = vd::blocked_reorder_in(ctx.c, xt);
        ggml_tensor* yb = (k == 1) ? vd::blocked_conv1x1(ctx.c, wt, xb, s, bt, false)
                                   : vd::blocked_conv3x3(ctx.c, wt, xb, (k - 1) / 2, s, bt, false);
        ggml_tensor* yt = vd::blocked_reorder_out(ctx.c, yb, OC);
        RAct y;
        y.C = OC;
        y.W = (int)yt->ne[0];
        y.H = (int)yt->ne[1];
        y.v.assign((const float*)yt->data, (const float*)yt->data + ggml_nelements(yt));
        return y;
    }
    void clamp(RAct& a) {
        const float hi = m->d.relu_clamp;
        for (float& v : a.v) v = v < 0.0f ? 0.0f : (v > hi ? hi : v);
    }
    RAct aff(const RAct& x, const RAct& ds) {
        RAct cat;
        cat.C = x.C + ds.C;
        cat.H = x.H;
        cat.W = x.W;
        cat.v = x.v;
        cat.v.insert(cat.v.end(), ds.v.begin(), ds.v.end());
        RAct z = conv(cat);
        for (float& v : z.v) v = v / (1.0f + std::exp(-v));
        RAct z2 = conv(z);
        RAct out = x;
        for (size_t i = 0; i < out.v.size(); ++i) {
            const float att = std::tanh(z2.v[i]);
            out.v[i] = (x.v[i] + ds.v[i]) + att * (x.v[i] - ds.v[i]);
        }
        return out;
    }
    RAct block(const RAct& x, int planes, int stride, bool is_aff, int& in_planes) {
        const int scale = m->d.scale;
        RAct out = conv(x);
        clamp(out);
        const int width = out.C / scale;
        const size_t hw = out.hw();
        RAct accum;
        accum.C = out.C;
        accum.H = out.H;
        accum.W = out.W;
        accum.v.assign(out.v.size(), 0.0f);
        RAct sp;
        for (int i = 0; i < scale; ++i) {
            RAct chunk;
            chunk.C = width;
            chunk.H = out.H;
            chunk.W = out.W;
            chunk.v.assign(out.v.begin() + (size_t)i * width * hw,
                           out.v.begin() + (size_t)(i + 1) * width * hw);
            RAct cur;
            if (i == 0) cur = chunk;
            else if (is_aff) cur = aff(sp, chunk);
            else {
                cur = chunk;
                for (size_t j = 0; j < cur.v.size(); ++j) cur.v[j] = sp.v[j] + chunk.v[j];
            }
            RAct cv = conv(cur);
            clamp(cv);
            std::copy(cv.v.begin(), cv.v.end(), accum.v.begin() + (size_t)i * width * hw);
            sp = cv;
        }
        RAct o3 = conv(accum);
        if (stride != 1 || in_planes != 2 * planes) {
            RAct r = conv(x);
            for (size_t j = 0; j < o3.v.size(); ++j) o3.v[j] += r.v[j];
        } else {
            for (size_t j = 0; j < o3.v.size(); ++j) o3.v[j] += x.v[j];
        }
        in_planes = 2 * planes;
        clamp(o3);
        return o3;
    }
    RAct layer(RAct x, int planes, int n, int stride, bool is_aff, int& in_planes) {
        for (int bi = 0; bi < n; ++bi) x = block(x, planes, bi == 0 ? stride : 1, is_aff, in_planes);
        return x;
    }
};

extern "C" {

void* vdref_eres2net_new(const vd_eres2net_desc* d) {
    RefERes2Net* m = new RefERes2Net();
    m->d = *d;
    for (int i = 0; i < d->n_convs; ++i) {
        m->ic.push_back(d->ic[i]);
        m->oc.push_back(d->oc[i]);
        m->k.push_back(d->k[i]);
        m->st.push_back(d->stride[i]);
        m->w.push_back(stable_copy(d->w[i], (size_t)d->oc[i] * d->ic[i] * d->k[i] * d->k[i]));
        m->b.push_back(d->b[i] ? stable_copy(d->b[i], (size_t)d->oc[i]) : nullptr);
    }
    m->seg_w = stable_copy(d->seg_w, (size_t)d->emb_dim * d->pooled_dim);
    m->seg_b = stable_copy(d->seg_b, (size_t)d->emb_dim);
    return m;
}

int vdref_eres2net_forward(void* handle, const float* feats, int T, int n_mels, float* emb,
                           float* prenorm) {
    RefERes2Net* m = (RefERes2Net*)handle;
    REnc e{m};
    const int M = m->d.m_channels;
    // stem: directconv_conv3x3 -> + bias -> ReLU (:203)
    RAct h;
    {
        Ctx ctx;
        ggml_tensor* x = shim_wrap_f32(ctx.c, const_cast<float*>(feats), T, n_mels, 1, 1);
        ggml_tensor* sw = shim_wrap_f32(ctx.c, m->w[0], 3, 3, 1, m->oc[0]);
        ggml_tensor* y = vd::directconv_conv3x3(ctx.c, sw, x, 1);
        add_bias_relu_nchw((float*)y->data, T, n_mels, m->oc[0], m->b[0], true);
        h.C = m->oc[0];
        h.H = n_mels;
        h.W = T;
        h.v.assign((const float*)y->data, (const float*)y->data + ggml_nelements(y));
        e.idx = 1;
    }
    int in_planes = M;
    const int* nb = m->d.num_blocks;
    RAct o1 = e.layer(h, M, nb[0], 1, false, in_planes);
    RAct o2 = e.layer(o1, 2 * M, nb[1], 2, false, in_planes);
    RAct o1d = e.conv(o1);
    RAct f12 = e.aff(o2, o1d);
    RAct o3 = e.layer(o2, 4 * M, nb[2], 2, true, in_planes);
    RAct f12d = e.conv(f12);
    RAct f123 = e.aff(o3, f12d);
    RAct o4 = e.layer(o3, 8 * M, nb[3], 2, true, in_planes);
    RAct f123d = e.conv(f123);
    RAct f = e.aff(o4, f123d);
    if (e.idx != m->d.n_convs) return 4;
    // TSTP + seg FC + L2 (:228-262), same restatement as the ResNet tail
    const int C = f.C, Hp = f.H, Wp = f.W, HC = Hp * C;
    if (2 * HC != m->d.pooled_dim) return 3;
    std::vector<float> pooled((size_t)2 * HC);
    for (int c = 0; c < C; ++c)
        for (int hh = 0; hh < Hp; ++hh) {
            const float* row = f.v.data() + ((size_t)c * Hp + hh) * Wp;
            double s = 0.0;
            for (int w = 0; w < Wp; ++w) s += row[w];
            const float mean = (float)(s / Wp);
            double s2 = 0.0;
            for (int w = 0; w < Wp; ++w) {
                const float dv = row[w] - mean;
                s2 += (double)(dv * dv);
            }
            float var = (float)(s2 / Wp);
            if (Wp > 1) var = var * ((float)Wp / (float)(Wp - 1));
            pooled[(size_t)c * Hp + hh] = mean;
            pooled[(size_t)HC + (size_t)c * Hp + hh] = std::sqrt(var + m->d.var_eps);
        }
    const int D = m->d.emb_dim;
    std::vector<float> out((size_t)D);
    for (int j = 0; j < D; ++j) {
        const float* wr = m->seg_w + (size_t)j * m->d.pooled_dim;
        double acc = 0.0;
        for (int i = 0; i < m->d.pooled_dim; ++i) acc += (double)wr[i] * (double)pooled[i];
        out[j] = (float)acc + m->seg_b[j];
    }
    if (prenorm) std::memcpy(prenorm, out.data(), out.size() * sizeof(float));
    if (m->d.l2_normalize) {
        double n2 = 0.0;
        for (float v : out) n2 += (double)v * (double)v;
        const double nrm = std::sqrt(n2);
        if (nrm > 0.0)
            for (float& v : out) v = (float)((double)v / nrm);
    }
    std::memcpy(emb, out.data(), out.size() * sizeof(float));
    return 0;
}

}  // extern "C"
