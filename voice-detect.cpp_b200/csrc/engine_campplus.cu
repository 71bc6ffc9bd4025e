// CAM++ on the B200 engine: the counterpart of the reference's CamPPlusEncoder
// (src/encoder_campplus.cpp:148-310) over a length-bucketed batch.
//
// Load. The GGUF carries a flat manifest (src/model_loader.cpp:165-172): conv
// weights / biases in forward-execution order and the prefixes of the runtime
// BatchNorms, consumed with running indices exactly as the reference's forward
// does. The dense blocks' layer counts are read off the manifest (a layer is the
// 1x1 conv followed by a k=3 conv; the 1x1 that is not is the transit), so the
// reference topology (12 / 24 / 16 layers, dilations 1 / 2 / 2) and smaller test
// models load through the same walk. 2-D weights become f16 [oc][kt*3+kf][ic],
// 1-D weights f16 [oc][k][ic], runtime BatchNorms f32 scale / shift, and the
// affine-free output BatchNorm is folded into the dense head.
//
// Forward of one bucket:
//   FBank -> CMN + stem (3x3, FPHASE output) -> FCM: two stages of
//   [BasicResBlock freq-stride 2 (conv1 | conv2 + 1x1 shortcut fused as a second
//   K segment), BasicResBlock (conv1 | conv2 + identity segment)], the last one
//   writing the next stage's FPHASE input -> FCM conv2 (freq stride 2) writing the
//   TDNN's time-phase input directly (channel f*M + c; the TDNN weight's columns are
//   permuted to match the reference's c*F + f order) -> TDNN (k=5, time stride 2) ->
//   3 dense blocks, per layer: 1x1 conv over the concatenated features with their
//   BN + ReLU applied to each A tile in shared memory (the conv's input prologue) +
//   bias + ReLU, CAM gate (one kernel per layer: segment sums -> context -> 2 FCs
//   -> sigmoid per 100-frame segment), k=3 dilated conv whose epilogue multiplies by the gate and stores into
//   the features' next 32 channels; transit (BN + ReLU prologue, 1x1) ->
//   statistics pooling (mean, unbiased std) -> dense head (output BN folded) -> L2.
#include <cuda_fp16.h>

#include <algorithm>
#include <cmath>
#include <string>

#include "engine.hpp"
#include "gguf.hpp"
#include "vdb_internal.h"

namespace vdb {
namespace {

constexpr int kSeg = 100;                  // CAM context segment (src/encoder_campplus.cpp:162-181)
constexpr int kBlockDil[3] = {1, 2, 2};    // dilation per dense block (:184-185)

size_t align256(size_t n) { return (n + 255) & ~(size_t)255; }
inline int half_ext(int n) { return (n - 1) / 2 + 1; }

}  // namespace

bool Engine::load_campplus(const Gguf& g, std::string& err) {
    CamppDev& E = campp_;
    const std::string pre = "voicedetect.campplus.";
    const auto wn = g.str_arr(pre + "conv_weight");
    const auto bn = g.str_arr(pre + "conv_bias");
    const auto bp = g.str_arr(pre + "bn_prefix");
    const float eps = g.f32(pre + "bn_eps", 1e-5f);
    if (wn.empty() || bn.size() != wn.size()) {
        err = "campplus: inconsistent voicedetect.campplus.conv_weight / conv_bias manifest";
        return false;
    }
    // One conv in torch order [OC][IC][KF][KT] (2-D) or [OC][IC][K] (1-D, kt = 1).
    struct Cv {
        std::vector<float> w, b;
        int oc = 0, ic = 0, k = 1;
        bool two_d = false;
    };
    auto read = [&](size_t i, Cv& c) -> bool {
        const GgufTensor* t = g.tensor(wn[i]);
        if (!t) {
            err = "missing tensor '" + wn[i] + "'";
            return false;
        }
        if (!g.to_f32(*t, c.w, err)) return false;
        const auto& ne = t->ne;
        if (ne.size() == 4) {
            if (ne[0] != ne[1]) {
                err = "campplus: '" + wn[i] + "' must be a square 2-D kernel";
                return false;
            }
            c.two_d = true;
            c.k = (int)ne[0];
            c.ic = (int)ne[2];
            c.oc = (int)ne[3];
        } else if (ne.size() == 3) {
            c.k = (int)ne[0];
            c.ic = (int)ne[1];
            c.oc = (int)ne[2];
        } else if (ne.size() == 2) {  // squeezed 1x1
            c.k = 1;
            c.ic = (int)ne[0];
            c.oc = (int)ne[1];
        } else {
            err = "campplus: '" + wn[i] + "' is not a conv weight";
            return false;
        }
        c.b.clear();
        if (!bn[i].empty()) {
            const GgufTensor* tb = g.tensor(bn[i]);
            if (!tb) {
                err = "missing tensor '" + bn[i] + "'";
                return false;
            }
            if (!g.to_f32(*tb, c.b, err)) return false;
            if ((int)c.b.size() != c.oc) {
                err = "campplus: bias '" + bn[i] + "' does not match its conv";
                return false;
            }
        }
        return true;
    };
    size_t ci = 0, bi = 0;
    auto next = [&](Cv& c, bool two_d, int k, int ic) -> bool {
        if (ci >= wn.size()) {
            err = "campplus: the manifest has fewer convs than the topology needs";
            return false;
        }
        const size_t i = ci++;
        if (!read(i, c)) return false;
        if (c.two_d != two_d || c.k != k || (ic >= 0 && c.ic != ic)) {
            err = "campplus conv " + std::to_string(i) + " ('" + wn[i] + "'): expected a " +
                  (two_d ? "2-D " : "1-D ") + std::to_string(k) + "-tap kernel from " +
                  std::to_string(ic) + " channels, got " + (c.two_d ? "2-D " : "1-D ") +
                  std::to_string(c.k) + " taps from " + std::to_string(c.ic);
            return false;
        }
        return true;
    };
    auto need16 = [&](int c, const char* what) -> bool {
        if (c <= 0 || c % 16 != 0) {
            err = std::string("campplus: ") + what + " must be a positive multiple of 16 (got " +
                  std::to_string(c) + ")";
            return false;
        }
        return true;
    };
    // runtime BatchNorm (bn1d_cm, :72-133): scale = w / sqrt(var + eps), shift = b - scale*mean
    auto bnorm = [&](int C, float** sc, float** sh) -> bool {
        if (bi >= bp.size()) {
            err = "campplus: the manifest has fewer BatchNorms than the topology needs";
            return false;
        }
        const std::string p = bp[bi++];
        std::vector<float> v[4];
        const char* sfx[4] = {".weight", ".bias", ".running_mean", ".running_var"};
        for (int k = 0; k < 4; ++k) {
            const GgufTensor* t = g.tensor(p + sfx[k]);
            if (!t) {
                err = "missing tensor '" + p + sfx[k] + "'";
                return false;
            }
            if (!g.to_f32(*t, v[k], err)) return false;
            if ((int)v[k].size() != C) {
                err = "campplus: BatchNorm '" + p + "' has " + std::to_string(v[k].size()) +
                      " channels, expected " + std::to_string(C);
                return false;
            }
        }
        std::vector<float> s(C), t(C);
        for (int i = 0; i < C; ++i) {
            s[i] = v[0][i] / std::sqrt(v[3][i] + eps);
            t[i] = v[1][i] - s[i] * v[2][i];
        }
        return upload_f32(s, sc, err) && upload_f32(t, sh, err);
    };
    // 2-D conv -> f16 [oc][kt*k + kf][ic]
    auto pack2d = [](const Cv& c) {
        std::vector<float> out((size_t)c.oc * c.k * c.k * c.ic);
        for (int o = 0; o < c.oc; ++o)
            for (int kf = 0; kf < c.k; ++kf)
                for (int kt = 0; kt < c.k; ++kt)
                    for (int i = 0; i < c.ic; ++i)
                        out[((size_t)o * c.k * c.k + (size_t)kt * c.k + kf) * c.ic + i] =
                            c.w[(((size_t)o * c.ic + i) * c.k + kf) * c.k + kt];
        return out;
    };
    // 1-D conv -> f16 [oc][k][ic]
    auto pack1d = [](const Cv& c) {
        std::vector<float> out((size_t)c.oc * c.k * c.ic);
        for (int o = 0; o < c.oc; ++o)
            for (int j = 0; j < c.k; ++j)
                for (int i = 0; i < c.ic; ++i)
                    out[((size_t)o * c.k + j) * c.ic + i] = c.w[((size_t)o * c.ic + i) * c.k + j];
        return out;
    };
    auto sum_bias = [&](const Cv& a, const Cv* b, float** out) -> bool {
        *out = nullptr;
        if (a.b.empty() && (!b || b->b.empty())) return true;
        std::vector<float> s((size_t)a.oc, 0.0f);
        for (size_t i = 0; i < a.b.size(); ++i) s[i] += a.b[i];
        if (b)
            for (size_t i = 0; i < b->b.size(); ++i) s[i] += b->b[i];
        return upload_f32(s, out, err);
    };
    auto conv2d_dev = [&](const Cv& c, Fcm2dDev& d) -> bool {
        d.ic = c.ic;
        d.oc = c.oc;
        d.k = c.k;
        return upload_f16(pack2d(c), &d.w, err);
    };
    auto tdnn_dev = [&](const Cv& c, TdnnDev& d, int dil) -> bool {
        d.ic = c.ic;
        d.oc = c.oc;
        d.k = c.k;
        d.dil = dil;
        if (!upload_f16(pack1d(c), &d.w, err)) return false;
        d.b = nullptr;
        return c.b.empty() || upload_f32(c.b, &d.b, err);
    };

    // FCM stem (:219): 3x3 from 1 channel, BN folded (bias), ReLU
    Cv c0;
    if (!next(c0, true, 3, 1)) return false;
    const int M = c0.oc;
    if (!(M == 16 || M == 32 || M == 64)) {
        err = "campplus: the FCM stem must have 16, 32 or 64 channels";
        return false;
    }
    E.M = M;
    {
        std::vector<float> sw((size_t)M * 9);
        for (int o = 0; o < M; ++o)
            for (int kf = 0; kf < 3; ++kf)
                for (int kt = 0; kt < 3; ++kt) sw[(size_t)o * 9 + kt * 3 + kf] = c0.w[(size_t)o * 9 + kf * 3 + kt];
        std::vector<float> sb = c0.b.empty() ? std::vector<float>((size_t)M, 0.0f) : c0.b;
        if (!upload_f32(sw, &E.stem_w, err) || !upload_f32(sb, &E.stem_b, err)) return false;
    }
    // two stages of [stride-2 block (conv1, conv2, 1x1 shortcut), stride-1 block]
    // (fcm_basicres, :220-223), then conv2 (:224)
    for (int s = 0; s < 2; ++s) {
        Cv a1, a2, sc, b1, b2;
        if (!next(a1, true, 3, M) || !next(a2, true, 3, M) || !next(sc, true, 1, M) ||
            !next(b1, true, 3, M) || !next(b2, true, 3, M))
            return false;
        if (a1.oc != M || a2.oc != M || sc.oc != M || b1.oc != M || b2.oc != M) {
            err = "campplus: FCM blocks must keep the stem's channel count";
            return false;
        }
        CamppStageDev& st = E.stages[s];
        if (!conv2d_dev(a1, st.c1) || !sum_bias(a1, nullptr, &st.c1.b) || !conv2d_dev(a2, st.c2) ||
            !sum_bias(a2, &sc, &st.c2.b) || !upload_f16(pack1d(sc), &st.sc_w, err) ||
            !conv2d_dev(b1, st.c3) || !sum_bias(b1, nullptr, &st.c3.b) || !conv2d_dev(b2, st.c4) ||
            !sum_bias(b2, nullptr, &st.c4.b))
            return false;
    }
    {
        Cv c2;
        if (!next(c2, true, 3, M)) return false;
        if (c2.oc != M) {
            err = "campplus: FCM conv2 must keep the channel count";
            return false;
        }
        if (!conv2d_dev(c2, E.fcm_out) || !sum_bias(c2, nullptr, &E.fcm_out.b)) return false;
    }
    int F = cfg_.n_mels;
    for (int s = 0; s < 3; ++s) F = half_ext(F);
    E.f_out = F;
    // TDNN (:238-241): k=5, stride 2, pad 2 over M*F channels ordered c*F + f; the
    // time-phase input from the FCM holds them as f*M + c, so the columns are permuted
    {
        Cv t;
        if (!next(t, false, 5, M * F)) return false;
        if (!need16(t.oc, "TDNN channels")) return false;
        Cv p = t;
        for (int o = 0; o < t.oc; ++o)
            for (int c = 0; c < M; ++c)
                for (int f = 0; f < F; ++f)
                    for (int j = 0; j < 5; ++j)
                        p.w[((size_t)o * t.ic + f * M + c) * 5 + j] =
                            t.w[((size_t)o * t.ic + c * F + f) * 5 + j];
        if (!tdnn_dev(p, E.tdnn, 1)) return false;
    }
    // dense blocks (:243-281)
    int C = E.tdnn.oc;
    E.blocks.clear();
    E.bnc = 0;
    E.growth = 0;
    E.cam_m = 0;
    for (int blk = 0; ci + 1 < wn.size(); ++blk) {
        if (blk >= 3) {
            err = "campplus: more than 3 dense blocks in the manifest";
            return false;
        }
        CamppBlockDev B;
        B.dil = kBlockDil[blk];
        B.c0 = C;
        // a layer: the 1x1 (linear1) followed by the k=3 linear_local
        for (;;) {
            Cv probe;
            if (ci + 1 >= wn.size() || !read(ci + 1, probe)) {
                if (!err.empty()) return false;
                break;
            }
            if (probe.two_d || probe.k != 3) break;
            CamppLayerDev L;
            L.c_in = C;
            if (!need16(C, "dense block channels") || !bnorm(C, &L.bn_scale, &L.bn_shift))
                return false;
            Cv l1, lo, m1, m2;
            if (!next(l1, false, 1, C) || !next(lo, false, 3, l1.oc) || !next(m1, false, 1, l1.oc) ||
                !next(m2, false, 1, m1.oc))
                return false;
            if (!need16(l1.oc, "bottleneck channels") || !need16(lo.oc, "growth rate") ||
                m2.oc != lo.oc || !lo.b.empty()) {
                if (err.empty())
                    err = "campplus: CAM linear2 must match linear_local, which has no bias";
                return false;
            }
            if ((E.bnc && E.bnc != l1.oc) || (E.growth && E.growth != lo.oc) ||
                (E.cam_m && E.cam_m != m1.oc)) {
                err = "campplus: every dense layer must have the same widths";
                return false;
            }
            E.bnc = l1.oc;
            E.growth = lo.oc;
            E.cam_m = m1.oc;
            if (!tdnn_dev(l1, L.lin1, 1) || !tdnn_dev(lo, L.local, B.dil)) return false;
            std::vector<float> mb1 = m1.b.empty() ? std::vector<float>(m1.oc, 0.0f) : m1.b;
            std::vector<float> mb2 = m2.b.empty() ? std::vector<float>(m2.oc, 0.0f) : m2.b;
            // CAM FCs stored transposed ([in][out]) for the gate kernel
            auto transpose = [](const std::vector<float>& w, int rows, int cols) {
                std::vector<float> t(w.size());
                for (int r = 0; r < rows; ++r)
                    for (int c = 0; c < cols; ++c) t[(size_t)c * rows + r] = w[(size_t)r * cols + c];
                return t;
            };
            if (!upload_f32(transpose(m1.w, m1.oc, m1.ic), &L.cam_w1, err) ||
                !upload_f32(mb1, &L.cam_b1, err) ||
                !upload_f32(transpose(m2.w, m2.oc, m2.ic), &L.cam_w2, err) ||
                !upload_f32(mb2, &L.cam_b2, err))
                return false;
            B.layers.push_back(L);
            C += E.growth;
        }
        if (B.layers.empty()) {
            err = "campplus: a dense block without layers";
            return false;
        }
        B.cmax = C;
        // transit (:273-280): BN -> ReLU -> 1x1 halving; the last one is biased + ReLU
        if (!bnorm(C, &B.tr_scale, &B.tr_shift)) return false;
        Cv tr;
        if (!next(tr, false, 1, C)) return false;
        if (!need16(tr.oc, "transit channels") || !tdnn_dev(tr, B.transit, 1)) return false;
        C = tr.oc;
        E.blocks.push_back(B);
    }
    if (E.blocks.size() != 3) {
        err = "campplus: expected 3 dense blocks, found " + std::to_string(E.blocks.size());
        return false;
    }
    E.c_out = C;
    // dense head (:294-298) with the affine-free output BN folded: e*s - s*mean
    {
        Cv d;
        if (!next(d, false, 1, 2 * C)) return false;
        if (d.oc != cfg_.emb_dim || !d.b.empty()) {
            err = "campplus: the dense head must map 2C channels to embedding_dim without a bias";
            return false;
        }
        std::vector<float> mu, var;
        const GgufTensor* tm = g.tensor(g.str(pre + "emb_bn_mean"));
        const GgufTensor* tv = g.tensor(g.str(pre + "emb_bn_var"));
        if (!tm || !tv || !g.to_f32(*tm, mu, err) || !g.to_f32(*tv, var, err) ||
            (int)mu.size() != d.oc || (int)var.size() != d.oc) {
            if (err.empty()) err = "campplus: missing or mis-sized output BatchNorm statistics";
            return false;
        }
        std::vector<float> w2((size_t)d.oc * d.ic), b2(d.oc);
        for (int o = 0; o < d.oc; ++o) {
            const float s = 1.0f / std::sqrt(var[o] + eps);
            for (int i = 0; i < d.ic; ++i) w2[(size_t)o * d.ic + i] = d.w[(size_t)o * d.ic + i] * s;
            b2[o] = -s * mu[o];
        }
        if (!upload_f32(w2, &E.fc_w, err) || !upload_f32(b2, &E.fc_b, err)) return false;
    }
    if (ci != wn.size() || bi != bp.size()) {
        err = "campplus: the manifest has " + std::to_string(wn.size() - ci) + " convs and " +
              std::to_string(bp.size() - bi) + " BatchNorms left over";
        return false;
    }
    // metadata levels: frames, TDNN frames
    levels_.assign(2, Level{});
    return true;
}

size_t Engine::campp_ws_bytes(int B, int t_max) const {
    const CamppDev& E = campp_;
    const int T = t_max, Tq = half_ext(T), P = E.pad;
    const int F0 = cfg_.n_mels, F1 = half_ext(F0), F2 = half_ext(F1), F3 = half_ext(F2);
    const size_t h = sizeof(__half), f = sizeof(float);
    const size_t M = (size_t)E.M;
    const size_t R = (size_t)vdb_seq_rows(B, Tq, P);
    int cmax = 0;
    for (const CamppBlockDev& b : E.blocks) cmax = std::max(cmax, b.cmax);
    const int nseg = (Tq + kSeg - 1) / kSeg;
    size_t n = 0;
    n += align256(2 * (size_t)B * (T + 2) * (F1 + 2) * M * h);            // stem FPHASE
    n += 3 * align256((size_t)vdb_grid_rows(B, T, F1) * M * h);           // stage 1 grids
    n += align256(2 * (size_t)B * (T + 2) * (F2 + 2) * M * h);            // stage 2 FPHASE
    n += 3 * align256((size_t)vdb_grid_rows(B, T, F2) * M * h);           // stage 2 grids
    n += align256(2 * (size_t)B * (T + 2) * (F3 + 2) * M * h);            // conv2 FPHASE
    n += align256(2 * R * F3 * M * h);                                    // TDNN TPHASE input
    n += 2 * align256(R * cmax * h);                                      // dense features
    n += align256(R * E.bnc * h);                                         // CAM input
    n += align256((size_t)B * nseg * E.growth * f);                       // CAM gate
    n += align256((size_t)B * 2 * E.c_out * f);                           // statistics
    n += align256((size_t)pool_fc_splits(B, 2 * E.c_out, cfg_.emb_dim) * B * cfg_.emb_dim * f);
    return n;
}

int Engine::run_campplus(int B, int t_max, const std::vector<long long>& tv_sum, cudaStream_t st,
                         float* d_out, long long& launches, std::string& err) {
    const CamppDev& E = campp_;
    const int T = t_max, Tq = half_ext(T), P = E.pad, M = E.M;
    const int F0 = cfg_.n_mels, F1 = half_ext(F0), F2 = half_ext(F1), F3 = half_ext(F2);
    const size_t R = (size_t)vdb_seq_rows(B, Tq, P);
    const int* tv = meta_;        // frames
    const int* tq = meta_ + B;    // TDNN frames
    const double frames = (double)tv_sum[0], qframes = (double)tv_sum[1];
    int cmax = 0;
    for (const CamppBlockDev& b : E.blocks) cmax = std::max(cmax, b.cmax);
    const int nseg = (Tq + kSeg - 1) / kSeg;
    char* cur = static_cast<char*>(ecapa_ws_);
    auto take = [&](size_t bytes) -> void* {
        void* p = cur;
        cur += align256(bytes);
        return p;
    };
    const size_t h = sizeof(__half), f = sizeof(float);
    __half* fp0 = (__half*)take(2 * (size_t)B * (T + 2) * (F1 + 2) * M * h);
    __half* g1[3];
    for (auto& p : g1) p = (__half*)take((size_t)vdb_grid_rows(B, T, F1) * M * h);
    __half* fp1 = (__half*)take(2 * (size_t)B * (T + 2) * (F2 + 2) * M * h);
    __half* g2[3];
    for (auto& p : g2) p = (__half*)take((size_t)vdb_grid_rows(B, T, F2) * M * h);
    __half* fp2 = (__half*)take(2 * (size_t)B * (T + 2) * (F3 + 2) * M * h);
    const size_t ts_bytes = 2 * R * F3 * M * h;
    __half* ts = (__half*)take(ts_bytes);
    __half* hb[2] = {(__half*)take(R * cmax * h), (__half*)take(R * cmax * h)};
    __half* cc = (__half*)take(R * E.bnc * h);
    float* gate = (float*)take((size_t)B * nseg * E.growth * f);
    float* stats = (float*)take((size_t)B * 2 * E.c_out * f);
    float* part = (float*)take((size_t)pool_fc_splits(B, 2 * E.c_out, cfg_.emb_dim) * B *
                               cfg_.emb_dim * f);
    auto fail = [&]() -> int {
        err = vdb_last_error();
        return 1;
    };

    // CMN + stem -> FPHASE
    {
        const int ps = prof_begin(st, 4);
        if (cmn_stem_launch(feats_, tv, B, T, F0, cfg_.cmn ? 1 : 0, E.stem_w, E.stem_b, M, mean_,
                            fp0, 1, st))
            return fail();
        prof_end(ps, st, 0.0);
        launches += cfg_.cmn ? 2 : 1;
    }
    // The TDNN's time-phase input has padding rows and slots no frame maps to.
    VDB_CHECK_CUDA(cudaMemsetAsync(ts, 0, ts_bytes, st));

    auto conv2d = [&](int f_out, int oc, int k0, int stride0, int ic0, const void* x0,
                      const __half* w0, const float* bias, void* y, int y_phase) {
        vdb_conv_args a{};
        a.batch = B;
        a.t_out = T;
        a.f_out = f_out;
        a.oc = oc;
        a.k0 = k0;
        a.stride0 = stride0;
        a.ic0 = ic0;
        a.x0 = x0;
        a.w0 = w0;
        a.bias = bias;
        a.relu = 1;
        a.tvalid = tv;
        a.y = y;
        a.y_phase = y_phase;
        a.err = errword_;
        return a;
    };
    auto run2d = [&](const vdb_conv_args& a, double flops) -> int {
        const int pe = prof_begin(st);
        if (vdb_conv(&a, st)) return fail();
        prof_end(pe, st, flops);
        ++launches;
        return 0;
    };
    // FCM stages
    const void* fin = fp0;
    int Fo = F1;
    for (int s = 0; s < 2; ++s) {
        const CamppStageDev& S = E.stages[s];
        __half** g = s == 0 ? g1 : g2;
        __half* fnext = s == 0 ? fp1 : fp2;
        const double px = frames * Fo;
        // block 0: conv1 (freq stride 2) | conv2 + 1x1 shortcut (freq stride 2)
        if (run2d(conv2d(Fo, M, 3, 3, M, fin, S.c1.w, S.c1.b, g[0], 0), 2.0 * M * M * 9 * px))
            return 1;
        {
            vdb_conv_args a = conv2d(Fo, M, 3, 1, M, g[0], S.c2.w, S.c2.b, g[1], 0);
            a.x1 = fin;
            a.w1 = S.sc_w;
            a.ic1 = M;
            a.stride1 = 3;
            if (run2d(a, 2.0 * M * M * 10 * px)) return 1;
        }
        // block 1: conv1 | conv2 + identity, written as the next stage's FPHASE input
        if (run2d(conv2d(Fo, M, 3, 1, M, g[1], S.c3.w, S.c3.b, g[2], 0), 2.0 * M * M * 9 * px))
            return 1;
        {
            vdb_conv_args a = conv2d(Fo, M, 3, 1, M, g[2], S.c4.w, S.c4.b, fnext, 2);
            const __half* id = identity(M, err);
            if (!id) return 1;
            a.x1 = g[1];
            a.w1 = id;
            a.ic1 = M;
            a.stride1 = 1;
            if (run2d(a, 2.0 * M * M * 9 * px)) return 1;
        }
        fin = fnext;
        Fo = half_ext(Fo);
    }
    // FCM conv2 (freq stride 2) -> the TDNN's TPHASE input
    {
        vdb_conv_args a = conv2d(F3, M, 3, 3, M, fin, E.fcm_out.w, E.fcm_out.b, ts, 3);
        a.y_pad = P;
        if (run2d(a, 2.0 * M * M * 9 * frames * F3)) return 1;
    }
    auto conv1 = [&](const TdnnDev& d, const __half* x, int ldx, void* y, int ldy) {
        vdb_conv1d_args a{};
        a.batch = B;
        a.t = Tq;
        a.pad = P;
        a.oc = d.oc;
        a.k0 = d.k;
        a.dil0 = d.dil;
        a.ic0 = d.ic;
        a.x0 = x;
        a.ldx0 = ldx;
        a.w0 = d.w;
        a.bias = d.b;
        a.act = 0;
        a.tvalid = tq;
        a.y = y;
        a.ldy = ldy;
        a.reflect = 2;
        a.err = errword_;
        return a;
    };
    auto run1d = [&](const vdb_conv1d_args& a, double flops) -> int {
        const int pe = prof_begin(st);
        if (vdb_conv1d(&a, st)) return fail();
        prof_end(pe, st, flops);
        ++launches;
        return 0;
    };
    // TDNN: k=5, time stride 2 -> block 0's features, channels [0, C0)
    int hi = 0;
    {
        vdb_conv1d_args a = conv1(E.tdnn, ts, E.tdnn.ic, hb[0], E.blocks[0].cmax);
        a.stride0 = 2;
        a.relu = 1;
        if (run1d(a, 2.0 * E.tdnn.oc * E.tdnn.ic * 5 * qframes)) return 1;
    }
    for (size_t bi = 0; bi < E.blocks.size(); ++bi) {
        const CamppBlockDev& Bk = E.blocks[bi];
        __half* hcur = hb[hi];
        const int ld = Bk.cmax;
        int C = Bk.c0;
        for (const CamppLayerDev& L : Bk.layers) {
            // nonlinear1 (BN + ReLU of the first C channels) as the 1x1 conv's input
            // prologue, then + bias, ReLU
            {
                vdb_conv1d_args a = conv1(L.lin1, hcur, ld, cc, E.bnc);
                a.x_scale = L.bn_scale;
                a.x_shift = L.bn_shift;
                a.relu = 1;
                if (run1d(a, 2.0 * E.bnc * C * qframes)) return 1;
            }
            const int pc = prof_begin(st, 3);
            if (campp_cam_gate(cc, E.bnc, tq, B, Tq, P, E.bnc, kSeg, nseg, L.cam_w1, L.cam_b1,
                               E.cam_m, L.cam_w2, L.cam_b2, E.growth, gate, st))
                return fail();
            prof_end(pc, st, 0.0);
            ++launches;
            {
                vdb_conv1d_args a = conv1(L.local, cc, E.bnc, hcur + C, ld);
                a.act = 5;
                a.gate = gate;
                a.gate_seg = kSeg;
                a.gate_nseg = nseg;
                if (run1d(a, 2.0 * E.growth * E.bnc * 3 * qframes)) return 1;
            }
            C += E.growth;
        }
        // transit (BN + ReLU prologue, 1x1) into the next block's features (or the
        // pooling input)
        hi ^= 1;
        const int ldn = bi + 1 < E.blocks.size() ? E.blocks[bi + 1].cmax : Bk.transit.oc;
        vdb_conv1d_args a = conv1(Bk.transit, hcur, ld, hb[hi], ldn);
        a.x_scale = Bk.tr_scale;
        a.x_shift = Bk.tr_shift;
        a.relu = bi + 1 == E.blocks.size() ? 1 : 0;
        if (run1d(a, 2.0 * Bk.transit.oc * C * qframes)) return 1;
    }
    // statistics pooling + dense head (output BN folded) + L2
    const int pp = prof_begin(st, 2);
    if (seq_meanstd_unbiased(hb[hi], E.c_out, tq, B, Tq, P, E.c_out, stats, st) ||
        fc_embed_launch(stats, B, 2 * E.c_out, E.fc_w, E.fc_b, nullptr, cfg_.emb_dim,
                        cfg_.l2 ? 1 : 0, meta_ + (size_t)levels_.size() * B, d_out, nullptr, part,
                        st))
        return fail();
    prof_end(pp, st, 0.0);
    launches += 3;
    return 0;
}

}  // namespace vdb
