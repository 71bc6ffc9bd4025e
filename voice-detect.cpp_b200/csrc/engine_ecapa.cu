// ECAPA-TDNN on the B200 engine: the counterpart of the reference's EcapaEncoder
// (src/encoder.cpp:157-340) over a length-bucketed batch.
//
// Load (src/encoder.cpp weight names, kept verbatim by the converter): every
// Conv1d becomes f16 [oc][k][ic] for vdb_conv1d, every eval BatchNorm a folded
// scale / shift (the reference's bn1d_eval arithmetic, :125-151), and the
// embedding head's asp_bn is folded into the fc weights. Two weights are split by
// columns so that no concatenation is ever materialised:
//   tdnn2       reads concat(x_0, y_1 .. y_{s-1}): group 0's columns are input
//               segment 0 (a channel slice of tdnn1's output), the rest segment 1
//               (the Res2Net output buffer from channel C/s on);
//   asp.tdnn    reads concat(x, mean, std): the x columns run on the tensor cores,
//               the mean / std columns become a per-clip bias (ecapa.cu, ASP note).
//
// Forward of one bucket (SEQ layout, pad = the widest conv reach):
//   CMN + pack -> stem (k=5) -> per SE-Res2Net block: tdnn1 -> scale-1 dilated
//   convs, each writing y_g into its slice and x_{g+1} + y_g (the next group's
//   input, reflect-padded) as a second output -> tdnn2 -> SE mean / FCs / apply
//   into its slice of the MFA input -> MFA -> global mean / std -> attention
//   tdnn (+ per-clip context bias, tanh) -> attention logits (f32) -> softmax
//   pooling -> fc (asp_bn folded) -> L2.
#include <cuda_fp16.h>

#include <algorithm>
#include <cmath>
#include <string>

#include "engine.hpp"
#include "gguf.hpp"
#include "vdb_internal.h"

namespace vdb {
namespace {

constexpr float kBnEps = 1e-5f;    // BatchNorm1d eps (src/encoder.cpp:13)
constexpr float kAspEps = 1e-12f;  // ASP variance floor (src/encoder.cpp:19)

size_t align256(size_t n) { return (n + 255) & ~(size_t)255; }

}  // namespace

bool Engine::load_ecapa(const Gguf& g, std::string& err) {
    EcapaDev& E = ecapa_;
    // Conv1d weight in torch order [OC][IC][K]. f32 tensors keep ggml ne = [K, IC, OC];
    // the converter stores quantised 1x1 weights squeezed to 2-D, ne = [IC, OC].
    auto conv1d = [&](const std::string& name, std::vector<float>& w, int& oc, int& ic,
                      int& k) -> bool {
        const GgufTensor* t = g.tensor(name);
        if (!t) {
            err = "missing tensor '" + name + "'";
            return false;
        }
        if (!g.to_f32(*t, w, err)) return false;
        if (t->ne.size() == 2) {
            k = 1;
            ic = (int)t->ne[0];
            oc = (int)t->ne[1];
        } else if (t->ne.size() == 3) {
            k = (int)t->ne[0];
            ic = (int)t->ne[1];
            oc = (int)t->ne[2];
        } else {
            err = "tensor '" + name + "': expected a Conv1d weight";
            return false;
        }
        return true;
    };
    auto vec = [&](const std::string& name, std::vector<float>& v, int n) -> bool {
        const GgufTensor* t = g.tensor(name);
        if (!t) {
            err = "missing tensor '" + name + "'";
            return false;
        }
        if (!g.to_f32(*t, v, err)) return false;
        if ((int)v.size() != n) {
            err = "tensor '" + name + "' has " + std::to_string(v.size()) + " elements, expected " +
                  std::to_string(n);
            return false;
        }
        return true;
    };
    // BatchNorm1d eval folded to scale / shift exactly as bn1d_eval (:130-142).
    auto bn = [&](const std::string& p, int C, std::vector<float>& sc,
                  std::vector<float>& sh) -> bool {
        std::vector<float> gm, bt, mu, var;
        if (!vec(p + ".weight", gm, C) || !vec(p + ".bias", bt, C) ||
            !vec(p + ".running_mean", mu, C) || !vec(p + ".running_var", var, C))
            return false;
        sc.resize(C);
        sh.resize(C);
        for (int i = 0; i < C; ++i) {
            const float inv = gm[i] / std::sqrt(var[i] + kBnEps);
            sc[i] = inv;
            sh[i] = bt[i] - inv * mu[i];
        }
        return true;
    };
    // torch [OC][IC][K] (columns [c0, c0 + n) of IC) -> [OC][K][n]
    auto pack = [](const std::vector<float>& w, int oc, int ic, int k, int c0, int n) {
        std::vector<float> out((size_t)oc * k * n);
        for (int o = 0; o < oc; ++o)
            for (int j = 0; j < k; ++j)
                for (int i = 0; i < n; ++i)
                    out[((size_t)o * k + j) * n + i] = w[((size_t)o * ic + c0 + i) * k + j];
        return out;
    };
    // One TDNN unit: <prefix>.conv.conv.{weight,bias} [+ <prefix>.norm.norm.*]
    auto tdnn = [&](const std::string& prefix, TdnnDev& d, int ic_expect, int dil, bool with_bn,
                    int col0, int ncols) -> bool {
        std::vector<float> w, b, sc, sh;
        int oc, ic, k;
        if (!conv1d(prefix + ".conv.conv.weight", w, oc, ic, k)) return false;
        if (ic_expect >= 0 && ic != ic_expect) {
            err = "'" + prefix + "': expected " + std::to_string(ic_expect) + " input channels, got " +
                  std::to_string(ic);
            return false;
        }
        if (!vec(prefix + ".conv.conv.bias", b, oc)) return false;
        if (with_bn && !bn(prefix + ".norm.norm", oc, sc, sh)) return false;
        if (ncols < 0) ncols = ic - col0;
        d.ic = ncols;
        d.oc = oc;
        d.k = k;
        d.dil = dil;
        if (!upload_f16(pack(w, oc, ic, k, col0, ncols), &d.w, err) || !upload_f32(b, &d.b, err))
            return false;
        if (with_bn && (!upload_f32(sc, &d.scale, err) || !upload_f32(sh, &d.shift, err)))
            return false;
        return true;
    };
    auto need16 = [&](int c, const char* what) -> bool {
        if (c <= 0 || c % 16 != 0) {
            err = std::string("ecapa: ") + what + " must be a positive multiple of 16 (got " +
                  std::to_string(c) + ")";
            return false;
        }
        return true;
    };

    const int nmel = cfg_.n_mels;
    if (!need16(nmel, "n_mels")) return false;
    // block0: TDNNBlock(k=5) (:303-307)
    if (!tdnn("blocks.0", E.stem, nmel, 1, true, 0, -1)) return false;
    if (E.stem.k % 2 == 0 || E.stem.k > 9) {
        err = "ecapa: blocks.0 kernel must be odd and <= 9";
        return false;
    }
    E.C = E.stem.oc;
    const int C = E.C;
    if (!need16(C, "channels")) return false;
    E.pad = (E.stem.k - 1) / 2;
    // SE-Res2Net blocks 1.. (:316-324), dilation idx + 1
    for (int i = 1; g.tensor("blocks." + std::to_string(i) + ".tdnn1.conv.conv.weight"); ++i) {
        const std::string p = "blocks." + std::to_string(i);
        EcapaBlockDev blk;
        blk.dil = i + 1;
        if (!tdnn(p + ".tdnn1", blk.tdnn1, C, 1, true, 0, -1)) return false;
        int scale = 1;
        while (g.tensor(p + ".res2net_block.blocks." + std::to_string(scale - 1) +
                        ".conv.conv.weight"))
            ++scale;
        if (blk.tdnn1.oc != C || blk.tdnn1.k != 1 || scale < 2 || C % scale != 0) {
            err = "ecapa: " + p + " must keep C channels with a 1x1 tdnn1 and a Res2Net scale "
                  "that divides C";
            return false;
        }
        const int w = C / scale;
        if (!need16(w, "Res2Net group width")) return false;
        if (E.scale && E.scale != scale) {
            err = "ecapa: every block must use the same Res2Net scale";
            return false;
        }
        E.scale = scale;
        for (int j = 0; j + 1 < scale; ++j) {
            TdnnDev gd;
            if (!tdnn(p + ".res2net_block.blocks." + std::to_string(j), gd, w, blk.dil, true, 0, -1))
                return false;
            if (gd.oc != w || gd.k % 2 == 0 || gd.k > 9) {
                err = "ecapa: Res2Net convs must keep the group width with an odd kernel <= 9";
                return false;
            }
            E.pad = std::max(E.pad, (gd.k - 1) / 2 * gd.dil);
            blk.groups.push_back(gd);
        }
        // tdnn2 split by input columns: group 0 | groups 1..
        if (!tdnn(p + ".tdnn2", blk.tdnn2, C, 1, true, 0, w)) return false;
        {
            std::vector<float> w2;
            int oc, ic, k;
            if (!conv1d(p + ".tdnn2.conv.conv.weight", w2, oc, ic, k)) return false;
            if (oc != C || k != 1) {
                err = "ecapa: " + p + ".tdnn2 must be a 1x1 conv to C channels";
                return false;
            }
            if (!upload_f16(pack(w2, oc, ic, 1, w, C - w), &blk.tdnn2_w_rest, err)) return false;
        }
        // SE block (:196-209): conv1 C->se, conv2 se->C, no BatchNorm
        {
            std::vector<float> w1, b1, w2, b2;
            int oc1, ic1, k1, oc2, ic2, k2;
            if (!conv1d(p + ".se_block.conv1.conv.weight", w1, oc1, ic1, k1) ||
                !conv1d(p + ".se_block.conv2.conv.weight", w2, oc2, ic2, k2))
                return false;
            if (ic1 != C || k1 != 1 || oc2 != C || ic2 != oc1 || k2 != 1) {
                err = "ecapa: " + p + ".se_block shapes do not match C";
                return false;
            }
            if (!vec(p + ".se_block.conv1.conv.bias", b1, oc1) ||
                !vec(p + ".se_block.conv2.conv.bias", b2, oc2))
                return false;
            blk.se = oc1;
            if (!upload_f32(w1, &blk.se_w1, err) || !upload_f32(b1, &blk.se_b1, err) ||
                !upload_f32(w2, &blk.se_w2, err) || !upload_f32(b2, &blk.se_b2, err))
                return false;
        }
        E.blocks.push_back(std::move(blk));
    }
    const int nb = (int)E.blocks.size();
    if (nb == 0) {
        err = "ecapa: no SE-Res2Net blocks (blocks.1.tdnn1.* missing)";
        return false;
    }
    // MFA over the concatenated block outputs (:327-334)
    if (!tdnn("mfa", E.mfa, nb * C, 1, true, 0, -1)) return false;
    E.Cm = E.mfa.oc;
    if (!need16(E.Cm, "MFA channels") || E.mfa.k != 1) {
        if (err.empty()) err = "ecapa: mfa must be a 1x1 conv";
        return false;
    }
    const int Cm = E.Cm;
    // ASP attention (:266-275): asp.tdnn over [x; mean; std] split by columns
    if (!tdnn("asp.tdnn", E.asp_tdnn, 3 * Cm, 1, true, 0, Cm)) return false;
    E.att = E.asp_tdnn.oc;
    if (!need16(E.att, "attention channels") || E.asp_tdnn.k != 1) {
        if (err.empty()) err = "ecapa: asp.tdnn must be a 1x1 conv";
        return false;
    }
    {
        std::vector<float> wa;
        int oc, ic, k;
        if (!conv1d("asp.tdnn.conv.conv.weight", wa, oc, ic, k)) return false;
        std::vector<float> ctx((size_t)oc * 2 * Cm);
        for (int o = 0; o < oc; ++o)
            for (int i = 0; i < 2 * Cm; ++i) ctx[(size_t)o * 2 * Cm + i] = wa[(size_t)o * ic + Cm + i];
        if (!upload_f32(ctx, &E.asp_ctx_w, err)) return false;
    }
    // asp.conv is a bare Conv1d: its tensors are asp.conv.conv.{weight,bias}
    if (!tdnn("asp", E.asp_conv, E.att, 1, false, 0, -1)) return false;
    if (E.asp_conv.oc != Cm || E.asp_conv.k != 1) {
        err = "ecapa: asp.conv must map the attention channels back to the MFA channels";
        return false;
    }
    // Head (:339-351): asp_bn over 2*Cm, then fc (fc.conv.{weight,bias}); asp_bn folded:
    // W' = W diag(s), b' = b + W t.
    {
        std::vector<float> sc, sh, fw, fb;
        if (!bn("asp_bn.norm", 2 * Cm, sc, sh)) return false;
        int oc, ic, k;
        if (!conv1d("fc.conv.weight", fw, oc, ic, k)) return false;
        if (ic != 2 * Cm || k != 1 || oc != cfg_.emb_dim) {
            err = "ecapa: fc must map 2*MFA channels to embedding_dim";
            return false;
        }
        if (!vec("fc.conv.bias", fb, oc)) return false;
        std::vector<float> w2((size_t)oc * ic), b2(oc);
        for (int o = 0; o < oc; ++o) {
            double acc = fb[o];
            for (int i = 0; i < ic; ++i) {
                w2[(size_t)o * ic + i] = fw[(size_t)o * ic + i] * sc[i];
                acc += (double)fw[(size_t)o * ic + i] * sh[i];
            }
            b2[o] = (float)acc;
        }
        if (!upload_f32(w2, &E.fc_w, err) || !upload_f32(b2, &E.fc_b, err)) return false;
    }
    // metadata: one level (frames)
    levels_.assign(1, Level{});
    return true;
}

// split-K partials of the per-clip FCs (SE squeeze / excite, attention context)
size_t Engine::ecapa_gemm_scratch(int B) const {
    const EcapaDev& E = ecapa_;
    size_t n = small_gemm_scratch_floats(B, 2 * E.Cm, E.att);
    for (const EcapaBlockDev& b : E.blocks)
        n = std::max({n, small_gemm_scratch_floats(B, E.C, b.se),
                      small_gemm_scratch_floats(B, b.se, E.C)});
    return n;
}

size_t Engine::ecapa_ws_bytes(int B, int t_max) const {
    const EcapaDev& E = ecapa_;
    const size_t R = (size_t)vdb_seq_rows(B, t_max, E.pad);
    const int nb = (int)E.blocks.size();
    const int w = E.C / E.scale;
    int se = 0;
    for (const EcapaBlockDev& b : E.blocks) se = std::max(se, b.se);
    const size_t h = sizeof(__half), f = sizeof(float);
    size_t n = 0;
    n += align256(R * cfg_.n_mels * h);                       // x0
    n += 4 * align256(R * E.C * h);                           // a0, t1, res2net out, h
    n += 2 * align256(R * w * h);                             // group input ping-pong
    n += align256(R * (size_t)nb * E.C * h);                  // MFA input
    n += align256(R * E.Cm * h);                              // MFA output
    n += align256(R * E.att * h);                             // attention tdnn
    n += align256(R * E.Cm * f);                              // attention logits
    n += 2 * align256((size_t)B * E.C * f) + align256((size_t)B * se * f);  // SE
    n += 2 * align256((size_t)B * 2 * E.Cm * f) + align256((size_t)B * E.att * f);
    n += align256((size_t)pool_fc_splits(B, 2 * E.Cm, cfg_.emb_dim) * B * cfg_.emb_dim * f);
    n += align256(ecapa_gemm_scratch(B) * f);
    return n;
}

int Engine::run_ecapa(int B, int t_max, const std::vector<long long>& tv_sum, cudaStream_t st,
                      float* d_out, long long& launches, std::string& err) {
    const EcapaDev& E = ecapa_;
    const int T = t_max, P = E.pad, C = E.C, Cm = E.Cm, att = E.att;
    const int nb = (int)E.blocks.size();
    const int w = C / E.scale;
    const size_t R = (size_t)vdb_seq_rows(B, T, P);
    const int* tv = meta_;
    const double frames = (double)tv_sum[0];
    // carve the workspace (ecapa_ws_bytes order)
    char* cur = static_cast<char*>(ecapa_ws_);
    auto take = [&](size_t bytes) -> void* {
        void* p = cur;
        cur += align256(bytes);
        return p;
    };
    const size_t h = sizeof(__half), f = sizeof(float);
    int se = 0;
    for (const EcapaBlockDev& b : E.blocks) se = std::max(se, b.se);
    __half* x0 = (__half*)take(R * cfg_.n_mels * h);
    __half* a0 = (__half*)take(R * C * h);
    __half* t1 = (__half*)take(R * C * h);
    __half* ro = (__half*)take(R * C * h);
    __half* hb = (__half*)take(R * C * h);
    __half* sbuf[2] = {(__half*)take(R * w * h), (__half*)take(R * w * h)};
    __half* cat = (__half*)take(R * (size_t)nb * C * h);
    __half* mf = (__half*)take(R * Cm * h);
    __half* at = (__half*)take(R * att * h);
    float* lg = (float*)take(R * Cm * f);
    float* se_s = (float*)take((size_t)B * C * f);
    float* se_g = (float*)take((size_t)B * C * f);
    float* se_z = (float*)take((size_t)B * se * f);
    float* stats = (float*)take((size_t)B * 2 * Cm * f);
    float* pooled = (float*)take((size_t)B * 2 * Cm * f);
    float* cb = (float*)take((size_t)B * att * f);
    float* part = (float*)take((size_t)pool_fc_splits(B, 2 * Cm, cfg_.emb_dim) * B *
                               cfg_.emb_dim * f);
    float* gpart = (float*)take(ecapa_gemm_scratch(B) * f);

    auto fail = [&]() -> int {
        err = vdb_last_error();
        return 1;
    };
    // one TDNN conv through vdb_conv1d
    auto conv = [&](const TdnnDev& d, const __half* x, int ldx, void* y, int ldy, int act,
                    int reflect) -> vdb_conv1d_args {
        vdb_conv1d_args a{};
        a.batch = B;
        a.t = T;
        a.pad = P;
        a.oc = d.oc;
        a.k0 = d.k;
        a.dil0 = d.dil;
        a.ic0 = d.ic;
        a.x0 = x;
        a.ldx0 = ldx;
        a.w0 = d.w;
        a.bias = d.b;
        a.bn_scale = d.scale;
        a.bn_shift = d.shift;
        a.act = act;
        a.tvalid = tv;
        a.y = y;
        a.ldy = ldy;
        a.reflect = reflect;
        a.err = errword_;
        return a;
    };
    auto launch = [&](const vdb_conv1d_args& a, double flops) -> int {
        const int pe = prof_begin(st);
        if (vdb_conv1d(&a, st)) return fail();
        prof_end(pe, st, flops);
        ++launches;
        return 0;
    };

    int pc = prof_begin(st, 4);
    if (ecapa_cmn_pack(feats_, tv, B, T, cfg_.n_mels, cfg_.cmn ? 1 : 0, P, x0, st)) return fail();
    prof_end(pc, st, 0.0);
    ++launches;
    // block0 (a CTA-pair tiling: its narrow K blocks make it feed-bound, and halving
    // each CTA's weight loads measured ~16% faster)
    {
        vdb_conv1d_args a = conv(E.stem, x0, cfg_.n_mels, a0, C, 3, 0);
        a.pair = 1;
        if (launch(a, 2.0 * C * cfg_.n_mels * E.stem.k * frames)) return 1;
    }
    const __half* in = a0;
    int ld_in = C;
    for (int bi = 0; bi < nb; ++bi) {
        const EcapaBlockDev& blk = E.blocks[bi];
        // tdnn1 (reflect-padded: group 1 reads a slice of it with dilated taps)
        if (launch(conv(blk.tdnn1, in, ld_in, t1, C, 3, 1), 2.0 * C * C * frames)) return 1;
        // Res2Net groups 1 .. scale-1 (:175-194)
        for (int gi = 1; gi < E.scale; ++gi) {
            const TdnnDev& gd = blk.groups[gi - 1];
            const __half* xs = gi == 1 ? t1 + w : sbuf[gi % 2];
            vdb_conv1d_args a = conv(gd, xs, gi == 1 ? C : w, ro + (size_t)gi * w, C, 3, 1);
            if (gi + 1 < E.scale) {
                a.ysum = sbuf[(gi + 1) % 2];
                a.ldsum = w;
                a.addend = t1 + (size_t)(gi + 1) * w;
                a.ldaddend = C;
            }
            if (launch(a, 2.0 * w * w * gd.k * frames)) return 1;
        }
        // tdnn2 over concat(x_0, y_1..): two input segments
        {
            vdb_conv1d_args a = conv(blk.tdnn2, t1, C, hb, C, 3, 0);
            a.x1 = ro + w;
            a.ldx1 = C;
            a.ic1 = C - w;
            a.w1 = blk.tdnn2_w_rest;
            if (launch(a, 2.0 * C * C * frames)) return 1;
        }
        // SE (:196-209) + residual (:229), written into the block's MFA input slice
        const int ps = prof_begin(st, 3);
        if (ecapa_seq_mean(hb, C, tv, B, T, P, C, se_s, st) ||
            small_gemm_launch(se_s, B, C, blk.se_w1, blk.se, blk.se_b1, 1, se_z, gpart, st) ||
            small_gemm_launch(se_z, B, blk.se, blk.se_w2, C, blk.se_b2, 2, se_g, gpart, st) ||
            ecapa_se_apply(hb, C, se_g, in, ld_in, tv, B, T, P, C, cat + (size_t)bi * C, nb * C,
                           st))
            return fail();
        prof_end(ps, st, 0.0);
        launches += 6;  // mean, 2 x (split-K GEMM + finish), apply
        in = cat + (size_t)bi * C;
        ld_in = nb * C;
    }
    // MFA (:327-334)
    if (launch(conv(E.mfa, cat, nb * C, mf, Cm, 3, 0), 2.0 * Cm * nb * C * frames)) return 1;
    // ASP (:246-285)
    const int pa = prof_begin(st, 2);
    if (ecapa_meanstd(mf, Cm, tv, B, T, P, Cm, kAspEps, stats, st) ||
        small_gemm_launch(stats, B, 2 * Cm, E.asp_ctx_w, att, E.asp_tdnn.b, 0, cb, gpart, st))
        return fail();
    prof_end(pa, st, 0.0);
    launches += 3;  // mean / std, split-K GEMM + finish
    {
        vdb_conv1d_args a = conv(E.asp_tdnn, mf, Cm, at, att, 4, 0);
        a.bias = nullptr;  // the conv bias is inside the per-clip context bias
        a.clip_bias = cb;
        if (launch(a, 2.0 * att * Cm * frames)) return 1;
    }
    {
        vdb_conv1d_args a = conv(E.asp_conv, at, att, lg, Cm, 0, 0);
        a.y_f32 = 1;
        if (launch(a, 2.0 * Cm * att * frames)) return 1;
    }
    const int pp = prof_begin(st, 2);
    if (ecapa_asp_pool(lg, Cm, mf, Cm, stats, tv, B, T, P, Cm, kAspEps, pooled, st)) return fail();
    // head: fc (asp_bn folded) + host-side-equivalent L2 (:339-372)
    if (fc_embed_launch(pooled, B, 2 * Cm, E.fc_w, E.fc_b, nullptr, cfg_.emb_dim,
                        cfg_.l2 ? 1 : 0, meta_ + (size_t)levels_.size() * B, d_out, nullptr, part,
                        st))
        return fail();
    prof_end(pp, st, 0.0);
    launches += 3;
    return 0;
}

}  // namespace vdb
