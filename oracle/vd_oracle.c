/* Plain-C restatement of the reference's conv + FBank hot path.
 *
 * TEST INFRASTRUCTURE ONLY (the checker, never the product): loaded by tests/,
 * __graft_entry__.smoke() and bench.py's CPU-baseline leg through ctypes. It is
 * pinned against the reference's own kernels (oracle/_ref/libvdref.so, built
 * from the unmodified reference sources by oracle/Makefile) and against
 * torchaudio golden fixtures (tests/golden/), see tests/test_oracle.py.
 *
 * Every function cites the reference file:line it follows. Where the reference
 * calls ggml graph ops (absent submodule; mean/sqrt/mul_mat in the pooling tail)
 * the arithmetic here is a restatement in f32 with f64 accumulation, so the
 * pooling/FC tail is "parity unpinned" at the ggml boundary.
 */
#include "vd_oracle.h"

#include <float.h>
#include <math.h>
#include <stdlib.h>
#include <string.h>

static const double kPI = 3.14159265358979323846;

/* Kaldi mel scale, src/fbank.cpp:25. */
static double mel_of(double f) { return 1127.0 * log(1.0 + f / 700.0); }

/* In-place radix-2 DIT FFT on double re/im, src/fbank.cpp:34-86 (bit reversal,
 * then per-stage twiddles w_j = exp(-2*pi*i*j/len)). */
static void fft_radix2(double* re, double* im, int n) {
    int logn = 0;
    while ((1 << logn) < n) ++logn;
    for (int i = 0; i < n; ++i) {
        int r = 0;
        for (int b = 0; b < logn; ++b)
            if (i & (1 << b)) r |= 1 << (logn - 1 - b);
        if (r > i) {
            double t = re[i]; re[i] = re[r]; re[r] = t;
            t = im[i]; im[i] = im[r]; im[r] = t;
        }
    }
    for (int len = 2; len <= n; len <<= 1) {
        const int m = len >> 1;
        for (int s = 0; s < n; s += len) {
            for (int j = 0; j < m; ++j) {
                const double ang = -2.0 * kPI * j / len;
                const double cwr = cos(ang), cwi = sin(ang);
                const int a = s + j, b = s + j + m;
                const double tr = cwr * re[b] - cwi * im[b];
                const double ti = cwr * im[b] + cwi * re[b];
                re[b] = re[a] - tr; im[b] = im[a] - ti;
                re[a] += tr;        im[a] += ti;
            }
        }
    }
}

/* FBank::compute, src/fbank.cpp:121-205. Output feat-major [n_mels, T]. */
int vdo_fbank(const float* pcm, int n, int sample_rate, int n_mels, int n_fft, int win,
              int hop, float preemph, float low_freq, float high_freq, int cmn,
              float* out, long out_cap, int* out_T) {
    if (out_T) *out_T = 0;
    if (win <= 0 || hop <= 0 || n_fft < win || n_mels <= 0) return 1;
    if (n < win) return 1;                                   /* :128 */
    const int T = 1 + (n - win) / hop;                       /* :130 snip_edges */
    if (out_T) *out_T = T;
    if (!out) return 0;
    if ((long)n_mels * T > out_cap) return 2;
    const int half = n_fft / 2;

    double* window = (double*)malloc(sizeof(double) * win);  /* :133-135 povey */
    for (int i = 0; i < win; ++i)
        window[i] = pow(0.5 - 0.5 * cos(2.0 * kPI * i / (win - 1)), 0.85);

    /* Triangular mel filterbank, :140-158. */
    const double lo = low_freq;
    const double hi = high_freq > 0.0f ? (double)high_freq : sample_rate / 2.0;
    const double mlo = mel_of(lo), mhi = mel_of(hi);
    const double mstep = (mhi - mlo) / (n_mels + 1);
    double* fb = (double*)calloc((size_t)n_mels * (half + 1), sizeof(double));
    for (int m = 0; m < n_mels; ++m) {
        const double l = mlo + m * mstep, c = mlo + (m + 1) * mstep, r = mlo + (m + 2) * mstep;
        for (int k = 0; k <= half; ++k) {
            const double mf = mel_of((double)k * sample_rate / n_fft);
            double w = 0.0;
            if (mf > l && mf <= c) w = (mf - l) / (c - l);
            else if (mf > c && mf < r) w = (r - mf) / (r - c);
            fb[(size_t)m * (half + 1) + k] = w;
        }
    }

    float* raw = (float*)malloc(sizeof(float) * win);
    double* re = (double*)malloc(sizeof(double) * n_fft);
    double* im = (double*)malloc(sizeof(double) * n_fft);
    double* ps = (double*)malloc(sizeof(double) * (half + 1));
    const double eps = (double)FLT_EPSILON;                  /* :163 */
    for (int t = 0; t < T; ++t) {
        const int off = t * hop;
        for (int i = 0; i < win; ++i) raw[i] = pcm[off + i];
        double mean = 0.0;                                   /* :169-173 DC removal */
        for (int i = 0; i < win; ++i) mean += raw[i];
        mean /= win;
        for (int i = 0; i < win; ++i) raw[i] -= (float)mean;
        for (int i = win - 1; i > 0; --i) raw[i] -= preemph * raw[i - 1];  /* :177-178 */
        raw[0] -= preemph * raw[0];
        for (int i = 0; i < n_fft; ++i) {                    /* :181-182 window + pad */
            const float f = (i < win) ? (float)(raw[i] * window[i]) : 0.0f;
            re[i] = f;
            im[i] = 0.0;
        }
        fft_radix2(re, im, n_fft);                           /* powspec :92-118 */
        for (int k = 0; k <= half; ++k) ps[k] = re[k] * re[k] + im[k] * im[k];
        for (int m = 0; m < n_mels; ++m) {                   /* :186-190 */
            double e = 0.0;
            const double* fr = fb + (size_t)m * (half + 1);
            for (int k = 0; k <= half; ++k) e += fr[k] * ps[k];
            out[(size_t)m * T + t] = (float)log(e > eps ? e : eps);
        }
    }
    if (cmn) {                                               /* :194-201 */
        for (int m = 0; m < n_mels; ++m) {
            double s = 0.0;
            for (int t = 0; t < T; ++t) s += out[(size_t)m * T + t];
            const float mu = (float)(s / T);
            for (int t = 0; t < T; ++t) out[(size_t)m * T + t] -= mu;
        }
    }
    free(window); free(fb); free(raw); free(re); free(im); free(ps);
    return 0;
}

/* Direct conv, NCHW f32, square kernel k (1 or 3), zero padding `pad`, stride s.
 * Each output accumulates in f32 FMA over (kh, kw, ic) in that order, the order
 * the reference microkernels use (src/directconv.cpp:534-537,684-686); the
 * optional bias (+ReLU) epilogue follows bemit (:544-549). Output size
 * (W + 2*pad - k)/s + 1 (:1500-1501, :1514-1515). */
void vdo_conv2d(const float* x, int W, int H, int IC, const float* w, int OC, int k,
                int stride, int pad, const float* bias, int relu, float* y) {
    const int Wo = (W + 2 * pad - k) / stride + 1;
    const int Ho = (H + 2 * pad - k) / stride + 1;
    const size_t HWi = (size_t)W * H, HWo = (size_t)Wo * Ho;
#pragma omp parallel for schedule(dynamic)
    for (int oc = 0; oc < OC; ++oc) {
        float* yo = y + (size_t)oc * HWo;
        for (size_t p = 0; p < HWo; ++p) yo[p] = 0.0f;
        for (int kh = 0; kh < k; ++kh)
            for (int kw = 0; kw < k; ++kw)
                for (int ic = 0; ic < IC; ++ic) {
                    /* ggml weight [KW, KH, IC, OC]: ((oc*IC + ic)*k + kh)*k + kw */
                    const float wv = w[(((size_t)oc * IC + ic) * k + kh) * k + kw];
                    const float* xc = x + (size_t)ic * HWi;
                    for (int oh = 0; oh < Ho; ++oh) {
                        const int ih = oh * stride + kh - pad;
                        if (ih < 0 || ih >= H) continue;
                        const float* xr = xc + (size_t)ih * W;
                        float* yr = yo + (size_t)oh * Wo;
                        for (int ow = 0; ow < Wo; ++ow) {
                            const int iw = ow * stride + kw - pad;
                            if (iw < 0 || iw >= W) continue;
                            yr[ow] = fmaf(wv, xr[iw], yr[ow]);
                        }
                    }
                }
        if (bias || relu) {
            const float b = bias ? bias[oc] : 0.0f;
            for (size_t p = 0; p < HWo; ++p) {
                float v = yo[p] + b;
                if (relu && v < 0.0f) v = 0.0f;
                yo[p] = v;
            }
        }
    }
}

/* ResNet34Encoder::forward_capture, src/encoder_resnet.cpp:94-185:
 * stem conv3x3 + bias + ReLU (:116-117); BasicBlocks (:54-73): conv1 (3x3, s,
 * +b, ReLU) -> conv2 (3x3, +b) -> + [1x1 s down (+b) | identity] -> ReLU;
 * TSTP (:143-157); FC - mean_vec (:162-170); L2 in double (:177-183). */
int vdo_resnet34_forward(const vd_resnet_desc* d, const float* feats, int T, int n_mels,
                         float* emb, float* prenorm) {
    int W = T, H = n_mels, C = d->stem_oc;
    float* cur = (float*)malloc(sizeof(float) * (size_t)W * H * C);
    vdo_conv2d(feats, W, H, 1, d->stem_w, C, 3, 1, 1, d->stem_b, 1, cur);
    for (int i = 0; i < d->n_blocks; ++i) {
        const int ic = d->in_ch[i], oc = d->out_ch[i], s = d->stride[i];
        const int Wo = (W + 2 - 3) / s + 1, Ho = (H + 2 - 3) / s + 1;
        const size_t n_out = (size_t)Wo * Ho * oc;
        float* h1 = (float*)malloc(sizeof(float) * n_out);
        float* h2 = (float*)malloc(sizeof(float) * n_out);
        vdo_conv2d(cur, W, H, ic, d->conv1_w[i], oc, 3, s, 1, d->conv1_b[i], 1, h1);
        vdo_conv2d(h1, Wo, Ho, oc, d->conv2_w[i], oc, 3, 1, 1, d->conv2_b[i], 0, h2);
        if (d->down_w[i]) {
            float* sc = (float*)malloc(sizeof(float) * n_out);
            vdo_conv2d(cur, W, H, ic, d->down_w[i], oc, 1, s, 0, d->down_b[i], 0, sc);
            for (size_t p = 0; p < n_out; ++p) {
                const float v = h2[p] + sc[p];
                h2[p] = v > 0.0f ? v : 0.0f;
            }
            free(sc);
        } else {
            for (size_t p = 0; p < n_out; ++p) {
                const float v = h2[p] + cur[p];
                h2[p] = v > 0.0f ? v : 0.0f;
            }
        }
        free(h1);
        free(cur);
        cur = h2;
        W = Wo; H = Ho; C = oc;
    }
    const int HC = H * C;
    if (2 * HC != d->pooled_dim) { free(cur); return 3; }
    float* pooled = (float*)malloc(sizeof(float) * 2 * (size_t)HC);
    for (int c = 0; c < C; ++c)
        for (int hh = 0; hh < H; ++hh) {
            const float* row = cur + ((size_t)c * H + hh) * W;
            double s1 = 0.0;
            for (int w = 0; w < W; ++w) s1 += row[w];
            const float mean = (float)(s1 / W);
            double s2 = 0.0;
            for (int w = 0; w < W; ++w) {
                const float dv = row[w] - mean;
                s2 += (double)(dv * dv);
            }
            float var = (float)(s2 / W);
            if (W > 1) var = var * ((float)W / (float)(W - 1));
            pooled[(size_t)c * H + hh] = mean;
            pooled[(size_t)HC + (size_t)c * H + hh] = sqrtf(var + d->var_eps);
        }
    for (int j = 0; j < d->emb_dim; ++j) {
        const float* wr = d->seg_w + (size_t)j * d->pooled_dim;
        double acc = 0.0;
        for (int i = 0; i < d->pooled_dim; ++i) acc += (double)wr[i] * (double)pooled[i];
        float v = (float)acc + d->seg_b[j];
        if (d->mean_vec) v -= d->mean_vec[j];
        emb[j] = v;
    }
    if (prenorm) memcpy(prenorm, emb, sizeof(float) * d->emb_dim);
    if (d->l2_normalize) {
        double n2 = 0.0;
        for (int j = 0; j < d->emb_dim; ++j) n2 += (double)emb[j] * (double)emb[j];
        const double nrm = sqrt(n2);
        if (nrm > 0.0)
            for (int j = 0; j < d->emb_dim; ++j) emb[j] = (float)((double)emb[j] / nrm);
    }
    free(pooled);
    free(cur);
    return 0;
}

/* resample_linear, src/audio_io.cpp:9-23. Returns the output length. */
long vdo_resample_linear(const float* in, long n, int in_sr, int out_sr, float* out,
                         long out_cap) {
    if (in_sr == out_sr || n <= 0) {
        if (out && out_cap >= n && n > 0) memcpy(out, in, sizeof(float) * n);
        return n > 0 ? n : 0;
    }
    const double ratio = (double)out_sr / (double)in_sr;
    const long n_out = (long)floor(n * ratio);
    if (!out || out_cap < n_out) return n_out;
    for (long i = 0; i < n_out; ++i) {
        const double src = i / ratio;
        const long i0 = (long)src;
        const double frac = src - i0;
        const float a = in[i0];
        const float b = (i0 + 1 < n) ? in[i0 + 1] : a;
        out[i] = (float)(a + (b - a) * frac);
    }
    return n_out;
}

/* Identify (no reference implementation exists; the C ABI advertises it,
 * README.md:15,44,59): f64 cosine of each query against every registry row,
 * top-k by descending score, ties broken by the lower registry index. */
void vdo_identify(const float* q, int n_q, const float* reg, int n_reg, int dim, int k,
                  int* out_idx, float* out_score) {
    double* rn = (double*)malloc(sizeof(double) * (n_reg > 0 ? n_reg : 1));
    for (int r = 0; r < n_reg; ++r) {
        double s = 0.0;
        for (int j = 0; j < dim; ++j) s += (double)reg[(size_t)r * dim + j] * reg[(size_t)r * dim + j];
        rn[r] = sqrt(s);
    }
#pragma omp parallel for schedule(dynamic)
    for (int i = 0; i < n_q; ++i) {
        const float* qi = q + (size_t)i * dim;
        double qn = 0.0;
        for (int j = 0; j < dim; ++j) qn += (double)qi[j] * qi[j];
        qn = sqrt(qn);
        double best_s[64];
        int best_i[64];
        const int kk = k < 64 ? k : 64;
        int nb = 0;
        for (int r = 0; r < n_reg; ++r) {
            double dot = 0.0;
            for (int j = 0; j < dim; ++j) dot += (double)qi[j] * reg[(size_t)r * dim + j];
            const double den = qn * rn[r];
            const double sc = den > 0.0 ? dot / den : 0.0;
            /* insert if strictly better than the current worst (ties keep lower r) */
            if (nb < kk || sc > best_s[nb - 1]) {
                int pos = nb < kk ? nb : kk - 1;
                while (pos > 0 && best_s[pos - 1] < sc) {
                    best_s[pos] = best_s[pos - 1];
                    best_i[pos] = best_i[pos - 1];
                    --pos;
                }
                best_s[pos] = sc;
                best_i[pos] = r;
                if (nb < kk) ++nb;
            }
        }
        for (int j = 0; j < k; ++j) {
            out_idx[(size_t)i * k + j] = j < nb ? best_i[j] : -1;
            out_score[(size_t)i * k + j] = j < nb ? (float)best_s[j] : -INFINITY;
        }
    }
    free(rn);
}

/* ---- ERes2Net, src/encoder_eres2net.cpp:36-264 ------------------------------ */

typedef struct {
    float* d;
    int C, H, W;
} Act;

static Act act_new(int C, int H, int W) {
    Act a;
    a.C = C; a.H = H; a.W = W;
    a.d = (float*)calloc((size_t)C * H * W, sizeof(float));
    return a;
}

typedef struct {
    const vd_eres2net_desc* d;
    int idx;
} ECtx;

/* next_conv (:36-54): conv i with its stride, pad (k-1)/2, optional bias. */
static Act e_next_conv(ECtx* e, const Act* x) {
    const int i = e->idx++;
    const vd_eres2net_desc* d = e->d;
    const int k = d->k[i], s = d->stride[i], pad = (k - 1) / 2;
    Act y = act_new(d->oc[i], (x->H + 2 * pad - k) / s + 1, (x->W + 2 * pad - k) / s + 1);
    vdo_conv2d(x->d, x->W, x->H, x->C, d->w[i], d->oc[i], k, s, pad, d->b[i], 0, y.d);
    return y;
}

/* hclamp = ggml_clamp(x, 0, hi) (:60-62) */
static void e_clamp(Act* a, float hi) {
    const size_t n = (size_t)a->C * a->H * a->W;
    for (size_t i = 0; i < n; ++i) {
        float v = a->d[i];
        v = v < 0.0f ? 0.0f : v;
        a->d[i] = v > hi ? hi : v;
    }
}

/* AFF (:91-101): z = conv(concat(x, ds)) -> SiLU -> conv -> tanh;
 * out = (x + ds) + tanh(z) * (x - ds). */
static Act e_aff(ECtx* e, const Act* x, const Act* ds) {
    const size_t hw = (size_t)x->H * x->W;
    Act cat = act_new(x->C + ds->C, x->H, x->W);
    memcpy(cat.d, x->d, sizeof(float) * x->C * hw);
    memcpy(cat.d + (size_t)x->C * hw, ds->d, sizeof(float) * ds->C * hw);
    Act z = e_next_conv(e, &cat);
    free(cat.d);
    const size_t nz = (size_t)z.C * hw;
    for (size_t i = 0; i < nz; ++i) z.d[i] = z.d[i] / (1.0f + expf(-z.d[i]));  /* ggml_silu */
    Act z2 = e_next_conv(e, &z);
    free(z.d);
    const size_t n = (size_t)x->C * hw;
    Act out = act_new(x->C, x->H, x->W);
    for (size_t i = 0; i < n; ++i) {
        const float att = tanhf(z2.d[i]);
        const float sum = x->d[i] + ds->d[i];
        const float diff = x->d[i] - ds->d[i];
        out.d[i] = sum + att * diff;
    }
    free(z2.d);
    return out;
}

/* res2net_block (:111-137) */
static Act e_block(ECtx* e, const Act* x, int planes, int stride, int is_aff, int* in_planes) {
    const float hi = e->d->relu_clamp;
    const int scale = e->d->scale;
    Act out = e_next_conv(e, x);
    e_clamp(&out, hi);
    const int width = out.C / scale;
    const size_t hw = (size_t)out.H * out.W;
    Act accum = act_new(out.C, out.H, out.W);
    Act sp = {NULL, 0, 0, 0};
    for (int i = 0; i < scale; ++i) {
        Act chunk = {out.d + (size_t)i * width * hw, width, out.H, out.W};
        Act cur;
        int own = 0;
        if (i == 0) {
            cur = chunk;
        } else if (is_aff) {
            cur = e_aff(e, &sp, &chunk);
            own = 1;
        } else {
            cur = act_new(width, out.H, out.W);
            for (size_t j = 0; j < (size_t)width * hw; ++j) cur.d[j] = sp.d[j] + chunk.d[j];
            own = 1;
        }
        Act cv = e_next_conv(e, &cur);
        e_clamp(&cv, hi);
        if (own) free(cur.d);
        memcpy(accum.d + (size_t)i * width * hw, cv.d, sizeof(float) * width * hw);
        if (sp.d) free(sp.d);
        sp = cv;
    }
    if (sp.d) free(sp.d);
    free(out.d);
    Act o3 = e_next_conv(e, &accum);
    free(accum.d);
    const size_t n = (size_t)o3.C * o3.H * o3.W;
    if (stride != 1 || *in_planes != 2 * planes) {
        Act r = e_next_conv(e, x);
        for (size_t j = 0; j < n; ++j) o3.d[j] += r.d[j];
        free(r.d);
    } else {
        for (size_t j = 0; j < n; ++j) o3.d[j] += x->d[j];
    }
    *in_planes = 2 * planes;
    e_clamp(&o3, hi);
    return o3;
}

static Act e_layer(ECtx* e, Act x, int planes, int n, int stride, int is_aff, int* in_planes,
                   int free_input) {
    for (int b = 0; b < n; ++b) {
        Act y = e_block(e, &x, planes, b == 0 ? stride : 1, is_aff, in_planes);
        if (b > 0 || free_input) free(x.d);
        x = y;
    }
    return x;
}

/* TSTP + FC + L2 over a [C][H][W] activation (shared by both encoders). */
static int tail_embed(const Act* a, const float* seg_w, const float* seg_b,
                      const float* mean_vec, int emb_dim, int pooled_dim, float var_eps,
                      int l2, float* emb, float* prenorm) {
    const int C = a->C, H = a->H, W = a->W, HC = H * C;
    if (2 * HC != pooled_dim) return 3;
    float* pooled = (float*)malloc(sizeof(float) * 2 * (size_t)HC);
    for (int c = 0; c < C; ++c)
        for (int hh = 0; hh < H; ++hh) {
            const float* row = a->d + ((size_t)c * H + hh) * W;
            double s1 = 0.0;
            for (int w = 0; w < W; ++w) s1 += row[w];
            const float mean = (float)(s1 / W);
            double s2 = 0.0;
            for (int w = 0; w < W; ++w) {
                const float dv = row[w] - mean;
                s2 += (double)(dv * dv);
            }
            float var = (float)(s2 / W);
            if (W > 1) var = var * ((float)W / (float)(W - 1));
            pooled[(size_t)c * H + hh] = mean;
            pooled[(size_t)HC + (size_t)c * H + hh] = sqrtf(var + var_eps);
        }
    for (int j = 0; j < emb_dim; ++j) {
        const float* wr = seg_w + (size_t)j * pooled_dim;
        double acc = 0.0;
        for (int i = 0; i < pooled_dim; ++i) acc += (double)wr[i] * (double)pooled[i];
        float v = (float)acc + seg_b[j];
        if (mean_vec) v -= mean_vec[j];
        emb[j] = v;
    }
    if (prenorm) memcpy(prenorm, emb, sizeof(float) * emb_dim);
    if (l2) {
        double n2 = 0.0;
        for (int j = 0; j < emb_dim; ++j) n2 += (double)emb[j] * (double)emb[j];
        const double nrm = sqrt(n2);
        if (nrm > 0.0)
            for (int j = 0; j < emb_dim; ++j) emb[j] = (float)((double)emb[j] / nrm);
    }
    free(pooled);
    return 0;
}

/* ERes2NetEncoder::forward_capture (:147-264) */
int vdo_eres2net_forward(const vd_eres2net_desc* d, const float* feats, int T, int n_mels,
                         float* emb, float* prenorm) {
    ECtx e = {d, 0};
    const int M = d->m_channels;
    Act x = {(float*)feats, 1, n_mels, T};
    Act h = e_next_conv(&e, &x);  /* stem -> plain ReLU (:203) */
    for (size_t i = 0; i < (size_t)h.C * h.H * h.W; ++i) h.d[i] = h.d[i] > 0.0f ? h.d[i] : 0.0f;
    int in_planes = M;
    Act o1 = e_layer(&e, h, M, d->num_blocks[0], 1, 0, &in_planes, 1);
    Act o2 = e_layer(&e, o1, 2 * M, d->num_blocks[1], 2, 0, &in_planes, 0);
    Act o1d = e_next_conv(&e, &o1);  /* layer1_downsample */
    free(o1.d);
    Act f12 = e_aff(&e, &o2, &o1d);
    free(o1d.d);
    Act o3 = e_layer(&e, o2, 4 * M, d->num_blocks[2], 2, 1, &in_planes, 0);
    free(o2.d);
    Act f12d = e_next_conv(&e, &f12);  /* layer2_downsample */
    free(f12.d);
    Act f123 = e_aff(&e, &o3, &f12d);
    free(f12d.d);
    Act o4 = e_layer(&e, o3, 8 * M, d->num_blocks[3], 2, 1, &in_planes, 0);
    free(o3.d);
    Act f123d = e_next_conv(&e, &f123);  /* layer3_downsample */
    free(f123.d);
    Act f1234 = e_aff(&e, &o4, &f123d);
    free(o4.d);
    free(f123d.d);
    if (e.idx != d->n_convs) {
        free(f1234.d);
        return 4;  /* manifest does not match the topology */
    }
    const int rc = tail_embed(&f1234, d->seg_w, d->seg_b, NULL, d->emb_dim, d->pooled_dim,
                              d->var_eps, d->l2_normalize, emb, prenorm);
    free(f1234.d);
    return rc;
}
