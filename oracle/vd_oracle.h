/* CPU oracle for the voice-detect conv + FBank hot path.
 *
 * TEST INFRASTRUCTURE ONLY. Two libraries implement this header's model
 * descriptor:
 *   - oracle/_build/libvdoracle.so : vd_oracle.c, a plain-C restatement of the
 *     reference algorithms (each function cites the reference file:line it
 *     follows);
 *   - oracle/_ref/libvdref.so      : ref_glue.cpp, the reference's own
 *     src/directconv.cpp, src/winograd.cpp and src/fbank.cpp compiled unmodified
 *     against a ggml shim.
 * Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg load
 * either one; the product library (libvoicedetect_b200.so) never does.
 *
 * Layouts follow the reference (ggml ne order, fastest first):
 *   activations x : [W=time, H=freq, C]        flat ((c*H + h)*W + w)
 *   3x3 weight    : [3(kw), 3(kh), IC, OC]     = torch (OC, IC, KH, KW)
 *   1x1 weight    : [IC, OC]                   = torch (OC, IC, 1, 1)
 *   FBank output  : feat-major [n_mels, T]     flat m*T + t
 */
#ifndef VD_ORACLE_H
#define VD_ORACLE_H
#ifdef __cplusplus
extern "C" {
#endif

typedef struct {
    int n_blocks;
    const float* stem_w; /* ggml [3,3,1,C0] */
    const float* stem_b; /* [C0] */
    int stem_oc;
    const float* const* conv1_w; /* per block ggml [3,3,IC,OC] */
    const float* const* conv1_b;
    const float* const* conv2_w; /* per block ggml [3,3,OC,OC] */
    const float* const* conv2_b;
    const float* const* down_w; /* per block ggml [1,1,IC,OC]; NULL = identity */
    const float* const* down_b;
    const int* in_ch;
    const int* out_ch;
    const int* stride;
    const float* seg_w;    /* ggml [pooled_dim, emb_dim] = torch (emb_dim, pooled_dim) */
    const float* seg_b;    /* [emb_dim] */
    const float* mean_vec; /* [emb_dim] or NULL */
    int emb_dim;
    int pooled_dim;
    float var_eps;
    int l2_normalize;
} vd_resnet_desc;

/* ERes2Net: the flat conv list in forward-execution order (the GGUF manifest,
 * src/model_loader.hpp:68-80). Conv i has torch weight (oc, ic, k, k) in w[i]
 * (ggml [k,k,ic,oc]), bias b[i] or NULL, stride[i]; padding is (k-1)/2. */
typedef struct {
    int n_convs;
    const float* const* w;
    const float* const* b;
    const int* ic;
    const int* oc;
    const int* k;
    const int* stride;
    int num_blocks[4];
    int m_channels;
    int scale;
    float relu_clamp;
    const float* seg_w; /* [emb_dim][pooled_dim] */
    const float* seg_b;
    int emb_dim;
    int pooled_dim;
    float var_eps;
    int l2_normalize;
} vd_eres2net_desc;

/* ---- vd_oracle.c (C restatement) ---------------------------------------- */
int vdo_eres2net_forward(const vd_eres2net_desc* d, const float* feats, int T, int n_mels,
                         float* emb, float* prenorm);
int vdo_fbank(const float* pcm, int n, int sample_rate, int n_mels, int n_fft, int win,
              int hop, float preemph, float low_freq, float high_freq, int cmn,
              float* out, long out_cap, int* out_T);
void vdo_conv2d(const float* x, int W, int H, int IC, const float* w, int OC, int k,
                int stride, int pad, const float* bias, int relu, float* y);
int vdo_resnet34_forward(const vd_resnet_desc* d, const float* feats, int T, int n_mels,
                         float* emb, float* prenorm);
long vdo_resample_linear(const float* in, long n, int in_sr, int out_sr, float* out,
                         long out_cap);
void vdo_identify(const float* q, int n_q, const float* reg, int n_reg, int dim, int k,
                  int* out_idx, float* out_score);

#ifdef __cplusplus
}
#endif
#endif
