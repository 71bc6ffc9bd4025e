/* Op-level C ABI of the B200 engine: the conv / FBank / pooling kernels that the
 * reference's encoders reach through ggml custom ops, re-dispatched as plain
 * C calls on device buffers (no torch types, plain pointers and sizes).
 *
 * Reference interfaces these entry points replace:
 *   vdb_conv            <- vd::blocked_conv3x3 / vd::blocked_conv1x1 /
 *                          vd::blocked_add_relu / vd::directconv_conv3x3 /
 *                          vd::winograd_conv3x3   (src/directconv.hpp:54,74-85,
 *                          src/winograd.hpp:32; routing src/backend.cpp:665-793)
 *   vdb_fbank           <- vd::FBank::compute without CMN (src/fbank.hpp:27-35,
 *                          src/fbank.cpp:121-191)
 *   vdb_cmn_stem        <- FBank CMN (src/fbank.cpp:194-201) + the ResNet stem
 *                          conv2d_bias + ReLU (src/encoder_resnet.cpp:116-117)
 *   vdb_pool_embed      <- TSTP + seg FC - mean_vec + host L2
 *                          (src/encoder_resnet.cpp:143-183)
 *
 * Every function returns 0 on success and a nonzero status on error; the
 * message is available from vdb_last_error() (thread-local). Pointers marked
 * "device" must be device memory; `stream` is a cudaStream_t (NULL = legacy
 * default stream). Calls are asynchronous with respect to the host.
 *
 * ---- Activation layouts (f16) ------------------------------------------------
 * GRID  G(B, T, F, C): a zero-bordered NHWC tensor with time as rows. Row
 *   r = (b*(T+2) + tp)*(F+2) + fp for tp in [0, T+2), fp in [0, F+2); element
 *   (r, c) lives at r*C + c. Pixel (b, t, f) (time t, mel/freq f) is stored at
 *   (tp, fp) = (t+1, f+1). Border positions and rows with t >= tvalid[b] hold 0.
 * PHASE P(B, T, F, C): the same data as a G(B, T, F, C) tensor, split into the
 *   4 stride-2 phases of its zero-bordered grid for a stride-2 consumer whose
 *   output extents are To = (T-1)/2+1, Fo = (F-1)/2+1. Plane q = 2*(tp&1)+(fp&1)
 *   is a G(B, To, Fo, C)-shaped block (planes contiguous, q-major); padded
 *   position (tp, fp) of image b sits in plane q at row
 *   (b*(To+2) + (tp>>1) + 1)*(Fo+2) + (fp>>1) + 1. Slots no position maps to
 *   are never read by a valid output.
 * FPHASE FP(B, T, F, C): the same data split into the 2 frequency phases for a
 *   consumer that strides 2 along frequency only (CAM++'s FCM, Conv2d stride (2, 1)),
 *   output extents (T, Fo = (F-1)/2+1). Plane q = fp&1 is a G(B, T, Fo, C)-shaped
 *   block; padded position (tp, fp) of image b sits in plane q at row
 *   (b*(T+2) + tp)*(Fo+2) + (fp>>1) + 1.
 * Weights: f16 [OC][k*k][IC] with tap index kt*k + kf (kt = time tap = the
 *   reference's kw, kf = freq tap = the reference's kh), i.e. torch
 *   w[oc][ic][kf][kt] -> W[oc][kt*k + kf][ic].
 */
#ifndef VDB_OPS_H
#define VDB_OPS_H
#include <stddef.h>
#include <stdint.h>
#ifdef __cplusplus
extern "C" {
#endif

const char* vdb_last_error(void);

/* Rows of a G(B, T, F, *) tensor and of a P(B, T, F, *) tensor. */
long long vdb_grid_rows(int batch, int t, int f);
long long vdb_phase_rows(int batch, int t, int f);

typedef struct vdb_conv_args {
    int batch;          /* B */
    int t_out, f_out;   /* output extents; output is G(B, t_out, f_out, oc) (or P when y_phase) */
    int oc;             /* output channels, multiple of 16 */
    /* segment 0: the conv itself */
    int k0;             /* kernel size: 3 (pad 1) or 1 (pad 0) */
    int stride0;        /* 1: x0 is G(B, t_out, f_out, ic0); 2: x0 is P(B, t_in, f_in, ic0)
                           whose stride-2 output extents are (t_out, f_out); 3 (stride 2 on
                           the frequency axis only): x0 is FP(B, t_out, f_in, ic0) */
    int ic0;            /* input channels, multiple of 16 */
    const void* x0;     /* device f16 */
    const void* w0;     /* device f16 [oc][k0*k0][ic0] */
    /* segment 1 (optional, x1 == NULL to disable): a 1x1 conv accumulated into the
       same outputs (the fused BasicBlock downsample shortcut) */
    int stride1;        /* 1: x1 is G(B, t_out, f_out, ic1); 2: x1 is P(...); 3: FP(...) */
    int ic1;
    const void* x1;
    const void* w1;     /* device f16 [oc][ic1] */
    /* epilogue: y = act(acc + bias [+ residual]) at valid pixels, 0 elsewhere */
    const float* bias;      /* device f32 [oc] (sum of both segments' biases), or NULL */
    const void* residual;   /* device f16 G(B, t_out, f_out, oc) or NULL */
    int relu;               /* 1: max(0, .) */
    float clamp_hi;         /* > 0: min(., clamp_hi) after ReLU (Hardtanh(0, hi)) */
    const int* tvalid;      /* device int32 [B]: valid time extent of the output */
    void* y;                /* device f16 output */
    int y_phase;            /* 0: y is G(B, t_out, f_out, oc); 1: y is P(B, t_out, f_out, oc);
                               2: y is FP(B, t_out, f_out, oc); 3: y is
                               TS(B, (t_out-1)/2+1, y_pad, f_out*oc) (pixel (t, f) channel c
                               at channel f*oc + c; grid border pixels are not stored) */
    int* err;               /* device int32 error word (may be NULL): kernel timeouts */
    /* tiling (0 = automatic) */
    int tile_m;             /* output rows per CTA tile: 0, 128 or 256 */
    int halo;               /* feed of a stride-1 3x3 (mode 1 also of stride-2 / 3 ones): 0 auto,
                               -1 never (one A tile per tap),
                               1 one input halo per channel block feeding all nine taps with
                               the weights resident (<= 96 KB), 2 the same halo with the
                               weights streamed per tap through a second ring */
    int ksplit;             /* 0 auto, else 1..16 independent partial accumulators per
                               128-row block, summed in the epilogue */
    /* channel slices and extra epilogue inputs / outputs (all 0 / NULL = off) */
    int ldx0, ldx1;         /* row pitch (elements) of x0 / x1 when they are channel
                               slices of wider tensors (0 = ic0 / ic1); the pointer then
                               points at the slice's first channel (16-byte aligned) */
    int ldy;                /* row pitch of y (0 = oc): y may be a channel slice */
    void* y2;               /* optional second output, P(B, t_out, f_out, oc) layout */
    int ldr;                /* row pitch of residual (0 = oc) */
    const void* residual2;  /* second epilogue input (GRID, pitch ldr2) for act = 2 */
    int ldr2;
    int act;                /* 0: [+residual] -> ReLU/clamp flags; 1: SiLU;
                               2: attentional fusion (x + ds) + tanh(acc + bias) * (x - ds)
                               with x = residual, ds = residual2 */
    /* optional sum output (NULL = off): ysum = f16(y + addend) per element, 0 at
       border / masked pixels; GRID layout of the output grid, row pitches ldsum /
       ldaddend (0 = oc). The Res2Net `sp + chunk` of the next chunk, written by the
       conv that produces sp (src/encoder_eres2net.cpp:126). */
    void* ysum;
    int ldsum;
    const void* addend;
    int ldaddend;
    int y_pad;              /* y_phase 3: padding rows P of the 1-D consumer's slots */
    int tile_n;             /* 0 auto (oc in <= 256-column tiles), else output columns per
                               tile: a multiple of 16 dividing oc (the HALO feeds need one
                               tile) */
    int pair;               /* CTA pairs (tcgen05 cta_group::2: two SMs share one 256-row
                               tile, each holding half of the weight columns): 0 auto,
                               1 on (one-tap-per-stage feed only), -1 off */
    int qpack;              /* 1: a ResNet stage-1 conv (3x3, stride 1, ic0 = oc = 32) over
                               the QPACK layout: x0, y (y_phase 0) and residual are
                               QP(B, t_out, f_out) rows of 128 channels (vdb_qpack_rows),
                               w0 is the packed weight of vdb_qpack_pack_weights, residual
                               (optional) is added before the ReLU, y_phase 1 writes the
                               PHASE layout instead; no second segment */
    /* q8_0 weights (NULL = f16 weights), 2-D convs only: w0 / w1 then hold int8 values
       in the same layout as the f16 weights ([oc][k*k][ic], or the QPACK packing) and
       w0_scale / w1_scale one f16 scale per 32 consecutive input channels of a tap
       (the gguf q8_0 block: weight = q * scale), block-major: [k*k*ic / 32][oc] (QPACK:
       one per packed row, [1152]). The segment's input channels must be a multiple of
       32. Resident weights (the automatic halo feeds, weights <= 96 KB, and QPACK) are
       expanded to f16 in each CTA's shared memory; streamed ones are expanded once per
       launch into w_scratch (2 bytes per weight of those segments, 256-byte aligned;
       stream-ordered, so one buffer serves every conv on a stream), then streamed as
       f16. Either way the f16 values are f16(float(q) * float(scale)). */
    const void* w0_scale;
    const void* w1_scale;
    void* w_scratch;
    long long w_scratch_bytes;
} vdb_conv_args;

/* QPACK layout QP(B, T, F): the zero-bordered grid of G(B, T, F, 32) with four
 * consecutive padded frequency pixels per row: row (b*(T+2) + t')*Wq + q holds
 * pixels f' = 4q + j, j = 0..3, as channels j*32 .. j*32 + 31 (Wq = ceil((F+2)/4);
 * the pixels past the padded grid are zero). A stage-1 conv then issues 18 tensor-core
 * MMAs of N = 32..96 per 512 output pixels and 32 input channels instead of 36 of
 * N = 32 (an N = 32 MMA is bound by fetching its A operand, not by its math). */
long long vdb_qpack_rows(int batch, int t, int f);

/* Packs a stage-1 conv weight for QPACK convs: w_taps device f16 [32][9][32] (the
 * vdb_conv layout [oc][kt*3 + kf][ic]) -> out device f16 [3][384][32]: for time tap kt
 * and input pixel shift u = -1..4 the rows (j, oc) for output pixel phases j with
 * 0 <= u - j + 1 <= 2 hold W[oc][kt*3 + (u - j + 1)][:]. Asynchronous on `stream`. */
int vdb_qpack_pack_weights(const void* w_taps, void* out, void* stream);

/* Implicit-GEMM conv on tcgen05 tensor cores (f16 in, f32 accumulate).
 * Launch ordering: vdb_conv and vdb_conv1d launch with programmatic stream
 * serialization, so a conv may start while the kernel launched just before it on
 * `stream` is still running. Before it waits for that kernel, the conv reads only
 * `bias`, `bn_scale` / `bn_shift` and `tvalid`: these must not be written by the
 * kernel launched immediately before the conv on the same stream (a copy, an event
 * from another stream, or any earlier kernel is fine). Every other input, the
 * weights included, is read after that kernel has completed. */
int vdb_conv(const vdb_conv_args* a, void* stream);

/* ---- 1-D (TDNN) convs: the ECAPA-TDNN path ---------------------------------------
 * Replaces the reference's conv1d_same + ReLU + bn1d_eval (+ tanh) graph pieces
 * (src/encoder.cpp:65-151, tdnn_block :157-167, ASP :246-258), f32 im2col + mul_mat
 * there, tensor-core implicit GEMM here.
 *
 * SEQ layout S(B, T, P, C): clip b owns rows [b*(T+2P), (b+1)*(T+2P)); frame t of
 *   clip b (time-major, C channels contiguous) is row b*(T+2P) + P + t. Frames
 *   t < tvalid[b] <= T are the clip's data. The P rows on either side of the valid
 *   frames hold their reflection (frame -j = frame j, frame tv-1+j = frame tv-1-j,
 *   1 <= j <= P: SpeechBrain's reflect padding at the clip's own length, which the
 *   reference builds with get_rows, src/encoder.cpp:32-50) when the tensor feeds a
 *   conv with k > 1; other rows are never read by a valid output.
 * With reflect = 2 the tensor is zero-padded instead: every row of the clip slots
 *   is stored, 0 outside the valid frames.
 * TPHASE TS(B, T, P, C): the input of a time-stride-2 conv whose output is
 *   S(B, T, P, *): two S(B, T, P, C) planes (contiguous, plane-major), input frame u
 *   of clip b in plane u&1 at row b*(T+2P) + P + (u>>1). Rows no frame maps to must
 *   hold 0 (the producer's caller clears the planes).
 * Weights: f16 [oc][k][ic], tap j at time offset (j - (k-1)/2) * dil (torch
 *   w[oc][ic][j] -> W[oc][j][ic]). */
long long vdb_seq_rows(int batch, int t, int pad);

typedef struct vdb_conv1d_args {
    int batch;              /* B */
    int t;                  /* T: frame slots per clip (the bucket length) */
    int pad;                /* P: padding rows on each side, >= (k0-1)/2 * dil0 */
    int oc;                 /* output channels, multiple of 16, <= 4096 */
    int k0, dil0;           /* segment 0: odd kernel size <= 9 and its dilation */
    int ic0;                /* multiple of 16 */
    const void* x0;         /* device f16 S(B, T, P, ic0) (or a channel slice, pitch ldx0) */
    int ldx0;
    const void* w0;         /* device f16 [oc][k0][ic0] */
    int ic1;                /* segment 1 (x1 == NULL: off): a 1x1 on x1 into the same sums */
    const void* x1;
    int ldx1;
    const void* w1;         /* device f16 [oc][ic1] */
    const float* bias;      /* device f32 [oc] or NULL */
    const float* clip_bias; /* device f32 [B][oc] added with the bias (act 3/4), or NULL */
    const float* bn_scale;  /* act 3/4: device f32 [oc] */
    const float* bn_shift;
    int act;                /* 0: acc + bias [+ residual], then ReLU if relu;
                               1: SiLU; 3: BN(ReLU(acc + bias + clip_bias)) with
                               BN(v) = v * bn_scale + bn_shift; 4: tanh of act 3;
                               5: (acc + bias) * gate[b][t / gate_seg][col] */
    int relu;
    const void* residual;   /* act 0/1: device f16 S(B, T, P, oc), pitch ldr; or NULL */
    int ldr;
    const int* tvalid;      /* device int32 [B] */
    void* y;                /* device S(B, T, P, oc): f16, or f32 when y_f32 */
    int ldy;
    int y_f32;
    int reflect;            /* 1: also write the P reflection rows on each side;
                               2: zero padding (every slot row stored, 0 outside the
                               valid frames); 0: valid frames only */
    void* ysum;             /* optional f16 f16(y + addend), same rows (and reflections) */
    int ldsum;
    const void* addend;
    int ldaddend;
    int* err;               /* device error word or NULL */
    int tile_m;             /* 0 auto, 128 or 256 */
    int tile_n;             /* 0 auto (oc split in <= 256-column tiles), else a divisor of oc */
    int pair;               /* 1: two SMs (a cluster of 2, tcgen05 cta_group::2) share each
                               256-row tile, each loading half of the tile's weight columns
                               (oc tiles multiples of 32, tile_m 0 or 256); 0 / -1: one CTA
                               per tile */
    int stride0;            /* 0 / 1: stride 1; 2: time stride 2, x0 is TS(B, T, P, ic0)
                               (output frame o reads input frames 2o + (j - (k-1)/2)*dil) */
    const float* gate;      /* act 5: device f32 [B][gate_nseg][oc], 16-byte aligned */
    int gate_seg;           /* act 5: frames per gate segment */
    int gate_nseg;          /* act 5: segments per clip in `gate` (>= ceil(T / gate_seg)) */
    const float* x_scale;   /* optional input prologue (1x1, one segment, no CTA pair): the
                               conv reads max(x0 * x_scale[c] + x_shift[c], 0) rounded to
                               f16 (scale and shift rounded to f16 first) instead of x0 (a
                               BatchNorm + ReLU on its input); device f32 [ic0], 16-byte
                               aligned, or NULL */
    const float* x_shift;
    int halo;               /* feed of a k > 1 stride-1 single-segment conv: 0 auto (the halo
                               for outputs of <= 64 columns), -1 one A tile per tap, 1 one
                               input halo of tile + (k-1)*dil rows per channel block feeding
                               every tap, weights resident (<= 96 KB) */
} vdb_conv1d_args;

/* Same launch ordering rule as vdb_conv. */
int vdb_conv1d(const vdb_conv1d_args* a, void* stream);

/* ---- Audio ingest ----------------------------------------------------------------
 * Device-side replacement for the reference's host audio path (drwav's int16 -> f32
 * scaling and vd::resample_linear, src/audio_io.cpp:9-23): `batch` mono clips, clip b
 * at element offset in_off[b] of `in` with n_in[b] samples at in_sr Hz (in_type 0: f32,
 * 1: int16 scaled by 2^-15), written as n_out[b] = vdb_resampled_length(n_in[b], in_sr,
 * out_sr) f32 samples at out_sr Hz to out + out_off[b]. Linear interpolation with the
 * reference's exact arithmetic (bitwise equal to the host computation). in_off, n_in,
 * out_off, n_out: device arrays; max_out >= every n_out[b]. */
long long vdb_resampled_length(long long n_in, int in_sr, int out_sr);
int vdb_pcm_ingest(const void* in, int in_type, const long long* in_off, const int* n_in,
                   int batch, int in_sr, int out_sr, const long long* out_off, const int* n_out,
                   int max_out, float* out, void* stream);

/* ---- FBank ----------------------------------------------------------------------
 * A plan holds the device tables of one FBank configuration (the GGUF
 * voicedetect.fbank.* keys, src/model_loader.cpp:126-136): Povey window, FFT
 * twiddles and the triangular mel filters. Only n_fft = 512 is supported. */
typedef struct vdb_fbank_plan vdb_fbank_plan;
vdb_fbank_plan* vdb_fbank_plan_create(int sample_rate, int n_mels, int n_fft, int win, int hop,
                                      float preemph, float low_freq, float high_freq);
void vdb_fbank_plan_destroy(vdb_fbank_plan* plan);
int vdb_fbank_plan_n_mels(const vdb_fbank_plan* plan);

/* Log-mel features of `batch` clips (16 kHz mono f32, concatenated in device
 * memory at offsets[b] with n_samples[b] samples; both arrays device int64 /
 * int32). Clip b yields T_b = 1 + (n_b - win)/hop frames (0 when n_b < win);
 * frame t < min(T_b, t_max) is written to feats[(b*t_max + t)*n_mels + m]
 * (device f32, time-major). No CMN here: see vdb_cmn_stem. */
int vdb_fbank(const vdb_fbank_plan* plan, const float* pcm, const long long* offsets,
              const int* n_samples, int batch, int t_max, float* feats, void* stream);

/* Per-utterance CMN + the ResNet stem conv (3x3, 1 -> oc, pad 1) + bias + ReLU.
 * feats: device f32 [batch][t_max][n_mels] from vdb_fbank; frames: device int32
 * [batch] valid frame counts (T_b); stem_w: device f32 [oc][9] with tap kt*3+kf;
 * stem_b: device f32 [oc]. mean_scratch: device f32 [batch][n_mels] working
 * memory (the per-clip CMN means). Output y: G(batch, t_max, n_mels, oc) f16. */
int vdb_cmn_stem(const float* feats, const int* frames, int batch, int t_max, int n_mels,
                 int cmn, const float* stem_w, const float* stem_b, int oc,
                 float* mean_scratch, void* y, void* stream);

/* vdb_cmn_stem with 32 stem channels and the output in the QPACK layout
 * QP(batch, t_max, n_mels) (vdb_qpack_rows x 128 channels): the input of the QPACK
 * stage-1 convs. Same arithmetic, so the values equal vdb_cmn_stem's. */
int vdb_cmn_stem_qpack(const float* feats, const int* frames, int batch, int t_max, int n_mels,
                       int cmn, const float* stem_w, const float* stem_b, float* mean_scratch,
                       void* y, void* stream);

/* The same CMN + stem as vdb_cmn_stem, for callers that cannot allocate device
 * memory: no counterpart exists in the reference. A streaming audio callback must
 * not call cudaMalloc/cudaFree (they can stall the whole device for an unbounded
 * time), and a host that manages all device memory through its own pool does not
 * let a library allocate behind its back. This entry point allocates nothing: the
 * per-clip CMN means go to a fixed array inside the library (65536 floats,
 * 256 KB, held on every GPU that loads the library until the process exits).
 *   - batch * n_mels must be <= 65536; larger calls fail with a clear error
 *     (use vdb_cmn_stem with caller-provided memory instead).
 *   - The first call on each device looks up the array's device address; make
 *     that first call before any stream capture. A lookup that fails is not
 *     remembered: the call returns an error and the next call tries again.
 *   - Every call uses the same array, and each call overwrites every entry it
 *     reads, so nothing carries over between calls. Calls whose kernels overlap
 *     on the GPU (concurrent streams, or threads sharing a device) race on the
 *     array: serialise them. */
int vdb_cmn_stem_noalloc(const float* feats, const int* frames, int batch, int t_max, int n_mels,
                         int cmn, const float* stem_w, const float* stem_b, int oc, void* y,
                         void* stream);

/* Temporal statistics pooling + embedding FC + L2 normalisation, one CTA per clip.
 * x: G(batch, t, f, c) f16 final backbone activation; tvalid: device int32 [batch]
 * valid time extent. pooled[c*f + h] = mean, pooled[c*f*... + c*f + h] = std
 * (unbiased, + var_eps inside the sqrt); emb = seg_w (f32 [emb_dim][2*c*f]) *
 * pooled + seg_b - mean_vec (mean_vec may be NULL); then L2-normalised when
 * l2 != 0. emb_out: device f32 [batch][emb_dim]; prenorm_out (may be NULL)
 * receives the embedding before normalisation. */
int vdb_pool_embed(const void* x, const int* tvalid, int batch, int t, int f, int c,
                   const float* seg_w, const float* seg_b, const float* mean_vec, int emb_dim,
                   float var_eps, int l2, float* emb_out, float* prenorm_out, void* stream);

/* y = a + b over `rows` rows of C f16 channels, each operand with its own row
 * pitch in elements (channel slices allowed; pitches and C multiples of 8, pointers
 * 16-byte aligned). The Res2Net chunk fusion sp + x_i (ggml_add in
 * src/encoder_eres2net.cpp:126) on GRID tensors, borders included. */
int vdb_add(const void* a, int lda, const void* b, int ldb, void* y, int ldy, long long rows,
            int C, void* stream);

/* Top-k cosine search (no reference counterpart exists; the additive C ABI
 * voicedetect_capi_identify calls it). q: device f32 [n_q][dim]; reg: device f32
 * [n_reg][dim]; out_idx / out_score: device [n_q][k], descending score, equal
 * scores ordered by the lower registry index, -1 / -inf past n_reg; 0 < k <= 64,
 * dim <= 1024. For dim <= 512 the candidates come from a tcgen05 f16 GEMM of the
 * unit-normalised rows with the top-(k + 8) kept per query in its epilogue; those
 * are rescored exactly (f64 dot over f64 norms) and the returned scores are exact
 * cosines. A row of the exact top k can be missed only if more than k + 8 rows
 * score within the f16 rounding of unit vectors (|error| <= 2^-10 per score,
 * about 2e-3 between two scores) of it. Allocates stream-ordered workspace. */
int vdb_identify(const float* q, int n_q, const float* reg, int n_reg, int dim, int k,
                 int* out_idx, float* out_score, void* stream);

#ifdef __cplusplus
}
#endif
#endif
