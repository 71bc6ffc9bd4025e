// Implicit-GEMM 3x3 / 1x1 convolution on sm_100a tensor cores (tcgen05 + TMEM),
// the B200 replacement for the reference's blocked direct conv microkernels
// (src/directconv.cpp:1072-1211 bconv3x3_compute, :1214-1280 bconv1x1_compute)
// and its fused bias / ReLU / residual-add epilogues (:544-549, :1366-1373).
//
// GEMM view. Rows (M) are the pixels of the output's zero-bordered grid
// (vdb_ops.h, GRID layout), columns (N) the output channels, and K runs over
// (tap, input channel). Because every activation carries a one-pixel zero border
// and is stored row-major over (time, freq), the A operand of tap (kt, kf) for BM
// consecutive output rows is BM consecutive input rows shifted by a constant:
//   stride 1: off = (kt-1)*(F+2) + (kf-1) in the same grid;
//   stride 2: the input is stored phase-split (PHASE layout), and the tap reads
//             plane 2*(kt&1) + (kf&1) at off = (kt>>1)*(F+2) + (kf>>1).
// The border zeros and TMA's out-of-bounds zero fill provide the padding. Rows on
// the grid border, or past a clip's valid length, are computed and then written
// as zeros, which keeps the next layer's padding exact under length-bucketed
// batching (ragged clips in one batch).
//
// Two ways to feed a K segment:
//   TAP  : one TMA box (KB channels x BM rows) per (tap, channel block) plus the
//          matching weight box (KB x BN). Used for stride-2 and wide layers,
//          where the weights dominate the traffic.
//   HALO : for stride-1 3x3 layers with few channels, one TMA load per channel
//          block brings the BM + 2*(F+2) + 2 input rows all nine taps need; the
//          nine MMAs read it through row-shifted shared-memory descriptors (the
//          tcgen05 swizzle is a function of the absolute shared-memory address,
//          so a descriptor may start at any 128 B row of a TMA-written tile). The
//          weights of all taps stay resident in shared memory for the whole
//          kernel. A traffic drops from 9*BM to BM + 2*(F+2) + 2 rows per block.
//
// Kernel structure (persistent, one CTA per SM, 12 warps):
//   warp 0 lane 0 : TMA producer, S-stage shared-memory ring
//   warp 1 lane 0 : tcgen05.mma issuer (M=128 per instruction, BM/128 row
//                   blocks, N=BN, K=16) into a double-buffered f32 TMEM
//                   accumulator; warp 1 also owns the TMEM allocation
//   warps 4..11   : epilogue, two warps per TMEM lane quadrant splitting the
//                   columns: tcgen05.ld -> + bias [+ residual] -> ReLU/clamp ->
//                   valid-pixel mask -> f16 store (plain or phase-split layout)
// An optional second K segment (a 1x1 conv on another input) accumulates into the
// same TMEM tile: that is how the BasicBlock downsample shortcut is fused into
// conv2 (reference: blocked_conv1x1 + blocked_add_relu, src/encoder_resnet.cpp:68-72).
#include <cuda_fp16.h>

#include <algorithm>
#include <cstdio>
#include <cstdlib>
#include <string>

#include "sm100_ptx.cuh"
#include "vdb_internal.h"
#include "vdb_ops.h"

namespace vdb {
namespace {

constexpr int kMB = 128;           // rows per MMA instruction
constexpr int kThreads = 384;      // 12 warps
constexpr int kEpiWarp0 = 4;
constexpr int kEpiThreads = 256;
constexpr int kMaxStages = 8;
constexpr int kSmemMax = 232448;   // 227 KB opt-in dynamic shared memory
// staged output: two 2 KB boxes per epilogue warp
constexpr uint32_t kOstageBytes = 8u * 2u * 2048u;

// Output store policy (VDB_CONV_TMA_STORE): 0 direct row stores only; 1 staged TMA box
// stores wherever they fit; unset or 2 staged where they leave enough pipeline slots.
int conv_tma_store_mode() {
    const char* e = std::getenv("VDB_CONV_TMA_STORE");
    return (e && (e[0] == '0' || e[0] == '1')) ? e[0] - '0' : 2;
}
constexpr int kMaxBatch = 8192;

// SEG_TAP: one A tile and one weight tile per (tap, channel block).
// SEG_HALO: one A halo per channel block feeds all nine taps; weights resident.
// SEG_HALO_S: one A halo per channel block, weights streamed per tap (two-ring
//   pipeline: A halos and weight tiles come through separate rings).
enum SegMode : int { SEG_TAP = 0, SEG_HALO = 1, SEG_HALO_S = 2 };

struct SegDev {
    int mode;
    int n_taps;
    int ic;
    int kb;          // channels per K block: 64 / 32 / 16 (128 / 64 / 32 B rows)
    int n_kb;        // ic / kb
    uint32_t bytes;  // TMA bytes per stage
    int plane[9];
    int off[9];      // TAP: global row offset per tap; HALO: row offset inside the halo
    int halo_back;   // HALO: rows before m0 covered by the halo
    uint32_t plane_bytes;  // HALO over FPHASE / PHASE: bytes between the planes' halos, else 0
    int halo_planes;       // HALO: planes loaded per channel block (1, FPHASE 2, PHASE 4)
    int halo_mode;         // HALO tap geometry: 0 stride 1, 1 FPHASE, 2 PHASE
    int dil;         // 1-D: tap j reads j*dil rows into a HALO (taps at (j - (k-1)/2)*dil)
    int n_box, box_rows;  // TMA A boxes per stage and their height (TAP: BM split in <= 256)
    uint32_t bres;   // HALO: resident weights, byte offset from the smem base
    uint32_t a_bytes, b_bytes;  // two-ring pipeline: A bytes per channel block, weight bytes per tap
    // q8_0 resident weights (wq != nullptr): int8 values in the f16 layout [oc][wk]
    // (wk = taps * ic, K-major) and one f16 scale per 32 of them, [wk / 32][wn] (wn =
    // oc); every CTA expands them to f16 in shared memory once
    const int8_t* wq;
    const __half* wd;
    int wk, wn;
};

struct ConvDev {
    int M;             // output grid rows
    int n_mt, n_nt, BN, BM, n_mblk, n_acc;
    int J;             // independent partial accumulators per row block (K split)
    int n_seg;
    SegDev seg[2];
    uint32_t stage0, stage_bytes, a_region, n_stages, tmem_cols, bres_bytes;
    uint32_t bres_tx;  // resident weight bytes loaded by TMA (the rest are q8_0-expanded)
    // two-ring pipeline (HALO_S): ra A slots of a_stride bytes from stage0, then rb
    // weight slots of b_stride bytes from b_ring0; barriers [0, ra) are the A
    // ring's, [ra, ra + rb) the weight ring's.
    int two_ring, ra, rb;
    uint32_t a_stride, b_stride, b_ring0;
    uint32_t bias_off, tv_off, bar_off;
    uint32_t ss_off;         // act 3/4: bn_scale then bn_shift in shared memory (0: none)
    const float* bias;       // may be null (no bias)
    const __half* residual;
    const __half* residual2;
    int ldr, ldr2, ldy;      // row pitches (elements)
    int act;                 // 0 ReLU/clamp flags, 1 SiLU, 2 attentional fusion
    __half* y;
    __half* y2;              // optional PHASE-layout second output
    __half* ysum;            // optional f16(y + addend) output (GRID rows, pitch ldsum)
    const __half* addend;
    int ldsum, ldadd;
    int y_phase;       // 0 GRID, 1 PHASE, 2 FPHASE, 3 TPHASE (see row_info)
    int Hp, Wp, T, F;  // output grid: Hp = T+2, Wp = F+2
    // n / (Hp*Wp) and n / Wp as (umulhi(n, mul) + n) >> sh, exact for 0 <= n < 2^31
    uint32_t img_mul, wp_mul;
    int img_sh, wp_sh;
    int Hq, Wq;        // phase-split output: consumer grid (TPHASE: rows per clip, F)
    int ypad;          // TPHASE: padding rows of the consumer's sequence slots
    long long plane_rows;
    const int* tvalid;
    int batch;
    int relu;
    float clamp_hi;
    int oc;
    int* err;
    // 1-D sequence geometry (seq != 0, vdb_conv1d): clip b owns rows
    // [b*Hp, (b+1)*Hp) with Hp = T + 2*pad, frame t at row b*Hp + pad + t, Wp = 1.
    // Only valid frames are stored; with `reflect` each stored row is also written
    // to the padding rows that mirror it (reflect padding at the clip's own length).
    int seq, pad, reflect, y_f32;
    const float* clip_bias;  // act 3/4: f32 [batch][oc] added before the ReLU
    const float* bn_scale;   // act 3/4: f32 [oc] per-channel affine after the ReLU
    const float* bn_shift;
    // act 5: y = (acc + bias) * gate[(b*gate_nseg + t/gate_seg)*oc + col] (a per-clip,
    // per-segment channel gate: the CAM++ context attention)
    const float* gate;
    int gate_seg, gate_nseg;
    // 1-D input prologue (xform != 0, 1x1 single-segment TAP convs): warps 2-3 rewrite
    // each landed A tile in shared memory as f16(max(x * x_scale[c] + x_shift[c], 0))
    // per input channel c before the MMAs read it (a BatchNorm + ReLU on the conv's
    // input, applied on the fly instead of in a separate pass over the tensor)
    int xform;
    const float* x_scale;
    const float* x_shift;
    int n_iss;               // MMA-issuing warps (2-D tiles of 2+ row blocks: 2)
    // QPACK (stage-1 3x3, 32 -> 32): rows of four frequency pixels x 32 channels. Wp is
    // then the row count per time step (Wq = ceil((F + 2) / 4)) and qp_res the optional
    // QPACK residual added in the epilogue (the BasicBlock identity shortcut).
    const __half* qp_res;
    // Output through TMA stores (GRID / QPACK y, no other output): each epilogue warp
    // stages its 32 rows x 32 columns in one of two 2 KB buffers at ostage_off (64-byte
    // swizzle) and one lane stores the box through the output map; 0 = the threads
    // store their rows directly
    uint32_t ostage_off;
};

// Division by a runtime-invariant divisor d (Granlund & Montgomery, "Division by
// invariant integers using multiplication", 1994): with l = ceil(log2 d) and
// mul = floor(2^32 (2^l - d) / d) + 1, n / d = (umulhi(n, mul) + n) >> l for every
// 0 <= n < 2^31 (the sum then stays below 2^32).
__device__ __forceinline__ int fdiv(int n, uint32_t mul, int sh) {
    return (int)((__umulhi((uint32_t)n, mul) + (uint32_t)n) >> sh);
}

// True when rows [m0, m0+BM) contain at least one pixel inside a clip's valid
// time range (conservative: border columns of those rows count). Every role
// evaluates it identically, so skipped tiles never touch the pipeline.
template <bool SEQ, bool QP = false>
__device__ __forceinline__ bool tile_live(const ConvDev& p, const int* tv, int m0) {
    const int img = p.Hp * p.Wp;
    const int mend = min(m0 + p.BM, p.M);
    for (int b = fdiv(m0, p.img_mul, p.img_sh); b * img < mend; ++b) {
        const int r0 = max(m0 - b * img, 0);
        const int r1 = min(mend - b * img, img);
        const int t = tv[b];
        if (t <= 0) continue;
        // QPACK: time row t' spans rows [t' * Wp, (t' + 1) * Wp)
        const int lo = SEQ ? p.pad : (QP ? p.Wp : p.Wp + 1);
        const int hi = SEQ ? p.pad + t : (QP ? p.Wp * (t + 1) : p.Wp * t + p.F + 1);
        if (r0 < hi && r1 > lo) return true;
    }
    return false;
}

__device__ __forceinline__ float h2f(uint32_t bits16) {
    return __half2float(__ushort_as_half((unsigned short)bits16));
}

struct RowInfo {
    bool in_range, valid;
    long long dst;    // row of y
    long long dst2;   // row of the PHASE-layout output (y2, or y when y_phase)
    int b;            // clip (1-D geometry)
    int t;            // frame within the clip (1-D geometry)
    long long refl[2];  // 1-D reflect: padding rows mirroring this row, or -1
};

template <bool SEQ>
__device__ __forceinline__ RowInfo row_info(const ConvDev& p, const int* tv, int m, bool live) {
    RowInfo ri{false, false, (long long)m, 0, 0, 0, {-1, -1}};
    if (m >= p.M) return ri;
    ri.in_range = true;
    if constexpr (SEQ) {
        const int b = fdiv(m, p.img_mul, p.img_sh);
        const int t = m - b * p.Hp - p.pad;
        const int tvb = min(tv[b], p.T);  // a length past the slot never writes outside it
        ri.b = b;
        ri.t = t;
        ri.valid = live && t >= 0 && t < tvb;
        if (p.reflect == 1 && ri.valid) {
            // frame -t mirrors frame t (1 <= t <= pad); frame 2*(tvb-1) - t mirrors
            // frame t when it lands in [tvb, tvb + pad)
            const long long row0 = (long long)b * p.Hp + p.pad;
            if (t >= 1 && t <= p.pad) ri.refl[0] = row0 - t;
            const int tr = 2 * (tvb - 1) - t;
            if (tr >= tvb && tr < tvb + p.pad) ri.refl[1] = row0 + tr;
        }
        return ri;
    }
    const int img = p.Hp * p.Wp;
    const int b = fdiv(m, p.img_mul, p.img_sh);
    const int r = m - b * img;
    const int tp = fdiv(r, p.wp_mul, p.wp_sh);
    const int fp = r - tp * p.Wp;
    ri.valid = live && tp >= 1 && tp <= tv[b] && fp >= 1 && fp <= p.F;
    if (p.y2 || p.y_phase == 1) {
        // PHASE: the 4 (time, freq) stride-2 planes of the padded grid
        const int q = ((tp & 1) << 1) | (fp & 1);
        ri.dst2 = (long long)q * p.plane_rows + ((long long)b * p.Hq + (tp >> 1) + 1) * p.Wq +
                  (fp >> 1) + 1;
        if (p.y_phase) ri.dst = ri.dst2;
    } else if (p.y_phase == 2) {
        // FPHASE: the 2 frequency stride-2 planes, time rows unchanged
        ri.dst2 = (long long)(fp & 1) * p.plane_rows + ((long long)b * p.Hq + tp) * p.Wq +
                  (fp >> 1) + 1;
        ri.dst = ri.dst2;
    } else if (p.y_phase == 3) {
        // TPHASE: frame t of pixel (t, f) to plane t&1, sequence row t>>1 of a
        // time-stride-2 1-D consumer, channels f*oc .. f*oc+oc-1 of that row. The grid
        // border has no slot there: those rows store nothing.
        if (tp >= 1 && tp <= p.T && fp >= 1 && fp <= p.F) {
            const int t = tp - 1;
            ri.dst2 = (long long)(t & 1) * p.plane_rows +
                      ((long long)b * p.Hq + p.ypad + (t >> 1)) * p.F + (fp - 1);
            ri.dst = ri.dst2;
        } else {
            ri.in_range = false;
        }
    }
    return ri;
}

template <int NC>
__device__ __forceinline__ void load_res(const __half* rrow, uint4 (&r)[NC / 8]) {
#pragma unroll
    for (int j = 0; j < NC / 8; ++j) r[j] = __ldg(reinterpret_cast<const uint4*>(rrow) + j);
}

// This thread's f16 row chunk: to global memory, or (sbuf != 0, NC = 32) to its row of
// the warp's staged 32 x 32 box: 16-byte chunk k of row r at r*64 + 16*(k ^ ((r >> 1)
// & 3)), the 64-byte swizzle the output map's TMA store reads (conflict-free stores).
template <int NC>
__device__ __forceinline__ void store_row(__half* yrow, const uint4 (&out)[NC / 8], uint32_t sbuf) {
    if constexpr (NC == 32) {
        if (sbuf) {
            const uint32_t r = threadIdx.x & 31;
            const uint32_t sw = (r >> 1) & 3;
#pragma unroll
            for (int k = 0; k < 4; ++k)
                st_shared_v4(sbuf + r * 64u + (((uint32_t)k ^ sw) << 4), out[k].x, out[k].y,
                             out[k].z, out[k].w);
            return;
        }
    }
    uint4* yp = reinterpret_cast<uint4*>(yrow);
#pragma unroll
    for (int j = 0; j < NC / 8; ++j) yp[j] = out[j];
}

// One epilogue chunk of NC (32 or 16) accumulator columns for this thread's row:
// TMEM (sum of the J partial accumulators) -> + bias [+ residual] -> ReLU / clamp
// -> mask -> f16 store. The TMEM loads are warp-collective, so every lane executes
// them whenever the tile is live.
// `res` holds this chunk's residual when has_res, else its addend when add_in_res
// (both prefetched one chunk ahead by epi_rows); sss is the shared-memory copy of
// bn_scale (sss[0, oc)) and bn_shift (sss[oc, 2*oc)) for act 3/4.
template <int NC, int J, bool SEQ, bool PLAIN>
__device__ __forceinline__ void epi_chunk(const ConvDev& p, bool live, const RowInfo& ri, int col,
                                          uint32_t taddr, const float* sbias, const float* sss,
                                          bool has_res, const uint4 (&res)[NC / 8],
                                          const __half* r2ptr, __half* yrow, __half* y2row,
                                          __half* srow, const __half* arow, bool add_in_res,
                                          uint32_t sbuf) {
    float f[NC];
#pragma unroll
    for (int i = 0; i < NC; ++i) f[i] = 0.0f;
    if (live) {
        if constexpr (NC == 32) {
#pragma unroll 1
            for (int j = 0; j < J; ++j) {
                uint32_t v[32];
                tmem_ld_32x32b_x32(taddr + (uint32_t)(j * p.BN), v);
#pragma unroll
                for (int i = 0; i < 32; ++i) f[i] += __uint_as_float(v[i]);
            }
        } else {
            // 16-column chunks: partials in pairs, one wait per pair
#pragma unroll
            for (int j = 0; j < J; j += 2) {
                uint32_t v[16], w[16];
                if (j + 1 < J) {
                    tmem_ld_32x32b_x16_pair(taddr + (uint32_t)(j * p.BN),
                                            taddr + (uint32_t)((j + 1) * p.BN), v, w);
#pragma unroll
                    for (int i = 0; i < 16; ++i) f[i] += __uint_as_float(v[i]) + __uint_as_float(w[i]);
                } else {
                    tmem_ld_32x32b_x16(taddr + (uint32_t)(j * p.BN), v);
#pragma unroll
                    for (int i = 0; i < 16; ++i) f[i] += __uint_as_float(v[i]);
                }
            }
        }
    }
    if (!ri.in_range) return;
    if constexpr (PLAIN) {
        // (acc + bias) [+ residual] -> ReLU -> valid-pixel mask -> f16: the ResNet
        // BasicBlock convs (every other epilogue mode compiled out, so the hot code stays
        // small); the residual is added in the general path's order
        const uint32_t keep = ri.valid ? 0xFFFFFFFFu : 0u;
        const __half2 zero2 = __float2half2_rn(0.0f);
        uint4 out[NC / 8];
#pragma unroll
        for (int j = 0; j < NC / 8; ++j) {
            const uint32_t w[4] = {res[j].x, res[j].y, res[j].z, res[j].w};
            __half2 h[4];
#pragma unroll
            for (int q = 0; q < 4; ++q) {
                float a0 = f[j * 8 + 2 * q] + sbias[j * 8 + 2 * q];
                float a1 = f[j * 8 + 2 * q + 1] + sbias[j * 8 + 2 * q + 1];
                if (has_res) {
                    a0 += h2f(w[q] & 0xFFFFu);
                    a1 += h2f(w[q] >> 16);
                }
                h[q] = __floats2half2_rn(a0, a1);
                if (p.relu) h[q] = __hmax2(h[q], zero2);
            }
            out[j] = make_uint4(*reinterpret_cast<uint32_t*>(&h[0]) & keep,
                                *reinterpret_cast<uint32_t*>(&h[1]) & keep,
                                *reinterpret_cast<uint32_t*>(&h[2]) & keep,
                                *reinterpret_cast<uint32_t*>(&h[3]) & keep);
        }
        store_row<NC>(yrow, out, sbuf);
        return;
    }
    if constexpr (SEQ) {
        // 1-D: padding rows hold reflections (or nothing used), unless the tensor is
        // zero-padded (reflect 2): then every row of the slots is stored, 0 outside
        // the valid frames
        if (!ri.valid && p.reflect != 2) return;
    }
    if (sbias) {
#pragma unroll
        for (int i = 0; i < NC; ++i) f[i] += sbias[i];
    }
    if (p.act == 2) {
        // attentional fusion: (x + ds) + tanh(z) * (x - ds), x = residual, ds = residual2
        if (ri.valid) {
#pragma unroll
            for (int j = 0; j < NC / 8; ++j) {
                const uint4 d4 = __ldg(reinterpret_cast<const uint4*>(r2ptr) + j);
                const uint32_t wx[4] = {res[j].x, res[j].y, res[j].z, res[j].w};
                const uint32_t wd[4] = {d4.x, d4.y, d4.z, d4.w};
#pragma unroll
                for (int h = 0; h < 8; ++h) {
                    const float x = h2f((h & 1) ? (wx[h >> 1] >> 16) : (wx[h >> 1] & 0xFFFFu));
                    const float d = h2f((h & 1) ? (wd[h >> 1] >> 16) : (wd[h >> 1] & 0xFFFFu));
                    const float att = tanhf(f[j * 8 + h]);
                    f[j * 8 + h] = (x + d) + att * (x - d);
                }
            }
        }
    } else {
        if (has_res) {
#pragma unroll
            for (int j = 0; j < NC / 8; ++j) {
                const uint32_t w[4] = {res[j].x, res[j].y, res[j].z, res[j].w};
#pragma unroll
                for (int h = 0; h < 4; ++h) {
                    f[j * 8 + 2 * h] += h2f(w[h] & 0xFFFFu);
                    f[j * 8 + 2 * h + 1] += h2f(w[h] >> 16);
                }
            }
        }
        if (p.act == 1) {
#pragma unroll
            for (int i = 0; i < NC; ++i) f[i] = f[i] / (1.0f + expf(-f[i]));  // SiLU
        } else if (SEQ && p.act == 5) {
            if (ri.valid) {
                const float4* g = reinterpret_cast<const float4*>(
                    p.gate + ((long long)ri.b * p.gate_nseg + ri.t / p.gate_seg) * p.oc + col);
#pragma unroll
                for (int j = 0; j < NC / 4; ++j) {
                    const float4 g4 = __ldg(g + j);
                    f[4 * j] *= g4.x;
                    f[4 * j + 1] *= g4.y;
                    f[4 * j + 2] *= g4.z;
                    f[4 * j + 3] *= g4.w;
                }
            }
        } else if (SEQ && (p.act == 3 || p.act == 4)) {
            // TDNN block: BatchNorm(ReLU(acc + bias [+ clip bias])), then tanh for act 4
            const float4* sc = reinterpret_cast<const float4*>(sss + col);
            const float4* sh = reinterpret_cast<const float4*>(sss + p.oc + col);
            const float4* cb = p.clip_bias ? reinterpret_cast<const float4*>(
                                                 p.clip_bias + (long long)ri.b * p.oc + col)
                                           : nullptr;
#pragma unroll
            for (int j = 0; j < NC / 4; ++j) {
                const float4 s4 = sc[j], h4 = sh[j];
                const float4 c4 = cb ? __ldg(cb + j) : make_float4(0.f, 0.f, 0.f, 0.f);
                const float sv[4] = {s4.x, s4.y, s4.z, s4.w};
                const float hv[4] = {h4.x, h4.y, h4.z, h4.w};
                const float cv[4] = {c4.x, c4.y, c4.z, c4.w};
#pragma unroll
                for (int q = 0; q < 4; ++q) {
                    float v = fmaxf(f[4 * j + q] + cv[q], 0.0f) * sv[q] + hv[q];
                    if (p.act == 4) v = tanhf(v);
                    f[4 * j + q] = v;
                }
            }
        }
    }
    if (SEQ && p.y_f32) {
        // f32 output (1-D geometry; no sum output): optional ReLU, valid rows only
        if (p.relu) {
#pragma unroll
            for (int i = 0; i < NC; ++i) f[i] = fmaxf(f[i], 0.0f);
        }
        float* yf = reinterpret_cast<float*>(p.y);
        const long long rows[3] = {ri.dst, ri.refl[0], ri.refl[1]};
#pragma unroll
        for (int k = 0; k < 3; ++k) {
            if (rows[k] < 0) continue;
            float4* yp = reinterpret_cast<float4*>(yf + rows[k] * p.ldy + col);
#pragma unroll
            for (int j = 0; j < NC / 4; ++j)
                yp[j] = make_float4(f[4 * j], f[4 * j + 1], f[4 * j + 2], f[4 * j + 3]);
        }
        return;
    }
    // Pack to f16 pairs, then ReLU / Hardtanh on the pairs: rounding to f16 is
    // monotone and 0 and clamp_hi are exact in f16, so max / min after rounding
    // equal rounding after max / min. Invalid pixels are zeroed with a bit mask.
    const uint32_t keep = ri.valid ? 0xFFFFFFFFu : 0u;
    const bool relu = p.act == 0 && p.relu;
    const bool clamp = p.act == 0 && p.clamp_hi > 0.0f;
    const __half2 zero2 = __float2half2_rn(0.0f);
    const __half2 hi2 = __float2half2_rn(p.clamp_hi);
    uint4 out[NC / 8];
#pragma unroll
    for (int j = 0; j < NC / 8; ++j) {
        __half2 h[4];
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            h[q] = __floats2half2_rn(f[j * 8 + 2 * q], f[j * 8 + 2 * q + 1]);
            if (relu) h[q] = __hmax2(h[q], zero2);
            if (clamp) h[q] = __hmin2(h[q], hi2);
        }
        out[j].x = *reinterpret_cast<uint32_t*>(&h[0]) & keep;
        out[j].y = *reinterpret_cast<uint32_t*>(&h[1]) & keep;
        out[j].z = *reinterpret_cast<uint32_t*>(&h[2]) & keep;
        out[j].w = *reinterpret_cast<uint32_t*>(&h[3]) & keep;
    }
    store_row<NC>(yrow, out, sbuf);
    if (y2row) {
        uint4* y2p = reinterpret_cast<uint4*>(y2row);
#pragma unroll
        for (int j = 0; j < NC / 8; ++j) y2p[j] = out[j];
    }
    uint4 so[NC / 8];
    if (srow) {
        // f16(y + addend) in f32, like a separate element-wise add of the stored y
        uint4* sp = reinterpret_cast<uint4*>(srow);
#pragma unroll
        for (int j = 0; j < NC / 8; ++j) {
            uint4 o = make_uint4(0u, 0u, 0u, 0u);
            if (arow) {
                const uint4 av = add_in_res ? res[j] : __ldg(reinterpret_cast<const uint4*>(arow) + j);
                const __half2* ho = reinterpret_cast<const __half2*>(&out[j]);
                const __half2* ha = reinterpret_cast<const __half2*>(&av);
                __half2* hs = reinterpret_cast<__half2*>(&o);
#pragma unroll
                for (int q = 0; q < 4; ++q) {
                    const float2 fo = __half22float2(ho[q]), fa = __half22float2(ha[q]);
                    hs[q] = __floats2half2_rn(fo.x + fa.x, fo.y + fa.y);
                }
            }
            so[j] = o;
            sp[j] = o;
        }
    }
    if (SEQ && p.reflect == 1) {
#pragma unroll
        for (int k = 0; k < 2; ++k) {
            if (ri.refl[k] < 0) continue;
            uint4* rp = reinterpret_cast<uint4*>(p.y + ri.refl[k] * p.ldy + col);
#pragma unroll
            for (int j = 0; j < NC / 8; ++j) rp[j] = out[j];
            if (srow) {
                uint4* rs = reinterpret_cast<uint4*>(p.ysum + ri.refl[k] * p.ldsum + col);
#pragma unroll
                for (int j = 0; j < NC / 8; ++j) rs[j] = so[j];
            }
        }
    }
}

// Epilogue of one (tile, row block) for this thread: columns [c_lo, c_hi) of the
// tile in chunks of NC, with the residual of the next chunk loaded before the
// current one is finished.
// Staged output (stage != 0): before a chunk, lane 0 waits until the store issued
// from the same buffer two chunks ago has read it; after it, the warp's box goes out
// by one TMA store from lane 0 (rows past M clipped by the map). One bulk group per
// chunk, even when empty, so the wait's count stays exact.
struct EpiStage {
    const CUtensorMap* map;
    uint32_t base;  // this warp's two 2 KB buffers; 0 = direct stores
    uint32_t n;     // chunks staged so far (buffer parity)
    int row0;       // first row of the warp's 32
};

__device__ __forceinline__ uint32_t stage_begin(EpiStage& st) {
    if (!st.base) return 0u;
    const uint32_t buf = st.base + (st.n & 1u) * 2048u;
    if ((threadIdx.x & 31) == 0) bulk_wait_read<1>();
    __syncwarp();
    return buf;
}

__device__ __forceinline__ void stage_end(EpiStage& st, uint32_t buf, int col, int M) {
    if (!st.base) return;
    fence_proxy_async_smem();
    __syncwarp();
    if ((threadIdx.x & 31) == 0) {
        if (st.row0 < M) tma_store_3d(st.map, buf, col, st.row0, 0);
        bulk_commit();
    }
    ++st.n;
}

template <int NC, int J, bool SEQ, bool PLAIN>
__device__ __forceinline__ void epi_rows(const ConvDev& p, bool live, const RowInfo& ri, int m,
                                         int n0, int c_lo, int c_hi, uint32_t tbase,
                                         const float* sbias, const float* sss, EpiStage& st) {
    if constexpr (PLAIN) {
        __half* yrow = p.y + ri.dst * p.ldy + n0;
        // the residual of the next chunk is loaded before the current one is finished
        const bool has_res = p.residual != nullptr && ri.valid;
        const __half* rrow = has_res ? p.residual + (long long)m * p.ldr + n0 : nullptr;
        uint4 res[NC / 8] = {};
        if (rrow) load_res<NC>(rrow + c_lo, res);
        for (int c = c_lo; c < c_hi; c += NC) {
            uint4 cur[NC / 8];
#pragma unroll
            for (int j = 0; j < NC / 8; ++j) cur[j] = res[j];
            if (rrow && c + NC < c_hi) load_res<NC>(rrow + c + NC, res);
            const uint32_t buf = stage_begin(st);
            epi_chunk<NC, J, SEQ, true>(p, live, ri, n0 + c, tbase + (uint32_t)c,
                                        sbias + n0 + c, sss, has_res, cur, nullptr, yrow + c,
                                        nullptr, nullptr, nullptr, false, buf);
            stage_end(st, buf, n0 + c, p.M);
        }
        return;
    }
    const bool has_res = p.residual != nullptr && ri.valid;
    const bool has_res2 = p.residual2 != nullptr && ri.valid;
    const __half* rrow = has_res ? p.residual + (long long)m * p.ldr + n0 : nullptr;
    const __half* r2row = has_res2 ? p.residual2 + (long long)m * p.ldr2 + n0 : nullptr;
    __half* yrow = p.y + ri.dst * p.ldy + n0;
    __half* y2row = (p.y2 && ri.in_range) ? p.y2 + ri.dst2 * p.oc + n0 : nullptr;
    __half* srow = (p.ysum && ri.in_range) ? p.ysum + (long long)m * p.ldsum + n0 : nullptr;
    const __half* arow = (p.ysum && ri.valid) ? p.addend + (long long)m * p.ldadd + n0 : nullptr;
    // The prefetch registers carry the residual, or else the sum output's addend.
    const bool add_in_res = !has_res && arow != nullptr;
    const __half* prow = has_res ? rrow : (add_in_res ? arow : nullptr);
    uint4 res[NC / 8];
    if (prow) load_res<NC>(prow + c_lo, res);
    for (int c = c_lo; c < c_hi; c += NC) {
        uint4 cur[NC / 8];
#pragma unroll
        for (int j = 0; j < NC / 8; ++j) cur[j] = res[j];
        if (prow && c + NC < c_hi) load_res<NC>(prow + c + NC, res);
        const uint32_t buf = stage_begin(st);
        epi_chunk<NC, J, SEQ, false>(p, live, ri, n0 + c, tbase + (uint32_t)c, sbias ? sbias + n0 + c : nullptr,
                         sss, has_res, cur, has_res2 ? r2row + c : nullptr, yrow + c,
                         y2row ? y2row + c : nullptr, srow ? srow + c : nullptr,
                         arow ? arow + c : nullptr, add_in_res, buf);
        stage_end(st, buf, n0 + c, p.M);
    }
}

// ---- q8_0 weights ------------------------------------------------------------
// 8 int8 values (two 32-bit words) times the f16 scale d as 8 f16, each the exact
// product q * d rounded once to nearest: the same bits as converting float(q) *
// float(d) (exact in f32) to f16 on the host. q becomes f16 exactly by the byte-plane
// construction 0x64 : (q + 128) = the f16 1024 + q + 128, minus 1152 (0x6480).
__device__ __forceinline__ uint4 q8_to_f16x8(uint2 q, __half d) {
    const uint32_t x0 = q.x ^ 0x80808080u, x1 = q.y ^ 0x80808080u;
    uint32_t w[4] = {__byte_perm(x0, 0x64646464u, 0x5140), __byte_perm(x0, 0x64646464u, 0x5342),
                     __byte_perm(x1, 0x64646464u, 0x5140), __byte_perm(x1, 0x64646464u, 0x5342)};
    const __half2 off2 = __half2half2(__ushort_as_half((unsigned short)0x6480));
    const __half2 d2 = __half2half2(d);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        __half2 h = __hmul2(__hsub2(*reinterpret_cast<__half2*>(&w[i]), off2), d2);
        w[i] = *reinterpret_cast<uint32_t*>(&h);
    }
    return make_uint4(w[0], w[1], w[2], w[3]);
}

// Rows [row0, row0 + R) x channels [k0, k0 + kb) of a q8_0 segment's weights, expanded
// into the f16 tile at shared address dst as TMA would have written it: rows of 2*kb
// bytes with the kb-dependent swizzle (16-byte chunk bits [4, 7) XOR address bits
// [7, 10), masked to the swizzle width). Threads t, t + nt, ... of the caller.
__device__ __forceinline__ void q8_expand(const SegDev& s, int kb, int row0, int R, int k0,
                                          uint32_t dst, int t, int nt) {
    const int cpr = kb >> 3;  // 16-byte chunks per row
    const int sh = cpr == 8 ? 3 : (cpr == 4 ? 2 : 1);
    const uint32_t mask = kb == 64 ? 7u : (kb == 32 ? 3u : 1u);
    for (int i = t; i < R * cpr; i += nt) {
        const int r = i >> sh, j = i & (cpr - 1);
        const long long row = (long long)row0 + r;
        const int k = k0 + 8 * j;
        const uint2 q = __ldg(reinterpret_cast<const uint2*>(s.wq + row * s.wk + k));
        const __half d = s.wd[(long long)(k >> 5) * s.wn + row];
        const uint4 o = q8_to_f16x8(q, d);
        const uint32_t off = (uint32_t)(r * kb * 2 + 16 * j);
        st_shared_v4(dst + (off ^ (((off >> 7) & mask) << 4)), o.x, o.y, o.z, o.w);
    }
}

// Streamed q8_0 weights: one pass per launch expands the segment's int8 values and
// scales into f16 [oc][K] in a scratch buffer (L2-resident, at most a few MB), which the
// conv then streams by TMA like f16 weights. Expanding them per stage in shared memory
// instead measured 2-4x slower on those convs: the expansion's shared-memory traffic
// (8 KB read + 16 KB written per stage, repeated for every M tile) competes with the
// tensor cores' operand fetch for shared-memory bandwidth.
__global__ void __launch_bounds__(256)
q8_dequant_kernel(const int8_t* __restrict__ q, const __half* __restrict__ d, int oc, int K,
                  __half* __restrict__ out) {
    const long long n8 = (long long)oc * K / 8;
    for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n8;
         i += (long long)gridDim.x * blockDim.x) {
        const long long e = i * 8;
        const int row = (int)(e / K), k = (int)(e - (long long)row * K);
        const uint2 qq = __ldg(reinterpret_cast<const uint2*>(q + e));
        const __half dd = d[(long long)(k >> 5) * oc + row];
        *reinterpret_cast<uint4*>(out + e) = q8_to_f16x8(qq, dd);
    }
}

// ---- QPACK ------------------------------------------------------------------
// A stage-1 conv (3x3, stride 1, 32 -> 32) over QPACK rows: row (b, t', q) holds the
// four padded frequency pixels f' = 4q + j (j = 0..3) x 32 channels. Output pixel
// (t', 4q + j) needs input (t' + kt - 1, 4q + u) with u = j + kf - 1 in [-1, 4], i.e.
// QPACK row (t' + kt - 1, q + floor(u / 4)) at pixel phase u & 3. So for each (kt, u)
// one MMA (K = that phase's 32 channels) produces the partial sums of every output
// pixel phase j it touches (j_min = max(0, u - 1) .. j_max = min(3, u + 1), N = 32 per
// phase) against packed weights W[kt][u][(j, oc)][ic] = W[oc][kt][u - j + 1][ic]:
// 18 MMAs of N = 32..96 per 128 rows and K step instead of 36 of N = 32, and a 128-row
// accumulator holds 512 output pixels. A stage is one 64-channel half of the rows
// (phases 2h, 2h + 1) as a halo of tile + 2 Wq + 2 rows; the packed weights (3 x 384
// rows of 32 channels) stay resident.
__host__ __device__ constexpr int qp_u(int half, int ui) {
    // stage 0 first issues u = 1 (columns 0..95) and u = 4 (96..127): together they
    // cover the accumulator, so they overwrite it and every later MMA accumulates
    return half == 0 ? (ui == 0 ? 1 : (ui == 1 ? 4 : 0)) : (ui == 0 ? -1 : (ui == 1 ? 2 : 3));
}
__host__ __device__ constexpr int qp_jmin(int u) { return u - 1 < 0 ? 0 : u - 1; }
__host__ __device__ constexpr int qp_jmax(int u) { return u + 1 > 3 ? 3 : u + 1; }
// first packed-weight row of (kt, u): blocks in u order -1..4 of 32 / 64 / 96 / 96 /
// 64 / 32 rows, 384 rows per kt
__host__ __device__ constexpr int qp_wrow(int kt, int u) {
    return kt * 384 + (u == -1 ? 0 : (u == 0 ? 32 : (u == 1 ? 96 : (u == 2 ? 192 : (u == 3 ? 288 : 352)))));
}

template <int NMB, int HALF, int MB0, int MBS>
__device__ __forceinline__ void issue_qpack(uint32_t d_tile, uint64_t a_desc, uint32_t wq_units,
                                            uint64_t b_desc, const uint32_t (&idn)[3],
                                            bool first) {
#pragma unroll
    for (int kt = 0; kt < 3; ++kt) {
#pragma unroll
        for (int ui = 0; ui < 3; ++ui) {
            const int u = qp_u(HALF, ui);
            const int jmin = qp_jmin(u), nn = qp_jmax(u) - jmin + 1;
            const int rsh = u < 0 ? 0 : (u > 3 ? 2 : 1);  // halo rows past kt * Wq
            // a 128-byte row is 8 descriptor units; phase u & 3 is the (u & 1)-th 32 channels
            const uint64_t at = a_desc + (uint64_t)(kt * wq_units + rsh * 8 + ((u & 3) & 1) * 4);
            const uint64_t bt = b_desc + (uint64_t)(qp_wrow(kt, u) * 4);  // 64-byte rows
            const uint32_t dt = d_tile + (uint32_t)(32 * jmin);
#pragma unroll
            for (int k = 0; k < 2; ++k) {
                const bool init = first && HALF == 0 && kt == 0 && ui < 2 && k == 0;
#pragma unroll
                for (int mb = MB0; mb < NMB; mb += MBS)
                    umma_f16(dt + (uint32_t)(mb * 128), at + (uint64_t)(mb * 128 * 8) + 2 * k,
                             bt + 2 * k, idn[nn - 1], init ? 0u : 1u);
            }
        }
    }
}

// Epilogue of pixel phase j of QPACK row m (accumulator columns [32 j, 32 j + 32) in
// v): + bias [+ residual] -> ReLU -> mask -> f16, stored to the same QPACK row
// (y_phase 0) or to the pixel's place in the PHASE layout (y_phase 1). res holds the
// residual's 32 channels when p.qp_res (prefetched by the caller).
// One QPACK output unit of a thread: row m, pixel phase j (its 32 channels): bias,
// the optional residual, ReLU and the padding mask applied, packed as f16 pairs.
// Returns false for a PHASE output pixel past the padded grid (nothing to store).
__device__ __forceinline__ bool qpack_pack(const ConvDev& p, const int* stv, int m, bool live,
                                           int j, const uint32_t (&v)[32], const float* sbias,
                                           const uint4 (&res)[4], uint32_t (&o)[16],
                                           __half** dst) {
    const int img = p.Hp * p.Wp;
    const int b = fdiv(m, p.img_mul, p.img_sh);
    const int r = m - b * img;
    const int tp = fdiv(r, p.wp_mul, p.wp_sh);
    const int fp = 4 * (r - tp * p.Wp) + j;
    const bool valid = live && tp >= 1 && tp <= stv[b] && fp >= 1 && fp <= p.F;
    if (p.y_phase == 1) {
        if (fp > p.F + 1) return false;  // past the padded grid: no PHASE slot
        const int q = ((tp & 1) << 1) | (fp & 1);
        *dst = p.y + ((long long)q * p.plane_rows + ((long long)b * p.Hq + (tp >> 1) + 1) * p.Wq +
                      (fp >> 1) + 1) * 32;
    } else {
        *dst = p.y + (long long)m * 128 + j * 32;
    }
    const uint32_t keep = valid ? 0xFFFFFFFFu : 0u;
    const __half2 zero2 = __float2half2_rn(0.0f);
#pragma unroll
    for (int c = 0; c < 4; ++c) {
        const uint32_t rw[4] = {res[c].x, res[c].y, res[c].z, res[c].w};
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            float a0 = __uint_as_float(v[c * 8 + 2 * q]) + sbias[c * 8 + 2 * q];
            float a1 = __uint_as_float(v[c * 8 + 2 * q + 1]) + sbias[c * 8 + 2 * q + 1];
            if (p.qp_res) {
                a0 += h2f(rw[q] & 0xFFFFu);
                a1 += h2f(rw[q] >> 16);
            }
            __half2 h = __floats2half2_rn(a0, a1);
            if (p.relu) h = __hmax2(h, zero2);
            o[c * 4 + q] = *reinterpret_cast<uint32_t*>(&h) & keep;
        }
    }
    return true;
}

// ---- MMA issue schedules ---------------------------------------------------
// The single issuing thread is on the critical path (a tcgen05.mma every ~60
// cycles at best), so each stage is one fully unrolled, branch-free sequence with
// descriptors derived by integer adds in 16-byte units from a per-stage base.
// Partial accumulator (mb, j) sits at TMEM column (mb*J + j)*BN of the tile, and
// consecutive MMAs rotate over the NMB*J partials so none waits on its
// predecessor. `first` marks the tile's first stage: the first MMA into each
// partial overwrites instead of accumulating.

// HALO stage: nine taps of a 3x3 stride-1 conv read one shared input halo through
// row-shifted descriptors; tap (kt, kf) starts kt*wp_units + kf*rb16 in.
// Tap (kt, kf) of a halo starts row(kt) + col(kf) 16-byte units in, by mode:
//   0 stride 1: kt*Wp + kf rows;
//   1 FPHASE (frequency-stride-2 input, 2 planes plane_units apart): plane kf&1,
//     kt*Wp + (kf>>1) rows;
//   2 PHASE (stride-2 input, 4 planes): plane 2*(kt&1) + (kf&1), (kt>>1)*Wp + (kf>>1)
//     rows.
template <int KS, int NMB, int J, int MB0 = 0, int MBS = 1>
__device__ __forceinline__ void issue_halo(uint32_t d_tile, uint32_t bn, uint64_t a_desc,
                                           uint32_t wp_units, uint32_t rb16, uint64_t b_desc,
                                           uint32_t b_tap_units, uint32_t idesc, bool first,
                                           int hmode, uint32_t plane_units) {
    // offsets of kt, kf = 1, 2 (0 for 0), chosen once: the loop below is the
    // issue-bound inner loop of the small-channel convs
    uint32_t row1 = wp_units, row2 = 2 * wp_units, col1 = rb16, col2 = 2 * rb16;
    if (hmode == 1) {
        col1 = plane_units;
        col2 = rb16;
    } else if (hmode == 2) {
        row1 = 2 * plane_units;
        row2 = wp_units;
        col1 = plane_units;
        col2 = rb16;
    }
#pragma unroll
    for (int tap = 0; tap < 9; ++tap) {
        const int kt = tap / 3, kf = tap % 3;
        const uint32_t row = kt == 0 ? 0u : (kt == 1 ? row1 : row2);
        const uint32_t col = kf == 0 ? 0u : (kf == 1 ? col1 : col2);
        const uint64_t at = a_desc + (uint64_t)(row + col);
        const uint64_t bt = b_desc + (uint64_t)(tap * b_tap_units);
#pragma unroll
        for (int k = 0; k < KS; ++k) {
            const int q = tap * KS + k;
            const int j = q % J;
#pragma unroll
            for (int mb = MB0; mb < NMB; mb += MBS)
                umma_f16(d_tile + (uint32_t)(mb * J + j) * bn,
                         at + (uint64_t)(mb * 128 * rb16) + 2 * k, bt + 2 * k, idesc,
                         (first && q < J) ? 0u : 1u);
        }
    }
}

// TAP stage: one (tap, channel block) A tile and its weight tile, rotating over
// JU = min(J, KS) partials. When this is the tile's first segment the host
// guarantees J <= KS, so the first stage initialises every partial.
template <int KS, int NMB, int J, bool PAIR, int MB0 = 0, int MBS = 1>
__device__ __forceinline__ void issue_tap(uint32_t d_tile, uint32_t bn, uint64_t a_desc,
                                          uint32_t rb16, uint64_t b_desc, uint32_t idesc,
                                          bool first) {
    constexpr int JU = J < KS ? J : KS;
#pragma unroll
    for (int k = 0; k < KS; ++k) {
        const int j = k % JU;
#pragma unroll
        for (int mb = MB0; mb < NMB; mb += MBS) {
            if constexpr (PAIR)
                umma_f16_pair(d_tile + (uint32_t)(mb * J + j) * bn,
                              a_desc + (uint64_t)(mb * 128 * rb16) + 2 * k, b_desc + 2 * k, idesc,
                              (first && k < JU) ? 0u : 1u);
            else
                umma_f16(d_tile + (uint32_t)(mb * J + j) * bn,
                         a_desc + (uint64_t)(mb * 128 * rb16) + 2 * k, b_desc + 2 * k, idesc,
                         (first && k < JU) ? 0u : 1u);
        }
    }
}

// 1-D HALO: n_taps taps, tap j starting j*dil rows (dil_units = dil*rb16) into the
// halo, which begins (k-1)/2*dil rows before the tile.
template <int KS, int NMB, int J, int MB0 = 0, int MBS = 1>
__device__ __forceinline__ void issue_halo1d(uint32_t d_tile, uint32_t bn, uint64_t a_desc,
                                             uint32_t rb16, uint64_t b_desc, uint32_t b_tap_units,
                                             uint32_t idesc, bool first, int n_taps,
                                             uint32_t dil_units) {
    for (int tap = 0; tap < n_taps; ++tap) {
        const uint64_t at = a_desc + (uint64_t)(tap * dil_units);
        const uint64_t bt = b_desc + (uint64_t)(tap * b_tap_units);
#pragma unroll
        for (int k = 0; k < KS; ++k) {
            const int q = tap * KS + k;
            const int j = q % J;
#pragma unroll
            for (int mb = MB0; mb < NMB; mb += MBS)
                umma_f16(d_tile + (uint32_t)(mb * J + j) * bn,
                         at + (uint64_t)(mb * 128 * rb16) + 2 * k, bt + 2 * k, idesc,
                         (first && q < J) ? 0u : 1u);
        }
    }
}

template <int NMB, int J, bool PAIR, int MB0 = 0, int MBS = 1>
__device__ __forceinline__ void issue_stage(bool halo, int ks, uint32_t d_tile, uint32_t bn,
                                            uint64_t a_desc, uint32_t wp_units, uint32_t rb16,
                                            uint64_t b_desc, uint32_t b_tap_units, uint32_t idesc,
                                            bool first, int hmode = 0, uint32_t plane_units = 0,
                                            int taps1d = 0, uint32_t dil_units = 0) {
    if (!PAIR && halo && taps1d) {
        if (ks == 4) issue_halo1d<4, NMB, J, MB0, MBS>(d_tile, bn, a_desc, rb16, b_desc, b_tap_units, idesc, first, taps1d, dil_units);
        else if (ks == 2) issue_halo1d<2, NMB, J, MB0, MBS>(d_tile, bn, a_desc, rb16, b_desc, b_tap_units, idesc, first, taps1d, dil_units);
        else issue_halo1d<1, NMB, J, MB0, MBS>(d_tile, bn, a_desc, rb16, b_desc, b_tap_units, idesc, first, taps1d, dil_units);
    } else if (!PAIR && halo) {
        if (ks == 4) issue_halo<4, NMB, J, MB0, MBS>(d_tile, bn, a_desc, wp_units, rb16, b_desc, b_tap_units, idesc, first, hmode, plane_units);
        else if (ks == 2) issue_halo<2, NMB, J, MB0, MBS>(d_tile, bn, a_desc, wp_units, rb16, b_desc, b_tap_units, idesc, first, hmode, plane_units);
        else issue_halo<1, NMB, J, MB0, MBS>(d_tile, bn, a_desc, wp_units, rb16, b_desc, b_tap_units, idesc, first, hmode, plane_units);
    } else {
        if (ks == 4) issue_tap<4, NMB, J, PAIR, MB0, MBS>(d_tile, bn, a_desc, rb16, b_desc, idesc, first);
        else if (ks == 2) issue_tap<2, NMB, J, PAIR, MB0, MBS>(d_tile, bn, a_desc, rb16, b_desc, idesc, first);
        else issue_tap<1, NMB, J, PAIR, MB0, MBS>(d_tile, bn, a_desc, rb16, b_desc, idesc, first);
    }
}

// The stage's MMAs for issuer `iss` of `n_iss`: with two issuing warps each takes
// every second row block (compile-time start and stride, so each issuer's unrolled
// sequence has the same shape as a single issuer's).
template <int NMB, int J, bool PAIR, bool SEQ>
__device__ __forceinline__ void issue_split(int n_iss, int iss, bool halo, int ks, uint32_t d_tile,
                                            uint32_t bn, uint64_t a_desc, uint32_t wp_units,
                                            uint32_t rb16, uint64_t b_desc, uint32_t b_tap_units,
                                            uint32_t idesc, bool first, int hmode = 0,
                                            uint32_t plane_units = 0, int taps1d = 0,
                                            uint32_t dil_units = 0) {
    if constexpr (NMB >= 2 && !PAIR && !SEQ) {
        if (n_iss == 2) {
            if (iss == 0)
                issue_stage<NMB, J, PAIR, 0, 2>(halo, ks, d_tile, bn, a_desc, wp_units, rb16,
                                                b_desc, b_tap_units, idesc, first, hmode,
                                                plane_units, taps1d, dil_units);
            else
                issue_stage<NMB, J, PAIR, 1, 2>(halo, ks, d_tile, bn, a_desc, wp_units, rb16,
                                                b_desc, b_tap_units, idesc, first, hmode,
                                                plane_units, taps1d, dil_units);
            return;
        }
    }
    issue_stage<NMB, J, PAIR>(halo, ks, d_tile, bn, a_desc, wp_units, rb16, b_desc, b_tap_units,
                              idesc, first, hmode, plane_units, taps1d, dil_units);
}

// The QPACK stage `half` for issuer `iss` of `n_iss` (two issuers take alternate row
// blocks, as issue_split).
template <int NMB>
__device__ __forceinline__ void qpack_stage(int n_iss, int iss, int half, uint32_t d_tile,
                                            uint64_t a_desc, uint32_t wq_units, uint64_t b_desc,
                                            const uint32_t (&idn)[3], bool first) {
    if constexpr (NMB >= 2) {
        if (n_iss == 2) {
            if (iss == 0) {
                if (half) issue_qpack<NMB, 1, 0, 2>(d_tile, a_desc, wq_units, b_desc, idn, first);
                else issue_qpack<NMB, 0, 0, 2>(d_tile, a_desc, wq_units, b_desc, idn, first);
            } else {
                if (half) issue_qpack<NMB, 1, 1, 2>(d_tile, a_desc, wq_units, b_desc, idn, first);
                else issue_qpack<NMB, 0, 1, 2>(d_tile, a_desc, wq_units, b_desc, idn, first);
            }
            return;
        }
    }
    if (half) issue_qpack<NMB, 1, 0, 1>(d_tile, a_desc, wq_units, b_desc, idn, first);
    else issue_qpack<NMB, 0, 0, 1>(d_tile, a_desc, wq_units, b_desc, idn, first);
}

// Persistent tile loop bounds. Read from the special registers at each loop rather
// than held in kernel-lifetime variables: keeping them live across the roles cost
// the epilogue-bound 2-D convs up to 15% (register pressure in the epilogue).
template <bool PAIR>
__device__ __forceinline__ int first_tile() {
    return PAIR ? (int)(blockIdx.x >> 1) : (int)blockIdx.x;
}
template <bool PAIR>
__device__ __forceinline__ int tile_stride() {
    return PAIR ? (int)(gridDim.x >> 1) : (int)gridDim.x;
}

// PAIR: the CTA is one half of a cta_group::2 pair (cluster of 2, TAP feeds only,
// NMB = J = 1). The pair computes a 256-row tile: each CTA loads its own 128 A rows
// and half of the tile's weight columns; the even CTA issues the pair MMAs and its
// commits arrive in both CTAs; every load of the pair completes on the even CTA's
// full barrier, and both CTAs' epilogue warps release the even CTA's accumulator.
template <int NMB, int J, bool PAIR, bool SEQ, bool PLAIN = false, bool QP = false>
__global__ void __launch_bounds__(kThreads, 1)
conv_tc_kernel(const __grid_constant__ CUtensorMap tmA0, const __grid_constant__ CUtensorMap tmB0,
               const __grid_constant__ CUtensorMap tmA1, const __grid_constant__ CUtensorMap tmB1,
               const __grid_constant__ CUtensorMap tmY, const __grid_constant__ ConvDev p) {
    extern __shared__ uint8_t smem_raw[];
    const uint32_t raw_u32 = smem_u32(smem_raw);
    const uint32_t base = (raw_u32 + 1023u) & ~1023u;
    uint8_t* smem = smem_raw + (base - raw_u32);
    const uint32_t S = p.n_stages;
    float* sbias = reinterpret_cast<float*>(smem + p.bias_off);
    int* stv = reinterpret_cast<int*>(smem + p.tv_off);
    float* sss = (SEQ && p.ss_off) ? reinterpret_cast<float*>(smem + p.ss_off) : nullptr;
    const uint32_t bar_full = base + p.bar_off;
    const uint32_t bar_empty = bar_full + 8 * S;
    const uint32_t bar_tfull = bar_empty + 8 * S;
    const uint32_t bar_tempty = bar_tfull + 16;
    const uint32_t bar_bres = bar_tempty + 16;
    const uint32_t bar_xfull = bar_bres + 8;  // [S]: stage transformed (xform)
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + p.bar_off + 8 * (3 * S + 5));
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const uint32_t rank = PAIR ? cluster_ctarank() : 0u;  // 0: the MMA-issuing CTA

    // QPACK: the 128 accumulator columns are 4 pixel phases x the 32 output channels
    for (int i = threadIdx.x; i < p.oc; i += blockDim.x)
        sbias[i] = p.bias ? p.bias[QP ? (i & 31) : i] : 0.0f;
    if (sss)
        for (int i = threadIdx.x; i < p.oc; i += blockDim.x) {
            sss[i] = p.bn_scale[i];
            sss[p.oc + i] = p.bn_shift[i];
        }
    for (int i = threadIdx.x; i < p.batch; i += blockDim.x) stv[i] = p.tvalid[i];
    if (threadIdx.x == 0) {
        const uint32_t n_iss = (SEQ || PAIR) ? 1u : (uint32_t)p.n_iss;  // commits per phase
        for (uint32_t s = 0; s < S; ++s) {
            mbar_init(bar_full + 8 * s, 1);
            mbar_init(bar_empty + 8 * s, n_iss);
            mbar_init(bar_xfull + 8 * s, 2);  // one arrival per transform warp
        }
        for (int a = 0; a < 2; ++a) {
            mbar_init(bar_tfull + 8 * a, n_iss);
            mbar_init(bar_tempty + 8 * a, PAIR ? 2 * (kEpiThreads / 32) : kEpiThreads);
        }
        mbar_init(bar_bres, 1);
        *abort_flag = 0;
        fence_barrier_init();
        fence_proxy_async_smem();
    }
    if (warp == 0 && lane == 0) {
        tma_prefetch_desc(&tmA0);
        tma_prefetch_desc(&tmB0);
        if (p.n_seg > 1) {
            tma_prefetch_desc(&tmA1);
            tma_prefetch_desc(&tmB1);
        }
    }
    if (warp == 1) {
        if constexpr (PAIR) tmem_alloc_pair(smem_u32(tmem_slot), p.tmem_cols);
        else tmem_alloc(smem_u32(tmem_slot), p.tmem_cols);
    }
    // resident q8_0 weights: every thread expands its share once (the weights predate
    // this kernel, so this may overlap the previous one's tail)
    {
        bool wrote = false;
        if (QP) {
            if (p.seg[0].wq) {
                // the packed rows: 32 channels (64 bytes, 64-byte swizzle) each
                q8_expand(p.seg[0], 32, 0, 1152, 0, base + p.seg[0].bres, threadIdx.x, blockDim.x);
                wrote = true;
            }
        } else {
            for (int sg = 0; sg < p.n_seg; ++sg) {
                const SegDev& s = p.seg[sg];
                if (s.mode != SEG_HALO || !s.wq) continue;
                const uint32_t box = (uint32_t)p.BN * s.kb * 2;
                for (int tap = 0; tap < s.n_taps; ++tap)
                    for (int kbi = 0; kbi < s.n_kb; ++kbi)
                        q8_expand(s, s.kb, 0, p.BN, tap * s.ic + kbi * s.kb,
                                  base + s.bres + (uint32_t)(tap * s.n_kb + kbi) * box,
                                  threadIdx.x, blockDim.x);
                wrote = true;
            }
        }
        if (wrote) fence_proxy_async_smem();  // generic writes -> the tensor cores' view
    }
    tc_fence_before();
    if constexpr (PAIR) cluster_sync();  // the peer's barriers exist before any signal
    else __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;
    // Everything above reads only data that existed before the previous kernel on the
    // stream started (weights, bias, BN scale / shift, per-clip lengths), so the next
    // conv may run up to this point while this one finishes (its CTAs take SMs as ours
    // leave); nothing below starts before the previous kernel has completed.
    if (threadIdx.x == 0) pdl_launch_dependents();
    pdl_wait();

    const int n_tiles = p.n_mt * p.n_nt;
    const uint32_t idesc = umma_idesc_f16(PAIR ? 2 * kMB : kMB, p.BN);
    const uint32_t acc_cols = (uint32_t)(NMB * J * p.BN);

    if (warp == 0) {
        if (lane == 0) {
            // ---------------- TMA producer ----------------
            // Resident weights of HALO segments: every (tap, channel block) box once.
            if (QP) {
                // QPACK: the packed weights, 9 boxes of 128 rows x 32 channels
                if (p.bres_tx) {
                    mbar_arrive_expect_tx(bar_bres, p.bres_tx);
                    for (int r = 0; r < 1152; r += 128)
                        tma_load_2d(base + p.seg[0].bres + (uint32_t)r * 64u, &tmB0, bar_bres, 0, r);
                }
            } else if (p.bres_tx) {
                mbar_arrive_expect_tx(bar_bres, p.bres_tx);
                for (int sg = 0; sg < p.n_seg; ++sg) {
                    const SegDev& s = p.seg[sg];
                    if (s.mode != SEG_HALO || s.wq) continue;
                    const CUtensorMap* tb = sg ? &tmB1 : &tmB0;
                    const uint32_t box = (uint32_t)p.BN * s.kb * 2;
                    for (int tap = 0; tap < s.n_taps; ++tap)
                        for (int kbi = 0; kbi < s.n_kb; ++kbi)
                            tma_load_2d(base + s.bres + (uint32_t)(tap * s.n_kb + kbi) * box, tb,
                                        bar_bres, tap * s.ic + kbi * s.kb, 0);
                }
            }
            uint32_t stage = 0, phase = 0;
            bool ok = true;
            if (p.two_ring) {
                // A halo (or the TAP segment's A rows) per channel block into the A
                // ring, then that block's weight tile per tap into the weight ring.
                uint32_t sa = 0, pa = 0, sb = 0, pb = 0;
                for (int tile = blockIdx.x; tile < n_tiles && ok; tile += gridDim.x) {
                    const int mt = tile / p.n_nt, nt = tile - mt * p.n_nt;
                    const int m0 = mt * p.BM, n0 = nt * p.BN;
                    if (!tile_live<SEQ, QP>(p, stv, m0)) continue;
                    for (int sg = 0; sg < p.n_seg && ok; ++sg) {
                        const SegDev& s = p.seg[sg];
                        const CUtensorMap* ta = sg ? &tmA1 : &tmA0;
                        const CUtensorMap* tb = sg ? &tmB1 : &tmB0;
                        const bool hs = s.mode == SEG_HALO_S;
                        const uint32_t box_bytes = (uint32_t)s.box_rows * s.kb * 2;
                        for (int kbi = 0; kbi < s.n_kb && ok; ++kbi) {
                            if (!mbar_wait(bar_empty + 8 * sa, pa ^ 1, p.err, VDB_ERR_TIMEOUT_EMPTY,
                                           abort_flag)) {
                                ok = false;
                                break;
                            }
                            const uint32_t fa = bar_full + 8 * sa;
                            const uint32_t da = base + p.stage0 + sa * p.a_stride;
                            mbar_arrive_expect_tx(fa, s.a_bytes);
                            for (int bx = 0; bx < s.n_box; ++bx)
                                tma_load_3d(da + bx * box_bytes, ta, fa, kbi * s.kb,
                                            (hs ? m0 - s.halo_back : m0 + s.off[0]) +
                                                bx * s.box_rows,
                                            hs ? 0 : s.plane[0]);
                            if (++sa == (uint32_t)p.ra) {
                                sa = 0;
                                pa ^= 1;
                            }
                            for (int tap = 0; tap < s.n_taps; ++tap) {
                                const uint32_t ib = (uint32_t)p.ra + sb;
                                if (!mbar_wait(bar_empty + 8 * ib, pb ^ 1, p.err,
                                               VDB_ERR_TIMEOUT_EMPTY, abort_flag)) {
                                    ok = false;
                                    break;
                                }
                                const uint32_t fw = bar_full + 8 * ib;
                                mbar_arrive_expect_tx(fw, s.b_bytes);
                                tma_load_2d(base + p.b_ring0 + sb * p.b_stride, tb, fw,
                                            tap * s.ic + kbi * s.kb, n0);
                                if (++sb == (uint32_t)p.rb) {
                                    sb = 0;
                                    pb ^= 1;
                                }
                            }
                        }
                    }
                }
                if (!ok) {
                    for (uint32_t i = 0; i < S; ++i)
                        mbar_wait_drain(bar_full + 8 * i, i < (uint32_t)p.ra ? pa : pb, 20000000ull);
                }
            }
            for (int tile = first_tile<PAIR>(); tile < n_tiles && ok && !p.two_ring; tile += tile_stride<PAIR>()) {
                const int mt = tile / p.n_nt, nt = tile - mt * p.n_nt;
                const int m0 = mt * p.BM, n0 = nt * p.BN;
                if (!tile_live<SEQ, QP>(p, stv, m0)) continue;
                // this CTA's A rows and weight rows (a pair splits both in halves)
                [[maybe_unused]] const int am0 = m0 + (int)rank * kMB;
                [[maybe_unused]] const int bn0 = n0 + (int)rank * (p.BN / 2);
                for (int sg = 0; sg < p.n_seg && ok; ++sg) {
                    const SegDev& s = p.seg[sg];
                    const CUtensorMap* ta = sg ? &tmA1 : &tmA0;
                    const CUtensorMap* tb = sg ? &tmB1 : &tmB0;
                    const int iters = s.mode == SEG_HALO ? s.n_kb : s.n_taps * s.n_kb;
                    for (int it = 0; it < iters; ++it) {
                        if (!mbar_wait(bar_empty + 8 * stage, phase ^ 1, p.err,
                                       VDB_ERR_TIMEOUT_EMPTY, abort_flag)) {
                            ok = false;
                            break;
                        }
                        const uint32_t fb = bar_full + 8 * stage;
                        const uint32_t sa = base + p.stage0 + stage * p.stage_bytes;
                        if constexpr (PAIR) {
                            // both CTAs' bytes complete on the even CTA's barrier
                            const uint32_t fl = mapa_shared(fb, 0);
                            if (rank == 0) mbar_arrive_expect_tx(fb, 2 * s.bytes);
                            const int tap = it / s.n_kb, kbi = it - tap * s.n_kb;
                            tma_load_3d_pair(sa, ta, fl, kbi * s.kb, am0 + s.off[tap], s.plane[tap]);
                            tma_load_2d_pair(sa + p.a_region, tb, fl, tap * s.ic + kbi * s.kb, bn0);
                            if (++stage == S) {
                                stage = 0;
                                phase ^= 1;
                            }
                            continue;
                        }
                        mbar_arrive_expect_tx(fb, s.bytes);
                        if (s.mode == SEG_HALO) {
                            const uint32_t box_bytes = (uint32_t)s.box_rows * s.kb * 2;
                            for (int bx = 0; bx < s.n_box; ++bx)
                                tma_load_3d(sa + bx * box_bytes, ta, fb, it * s.kb,
                                            m0 - s.halo_back + bx * s.box_rows, 0);
                            // FPHASE / PHASE: the other planes' halos
                            for (int q = 1; q < s.halo_planes; ++q)
                                for (int bx = 0; bx < s.n_box; ++bx)
                                    tma_load_3d(sa + q * s.plane_bytes + bx * box_bytes, ta, fb,
                                                it * s.kb, m0 - s.halo_back + bx * s.box_rows, q);
                        } else {
                            const int tap = it / s.n_kb, kbi = it - tap * s.n_kb;
                            const uint32_t box_bytes = (uint32_t)s.box_rows * s.kb * 2;
                            for (int bx = 0; bx < s.n_box; ++bx)
                                tma_load_3d(sa + bx * box_bytes, ta, fb, kbi * s.kb,
                                            m0 + s.off[tap] + bx * s.box_rows, s.plane[tap]);
                            tma_load_2d(sa + p.a_region, tb, fb, tap * s.ic + kbi * s.kb, n0);
                        }
                        if (++stage == S) {
                            stage = 0;
                            phase ^= 1;
                        }
                    }
                }
            }
            if (!ok && !p.two_ring) {
                // Let copies already issued land before the CTA can exit.
                for (uint32_t i = 0; i < S; ++i) mbar_wait_drain(bar_full + 8 * i, phase, 20000000ull);
            }
        }
    } else if (warp == 1 || (!SEQ && !PAIR && warp == 2 && p.n_iss == 2)) {
        // One MMA-issuing thread paces small-N tiles (an N = 32 MMA every ~57 cycles
        // from one thread against the tensor pipe's 40): 2-D tiles of two or more row
        // blocks split them over warps 1 and 2, each committing to every barrier.
        const int n_iss = (SEQ || PAIR) ? 1 : p.n_iss;
        const int iss = warp - 1;
        if (lane == 0 && rank == 0) {
            // ---------------- MMA issuer ----------------
            uint32_t stage = 0, phase = 0;
            uint32_t acc = 0, acc_phase = 0;
            uint32_t sa = 0, pa = 0, sb = 0, pb = 0;  // two-ring slots and phases
            [[maybe_unused]] const uint32_t qp_idn[3] = {umma_idesc_f16(kMB, 32), umma_idesc_f16(kMB, 64),
                                                         umma_idesc_f16(kMB, 96)};
            bool ok = true, issued = false;
            if (p.bres_tx &&
                !mbar_wait(bar_bres, 0, p.err, VDB_ERR_TIMEOUT_FULL, abort_flag))
                ok = false;
            for (int tile = first_tile<PAIR>(); tile < n_tiles && ok; tile += tile_stride<PAIR>()) {
                const int mt = tile / p.n_nt;
                if (!tile_live<SEQ, QP>(p, stv, mt * p.BM)) continue;
                if (!mbar_wait(bar_tempty + 8 * acc, acc_phase ^ 1, p.err,
                               VDB_ERR_TIMEOUT_TEMPTY, abort_flag)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                const uint32_t d_tile = tmem_base + acc * acc_cols;
                bool first = true;
                for (int sg = 0; sg < p.n_seg && ok; ++sg) {
                    const SegDev& s = p.seg[sg];
                    const bool halo = s.mode == SEG_HALO;
                    const int row_bytes = s.kb * 2;
                    const uint32_t rb16 = (uint32_t)s.kb / 8;  // a row in 16-byte units
                    const int ksteps = s.kb / 16;
                    const int iters = halo ? s.n_kb : s.n_taps * s.n_kb;
                    const uint64_t a_desc0 = umma_sdesc(base + p.stage0, row_bytes);
                    const uint64_t bres_desc = umma_sdesc(base + s.bres, row_bytes);
                    const uint32_t wp_units = (uint32_t)p.Wp * rb16;
                    const uint32_t b_kb_units = (uint32_t)p.BN * rb16;
                    const uint32_t b_tap_units = (uint32_t)s.n_kb * b_kb_units;
                    if (p.two_ring) {
                        const bool hs = s.mode == SEG_HALO_S;
                        for (int kbi = 0; kbi < s.n_kb && ok; ++kbi) {
                            if (!mbar_wait(bar_full + 8 * sa, pa, p.err, VDB_ERR_TIMEOUT_FULL,
                                           abort_flag)) {
                                ok = false;
                                break;
                            }
                            tc_fence_after();
                            const uint64_t a_slot =
                                umma_sdesc(base + p.stage0 + sa * p.a_stride, row_bytes);
                            for (int tap = 0; tap < s.n_taps; ++tap) {
                                const uint32_t ib = (uint32_t)p.ra + sb;
                                if (!mbar_wait(bar_full + 8 * ib, pb, p.err, VDB_ERR_TIMEOUT_FULL,
                                               abort_flag)) {
                                    ok = false;
                                    break;
                                }
                                tc_fence_after();
                                // tap (kt, kf) of a halo starts kt*Wp + kf rows in
                                const uint64_t a_desc =
                                    a_slot + (hs ? (uint64_t)((tap / 3) * wp_units + (tap % 3) * rb16)
                                                 : 0ull);
                                const uint64_t b_desc =
                                    umma_sdesc(base + p.b_ring0 + sb * p.b_stride, row_bytes);
                                issue_split<NMB, J, false, SEQ>(n_iss, iss, false, ksteps, d_tile,
                                                                (uint32_t)p.BN, a_desc, wp_units,
                                                                rb16, b_desc, b_tap_units, idesc,
                                                                first);
                                first = false;
                                umma_commit(bar_empty + 8 * ib);
                                issued = true;
                                if (++sb == (uint32_t)p.rb) {
                                    sb = 0;
                                    pb ^= 1;
                                }
                            }
                            if (!ok) break;
                            umma_commit(bar_empty + 8 * sa);
                            if (++sa == (uint32_t)p.ra) {
                                sa = 0;
                                pa ^= 1;
                            }
                        }
                        continue;
                    }
                    // with the input prologue, a stage is ready once both transform
                    // warps have rewritten it (they wait for its TMA bytes themselves)
                    const uint32_t ready = p.xform ? bar_xfull : bar_full;
                    for (int it = 0; it < iters; ++it) {
                        if (!mbar_wait(ready + 8 * stage, phase, p.err, VDB_ERR_TIMEOUT_FULL,
                                       abort_flag)) {
                            ok = false;
                            break;
                        }
                        tc_fence_after();
                        const uint64_t a_desc = a_desc0 + (uint64_t)(stage * (p.stage_bytes >> 4));
                        if constexpr (QP) {
                            if (sg == 0) {
                                // stage `it` = channel half `it` of the QPACK halo
                                qpack_stage<NMB>(n_iss, iss, it, d_tile, a_desc, wp_units,
                                                 umma_sdesc(base + s.bres, 64), qp_idn, first);
                                goto stage_issued;
                            }
                        }
                        {
                        const uint64_t b_desc = halo ? bres_desc + (uint64_t)(it * b_kb_units)
                                                     : a_desc + (uint64_t)(p.a_region >> 4);
                        issue_split<NMB, J, PAIR, SEQ>(n_iss, iss, halo, ksteps, d_tile,
                                                       (uint32_t)p.BN, a_desc, wp_units, rb16,
                                                       b_desc, b_tap_units, idesc, first,
                                                       s.halo_mode, s.plane_bytes >> 4,
                                                       SEQ ? s.n_taps : 0,
                                                       SEQ ? (uint32_t)s.dil * rb16 : 0u);
                        }
                    stage_issued:
                        first = false;
                        if constexpr (PAIR) umma_commit_pair(bar_empty + 8 * stage, 0x3);
                        else umma_commit(bar_empty + 8 * stage);
                        issued = true;
                        if (++stage == S) {
                            stage = 0;
                            phase ^= 1;
                        }
                    }
                }
                if (!ok) break;
                if constexpr (PAIR) umma_commit_pair(bar_tfull + 8 * acc, 0x3);
                else umma_commit(bar_tfull + 8 * acc);
                if (p.n_acc == 2 && ++acc == 2) {
                    acc = 0;
                    acc_phase ^= 1;
                } else if (p.n_acc == 1) {
                    acc_phase ^= 1;
                }
            }
            if (!ok && issued) {
                // Make sure no MMA is still writing TMEM before teardown: wait for the
                // commit that followed the last issued MMAs.
                if (p.two_ring) {
                    const uint32_t lb = (sb + (uint32_t)p.rb - 1) % (uint32_t)p.rb;
                    mbar_wait_drain(bar_empty + 8 * ((uint32_t)p.ra + lb), sb == 0 ? pb ^ 1u : pb,
                                    20000000ull);
                } else {
                    const uint32_t last = (stage + S - 1) % S;
                    mbar_wait_drain(bar_empty + 8 * last, phase ^ (stage == 0 ? 1u : 0u),
                                    20000000ull);
                }
            }
        }
    } else if (warp == 2 || warp == 3) {
        if constexpr (SEQ && !PAIR) {
            if (p.xform) {
                // ---------------- input prologue (BN + ReLU of the A tiles) ----------
                // Thread t owns the 16-byte chunks at byte offsets t*16 + 1024*k of each
                // A tile. The tile is 1024-byte aligned and the TMA swizzle XORs the
                // chunk index within a row with address bits [7, 10), so every chunk a
                // thread owns holds the same 8 input channels: chunk ((t ^ (t >> 3)) &
                // (row chunks - 1)) of the row.
                const SegDev& s = p.seg[0];
                const int t = (int)threadIdx.x - 64;
                const uint32_t rowbytes = (uint32_t)s.kb * 2;
                const uint32_t o0 = (uint32_t)t * 16u;
                const int lchunk = (int)(((o0 >> 4) ^ (o0 >> 7)) & (rowbytes / 16 - 1));
                const uint32_t a_bytes = (uint32_t)(s.n_box * s.box_rows) * rowbytes;
                uint32_t stage = 0, phase = 0;
                bool ok = true;
                for (int tile = first_tile<false>(); tile < n_tiles && ok;
                     tile += tile_stride<false>()) {
                    const int mt = tile / p.n_nt;
                    if (!tile_live<SEQ, QP>(p, stv, mt * p.BM)) continue;
                    for (int it = 0; it < s.n_kb; ++it) {
                        if (!mbar_wait(bar_full + 8 * stage, phase, p.err, VDB_ERR_TIMEOUT_XFORM,
                                       abort_flag)) {
                            ok = false;
                            break;
                        }
                        const int c0 = it * s.kb + lchunk * 8;
                        const float4 s0 = __ldg(reinterpret_cast<const float4*>(p.x_scale + c0));
                        const float4 s1 = __ldg(reinterpret_cast<const float4*>(p.x_scale + c0 + 4));
                        const float4 h0 = __ldg(reinterpret_cast<const float4*>(p.x_shift + c0));
                        const float4 h1 = __ldg(reinterpret_cast<const float4*>(p.x_shift + c0 + 4));
                        // f16x2 fused multiply-add with ReLU (one rounding of the exact
                        // x*scale + shift, with scale and shift rounded to f16): a third of
                        // the instructions of the f32 form, which two warps could not
                        // issue as fast as the tensor cores consume the tiles
                        const __half2 sc[4] = {__floats2half2_rn(s0.x, s0.y), __floats2half2_rn(s0.z, s0.w),
                                               __floats2half2_rn(s1.x, s1.y), __floats2half2_rn(s1.z, s1.w)};
                        const __half2 sh[4] = {__floats2half2_rn(h0.x, h0.y), __floats2half2_rn(h0.z, h0.w),
                                               __floats2half2_rn(h1.x, h1.y), __floats2half2_rn(h1.z, h1.w)};
                        uint8_t* a = smem + p.stage0 + stage * p.stage_bytes;
#pragma unroll 4
                        for (uint32_t o = o0; o < a_bytes; o += 1024u) {
                            uint4 v = *reinterpret_cast<const uint4*>(a + o);
                            __half2* hv = reinterpret_cast<__half2*>(&v);
#pragma unroll
                            for (int q = 0; q < 4; ++q) hv[q] = __hfma2_relu(hv[q], sc[q], sh[q]);
                            *reinterpret_cast<uint4*>(a + o) = v;
                        }
                        // generic-proxy writes -> visible to the tensor cores' async proxy
                        fence_proxy_async_smem();
                        __syncwarp();
                        if (lane == 0) mbar_arrive(bar_xfull + 8 * stage);
                        if (++stage == S) {
                            stage = 0;
                            phase ^= 1;
                        }
                    }
                }
            }
        }
    } else if (warp >= kEpiWarp0) {
        // ---------------- epilogue ----------------
        const int ew = warp - kEpiWarp0;
        const int quad = warp & 3;        // TMEM lane quadrant this warp may access
        const int half = ew >> 2;
        // Several 128-row blocks: warp half h drains blocks h, h+2, ... over all
        // columns, so each row's index math is done once. One block: the halves
        // split the columns (multiples of 16), or the first half takes them all.
        const bool mb_split = NMB >= 2;
        const bool split = !mb_split && p.BN % 32 == 0;
        const int c_lo = split ? half * (p.BN / 2) : 0;
        const int c_hi = mb_split ? p.BN : (split ? c_lo + p.BN / 2 : (half == 0 ? p.BN : 0));
        uint32_t acc = 0, acc_phase = 0;
        // staged output: this warp's two buffers and the chunks it has staged
        const uint32_t stage_base = base + p.ostage_off + (uint32_t)ew * 4096u;
        uint32_t stage_n = 0;
        for (int tile = first_tile<PAIR>(); tile < n_tiles; tile += tile_stride<PAIR>()) {
            const int mt = tile / p.n_nt, nt = tile - mt * p.n_nt;
            const int m0 = mt * p.BM + (int)rank * kMB, n0 = nt * p.BN;
            const bool live = tile_live<SEQ, QP>(p, stv, mt * p.BM);
            // QPACK residual: the (mb, 32-column chunk) units this thread stores, in
            // order; the first unit's residual is loaded before the accumulator wait and
            // each next one while the current unit is converted, so the residual read
            // overlaps the MMAs and the stores instead of following them
            const int qp_mb0 = mb_split ? half : 0, qp_mbs = mb_split ? 2 : 1;
            const int qp_nc = (c_hi - c_lo) >> 5;
            const int qp_units = QP ? ((NMB - qp_mb0 + qp_mbs - 1) / qp_mbs) * qp_nc : 0;
            uint4 res[4] = {};
            auto qp_res_load = [&](int u, uint4 (&r)[4]) {
                const int mb = qp_mb0 + (u / qp_nc) * qp_mbs;
                const int c = c_lo + (u % qp_nc) * 32;
                const int m = m0 + mb * kMB + quad * 32 + lane;
                if (p.qp_res && m < p.M) {
                    const uint4* rp = reinterpret_cast<const uint4*>(p.qp_res + (long long)m * 128 + c);
#pragma unroll
                    for (int q = 0; q < 4; ++q) r[q] = __ldg(rp + q);
                }
            };
            if constexpr (QP) {
                if (qp_units > 0) qp_res_load(0, res);
            }
            if (live) {
                if (!mbar_wait(bar_tfull + 8 * acc, acc_phase, p.err, VDB_ERR_TIMEOUT_TFULL,
                               abort_flag))
                    break;
                tc_fence_after();
            }
            if constexpr (QP) {
                for (int u = 0; u < qp_units; ++u) {
                    const int mb = qp_mb0 + (u / qp_nc) * qp_mbs;
                    const int c = c_lo + (u % qp_nc) * 32;
                    const int m = m0 + mb * kMB + quad * 32 + lane;
                    const uint32_t tb = tmem_base + ((uint32_t)(quad * 32) << 16) + acc * acc_cols +
                                        (uint32_t)(mb * p.BN);
                    uint4 nres[4] = {};
                    if (u + 1 < qp_units) qp_res_load(u + 1, nres);
                    uint32_t v[32];
                    if (live) {
                        tmem_ld_32x32b_x32(tb + (uint32_t)c, v);
                    } else {
#pragma unroll
                        for (int i = 0; i < 32; ++i) v[i] = 0u;
                    }
                    uint32_t o[16] = {};
                    __half* dst = nullptr;
                    const bool has = m < p.M &&
                                     qpack_pack(p, stv, m, live, c >> 5, v, sbias + c, res, o, &dst);
                    if (p.ostage_off) {
                        // the warp's 32 consecutive rows x these 32 columns are one box of
                        // the output map: stage it (64-byte swizzle: 16-byte chunk k of
                        // row r at r*64 + 16*(k ^ ((r >> 1) & 3)), conflict-free) and let
                        // one lane store it; rows past M are clipped by the map
                        const uint32_t buf = stage_base + (stage_n & 1u) * 2048u;
                        if (lane == 0) bulk_wait_read<1>();  // this buffer's last store has read it
                        __syncwarp();
                        const uint32_t sw = (uint32_t)((lane >> 1) & 3);
#pragma unroll
                        for (int k = 0; k < 4; ++k)
                            st_shared_v4(buf + (uint32_t)lane * 64u + (((uint32_t)k ^ sw) << 4),
                                         o[4 * k], o[4 * k + 1], o[4 * k + 2], o[4 * k + 3]);
                        fence_proxy_async_smem();
                        __syncwarp();
                        if (lane == 0) {
                            const int row0 = m0 + mb * kMB + quad * 32;
                            if (row0 < p.M) tma_store_3d(&tmY, buf, c, row0, 0);
                            bulk_commit();  // one group per unit, even when empty
                        }
                        ++stage_n;
                    } else if (has) {
                        uint4* yp = reinterpret_cast<uint4*>(dst);
#pragma unroll
                        for (int k = 0; k < 4; ++k)
                            yp[k] = make_uint4(o[4 * k], o[4 * k + 1], o[4 * k + 2], o[4 * k + 3]);
                    }
#pragma unroll
                    for (int q = 0; q < 4; ++q) res[q] = nres[q];
                }
                goto tile_done;
            }
            for (int mb = 0; mb < NMB; ++mb) {
                if (mb_split && (mb & 1) != half) continue;
                const int m = m0 + mb * kMB + quad * 32 + lane;
                const uint32_t tbase = tmem_base + ((uint32_t)(quad * 32) << 16) +
                                       acc * acc_cols + (uint32_t)(mb * J * p.BN);
                const RowInfo ri = row_info<SEQ>(p, stv, m, live);
                // the host stages only outputs whose chunks are 32 columns wide
                // (the 1-D and K-split kernels store directly: a compile-time 0 folds the
                // staging code away there)
                EpiStage st{&tmY, (!SEQ && J == 1 && p.ostage_off && (c_hi - c_lo) % 32 == 0)
                                      ? stage_base : 0u,
                            stage_n, m0 + mb * kMB + quad * 32};
                if ((c_hi - c_lo) % 32 == 0)
                    epi_rows<32, J, SEQ, PLAIN>(p, live, ri, m, n0, c_lo, c_hi, tbase, sbias, sss, st);
                else
                    epi_rows<16, J, SEQ, PLAIN>(p, live, ri, m, n0, c_lo, c_hi, tbase, sbias, sss, st);
                stage_n = st.n;
            }
        tile_done:
            if (live) {
                tc_fence_before();
                if constexpr (PAIR) {
                    // one arrival per warp on the MMA-issuing CTA's barrier
                    __syncwarp();
                    if (lane == 0) mbar_arrive_cluster(mapa_shared(bar_tempty + 8 * acc, 0));
                } else {
                    mbar_arrive(bar_tempty + 8 * acc);
                }
                if (p.n_acc == 2 && ++acc == 2) {
                    acc = 0;
                    acc_phase ^= 1;
                } else if (p.n_acc == 1) {
                    acc_phase ^= 1;
                }
            }
        }
        // the staged TMA stores have written global memory before the CTA retires
        if (p.ostage_off && lane == 0) bulk_wait<0>();
    }

    tc_fence_before();
    // A pair's MMAs read both CTAs' shared memory and write both TMEMs: neither CTA
    // releases either until the whole pair is done.
    if constexpr (PAIR) cluster_sync();
    else __syncthreads();
    if (warp == 1) {
        __syncwarp();
        tc_fence_after();
        if constexpr (PAIR) tmem_dealloc_pair(tmem_base, p.tmem_cols);
        else tmem_dealloc(tmem_base, p.tmem_cols);
    }
}

// Host side of fdiv: the multiplier and shift for divisor d (1 <= d < 2^31).
void magic_div(uint32_t d, uint32_t& mul, int& sh) {
    int l = 0;
    while ((1ull << l) < d) ++l;
    mul = (uint32_t)(((1ull << 32) * ((1ull << l) - d)) / d + 1);
    sh = l;
}

CUtensorMapSwizzle swizzle_for(int kb) {
    return kb == 64 ? CU_TENSOR_MAP_SWIZZLE_128B
                    : (kb == 32 ? CU_TENSOR_MAP_SWIZZLE_64B : CU_TENSOR_MAP_SWIZZLE_32B);
}

// A operand view: C channels of rows with pitch ld elements (ld > C when the
// tensor is a channel slice of a wider one), in 1 or 4 planes.
bool make_map_a(CUtensorMap* m, const void* ptr, int C, int ld, long long rows, int planes,
                int kb, int box_rows) {
    cuuint64_t dims[3] = {(cuuint64_t)C, (cuuint64_t)rows, (cuuint64_t)planes};
    cuuint64_t strides[2] = {(cuuint64_t)ld * 2, (cuuint64_t)rows * ld * 2};
    cuuint32_t box[3] = {(cuuint32_t)kb, (cuuint32_t)box_rows, 1};
    cuuint32_t estr[3] = {1, 1, 1};
    CUresult r = encode_tiled_fn()(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, const_cast<void*>(ptr),
                                   dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                                   swizzle_for(kb), CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS;
}

bool make_map_b(CUtensorMap* m, const void* ptr, int kcols, int oc, int bn, int kb) {
    cuuint64_t dims[2] = {(cuuint64_t)kcols, (cuuint64_t)oc};
    cuuint64_t strides[1] = {(cuuint64_t)kcols * 2};
    cuuint32_t box[2] = {(cuuint32_t)kb, (cuuint32_t)bn};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = encode_tiled_fn()(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void*>(ptr),
                                   dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                                   swizzle_for(kb), CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS;
}

void fill_taps(SegDev& s, int k, int stride, int ic, int Wp_out) {
    s.ic = ic;
    s.kb = (ic % 64 == 0) ? 64 : ((ic % 32 == 0) ? 32 : 16);
    s.n_kb = ic / s.kb;
    s.n_taps = k * k;
    for (int kt = 0; kt < k; ++kt)
        for (int kf = 0; kf < k; ++kf) {
            const int tap = kt * k + kf;
            if (k == 1) {
                // 1x1: stride 1 reads the same grid row; stride 2 reads padded
                // position (2t+1, 2f+1) = plane 3 at the output's own row; the
                // frequency-only stride 3 reads (t+1, 2f+1) = plane 1 of FPHASE.
                s.plane[tap] = (stride == 2) ? 3 : (stride == 3 ? 1 : 0);
                s.off[tap] = 0;
            } else if (stride == 1) {
                s.plane[tap] = 0;
                s.off[tap] = (kt - 1) * Wp_out + (kf - 1);
            } else if (stride == 3) {
                // FPHASE: padded input (to + kt, 2*fo + kf) is plane kf&1 at the
                // output's row shifted by kt - 1 time rows and kf>>1 columns
                s.plane[tap] = kf & 1;
                s.off[tap] = (kt - 1) * Wp_out + (kf >> 1);
            } else {
                s.plane[tap] = ((kt & 1) << 1) | (kf & 1);
                s.off[tap] = (kt >> 1) * Wp_out + (kf >> 1);
            }
        }
}

// 1-D taps of a k-wide conv with dilation d: row offsets (j - (k-1)/2) * d. With
// stride 2 the input is TPHASE (frame u of the input for output frame o is
// 2*o + u): tap offset u = (j - (k-1)/2) * d reads plane u & 1 at row offset
// floor(u / 2).
void fill_taps_1d(SegDev& s, int k, int dil, int ic, int stride = 1) {
    s.ic = ic;
    s.kb = (ic % 64 == 0) ? 64 : ((ic % 32 == 0) ? 32 : 16);
    s.n_kb = ic / s.kb;
    s.n_taps = k;
    s.dil = dil;
    for (int j = 0; j < k; ++j) {
        const int u = (j - (k - 1) / 2) * dil;
        s.plane[j] = stride == 2 ? (u & 1) : 0;
        s.off[j] = stride == 2 ? (u >> 1) : u;  // arithmetic shift: floor division
    }
}

int round_up(int x, int m) { return (x + m - 1) / m * m; }

// Extras of the 1-D sequence geometry (vdb_conv1d); nullptr for the 2-D grid.
struct SeqArgs {
    int pad, dil0, reflect, y_f32, tile_n, pair, stride0;
    const float* gate;
    int gate_seg, gate_nseg;
    const float* x_scale;
    const float* x_shift;
    const float* clip_bias;
    const float* bn_scale;
    const float* bn_shift;
};

int conv_impl(const vdb_conv_args* a, const SeqArgs* sq, void* stream);
int conv_qpack_impl(const vdb_conv_args* a, void* stream);

}  // namespace
}  // namespace vdb

using namespace vdb;

extern "C" long long vdb_grid_rows(int batch, int t, int f) {
    return (long long)batch * (t + 2) * (f + 2);
}

extern "C" long long vdb_phase_rows(int batch, int t, int f) {
    const int to = (t - 1) / 2 + 1, fo = (f - 1) / 2 + 1;
    return 4LL * batch * (to + 2) * (fo + 2);
}

namespace vdb {
namespace {
thread_local int g_conv_launches = 0;
}
int last_conv_launches() { return g_conv_launches; }
}  // namespace vdb

extern "C" int vdb_conv(const vdb_conv_args* a, void* stream) {
    g_conv_launches = 1;
    if (!a) {
        set_error("vdb_conv: NULL args");
        return 1;
    }
    if (a->qpack) return conv_qpack_impl(a, stream);
    return conv_impl(a, nullptr, stream);
}

extern "C" long long vdb_qpack_rows(int batch, int t, int f) {
    return (long long)batch * (t + 2) * ((f + 2 + 3) / 4);
}

namespace vdb {
namespace {
// out[kt][r][ic], r = the packed row of (u, j, oc) (see qp_wrow): W[oc][kt*3 + u - j + 1][ic]
__global__ void qpack_pack_kernel(const __half* __restrict__ w, __half* __restrict__ out) {
    const int e = blockIdx.x * blockDim.x + threadIdx.x;
    if (e >= 3 * 384 * 32) return;
    const int ic = e & 31, r = (e >> 5) % 384, kt = (e >> 5) / 384;
    int u = -1;
    for (int c = 0; c <= 4; ++c)
        if (r >= qp_wrow(0, c)) u = c;
    const int rr = r - qp_wrow(0, u);
    const int j = qp_jmin(u) + rr / 32, oc = rr & 31;
    out[e] = w[((size_t)oc * 9 + kt * 3 + (u - j + 1)) * 32 + ic];
}
}  // namespace
}  // namespace vdb

extern "C" int vdb_qpack_pack_weights(const void* w_taps, void* out, void* stream) {
    if (!w_taps || !out) {
        set_error("vdb_qpack_pack_weights: NULL argument");
        return 1;
    }
    qpack_pack_kernel<<<(3 * 384 * 32 + 255) / 256, 256, 0, static_cast<cudaStream_t>(stream)>>>(
        static_cast<const __half*>(w_taps), static_cast<__half*>(out));
    VDB_CHECK_CUDA(cudaGetLastError());
    return 0;
}

extern "C" long long vdb_seq_rows(int batch, int t, int pad) {
    return (long long)batch * (t + 2LL * pad);
}

extern "C" int vdb_conv1d(const vdb_conv1d_args* c, void* stream) {
    g_conv_launches = 1;
    if (!c) {
        set_error("vdb_conv1d: NULL args");
        return 1;
    }
    if (c->pad < 0 || c->k0 < 1 || c->k0 > 9 || c->k0 % 2 == 0 || c->dil0 < 1 ||
        (c->k0 - 1) / 2 * c->dil0 > c->pad) {
        set_error("vdb_conv1d: k0 must be odd in [1, 9], dil0 >= 1 and (k0-1)/2 * dil0 <= pad");
        return 1;
    }
    if (c->act != 0 && c->act != 1 && c->act != 3 && c->act != 4 && c->act != 5) {
        set_error("vdb_conv1d: act must be 0, 1, 3, 4 or 5");
        return 1;
    }
    if (c->act == 5 && (!c->gate || c->gate_seg < 1 || c->gate_nseg < 1 ||
                        (c->t - 1) / c->gate_seg >= c->gate_nseg ||
                        (reinterpret_cast<uintptr_t>(c->gate) & 15u) != 0)) {
        set_error("vdb_conv1d: act 5 needs a 16-byte aligned gate [batch][gate_nseg][oc] with "
                  "gate_seg >= 1 and gate_nseg * gate_seg >= t");
        return 1;
    }
    if (c->halo < -1 || c->halo > 1) {
        set_error("vdb_conv1d: halo must be -1 (per-tap tiles), 0 (auto) or 1 (one halo)");
        return 1;
    }
    if (c->reflect < 0 || c->reflect > 2 || c->stride0 < 0 || c->stride0 > 2) {
        set_error("vdb_conv1d: reflect must be 0, 1 or 2 and stride0 0, 1 or 2");
        return 1;
    }
    if (c->stride0 == 2 && c->x1) {
        set_error("vdb_conv1d: a stride-2 conv takes one input segment");
        return 1;
    }
    if (!c->x_scale != !c->x_shift ||
        (c->x_scale && ((reinterpret_cast<uintptr_t>(c->x_scale) & 15u) != 0 ||
                        (reinterpret_cast<uintptr_t>(c->x_shift) & 15u) != 0))) {
        set_error("vdb_conv1d: x_scale and x_shift go together, 16-byte aligned");
        return 1;
    }
    if (c->reflect == 2 && c->y_f32) {
        set_error("vdb_conv1d: zero padding (reflect 2) needs the f16 output");
        return 1;
    }
    if ((c->act == 3 || c->act == 4) && (!c->bn_scale || !c->bn_shift)) {
        set_error("vdb_conv1d: act 3/4 need bn_scale and bn_shift");
        return 1;
    }
    if (c->clip_bias && c->act != 3 && c->act != 4) {
        set_error("vdb_conv1d: clip_bias needs act 3 or 4");
        return 1;
    }
    if (c->y_f32 && c->ysum) {
        set_error("vdb_conv1d: an f32 output has no sum output");
        return 1;
    }
    auto misaligned = [](const void* q) { return (reinterpret_cast<uintptr_t>(q) & 15u) != 0; };
    if ((c->bn_scale && misaligned(c->bn_scale)) || (c->bn_shift && misaligned(c->bn_shift)) ||
        (c->clip_bias && misaligned(c->clip_bias))) {
        set_error("vdb_conv1d: bn_scale / bn_shift / clip_bias must be 16-byte aligned");
        return 1;
    }
    vdb_conv_args a{};
    a.batch = c->batch;
    a.t_out = c->t;
    a.f_out = 1;
    a.oc = c->oc;
    a.k0 = c->k0;
    a.stride0 = 1;
    a.ic0 = c->ic0;
    a.x0 = c->x0;
    a.ldx0 = c->ldx0;
    a.w0 = c->w0;
    a.stride1 = 1;
    a.ic1 = c->ic1;
    a.x1 = c->x1;
    a.ldx1 = c->ldx1;
    a.w1 = c->w1;
    a.bias = c->bias;
    a.residual = c->residual;
    a.ldr = c->ldr;
    a.relu = c->relu;
    a.tvalid = c->tvalid;
    a.y = c->y;
    a.ldy = c->ldy;
    a.err = c->err;
    a.tile_m = c->tile_m;
    a.halo = c->halo;
    a.act = c->act;
    a.ysum = c->ysum;
    a.ldsum = c->ldsum;
    a.addend = c->addend;
    a.ldaddend = c->ldaddend;
    SeqArgs sq{c->pad,  c->dil0,     c->reflect,   c->y_f32 ? 1 : 0, c->tile_n,
               c->pair, c->stride0 == 2 ? 2 : 1, c->gate,    c->gate_seg, c->gate_nseg,
               c->x_scale, c->x_shift, c->clip_bias, c->bn_scale, c->bn_shift};
    return conv_impl(&a, &sq, stream);
}

namespace vdb {
namespace {

int conv_impl(const vdb_conv_args* a, const SeqArgs* sq, void* stream) {
    const bool seq = sq != nullptr;
    if (a->batch <= 0 || a->batch > kMaxBatch || a->t_out <= 0 || a->f_out <= 0) {
        set_error("vdb_conv: batch must be in [1, 8192] and the output non-empty");
        return 1;
    }
    const int oc_max = seq ? 4096 : 1024;
    if (a->oc % 16 != 0 || a->oc <= 0 || a->oc > oc_max) {
        set_error("vdb_conv: oc must be a positive multiple of 16 (<= 1024; <= 4096 for 1-D)");
        return 1;
    }
    if (a->ic0 % 16 != 0 || a->ic0 <= 0 || (a->x1 && (a->ic1 % 16 != 0 || a->ic1 <= 0))) {
        set_error("vdb_conv: input channels must be positive multiples of 16");
        return 1;
    }
    if (!seq && (!(a->k0 == 3 || a->k0 == 1) || a->stride0 < 1 || a->stride0 > 3 ||
                 (a->x1 && (a->stride1 < 1 || a->stride1 > 3)))) {
        set_error("vdb_conv: unsupported kernel/stride");
        return 1;
    }
    if (!seq && (a->y_phase < 0 || a->y_phase > 3 || (a->y2 && a->y_phase > 1) ||
                 (a->y_phase == 3 && (a->y_pad < 1 || a->y_pad > 64)))) {
        set_error("vdb_conv: y_phase must be 0..3 (y2 only with 0 / 1; 3 needs y_pad in [1, 64])");
        return 1;
    }
    if (!a->x0 || !a->w0 || !a->tvalid || !a->y || (a->x1 && !a->w1)) {
        set_error("vdb_conv: NULL buffer");
        return 1;
    }
    if ((a->ldx0 && a->ldx0 < a->ic0) || (a->x1 && a->ldx1 && a->ldx1 < a->ic1) ||
        (a->ldy && a->ldy < a->oc) || (a->ldr && a->ldr < a->oc) || (a->ldr2 && a->ldr2 < a->oc) ||
        (a->ldx0 | a->ldx1 | a->ldy | a->ldr | a->ldr2) % 8 != 0) {
        set_error("vdb_conv: row pitches must be >= the channel count and multiples of 8");
        return 1;
    }
    auto misaligned = [](const void* q) { return (reinterpret_cast<uintptr_t>(q) & 15u) != 0; };
    if (a->ysum && (!a->addend || (a->ldsum && a->ldsum < a->oc) ||
                    (a->ldaddend && a->ldaddend < a->oc) || (a->ldsum | a->ldaddend) % 8 != 0 ||
                    misaligned(a->ysum) || misaligned(a->addend))) {
        set_error("vdb_conv: ysum needs addend, pitches >= oc and multiples of 8, 16-byte "
                  "aligned pointers");
        return 1;
    }
    if (misaligned(a->x0) || (a->x1 && misaligned(a->x1)) || misaligned(a->y) ||
        (a->y2 && misaligned(a->y2)) || (a->residual && misaligned(a->residual)) ||
        (a->residual2 && misaligned(a->residual2))) {
        set_error("vdb_conv: activation pointers must be 16-byte aligned");
        return 1;
    }
    if (!seq && (a->act < 0 || a->act > 2 || (a->act == 2 && (!a->residual || !a->residual2)))) {
        set_error("vdb_conv: act must be 0, 1 or 2 (2 needs residual and residual2)");
        return 1;
    }
    if (seq && (a->y2 || a->y_phase || a->residual2)) {
        set_error("vdb_conv1d: no PHASE outputs or second residual in the 1-D geometry");
        return 1;
    }
    int n_nt = (a->oc + 255) / 256;
    const int tile_n = seq ? sq->tile_n : a->tile_n;
    if (tile_n) {
        if (tile_n % 16 != 0 || tile_n > 256 || a->oc % tile_n != 0) {
            set_error("vdb_conv: tile_n must be a multiple of 16, <= 256, dividing oc");
            return 1;
        }
        n_nt = a->oc / tile_n;
    }
    const int BN = a->oc / n_nt;
    if (BN % 16 != 0 || BN * n_nt != a->oc) {
        set_error("vdb_conv: oc does not split into tcgen05 N tiles");
        return 1;
    }
    // Row indices (and the fdiv fast division) are 32-bit: keep every tensor's row
    // count, plus one tile of slack, below 2^31.
    const long long kMaxRows = (1LL << 31) - 1024;
    if (seq ? vdb_seq_rows(a->batch, a->t_out, sq->pad) > kMaxRows
            : (vdb_grid_rows(a->batch, a->t_out, a->f_out) > kMaxRows ||
               vdb_phase_rows(a->batch, a->t_out, a->f_out) > kMaxRows ||
               vdb_grid_rows(a->batch, 2 * a->t_out, 2 * a->f_out) > kMaxRows)) {
        set_error("vdb_conv: tensor too large (more than 2^31 rows); split the batch");
        return 1;
    }
    ConvDev p{};
    const int Hp = seq ? a->t_out + 2 * sq->pad : a->t_out + 2;
    const int Wp = seq ? 1 : a->f_out + 2;
    p.M = seq ? (int)vdb_seq_rows(a->batch, a->t_out, sq->pad)
              : (int)vdb_grid_rows(a->batch, a->t_out, a->f_out);
    p.n_nt = n_nt;
    p.BN = BN;
    p.n_seg = a->x1 ? 2 : 1;
    if (seq) {
        fill_taps_1d(p.seg[0], a->k0, sq->dil0, a->ic0, sq->stride0);
        if (a->x1) fill_taps_1d(p.seg[1], 1, 1, a->ic1);
    } else {
        fill_taps(p.seg[0], a->k0, a->stride0, a->ic0, Wp);
        if (a->x1) fill_taps(p.seg[1], 1, a->stride1, a->ic1, Wp);
    }

    // HALO for stride-1 3x3 segments whose weights fit in shared memory.
    const uint32_t w_bytes0 = (uint32_t)9 * a->ic0 * BN * 2;
    // Feed of segment 0: HALO (one A halo per channel block, resident weights) when
    // the weights fit; else, for stride-1 3x3 convs of up to 128 columns, HALO_S (the
    // halo with the weights streamed per tap through a second ring: ~9x less A
    // traffic than TAP); else TAP. a->halo: 0 auto, 1 force HALO, 2 force HALO_S,
    // -1 TAP.
    // The resident-weight HALO also feeds the frequency-stride-2 conv over FPHASE
    // (stride 3): one halo per plane, the 9 taps as row shifts inside them.
    const bool hs_ok = !seq && a->k0 == 3 && a->stride0 == 1 && n_nt == 1;
    const bool fph = !seq && a->k0 == 3 && a->stride0 == 3;
    const bool ph2 = !seq && a->k0 == 3 && a->stride0 == 2;  // PHASE: 4 plane halos
    const int hplanes = ph2 ? 4 : (fph ? 2 : 1);
    // 1-D: one halo of tile + 2*reach rows per channel block feeds every tap (weights
    // resident); automatic for narrow outputs (<= 64 columns: CAM++'s 32-column k=3
    // convs), where the per-tap stages cost more than their MMAs.
    const bool seq_halo_ok = seq && a->k0 > 1 && sq->stride0 == 1 && !a->x1 && n_nt == 1 &&
                             !sq->x_scale && sq->pair != 1 &&
                             (uint32_t)a->k0 * a->ic0 * BN * 2 <= 96 * 1024;
    const bool halo_ok = seq ? seq_halo_ok
                             : (hs_ok || ((fph || ph2) && n_nt == 1)) && w_bytes0 <= 96 * 1024;
    if (a->halo < -1 || a->halo > 2 || (seq && a->halo > 1)) {
        set_error("vdb_conv: halo must be -1, 0, 1 or 2");
        return 1;
    }
    const bool halo = a->halo == 0 ? halo_ok && (!seq || BN <= 64) : (a->halo == 1 && halo_ok);
    // Stride-1 3x3 convs whose weights do not fit resident take the halo with streamed
    // weights automatically up to 128 columns (ResNet34 128 -> 128 at batch 512 x 300
    // frames: 972 -> 1074 TFLOP/s; with the fused downsample 956 -> 1035); 256-column
    // tiles run as CTA pairs instead (1152 against 1082 for the streamed halo).
    const bool auto_two_ring = a->halo == 0 && !seq && hs_ok && !halo_ok && BN <= 128 &&
                               a->ksplit <= 1 && (a->tile_m == 0 || a->tile_m == 256) &&
                               a->pair != 1;
    const bool two_ring = (a->halo == 2 && hs_ok) || auto_two_ring;
    if ((a->halo == 1 && !halo_ok) || (a->halo == 2 && !hs_ok)) {
        set_error("vdb_conv: HALO modes need a 3x3 conv with oc <= 256, stride 1 (or stride "
                  "2 / the frequency-only stride 3 for the resident HALO) and weights <= 96 KB "
                  "for the resident HALO");
        return 1;
    }
    // Tiling. A tcgen05.mma that accumulates into the same TMEM tile as the one
    // before it waits for it (~180 cycles per MMA on B200), while independent
    // accumulators overlap down to ~60 cycles per MMA. So the tile carries
    // n_mblk * J independent f32 accumulators (row blocks x K-split partials,
    // summed in the epilogue), double-buffered when TMEM's 512 columns allow.
    // tile_m = 256 also halves the weight traffic per output row.
    // HALO tiles may be taller (tile_m up to 1024 = 8 row blocks): with small N the
    // issuer needs more independent accumulators than two, and more row blocks
    // give them without K partials. The automatic choice takes the most row blocks
    // that keep the accumulators double-buffered, two pipeline stages in shared
    // memory and at least two tiles per SM.
    int BM = a->tile_m;
    // 1-D convs with 256-column tiles: 128-row tiles keep two accumulators in TMEM so
    // the epilogue of one tile overlaps the MMAs of the next (measured 10-20% faster
    // on the ECAPA 1024- and 1536-channel convs than 256-row single-buffered tiles).
    if (BM == 0 && seq) BM = BN > 128 ? 128 : 256;
    if (BM == 0) {
        BM = 256;
        if (halo && a->ksplit <= 1) {
            const int Hs = fph ? Wp : Wp + 1;
            const int w_res = 9 * a->ic0 * BN * 2;
            const long long rows = vdb_grid_rows(a->batch, a->t_out, a->f_out);
            const int tail = round_up(a->oc * 4, 16) + round_up(a->batch * 4, 16) +
                             8 * (3 * kMaxStages + 5) + 16;
            for (int cand : {8, 4, 3}) {
                const int H = ph2 ? cand * kMB + Wp + 1 : cand * kMB + 2 * Hs + (fph ? 1 : 0);
                const int nbox = (H + 255) / 256;
                const int box = round_up((H + nbox - 1) / nbox, 8);
                const int kb = a->ic0 % 64 == 0 ? 64 : (a->ic0 % 32 == 0 ? 32 : 16);
                long long a_b = (long long)nbox * box * kb * 2, b_b = 0;
                a_b += (long long)(hplanes - 1) * round_up((int)a_b, 1024);  // other planes
                if (a->x1) {  // segment 1 stages hold its A rows and a weight tile
                    const int kb1 = a->ic1 % 64 == 0 ? 64 : (a->ic1 % 32 == 0 ? 32 : 16);
                    a_b = std::max<long long>(a_b, (long long)cand * kMB * kb1 * 2);
                    b_b = (long long)BN * kb1 * 2;
                }
                const long long stage = round_up((int)a_b, 1024) + round_up((int)b_b, 1024);
                const long long fit = (kSmemMax - 1024 - round_up(w_res, 1024) - tail) / stage;
                // two tiles in flight: a tile takes 1 stage per channel block of each segment
                const int per_tile = (a->ic0 / kb) + (a->x1 ? a->ic1 / (a->ic1 % 64 == 0 ? 64 : (a->ic1 % 32 == 0 ? 32 : 16)) : 0);
                if (2 * cand * BN <= 512 && fit >= 2 * per_tile &&
                    (rows + cand * kMB - 1) / (cand * kMB) >= 2LL * num_sms()) {
                    BM = cand * kMB;
                    break;
                }
            }
        }
    }
    if (!(BM == 128 || BM == 256 || BM == 384 || BM == 512 || BM == 1024)) {
        set_error("vdb_conv: tile_m must be 0 (auto), 128, 256, 384, 512 or 1024");
        return 1;
    }
    if (BM > 256 && !halo) {
        set_error("vdb_conv: tile_m above 256 needs the HALO feed (stride-1 3x3, resident weights)");
        return 1;
    }
    if ((BM / kMB) * BN > 512) BM = kMB;
    const int nmb = BM / kMB;
    const int ks0 = p.seg[0].kb / 16;  // MMA K-steps per stage of segment 0
    // Measured on the ResNet34 shapes (batch 64): two 128-row blocks already give
    // the issuer two independent chains, and extra K partials cost more in the
    // epilogue than they save, so the automatic choice is J = 1.
    int J = a->ksplit;
    if (J == 0) J = 1;
    if (!(J == 1 || J == 2 || J == 4 || J == 8) || nmb * J * BN > 512) {
        set_error("vdb_conv: ksplit must be 1, 2, 4 or 8 and tile_m/128 * ksplit * N <= 512");
        return 1;
    }
    if ((!halo || two_ring) && J > ks0) {
        set_error("vdb_conv: ksplit may not exceed the K-steps per stage (channel block / 16)");
        return 1;
    }
    // CTA pairs (cta_group::2, 1-D convs): a 256-row tile per pair, each CTA loading
    // its 128 rows and half the weight columns, so a CTA moves 1.5x fewer bytes per
    // MMA than a 128 x BN tile of its own. Measured on the ECAPA shapes (B200, batch
    // 512 x 398 frames) it only pays off for the 80-channel k=5 stem (16-channel K
    // blocks: 528 -> 444 us); the 1024/1536-channel 1x1 convs run at the same speed
    // and the 128-channel ones slower, so it is opt-in. sq->pair: 1 on, 0 / -1 off.
    // 2-D convs with 256-column tiles take pairs automatically: a 256-row, 256-column
    // tile then needs 256 TMEM columns per CTA instead of 512, so the accumulator is
    // double-buffered (the epilogue overlaps the next tile's MMAs), and each SM
    // fetches half the weight operand per MMA (256 -> 256 convs 999 -> 1127 TFLOP/s,
    // 128 -> 256 stride 2 745 -> 881 at batch 512 x 300 frames). With 128 columns it
    // measured slower (916 -> 727 TFLOP/s on 128 -> 128).
    const int want_pair = seq ? sq->pair : a->pair;
    const bool auto_pair = want_pair == 0 && !seq && BN == 256 && a->tile_m == 0 &&
                           a->ksplit <= 1;
    const bool pair = (want_pair == 1 || auto_pair) && !halo && !two_ring && J == 1 &&
                      BN % 32 == 0 && (a->tile_m == 0 || a->tile_m == 256) && num_sms() >= 2;
    if (want_pair == 1 && !pair) {
        set_error("vdb_conv: a CTA pair needs the one-tap-per-stage feed, oc tiles that are "
                  "multiples of 32 and tile_m 0 or 256");
        return 1;
    }
    if (pair) BM = 2 * kMB;
    p.BM = BM;
    p.n_mblk = pair ? 1 : BM / kMB;
    p.n_iss = (!seq && !pair && p.n_mblk >= 2) ? 2 : 1;
    // q8_0 weights (2-D convs): an f16 scale per 32 input channels of a tap
    const void* wsc[2] = {a->w0_scale, a->x1 ? a->w1_scale : nullptr};
    if (wsc[0] || wsc[1]) {
        if (seq) {
            set_error("vdb_conv1d: q8_0 weights are supported by the 2-D conv only");
            return 1;
        }
        if ((wsc[0] && a->ic0 % 32) || (wsc[1] && a->ic1 % 32)) {
            set_error("vdb_conv: q8_0 weights need input channels that are a multiple of 32");
            return 1;
        }
    }
    p.J = J;
    p.n_acc = (2 * p.n_mblk * J * BN <= 512) ? 2 : 1;
    const int cta_rows = pair ? kMB : BM;   // A rows one CTA loads per stage
    const int cta_bn = pair ? BN / 2 : BN;  // weight rows one CTA loads per stage
    p.n_mt = (p.M + BM - 1) / BM;

    uint32_t off = 0;
    p.bres_bytes = 0;
    uint32_t a_bytes = 0, b_bytes = 0;
    for (int sg = 0; sg < p.n_seg; ++sg) {
        SegDev& s = p.seg[sg];
        const uint32_t row_bytes = (uint32_t)s.kb * 2;
        if (sg == 0 && two_ring) {
            s.mode = SEG_HALO_S;
            const int H = BM + 2 * Wp + 2;
            s.halo_back = Wp + 1;
            s.n_box = (H + 255) / 256;
            s.box_rows = round_up((H + s.n_box - 1) / s.n_box, 8);
            for (int t = 0; t < 9; ++t) s.off[t] = (t / 3) * Wp + (t % 3);  // kt*Wp + kf
            s.a_bytes = (uint32_t)s.n_box * s.box_rows * row_bytes;
            s.b_bytes = (uint32_t)BN * row_bytes;
            s.bytes = s.a_bytes;
        } else if (sg == 0 && halo) {
            s.mode = SEG_HALO;
            // stride 1: taps at kt*Wp + kf rows into a halo from m0 - (Wp + 1); FPHASE:
            // taps at kt*Wp + (kf>>1) rows into plane kf&1's halo from m0 - Wp
            const int reach = seq ? (a->k0 - 1) / 2 * sq->dil0 : 0;
            // PHASE: taps at (kt>>1)*Wp + (kf>>1) rows into plane 2(kt&1)+(kf&1)'s
            // halo from m0
            const int H = seq ? BM + 2 * reach
                              : (ph2 ? BM + Wp + 1 : (fph ? BM + 2 * Wp + 1 : BM + 2 * Wp + 2));
            s.halo_back = seq ? reach : (ph2 ? 0 : (fph ? Wp : Wp + 1));
            s.n_box = (H + 255) / 256;
            s.box_rows = round_up((H + s.n_box - 1) / s.n_box, 8);
            for (int t = 0; t < 9; ++t) s.off[t] = (t / 3) * Wp + (t % 3);  // kt*Wp + kf
            const uint32_t one = (uint32_t)s.n_box * s.box_rows * row_bytes;
            s.halo_planes = seq ? 1 : hplanes;
            s.halo_mode = seq ? 0 : (ph2 ? 2 : (fph ? 1 : 0));
            s.plane_bytes = s.halo_planes > 1 ? (uint32_t)round_up((int)one, 1024) : 0u;
            s.bytes = (uint32_t)s.halo_planes * one;
            s.bres = off;
            const uint32_t w = (uint32_t)s.n_taps * s.n_kb * BN * row_bytes;
            off += w;
            p.bres_bytes += w;
            if (!wsc[sg]) p.bres_tx += w;  // q8_0 weights are expanded, not loaded
            a_bytes = std::max(a_bytes, (uint32_t)(s.halo_planes - 1) * s.plane_bytes + one);
        } else {
            s.mode = SEG_TAP;
            s.n_box = (cta_rows + 255) / 256;
            s.box_rows = cta_rows / s.n_box;
            s.bytes = (uint32_t)(cta_rows + cta_bn) * row_bytes;
            s.a_bytes = (uint32_t)cta_rows * row_bytes;
            s.b_bytes = (uint32_t)cta_bn * row_bytes;
            a_bytes = std::max(a_bytes, (uint32_t)cta_rows * row_bytes);
            b_bytes = std::max(b_bytes, (uint32_t)cta_bn * row_bytes);
        }
    }
    // q8_0 segments: resident (HALO) weights are expanded to f16 in shared memory by
    // every CTA (q8_expand); streamed ones are expanded once for this launch into the
    // caller's scratch (q8_dequant_kernel, below) and then streamed as f16
    const void* wseg[2] = {a->w0, a->x1 ? a->w1 : nullptr};
    size_t scratch_need[2] = {0, 0};
    for (int sg = 0; sg < p.n_seg; ++sg) {
        SegDev& s = p.seg[sg];
        if (!wsc[sg]) continue;
        if (s.mode == SEG_HALO) {
            s.wq = static_cast<const int8_t*>(wseg[sg]);
            s.wd = static_cast<const __half*>(wsc[sg]);
            s.wk = s.n_taps * s.ic;
            s.wn = a->oc;
        } else {
            scratch_need[sg] = (size_t)round_up(a->oc * s.n_taps * s.ic * 2, 256);
        }
    }
    if (scratch_need[0] + scratch_need[1] > 0 &&
        (!a->w_scratch || (long long)(scratch_need[0] + scratch_need[1]) > a->w_scratch_bytes ||
         (reinterpret_cast<uintptr_t>(a->w_scratch) & 255u))) {
        set_error("vdb_conv: q8_0 weights this conv streams need w_scratch (256-byte aligned) "
                  "of at least 2 bytes per weight of those segments");
        return 1;
    }
    off = (uint32_t)round_up((int)off, 1024);
    p.stage0 = off;
    p.a_region = (uint32_t)round_up((int)a_bytes, 1024);
    p.stage_bytes = p.a_region + (uint32_t)round_up((int)b_bytes, 1024);
    const bool has_bn = seq && sq->bn_scale != nullptr;
    const uint32_t ss_bytes = has_bn ? 2u * (uint32_t)round_up(a->oc * 4, 16) : 0u;
    const uint32_t tail = (uint32_t)round_up(a->oc * 4, 16) + (uint32_t)round_up(a->batch * 4, 16) +
                          ss_bytes + 8 * (3 * kMaxStages + 5) + 16;
    uint32_t ab = 0, bb = 0;  // two-ring slot sizes
    for (int sg = 0; sg < p.n_seg; ++sg) {
        ab = std::max(ab, p.seg[sg].a_bytes);
        bb = std::max(bb, p.seg[sg].b_bytes);
    }
    // pipeline slots that fit a budget: weight slots (two-ring) or stages
    auto slots = [&](int bud) {
        return two_ring ? std::min<int>(kMaxStages - 2, (bud - 2 * round_up((int)ab, 1024)) /
                                                            round_up((int)bb, 1024))
                        : std::min<int>(kMaxStages, bud / (int)p.stage_bytes);
    };
    // Staged output (GRID y only, 32-column chunks, a 16-byte aligned row pitch): the
    // epilogue warps' stores become one TMA box store per 32 rows x 32 columns instead
    // of 32 row stores of 64 bytes, which otherwise saturate the LSU data path on the
    // small-channel convs. Taken when it leaves at least min(3, the slots without it)
    // pipeline slots.
    const bool chunk32 = BN % 64 == 0 || (p.n_mblk >= 2 && BN % 32 == 0);
    const int ldy_el = a->ldy ? a->ldy : a->oc;
    const int store_mode = conv_tma_store_mode();
    bool staged = store_mode != 0 && !seq && J == 1 && a->y_phase == 0 && !a->y2 && !a->ysum && chunk32 &&
                  (reinterpret_cast<uintptr_t>(a->y) & 15u) == 0 && ldy_el % 8 == 0;
    const int budget0 = kSmemMax - 1024 - (int)off - (int)tail;
    if (staged) {
        const int with = slots(budget0 - (int)kOstageBytes), without = slots(budget0);
        staged = with >= 2 && (store_mode == 1 || with >= std::min(3, without));
    }
    const uint32_t ostage_bytes = staged ? kOstageBytes : 0u;
    const int budget = budget0 - (int)ostage_bytes;
    p.two_ring = two_ring ? 1 : 0;
    if (two_ring) {
        // 2 A slots (a halo per channel block) + as many weight slots as fit
        p.ra = 2;
        p.a_stride = (uint32_t)round_up((int)ab, 1024);
        p.b_stride = (uint32_t)round_up((int)bb, 1024);
        p.rb = std::min<int>(kMaxStages - p.ra, (budget - p.ra * (int)p.a_stride) / (int)p.b_stride);
        if (p.rb < 2) {
            set_error("vdb_conv: tile does not fit in shared memory");
            return 1;
        }
        p.b_ring0 = p.stage0 + p.ra * p.a_stride;
        p.n_stages = (uint32_t)(p.ra + p.rb);
        p.stage_bytes = p.a_stride;  // unused by the two-ring path
        off = p.b_ring0 + p.rb * p.b_stride;
    } else {
        p.n_stages = (uint32_t)std::min<int>(kMaxStages, budget / (int)p.stage_bytes);
        if (p.n_stages < 2) {
            set_error("vdb_conv: tile does not fit in shared memory");
            return 1;
        }
        off += p.n_stages * p.stage_bytes;
    }
    p.ostage_off = staged ? off : 0u;  // 1024-byte aligned: every slot is
    off += ostage_bytes;
    p.bias_off = off;
    off += (uint32_t)round_up(a->oc * 4, 16);
    p.tv_off = off;
    off += (uint32_t)round_up(a->batch * 4, 16);
    p.ss_off = has_bn ? off : 0u;
    off += ss_bytes;
    p.bar_off = (uint32_t)round_up((int)off, 8);
    off = p.bar_off + 8 * (3 * p.n_stages + 5) + 16;
    const size_t smem = (size_t)off + 1024;

    uint32_t cols = 32;
    while (cols < (uint32_t)(p.n_acc * p.n_mblk * J * BN)) cols <<= 1;
    p.tmem_cols = cols;
    p.bias = a->bias;
    p.residual = static_cast<const __half*>(a->residual);
    p.residual2 = static_cast<const __half*>(a->residual2);
    p.ldr = a->ldr ? a->ldr : a->oc;
    p.ldr2 = a->ldr2 ? a->ldr2 : a->oc;
    p.ldy = a->ldy ? a->ldy : a->oc;
    p.act = a->act;
    p.y = static_cast<__half*>(a->y);
    p.y2 = static_cast<__half*>(a->y2);
    p.ysum = static_cast<__half*>(a->ysum);
    p.addend = static_cast<const __half*>(a->addend);
    p.ldsum = a->ldsum ? a->ldsum : a->oc;
    p.ldadd = a->ldaddend ? a->ldaddend : a->oc;
    p.y_phase = a->y_phase;
    p.Hp = Hp;
    p.Wp = Wp;
    magic_div((uint32_t)Hp * (uint32_t)Wp, p.img_mul, p.img_sh);
    magic_div((uint32_t)Wp, p.wp_mul, p.wp_sh);
    p.T = a->t_out;
    p.F = a->f_out;
    if (a->y_phase == 2) {         // FPHASE for a frequency-stride-2 consumer
        p.Hq = a->t_out + 2;
        p.Wq = (a->f_out - 1) / 2 + 1 + 2;
    } else if (a->y_phase == 3) {  // TPHASE for a time-stride-2 1-D consumer
        p.ypad = a->y_pad;
        p.Hq = (a->t_out - 1) / 2 + 1 + 2 * a->y_pad;
        p.Wq = a->f_out;
    } else {                       // PHASE
        p.Hq = (a->t_out - 1) / 2 + 1 + 2;
        p.Wq = (a->f_out - 1) / 2 + 1 + 2;
    }
    p.plane_rows = (long long)a->batch * p.Hq * p.Wq;
    p.tvalid = a->tvalid;
    p.batch = a->batch;
    p.relu = a->relu;
    p.clamp_hi = a->clamp_hi;
    p.oc = a->oc;
    p.err = a->err;
    if (seq) {
        p.seq = 1;
        p.pad = sq->pad;
        p.reflect = sq->reflect;
        p.y_f32 = sq->y_f32;
        p.clip_bias = sq->clip_bias;
        p.bn_scale = sq->bn_scale;
        p.bn_shift = sq->bn_shift;
        p.gate = sq->gate;
        p.gate_seg = sq->gate_seg;
        p.gate_nseg = sq->gate_nseg;
        if (sq->x_scale) {
            if (a->k0 != 1 || a->x1 || pair || p.seg[0].mode != SEG_TAP) {
                set_error("vdb_conv1d: the input BN + ReLU prologue needs a single-segment "
                          "1x1 conv without CTA pairs");
                return 1;
            }
            p.xform = 1;
            p.x_scale = sq->x_scale;
            p.x_shift = sq->x_shift;
        }
        magic_div((uint32_t)Hp, p.img_mul, p.img_sh);
    }

    // Input row extents: stride 1 reads G(B, t_out, f_out); stride 2 reads the
    // 4 planes of a PHASE tensor, each shaped like the output grid.
    const long long rows_out = p.M;
    CUtensorMap tm[5];
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    for (int sg = 0; sg < p.n_seg; ++sg) {
        if (!scratch_need[sg]) continue;
        const SegDev& s = p.seg[sg];
        __half* dst = reinterpret_cast<__half*>(static_cast<char*>(a->w_scratch) +
                                                (sg ? scratch_need[0] : 0));
        const int K = s.n_taps * s.ic;
        const long long n8 = (long long)a->oc * K / 8;
        const int blocks = (int)std::min<long long>((n8 + 255) / 256, (long long)num_sms() * 8);
        q8_dequant_kernel<<<blocks, 256, 0, st>>>(static_cast<const int8_t*>(wseg[sg]),
                                                   static_cast<const __half*>(wsc[sg]), a->oc, K,
                                                   dst);
        VDB_CHECK_CUDA(cudaGetLastError());
        ++g_conv_launches;
        wseg[sg] = dst;  // this segment streams the f16 expansion
    }
    for (int sg = 0; sg < p.n_seg; ++sg) {
        const SegDev& s = p.seg[sg];
        const void* x = sg ? a->x1 : a->x0;
        const void* w = wseg[sg];
        const int stride = sg ? a->stride1 : a->stride0;
        const int box_rows = s.box_rows;
        const int ldx = sg ? (a->ldx1 ? a->ldx1 : a->ic1) : (a->ldx0 ? a->ldx0 : a->ic0);
        // planes: PHASE 4, FPHASE 2 (2-D stride 3), TPHASE 2 (1-D stride 2)
        const int planes = seq ? ((sg == 0 && sq->stride0 == 2) ? 2 : 1)
                               : (stride == 2 ? 4 : (stride == 3 ? 2 : 1));
        // q8_0 resident weights are expanded from global memory (no weight map)
        const bool q8_res = s.wq != nullptr;
        if (!make_map_a(&tm[2 * sg], x, s.ic, ldx, rows_out, planes, s.kb, box_rows) ||
            (!q8_res && !make_map_b(&tm[2 * sg + 1], w, s.n_taps * s.ic, a->oc, cta_bn, s.kb))) {
            set_error("vdb_conv: cuTensorMapEncodeTiled failed");
            return 1;
        }
        if (q8_res) tm[2 * sg + 1] = tm[2 * sg];
    }
    if (p.n_seg == 1) {
        tm[2] = tm[0];
        tm[3] = tm[1];
    }
    if (staged) {
        if (!make_map_a(&tm[4], a->y, a->oc, ldy_el, rows_out, 1, 32, 32)) {
            set_error("vdb_conv: cuTensorMapEncodeTiled failed");
            return 1;
        }
    } else {
        tm[4] = tm[0];
    }
    // One CTA per SM: more than 256 TMEM columns, or most of shared memory.
    const size_t smem_launch = std::max<size_t>(smem, 120 * 1024);
    const int n_tiles = p.n_mt * p.n_nt;
    const int grid = pair ? 2 * std::max(1, std::min(n_tiles, num_sms() / 2))
                          : std::max(1, std::min(n_tiles, num_sms()));
    auto launch = [&](auto kern) -> int {
        // The shared-memory opt-in. While a stream is being captured into a CUDA graph
        // it is skipped: the engine captures a bucket only after launching it plainly
        // once, which set it.
        cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
        VDB_CHECK_CUDA(cudaStreamIsCapturing(st, &cs));
        if (cs == cudaStreamCaptureStatusNone)
            VDB_CHECK_CUDA(
                cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemMax));
        // programmatic stream serialization: the prologue (barriers, TMEM, bias and
        // lengths in shared memory) overlaps the previous conv's last tiles
        cudaLaunchConfig_t cfg{};
        cfg.gridDim = dim3((unsigned)grid);
        cfg.blockDim = dim3(kThreads);
        cfg.dynamicSmemBytes = smem_launch;
        cfg.stream = st;
        cudaLaunchAttribute attr[1];
        attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[0].val.programmaticStreamSerializationAllowed = 1;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
        VDB_CHECK_CUDA(cudaLaunchKernelEx(&cfg, kern, tm[0], tm[1], tm[2], tm[3], tm[4], p));
        return 0;
    };
    // The plain epilogue (bias, optional residual, ReLU, mask, GRID / PHASE store): every
    // ResNet34 conv.
    const bool plain = !seq && a->act == 0 && !a->residual2 && !a->y2 && !a->ysum &&
                       a->clamp_hi <= 0.0f && (a->y_phase == 0 || a->y_phase == 1);
    if (pair) {
        auto kern = seq ? conv_tc_kernel<1, 1, true, true>
                        : (plain ? conv_tc_kernel<1, 1, true, false, true>
                                 : conv_tc_kernel<1, 1, true, false>);
        cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
        VDB_CHECK_CUDA(cudaStreamIsCapturing(st, &cs));
        if (cs == cudaStreamCaptureStatusNone)
            VDB_CHECK_CUDA(
                cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemMax));
        cudaLaunchConfig_t cfg{};
        cfg.gridDim = dim3((unsigned)grid);
        cfg.blockDim = dim3(kThreads);
        cfg.dynamicSmemBytes = smem_launch;
        cfg.stream = st;
        cudaLaunchAttribute attr[2];
        attr[0].id = cudaLaunchAttributeClusterDimension;
        attr[0].val.clusterDim.x = 2;
        attr[0].val.clusterDim.y = 1;
        attr[0].val.clusterDim.z = 1;
        attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[1].val.programmaticStreamSerializationAllowed = 1;
        cfg.attrs = attr;
        cfg.numAttrs = 2;
        VDB_CHECK_CUDA(cudaLaunchKernelEx(&cfg, kern, tm[0], tm[1], tm[2], tm[3], tm[4], p));
        return 0;
    }
    if (seq) {
        if (J != 1 || p.n_mblk > 2) {
            set_error("vdb_conv1d: 1-D tiles are 128 or 256 rows with one accumulator");
            return 1;
        }
        return p.n_mblk == 2 ? launch(conv_tc_kernel<2, 1, false, true>)
                             : launch(conv_tc_kernel<1, 1, false, true>);
    }
    const int key = p.n_mblk * 100 + J;
    if (plain) {
        switch (key) {
            case 101: return launch(conv_tc_kernel<1, 1, false, false, true>);
            case 201: return launch(conv_tc_kernel<2, 1, false, false, true>);
            case 301: return launch(conv_tc_kernel<3, 1, false, false, true>);
            case 401: return launch(conv_tc_kernel<4, 1, false, false, true>);
            case 801: return launch(conv_tc_kernel<8, 1, false, false, true>);
            default: break;  // ksplit > 1: the general epilogue
        }
    }
    switch (key) {
        case 101: return launch(conv_tc_kernel<1, 1, false, false>);
        case 102: return launch(conv_tc_kernel<1, 2, false, false>);
        case 104: return launch(conv_tc_kernel<1, 4, false, false>);
        case 108: return launch(conv_tc_kernel<1, 8, false, false>);
        case 201: return launch(conv_tc_kernel<2, 1, false, false>);
        case 202: return launch(conv_tc_kernel<2, 2, false, false>);
        case 204: return launch(conv_tc_kernel<2, 4, false, false>);
        case 208: return launch(conv_tc_kernel<2, 8, false, false>);
        case 301: return launch(conv_tc_kernel<3, 1, false, false>);
        case 401: return launch(conv_tc_kernel<4, 1, false, false>);
        case 801: return launch(conv_tc_kernel<8, 1, false, false>);
        default:
            set_error("vdb_conv: ksplit must be 1, 2, 4 or 8 (1 for tile_m above 256)");
            return 1;
    }
}


// Stage-1 conv over QPACK rows (vdb_conv_args.qpack): see the QPACK section above.

int conv_qpack_impl(const vdb_conv_args* a, void* stream) {
    if (a->k0 != 3 || a->stride0 != 1 || a->ic0 != 32 || a->oc != 32 || a->x1 || a->act != 0 ||
        a->y2 || a->ysum || a->residual2 || a->clamp_hi > 0.0f ||
        !(a->y_phase == 0 || a->y_phase == 1) || (a->ldx0 && a->ldx0 != 128) ||
        (a->ldy && a->ldy != 128) || (a->ldr && a->ldr != 128) || a->pair == 1 ||
        (a->halo != 0 && a->halo != 1) || a->ksplit > 1 || a->tile_n) {
        set_error("vdb_conv: a QPACK conv is 3x3, stride 1, 32 -> 32 channels, one segment, "
                  "act 0, y_phase 0 or 1, an optional QPACK residual, no other options");
        return 1;
    }
    if (a->batch <= 0 || a->batch > kMaxBatch || a->t_out <= 0 || a->f_out <= 0) {
        set_error("vdb_conv: batch must be in [1, 8192] and the output non-empty");
        return 1;
    }
    if (!a->x0 || !a->w0 || !a->tvalid || !a->y) {
        set_error("vdb_conv: NULL buffer");
        return 1;
    }
    auto misaligned = [](const void* q) { return (reinterpret_cast<uintptr_t>(q) & 15u) != 0; };
    if (misaligned(a->x0) || misaligned(a->y) || (a->residual && misaligned(a->residual))) {
        set_error("vdb_conv: activation pointers must be 16-byte aligned");
        return 1;
    }
    const int Wq = (a->f_out + 2 + 3) / 4;
    const long long rows = vdb_qpack_rows(a->batch, a->t_out, a->f_out);
    if (rows > (1LL << 31) - 1024 || vdb_phase_rows(a->batch, a->t_out, a->f_out) > (1LL << 31) - 1024) {
        set_error("vdb_conv: tensor too large (more than 2^31 rows); split the batch");
        return 1;
    }
    int BM = a->tile_m ? a->tile_m : 256;
    if (BM != 128 && BM != 256) {
        set_error("vdb_conv: a QPACK conv takes tile_m 0, 128 or 256");
        return 1;
    }
    ConvDev p{};
    p.M = (int)rows;
    p.n_nt = 1;
    p.BN = 128;  // 4 pixel phases x 32 output channels
    p.n_seg = 1;
    SegDev& s = p.seg[0];
    s.mode = SEG_HALO;
    s.ic = 128;
    s.kb = 64;
    s.n_kb = 2;
    s.n_taps = 9;
    const int H = BM + 2 * Wq + 2;
    s.halo_back = Wq + 1;
    s.n_box = (H + 255) / 256;
    s.box_rows = round_up((H + s.n_box - 1) / s.n_box, 8);
    s.halo_planes = 1;
    s.halo_mode = 0;
    s.plane_bytes = 0;
    s.bytes = (uint32_t)s.n_box * s.box_rows * 128u;
    s.bres = 0;
    p.bres_bytes = 1152u * 64u;  // 3 x 384 rows of 32 channels
    if (a->w0_scale) {
        // q8_0: one f16 scale per packed row (32 channels), expanded once per CTA
        s.wq = static_cast<const int8_t*>(a->w0);
        s.wd = static_cast<const __half*>(a->w0_scale);
        s.wk = 32;
        s.wn = 1152;  // scales [1][1152]: one per packed row
    } else {
        p.bres_tx = p.bres_bytes;
    }
    uint32_t off = p.bres_bytes;   // 72 KB: 1024-byte aligned
    p.stage0 = off;
    p.a_region = (uint32_t)round_up((int)s.bytes, 1024);
    p.stage_bytes = p.a_region;
    // y_phase 0 stores through TMA from 2 staging buffers of 2 KB per epilogue warp
    const bool staged = a->y_phase == 0 && conv_tma_store_mode() != 0;
    const uint32_t ostage_bytes = staged ? kOstageBytes : 0u;
    const uint32_t tail = ostage_bytes + (uint32_t)round_up(128 * 4, 16) +
                          (uint32_t)round_up(a->batch * 4, 16) + 8 * (3 * kMaxStages + 5) + 16;
    const int budget = kSmemMax - 1024 - (int)off - (int)tail;
    p.n_stages = (uint32_t)std::min<int>(kMaxStages, budget / (int)p.stage_bytes);
    if (p.n_stages < 2) {
        set_error("vdb_conv: QPACK tile does not fit in shared memory");
        return 1;
    }
    off += p.n_stages * p.stage_bytes;
    p.ostage_off = staged ? off : 0u;  // 1024-byte aligned: the stages are
    off += ostage_bytes;
    p.bias_off = off;
    off += (uint32_t)round_up(128 * 4, 16);
    p.tv_off = off;
    off += (uint32_t)round_up(a->batch * 4, 16);
    p.ss_off = 0;
    p.bar_off = (uint32_t)round_up((int)off, 8);
    off = p.bar_off + 8 * (3 * p.n_stages + 5) + 16;
    const size_t smem = (size_t)off + 1024;
    p.BM = BM;
    p.n_mblk = BM / kMB;
    p.J = 1;
    p.n_acc = 2;
    p.n_iss = p.n_mblk >= 2 ? 2 : 1;
    p.n_mt = (p.M + BM - 1) / BM;
    uint32_t cols = 32;
    while (cols < (uint32_t)(p.n_acc * p.n_mblk * 128)) cols <<= 1;
    p.tmem_cols = cols;
    p.bias = a->bias;
    p.relu = a->relu;
    p.y = static_cast<__half*>(a->y);
    p.ldy = 128;
    p.act = 0;
    p.y_phase = a->y_phase;
    p.Hp = a->t_out + 2;
    p.Wp = Wq;
    magic_div((uint32_t)p.Hp * (uint32_t)Wq, p.img_mul, p.img_sh);
    magic_div((uint32_t)Wq, p.wp_mul, p.wp_sh);
    p.T = a->t_out;
    p.F = a->f_out;
    p.Hq = (a->t_out - 1) / 2 + 1 + 2;  // PHASE output: the stride-2 consumer's grid
    p.Wq = (a->f_out - 1) / 2 + 1 + 2;
    p.plane_rows = (long long)a->batch * p.Hq * p.Wq;
    p.tvalid = a->tvalid;
    p.batch = a->batch;
    p.oc = 128;
    p.err = a->err;
    p.qp_res = static_cast<const __half*>(a->residual);
    CUtensorMap tm[5];
    if (!make_map_a(&tm[0], a->x0, 128, 128, rows, 1, 64, s.box_rows) ||
        (!s.wq && !make_map_b(&tm[1], a->w0, 32, 1152, 128, 32))) {
        set_error("vdb_conv: cuTensorMapEncodeTiled failed");
        return 1;
    }
    if (s.wq) tm[1] = tm[0];  // q8_0 weights are expanded, not loaded by TMA
    tm[2] = tm[0];
    tm[3] = tm[1];
    if (staged) {
        if (!make_map_a(&tm[4], a->y, 128, 128, rows, 1, 32, 32)) {
            set_error("vdb_conv: cuTensorMapEncodeTiled failed");
            return 1;
        }
    } else {
        tm[4] = tm[0];
    }
    const size_t smem_launch = std::max<size_t>(smem, 120 * 1024);
    const int grid = std::max(1, std::min(p.n_mt, num_sms()));
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    auto kern = p.n_mblk == 2 ? conv_tc_kernel<2, 1, false, false, true, true>
                              : conv_tc_kernel<1, 1, false, false, true, true>;
    cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
    VDB_CHECK_CUDA(cudaStreamIsCapturing(st, &cs));
    if (cs == cudaStreamCaptureStatusNone)
        VDB_CHECK_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemMax));
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3((unsigned)grid);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = smem_launch;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    VDB_CHECK_CUDA(cudaLaunchKernelEx(&cfg, kern, tm[0], tm[1], tm[2], tm[3], tm[4], p));
    return 0;
}

}  // namespace
}  // namespace vdb
