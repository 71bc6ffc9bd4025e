// Implicit-GEMM 3x3 / 1x1 convolution on sm_100a tensor cores (tcgen05 + TMEM),
// the B200 replacement for the reference's blocked direct conv microkernels
// (src/directconv.cpp:1072-1211 bconv3x3_compute, :1214-1280 bconv1x1_compute)
// and its fused bias / ReLU / residual-add epilogues (:544-549, :1366-1373).
//
// GEMM view. Rows (M) are the pixels of the output's zero-bordered grid
// (vdb_ops.h, GRID layout), columns (N) the output channels, and K runs over
// (tap, input channel). Because every activation carries a one-pixel zero border
// and is stored row-major over (time, freq), the A tile of tap (kt, kf) for 128
// consecutive output rows is 128 consecutive input rows shifted by a constant:
//   stride 1: off = (kt-1)*(F+2) + (kf-1) in the same grid;
//   stride 2: the input is stored phase-split (PHASE layout), and the tap reads
//             plane 2*(kt&1) + (kf&1) at off = (kt>>1)*(F+2) + (kf>>1).
// So every A tile is ONE rectangular TMA box (channels x 128 rows); the border
// zeros and TMA's out-of-bounds zero fill provide the convolution padding. Rows
// that fall on the grid border, or past a clip's valid length, are computed and
// then written as zeros, which keeps the next layer's padding exact under
// length-bucketed batching (ragged clips in one batch).
//
// Kernel structure (persistent, one CTA per SM, 8 warps):
//   warp 0 lane 0 : TMA producer, S-stage smem ring (A tile + B tile per stage)
//   warp 1 lane 0 : tcgen05.mma issuer (M=128, N=BN, K=16 per instruction) into
//                   a double-buffered f32 TMEM accumulator; also owns TMEM alloc
//   warps 4..7    : epilogue: tcgen05.ld -> + bias [+ residual] -> ReLU/clamp ->
//                   valid-pixel mask -> f16 store (plain or phase-split layout)
// A second, optional K segment (a 1x1 conv on another input) accumulates into the
// same TMEM tile: that is how the BasicBlock downsample shortcut is fused into
// conv2 (reference: blocked_conv1x1 + blocked_add_relu, src/encoder_resnet.cpp:68-72).
#include <cuda_fp16.h>

#include <algorithm>
#include <cstdio>
#include <string>

#include "sm100_ptx.cuh"
#include "vdb_internal.h"
#include "vdb_ops.h"

namespace vdb {
namespace {

constexpr int kBM = 128;
constexpr int kThreads = 256;
constexpr int kMaxStages = 8;
constexpr int kSmemBudget = 200 * 1024;

struct SegDev {
    int n_taps;
    int ic;
    int kb;      // channels per K block: 64 / 32 / 16 (128 / 64 / 32 B rows)
    int n_kb;    // ic / kb
    int kcols;   // B matrix K extent = n_taps * ic
    uint32_t bytes;  // TMA bytes per k-iteration (A + B)
    int plane[9];
    int off[9];
};

struct ConvDev {
    int M;          // output grid rows
    int n_mt, n_nt, BN;
    int n_seg;
    SegDev seg[2];
    uint32_t stage_bytes, a_region, n_stages, tmem_cols;
    const float* bias;
    const __half* residual;
    __half* y;
    int y_phase;
    int Hp, Wp, T, F;   // output grid: Hp = T+2, Wp = F+2
    int Hq, Wq;         // phase-split output: consumer grid
    long long plane_rows;
    const int* tvalid;
    int relu;
    float clamp_hi;
    int oc;
    int* err;
};

// True when rows [m0, m0+128) contain at least one pixel inside a clip's valid
// time range (conservative: border columns of those rows count). Every role
// evaluates it identically, so skipped tiles never touch the pipeline.
__device__ __forceinline__ bool tile_live(const ConvDev& p, int m0) {
    const int img = p.Hp * p.Wp;
    const int mend = min(m0 + kBM, p.M);
    for (int b = m0 / img; b * img < mend; ++b) {
        const int r0 = max(m0 - b * img, 0);
        const int r1 = min(mend - b * img, img);
        const int tv = p.tvalid[b];
        if (tv <= 0) continue;
        const int lo = p.Wp + 1;
        const int hi = p.Wp * tv + p.F + 1;
        if (r0 < hi && r1 > lo) return true;
    }
    return false;
}

__device__ __forceinline__ float h2f(uint32_t bits16) {
    return __half2float(__ushort_as_half((unsigned short)bits16));
}

// One epilogue chunk of NC (32 or 16) accumulator columns for this thread's row:
// TMEM -> + bias [+ residual] -> ReLU / clamp -> mask -> f16 store. The TMEM load
// is warp-collective, so every lane executes it whenever the tile is live.
template <int NC>
__device__ __forceinline__ void epi_chunk(const ConvDev& p, bool live, bool in_range, bool valid,
                                          uint32_t taddr, int ch0, const __half* rrow,
                                          __half* yrow) {
    uint32_t v[NC];
    if (live) {
        if constexpr (NC == 32) tmem_ld_32x32b_x32(taddr, v);
        else tmem_ld_32x32b_x16(taddr, v);
    }
    if (!in_range) return;
    float f[NC];
    if (valid) {
#pragma unroll
        for (int i = 0; i < NC; ++i) f[i] = __uint_as_float(v[i]) + __ldg(p.bias + ch0 + i);
        if (rrow) {
            const uint4* rp = reinterpret_cast<const uint4*>(rrow);
#pragma unroll
            for (int j = 0; j < NC / 8; ++j) {
                const uint4 q = __ldg(rp + j);
                const uint32_t w[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
                for (int h = 0; h < 4; ++h) {
                    f[j * 8 + 2 * h] += h2f(w[h] & 0xFFFFu);
                    f[j * 8 + 2 * h + 1] += h2f(w[h] >> 16);
                }
            }
        }
        if (p.relu) {
#pragma unroll
            for (int i = 0; i < NC; ++i) f[i] = fmaxf(f[i], 0.0f);
        }
        if (p.clamp_hi > 0.0f) {
#pragma unroll
            for (int i = 0; i < NC; ++i) f[i] = fminf(f[i], p.clamp_hi);
        }
    } else {
#pragma unroll
        for (int i = 0; i < NC; ++i) f[i] = 0.0f;
    }
    uint4* yp = reinterpret_cast<uint4*>(yrow);
#pragma unroll
    for (int j = 0; j < NC / 8; ++j) {
        uint4 q;
        __half2 h0 = __floats2half2_rn(f[j * 8 + 0], f[j * 8 + 1]);
        __half2 h1 = __floats2half2_rn(f[j * 8 + 2], f[j * 8 + 3]);
        __half2 h2 = __floats2half2_rn(f[j * 8 + 4], f[j * 8 + 5]);
        __half2 h3 = __floats2half2_rn(f[j * 8 + 6], f[j * 8 + 7]);
        q.x = *reinterpret_cast<uint32_t*>(&h0);
        q.y = *reinterpret_cast<uint32_t*>(&h1);
        q.z = *reinterpret_cast<uint32_t*>(&h2);
        q.w = *reinterpret_cast<uint32_t*>(&h3);
        yp[j] = q;
    }
}

__global__ void __launch_bounds__(kThreads, 1)
conv_tc_kernel(const __grid_constant__ CUtensorMap tmA0, const __grid_constant__ CUtensorMap tmB0,
               const __grid_constant__ CUtensorMap tmA1, const __grid_constant__ CUtensorMap tmB1,
               const __grid_constant__ ConvDev p) {
    extern __shared__ uint8_t smem_raw[];
    const uint32_t raw_u32 = smem_u32(smem_raw);
    const uint32_t base = (raw_u32 + 1023u) & ~1023u;
    uint8_t* smem = smem_raw + (base - raw_u32);
    const uint32_t S = p.n_stages;
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + S * p.stage_bytes);
    const uint32_t bar_full = smem_u32(bars);
    const uint32_t bar_empty = bar_full + 8 * S;
    const uint32_t bar_tfull = bar_empty + 8 * S;
    const uint32_t bar_tempty = bar_tfull + 16;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2 * S + 4);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;

    if (threadIdx.x == 0) {
        for (uint32_t s = 0; s < S; ++s) {
            mbar_init(bar_full + 8 * s, 1);
            mbar_init(bar_empty + 8 * s, 1);
        }
        for (int a = 0; a < 2; ++a) {
            mbar_init(bar_tfull + 8 * a, 1);
            mbar_init(bar_tempty + 8 * a, 128);
        }
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
    if (warp == 1) tmem_alloc(smem_u32(tmem_slot), p.tmem_cols);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;

    const int n_tiles = p.n_mt * p.n_nt;
    const uint32_t idesc = umma_idesc_f16(kBM, p.BN);

    if (warp == 0) {
        if (lane == 0) {
            // ---------------- TMA producer ----------------
            uint32_t stage = 0, phase = 0;
            bool ok = true;
            int inflight = 0;  // stages issued and not yet confirmed consumed
            for (int tile = blockIdx.x; tile < n_tiles && ok; tile += gridDim.x) {
                const int mt = tile / p.n_nt, nt = tile - mt * p.n_nt;
                const int m0 = mt * kBM, n0 = nt * p.BN;
                if (!tile_live(p, m0)) continue;
                for (int sg = 0; sg < p.n_seg && ok; ++sg) {
                    const SegDev& s = p.seg[sg];
                    const CUtensorMap* ta = sg ? &tmA1 : &tmA0;
                    const CUtensorMap* tb = sg ? &tmB1 : &tmB0;
                    for (int tap = 0; tap < s.n_taps && ok; ++tap) {
                        for (int kbi = 0; kbi < s.n_kb; ++kbi) {
                            if (!mbar_wait(bar_empty + 8 * stage, phase ^ 1, p.err,
                                           VDB_ERR_TIMEOUT_EMPTY, abort_flag)) {
                                ok = false;
                                break;
                            }
                            const uint32_t fb = bar_full + 8 * stage;
                            const uint32_t sa = base + stage * p.stage_bytes;
                            mbar_arrive_expect_tx(fb, s.bytes);
                            tma_load_3d(sa, ta, fb, kbi * s.kb, m0 + s.off[tap], s.plane[tap]);
                            tma_load_2d(sa + p.a_region, tb, fb, tap * s.ic + kbi * s.kb, n0);
                            inflight = min(inflight + 1, (int)S);
                            if (++stage == S) {
                                stage = 0;
                                phase ^= 1;
                            }
                        }
                    }
                }
            }
            if (!ok) {
                // Let copies already issued land before the CTA can exit.
                for (int i = 0; i < inflight; ++i) {
                    stage = (stage + S - 1) % S;
                    mbar_wait_drain(bar_full + 8 * stage, 0, 50000000ull);
                    mbar_wait_drain(bar_full + 8 * stage, 1, 1000ull);
                }
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {
            // ---------------- MMA issuer ----------------
            uint32_t stage = 0, phase = 0;
            uint32_t acc = 0, acc_phase = 0;
            bool ok = true;
            bool issued = false;
            for (int tile = blockIdx.x; tile < n_tiles && ok; tile += gridDim.x) {
                const int mt = tile / p.n_nt;
                const int m0 = mt * kBM;
                if (!tile_live(p, m0)) continue;
                if (!mbar_wait(bar_tempty + 8 * acc, acc_phase ^ 1, p.err,
                               VDB_ERR_TIMEOUT_TEMPTY, abort_flag)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                const uint32_t d_tmem = tmem_base + acc * (uint32_t)p.BN;
                uint32_t first = 1;
                for (int sg = 0; sg < p.n_seg && ok; ++sg) {
                    const SegDev& s = p.seg[sg];
                    const int row_bytes = s.kb * 2;
                    const int ksteps = s.kb / 16;
                    const int iters = s.n_taps * s.n_kb;
                    for (int it = 0; it < iters; ++it) {
                        if (!mbar_wait(bar_full + 8 * stage, phase, p.err, VDB_ERR_TIMEOUT_FULL,
                                       abort_flag)) {
                            ok = false;
                            break;
                        }
                        tc_fence_after();
                        const uint32_t sa = base + stage * p.stage_bytes;
                        const uint64_t ad = umma_sdesc(sa, row_bytes);
                        const uint64_t bd = umma_sdesc(sa + p.a_region, row_bytes);
                        for (int k = 0; k < ksteps; ++k) {
                            // advance 16 f16 = 32 B along K: +2 in the (addr >> 4) field
                            umma_f16(d_tmem, ad + 2 * k, bd + 2 * k, idesc, first ? 0u : 1u);
                            first = 0;
                        }
                        umma_commit(bar_empty + 8 * stage);
                        issued = true;
                        if (++stage == S) {
                            stage = 0;
                            phase ^= 1;
                        }
                    }
                }
                if (!ok) break;
                umma_commit(bar_tfull + 8 * acc);
                if (++acc == 2) {
                    acc = 0;
                    acc_phase ^= 1;
                }
            }
            if (!ok && issued) {
                // Make sure no MMA is still writing TMEM before teardown.
                const uint32_t last = (stage + S - 1) % S;
                mbar_wait_drain(bar_empty + 8 * last, 0, 50000000ull);
                mbar_wait_drain(bar_empty + 8 * last, 1, 1000ull);
            }
        }
    } else if (warp >= 4) {
        // ---------------- epilogue ----------------
        const int quad = warp & 3;  // TMEM lane quadrant this warp may access
        uint32_t acc = 0, acc_phase = 0;
        const int img = p.Hp * p.Wp;
        for (int tile = blockIdx.x; tile < n_tiles; tile += gridDim.x) {
            const int mt = tile / p.n_nt, nt = tile - mt * p.n_nt;
            const int m0 = mt * kBM, n0 = nt * p.BN;
            const bool live = tile_live(p, m0);
            const int m = m0 + quad * 32 + lane;
            bool valid = false;
            long long dst = m;
            if (m < p.M) {
                const int b = m / img;
                const int r = m - b * img;
                const int tp = r / p.Wp;
                const int fp = r - tp * p.Wp;
                valid = live && tp >= 1 && tp <= p.tvalid[b] && fp >= 1 && fp <= p.F;
                if (p.y_phase) {
                    const int q = ((tp & 1) << 1) | (fp & 1);
                    dst = (long long)q * p.plane_rows +
                          ((long long)b * p.Hq + (tp >> 1) + 1) * p.Wq + (fp >> 1) + 1;
                }
            }
            __half* yrow = p.y + dst * p.oc + n0;
            const __half* rrow =
                (p.residual && m < p.M) ? p.residual + (long long)m * p.oc + n0 : nullptr;
            if (live) {
                if (!mbar_wait(bar_tfull + 8 * acc, acc_phase, p.err, VDB_ERR_TIMEOUT_TFULL,
                               abort_flag))
                    break;
                tc_fence_after();
            }
            const uint32_t trow = tmem_base + ((uint32_t)(quad * 32) << 16) + acc * (uint32_t)p.BN;
            int c0 = 0;
            for (; c0 + 32 <= p.BN; c0 += 32)
                epi_chunk<32>(p, live, m < p.M, valid, trow + (uint32_t)c0, n0 + c0,
                              rrow ? rrow + c0 : nullptr, yrow + c0);
            if (c0 < p.BN)
                epi_chunk<16>(p, live, m < p.M, valid, trow + (uint32_t)c0, n0 + c0,
                              rrow ? rrow + c0 : nullptr, yrow + c0);
            if (live) {
                tc_fence_before();
                mbar_arrive(bar_tempty + 8 * acc);
                if (++acc == 2) {
                    acc = 0;
                    acc_phase ^= 1;
                }
            }
        }
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        __syncwarp();
        tc_fence_after();
        tmem_dealloc(tmem_base, p.tmem_cols);
    }
}

CUtensorMapSwizzle swizzle_for(int kb) {
    return kb == 64 ? CU_TENSOR_MAP_SWIZZLE_128B
                    : (kb == 32 ? CU_TENSOR_MAP_SWIZZLE_64B : CU_TENSOR_MAP_SWIZZLE_32B);
}

bool make_map_a(CUtensorMap* m, const void* ptr, int C, long long rows, int planes, int kb) {
    cuuint64_t dims[3] = {(cuuint64_t)C, (cuuint64_t)rows, (cuuint64_t)planes};
    cuuint64_t strides[2] = {(cuuint64_t)C * 2, (cuuint64_t)rows * C * 2};
    cuuint32_t box[3] = {(cuuint32_t)kb, (cuuint32_t)kBM, 1};
    cuuint32_t estr[3] = {1, 1, 1};
    CUresult r = encode_tiled_fn()(
        m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, const_cast<void*>(ptr), dims, strides, box, estr,
        CU_TENSOR_MAP_INTERLEAVE_NONE,
        swizzle_for(kb),
        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS;
}

bool make_map_b(CUtensorMap* m, const void* ptr, int kcols, int oc, int bn, int kb) {
    cuuint64_t dims[2] = {(cuuint64_t)kcols, (cuuint64_t)oc};
    cuuint64_t strides[1] = {(cuuint64_t)kcols * 2};
    cuuint32_t box[2] = {(cuuint32_t)kb, (cuuint32_t)bn};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = encode_tiled_fn()(
        m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void*>(ptr), dims, strides, box, estr,
        CU_TENSOR_MAP_INTERLEAVE_NONE,
        swizzle_for(kb),
        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS;
}

bool fill_seg(SegDev& s, int k, int stride, int ic, int Wp_out, int bn) {
    s.ic = ic;
    s.kb = (ic % 64 == 0) ? 64 : ((ic % 32 == 0) ? 32 : 16);
    s.n_kb = ic / s.kb;
    s.n_taps = k * k;
    s.kcols = s.n_taps * ic;
    s.bytes = (uint32_t)(kBM + bn) * (uint32_t)s.kb * 2u;
    for (int kt = 0; kt < k; ++kt)
        for (int kf = 0; kf < k; ++kf) {
            const int tap = kt * k + kf;
            if (k == 1) {
                // 1x1: stride 1 reads the same grid row; stride 2 reads padded
                // position (2t+1, 2f+1) = plane 3 at the output's own row.
                s.plane[tap] = (stride == 2) ? 3 : 0;
                s.off[tap] = 0;
            } else if (stride == 1) {
                s.plane[tap] = 0;
                s.off[tap] = (kt - 1) * Wp_out + (kf - 1);
            } else {
                s.plane[tap] = ((kt & 1) << 1) | (kf & 1);
                s.off[tap] = (kt >> 1) * Wp_out + (kf >> 1);
            }
        }
    return true;
}

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

extern "C" int vdb_conv(const vdb_conv_args* a, void* stream) {
    if (!a) {
        set_error("vdb_conv: NULL args");
        return 1;
    }
    if (a->batch <= 0 || a->t_out <= 0 || a->f_out <= 0) {
        set_error("vdb_conv: empty output");
        return 1;
    }
    if (a->oc % 16 != 0 || a->oc <= 0) {
        set_error("vdb_conv: oc must be a positive multiple of 16");
        return 1;
    }
    if (a->ic0 % 16 != 0 || a->ic0 <= 0 || (a->x1 && (a->ic1 % 16 != 0 || a->ic1 <= 0))) {
        set_error("vdb_conv: input channels must be positive multiples of 16");
        return 1;
    }
    if (!(a->k0 == 3 || a->k0 == 1) || !(a->stride0 == 1 || a->stride0 == 2) ||
        (a->x1 && !(a->stride1 == 1 || a->stride1 == 2))) {
        set_error("vdb_conv: unsupported kernel/stride");
        return 1;
    }
    if (!a->x0 || !a->w0 || !a->bias || !a->tvalid || !a->y || (a->x1 && !a->w1)) {
        set_error("vdb_conv: NULL buffer");
        return 1;
    }
    const int n_nt = (a->oc + 255) / 256;
    const int BN = a->oc / n_nt;
    if (BN % 16 != 0 || BN * n_nt != a->oc) {
        set_error("vdb_conv: oc does not split into tcgen05 N tiles");
        return 1;
    }
    ConvDev p{};
    const int Hp = a->t_out + 2, Wp = a->f_out + 2;
    p.M = (int)vdb_grid_rows(a->batch, a->t_out, a->f_out);
    p.n_mt = (p.M + kBM - 1) / kBM;
    p.n_nt = n_nt;
    p.BN = BN;
    p.n_seg = a->x1 ? 2 : 1;
    fill_seg(p.seg[0], a->k0, a->stride0, a->ic0, Wp, BN);
    if (a->x1) fill_seg(p.seg[1], 1, a->stride1, a->ic1, Wp, BN);
    int kbmax = p.seg[0].kb;
    if (a->x1) kbmax = std::max(kbmax, p.seg[1].kb);
    p.a_region = (uint32_t)kBM * kbmax * 2;
    p.stage_bytes = p.a_region + (uint32_t)BN * kbmax * 2;
    p.n_stages = std::min<uint32_t>(kMaxStages, kSmemBudget / p.stage_bytes);
    if (p.n_stages < 2) {
        set_error("vdb_conv: stage does not fit in shared memory");
        return 1;
    }
    uint32_t cols = 32;
    while (cols < 2u * (uint32_t)BN) cols <<= 1;
    p.tmem_cols = cols;
    p.bias = a->bias;
    p.residual = static_cast<const __half*>(a->residual);
    p.y = static_cast<__half*>(a->y);
    p.y_phase = a->y_phase;
    p.Hp = Hp;
    p.Wp = Wp;
    p.T = a->t_out;
    p.F = a->f_out;
    p.Hq = (a->t_out - 1) / 2 + 1 + 2;
    p.Wq = (a->f_out - 1) / 2 + 1 + 2;
    p.plane_rows = (long long)a->batch * p.Hq * p.Wq;
    p.tvalid = a->tvalid;
    p.relu = a->relu;
    p.clamp_hi = a->clamp_hi;
    p.oc = a->oc;
    p.err = a->err;

    // Input row extents: stride 1 reads G(B, t_out, f_out); stride 2 reads the
    // 4 planes of a PHASE tensor, each shaped like the output grid.
    const long long rows_out = p.M;
    CUtensorMap tmA0, tmB0, tmA1, tmB1;
    if (!make_map_a(&tmA0, a->x0, a->ic0, rows_out, a->stride0 == 2 ? 4 : 1, p.seg[0].kb) ||
        !make_map_b(&tmB0, a->w0, p.seg[0].kcols, a->oc, BN, p.seg[0].kb)) {
        set_error("vdb_conv: cuTensorMapEncodeTiled failed (segment 0)");
        return 1;
    }
    if (a->x1) {
        if (!make_map_a(&tmA1, a->x1, a->ic1, rows_out, a->stride1 == 2 ? 4 : 1,
                        p.seg[1].kb) ||
            !make_map_b(&tmB1, a->w1, p.seg[1].kcols, a->oc, BN, p.seg[1].kb)) {
            set_error("vdb_conv: cuTensorMapEncodeTiled failed (segment 1)");
            return 1;
        }
    } else {
        tmA1 = tmA0;
        tmB1 = tmB0;
    }
    // stages + 1 KB alignment slack + barriers (2S + 4) * 8 B + TMEM slot / abort flag
    const size_t smem = (size_t)p.n_stages * p.stage_bytes + 1024 + (2 * p.n_stages + 4) * 8 + 16;
    static bool attr_set = false;
    if (!attr_set) {
        VDB_CHECK_CUDA(cudaFuncSetAttribute(conv_tc_kernel,
                                            cudaFuncAttributeMaxDynamicSharedMemorySize,
                                            227 * 1024));
        attr_set = true;
    }
    // TMEM: more than 256 columns per CTA must not share an SM with another CTA.
    size_t smem_launch = smem;
    if (p.tmem_cols > 256) smem_launch = std::max<size_t>(smem, 120 * 1024);
    int occ = 1;
    VDB_CHECK_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, conv_tc_kernel, kThreads,
                                                                  smem_launch));
    occ = std::max(1, std::min(occ, (int)(512 / p.tmem_cols)));
    const int n_tiles = p.n_mt * p.n_nt;
    const int grid = std::max(1, std::min(n_tiles, num_sms() * occ));
    conv_tc_kernel<<<grid, kThreads, smem_launch, static_cast<cudaStream_t>(stream)>>>(
        tmA0, tmB0, tmA1, tmB1, p);
    VDB_CHECK_CUDA(cudaGetLastError());
    return 0;
}
