// Identify: top-k cosine search of query embeddings against a registry. The
// reference advertises identify (README.md:15,44,59) but has no implementation, so
// the semantics are the oracle's (oracle/vd_oracle.c, vdo_identify): cosine =
// dot / (|q| |r|) (0 when a norm is 0), top-k by descending score, equal scores
// ordered by the lower registry index.
//
// Tensor-core path (dim <= 512), three kernels:
//   1. normalize_rows_kernel: every query and registry row to a unit-norm f16 row
//      (zero-padded to a multiple of 64 dims) and its f64 norm.
//   2. identify_tc_kernel: a persistent tcgen05 GEMM. A CTA holds 256 queries (128
//      when dim > 256) resident in shared memory and streams 128-row registry tiles
//      through a TMA ring; each tile's scores land in a double-buffered TMEM
//      accumulator (M = 128 queries x N = 128 registry rows per MMA, f32), and eight
//      epilogue warps read them with tcgen05.ld and keep, per query, a running list of
//      the best L = k + 8 (score, index) pairs. The score matrix is never written.
//      Work items are (query block, registry slice); each writes its lists once.
//   3. merge_rescore_kernel: per query, the best L candidates over all slices by the
//      f16 scores, each rescored exactly (f64 dot of the f32 inputs over the f64
//      norms), then the top k of those by (exact score desc, index asc).
// Returned scores are exact cosines of the returned rows. The f16 candidate search
// can only miss a true top-k row if f16 rounding (|error| <= 2^-10 on unit vectors)
// reorders it behind 8 or more other rows, i.e. when more than k + 8 rows score
// within about 2e-3 of the k-th best; ties between identical rows stay exact.
// dim > 512 uses the CUDA-core path: an f32 tiled score GEMM into a bounded scratch
// chunk plus a warp-per-query top-k merge.
#include <cuda_fp16.h>

#include <algorithm>
#include <cfloat>
#include <climits>
#include <mutex>

#include "sm100_ptx.cuh"
#include "vdb_internal.h"
#include "vdb_ops.h"

namespace vdb {
namespace {

constexpr int kMaxK = 64;
constexpr int kExtra = 8;          // candidates per query beyond k kept for rescoring
constexpr int kMaxL = kMaxK + kExtra;

__device__ __forceinline__ bool better(float s, int i, float t, int j) {
    return s > t || (s == t && i < j);
}

// Order-preserving map of a float to an int (a < b  <=>  key(a) < key(b)), for
// atomicMax on scores of either sign.
__device__ __forceinline__ int score_key(float f) {
    const int i = __float_as_int(f);
    return i >= 0 ? i : i ^ 0x7FFFFFFF;
}
__device__ __forceinline__ float key_score(int k) {
    return __int_as_float(k >= 0 ? k : k ^ 0x7FFFFFFF);
}

// ---------------------------------------------------------------------------
// 1. unit-norm f16 rows
// ---------------------------------------------------------------------------
// One warp per row: |x| in f64 (lanes stride the dims, fixed-order reduction), then
// f16(x / |x|) into xh [rows_pad][dim_pad] (padding dims 0; a zero row stays 0) and
// |x| into nrm. Rows past n (up to the padded count) are written as zeros.
__global__ void __launch_bounds__(256)
normalize_rows_kernel(const float* __restrict__ x, int n, int n_pad, int dim, int dim_pad,
                      __half* __restrict__ xh, double* __restrict__ nrm, int* __restrict__ thr) {
    const int row = blockIdx.x * 8 + (threadIdx.x >> 5);
    const int lane = threadIdx.x & 31;
    if (row >= n_pad) return;
    if (thr && lane == 0) thr[row] = score_key(-INFINITY);
    __half* out = xh + (long long)row * dim_pad;
    if (row >= n) {
        for (int d = lane; d < dim_pad; d += 32) out[d] = __float2half_rn(0.0f);
        return;
    }
    const float* r = x + (long long)row * dim;
    double s = 0.0;
    for (int d = lane; d < dim; d += 32) s += (double)r[d] * (double)r[d];
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    const double norm = sqrt(s);
    if (lane == 0) nrm[row] = norm;
    const double inv = norm > 0.0 ? 1.0 / norm : 0.0;
    for (int d = lane; d < dim_pad; d += 32)
        out[d] = __float2half_rn(d < dim ? (float)((double)r[d] * inv) : 0.0f);
}

// ---------------------------------------------------------------------------
// 2. tensor-core scores with the running top-L in the epilogue
// ---------------------------------------------------------------------------
constexpr int kThreads = 384;        // warp 0 TMA, warp 1 MMA, warps 4..11 epilogue
constexpr int kRows = 128;           // registry rows per tile (MMA N) and queries per row block
constexpr int kKc = 64;              // dims per K chunk (128-byte swizzled rows)
constexpr uint32_t kChunkBytes = kRows * kKc * 2;  // one 128 x 64 f16 box: 16 KB
constexpr int kStages = 5;
constexpr uint32_t kStageBytes = 8 * 32 * 17 * 4;  // 16 scores per epilogue thread, padded

struct IdDev {
    int n_q, n_reg, n_rt;     // queries, registry rows, registry tiles of 128
    int n_kc;                 // K chunks of 64 dims
    int nrb;                  // query row blocks per item (2: 256 queries, 1: 128)
    int n_qb, n_sl;           // query blocks, registry slices
    int L;                    // candidates kept per query and item (the reservoir size)
    float* part_s;            // [n_sl][n_q_pad][L] f16-scored candidates
    int* part_i;
    int n_q_pad;
    int* thr;                 // [n_q_pad] per-query lower bound on its L-th best f16
                              // score, as an order-preserving int (atomicMax)
    int seed;                 // 1: only raise thr (no candidate lists written)
    int* err;
};


// Candidate reservoir of one query: the LR best (score desc, index asc) of the values
// admitted so far, unsorted, in registers; `mn` / `mi` / `mpos` are its worst entry
// (lowest score, highest index among equal scores) once it is full.
template <int LR>
struct Reservoir {
    float s[LR];
    int i[LR];
    int n;
    float mn;
    int mi, mpos;

    __device__ __forceinline__ void reset() {
        n = 0;
        mn = -INFINITY;
        mi = INT_MAX;
        mpos = 0;
#pragma unroll
        for (int j = 0; j < LR; ++j) {
            s[j] = -INFINITY;
            i[j] = -1;
        }
    }
    __device__ __forceinline__ void find_worst() {
        mn = s[0];
        mi = i[0];
        mpos = 0;
#pragma unroll
        for (int j = 1; j < LR; ++j) {
            const bool w = s[j] < mn || (s[j] == mn && i[j] > mi);
            mn = w ? s[j] : mn;
            mi = w ? i[j] : mi;
            mpos = w ? j : mpos;
        }
    }
    // Called only for v above the admission threshold: appends, or replaces the worst.
    __device__ __forceinline__ void add(float v, int idx) {
        const int slot = n < LR ? n : mpos;
#pragma unroll
        for (int j = 0; j < LR; ++j) {
            const bool here = j == slot;
            s[j] = here ? v : s[j];
            i[j] = here ? idx : i[j];
        }
        if (n < LR) ++n;
        if (n == LR) find_worst();
    }
};

template <int LR>
__global__ void __launch_bounds__(kThreads, 1)
identify_tc_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmR,
                   const __grid_constant__ IdDev p) {
    extern __shared__ uint8_t smem_raw[];
    const uint32_t raw_u32 = smem_u32(smem_raw);
    const uint32_t base = (raw_u32 + 1023u) & ~1023u;
    uint8_t* smem = smem_raw + (base - raw_u32);
    const uint32_t q_bytes = (uint32_t)p.nrb * p.n_kc * kChunkBytes;
    const uint32_t stage0 = q_bytes;
    const uint32_t stage_off = stage0 + kStages * kChunkBytes;  // epilogue value staging
    const uint32_t bar0 = stage_off + kStageBytes;
    const uint32_t bar_full = base + bar0;
    const uint32_t bar_empty = bar_full + 8 * kStages;
    const uint32_t bar_tfull = bar_empty + 8 * kStages;
    const uint32_t bar_tempty = bar_tfull + 16;
    const uint32_t bar_qfull = bar_tempty + 16;
    const uint32_t bar_qempty = bar_qfull + 8;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + bar0 + 8 * (2 * kStages + 6));
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t acc_cols = (uint32_t)p.nrb * kRows;  // one accumulator buffer

    if (threadIdx.x == 0) {
        for (int s = 0; s < kStages; ++s) {
            mbar_init(bar_full + 8 * s, 1);
            mbar_init(bar_empty + 8 * s, 1);
        }
        for (int a = 0; a < 2; ++a) {
            mbar_init(bar_tfull + 8 * a, 1);
            mbar_init(bar_tempty + 8 * a, 8 * 32);
        }
        mbar_init(bar_qfull, 1);
        mbar_init(bar_qempty, 1);
        *abort_flag = 0;
        fence_barrier_init();
        fence_proxy_async_smem();
    }
    if (warp == 0 && lane == 0) {
        tma_prefetch_desc(&tmQ);
        tma_prefetch_desc(&tmR);
    }
    if (warp == 1) tmem_alloc(smem_u32(tmem_slot), 2 * acc_cols < 256 ? 256 : 2 * acc_cols);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;
    const int n_items = p.n_qb * p.n_sl;

    if (warp == 0) {
        if (lane == 0) {
            // ---------------- TMA producer ----------------
            uint32_t stage = 0, phase = 0, qphase = 0;
            bool ok = true;
            for (int item = blockIdx.x; item < n_items && ok; item += gridDim.x) {
                const int qb = item / p.n_sl, sl = item - qb * p.n_sl;
                const int t0 = (int)((long long)sl * p.n_rt / p.n_sl);
                const int t1 = (int)((long long)(sl + 1) * p.n_rt / p.n_sl);
                // the previous item's MMAs are done with the resident queries
                if (!mbar_wait(bar_qempty, qphase ^ 1, p.err, VDB_ERR_TIMEOUT_EMPTY, abort_flag)) {
                    ok = false;
                    break;
                }
                qphase ^= 1;
                mbar_arrive_expect_tx(bar_qfull, q_bytes);
                for (int rb = 0; rb < p.nrb; ++rb)
                    for (int c = 0; c < p.n_kc; ++c)
                        tma_load_2d(base + (uint32_t)(rb * p.n_kc + c) * kChunkBytes, &tmQ,
                                    bar_qfull, c * kKc, (qb * p.nrb + rb) * kRows);
                for (int t = t0; t < t1 && ok; ++t)
                    for (int c = 0; c < p.n_kc; ++c) {
                        if (!mbar_wait(bar_empty + 8 * stage, phase ^ 1, p.err,
                                       VDB_ERR_TIMEOUT_EMPTY, abort_flag)) {
                            ok = false;
                            break;
                        }
                        mbar_arrive_expect_tx(bar_full + 8 * stage, kChunkBytes);
                        tma_load_2d(base + stage0 + stage * kChunkBytes, &tmR, bar_full + 8 * stage,
                                    c * kKc, t * kRows);
                        if (++stage == kStages) {
                            stage = 0;
                            phase ^= 1;
                        }
                    }
            }
            if (!ok) {
                for (int i = 0; i < kStages; ++i)
                    mbar_wait_drain(bar_full + 8 * i, phase, 20000000ull);
                mbar_wait_drain(bar_qfull, qphase ^ 1, 20000000ull);
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {
            // ---------------- MMA issuer ----------------
            const uint32_t idesc = umma_idesc_f16(kRows, kRows);
            uint32_t stage = 0, phase = 0, qphase = 0, acc = 0, acc_phase = 0;
            bool ok = true, issued = false;
            const uint64_t q_desc = umma_sdesc(base, 128);
            const uint64_t s_desc = umma_sdesc(base + stage0, 128);
            const uint32_t chunk_units = kChunkBytes >> 4;
            for (int item = blockIdx.x; item < n_items && ok; item += gridDim.x) {
                const int sl = item % p.n_sl;
                const int t0 = (int)((long long)sl * p.n_rt / p.n_sl);
                const int t1 = (int)((long long)(sl + 1) * p.n_rt / p.n_sl);
                if (!mbar_wait(bar_qfull, qphase, p.err, VDB_ERR_TIMEOUT_FULL, abort_flag)) {
                    ok = false;
                    break;
                }
                qphase ^= 1;
                tc_fence_after();
                for (int t = t0; t < t1 && ok; ++t) {
                    if (!mbar_wait(bar_tempty + 8 * acc, acc_phase ^ 1, p.err,
                                   VDB_ERR_TIMEOUT_TEMPTY, abort_flag)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t d = tmem_base + acc * acc_cols;
                    for (int c = 0; c < p.n_kc; ++c) {
                        if (!mbar_wait(bar_full + 8 * stage, phase, p.err, VDB_ERR_TIMEOUT_FULL,
                                       abort_flag)) {
                            ok = false;
                            break;
                        }
                        tc_fence_after();
                        const uint64_t b = s_desc + (uint64_t)(stage * chunk_units);
                        const uint64_t a0 = q_desc + (uint64_t)(c * chunk_units);
#pragma unroll
                        for (int k = 0; k < kKc / 16; ++k) {
                            umma_f16(d, a0 + 2 * k, b + 2 * k, idesc, (c | k) ? 1u : 0u);
                            if (p.nrb == 2)
                                umma_f16(d + kRows, a0 + (uint64_t)(p.n_kc * chunk_units) + 2 * k,
                                         b + 2 * k, idesc, (c | k) ? 1u : 0u);
                        }
                        umma_commit(bar_empty + 8 * stage);
                        issued = true;
                        if (++stage == kStages) {
                            stage = 0;
                            phase ^= 1;
                        }
                    }
                    if (!ok) break;
                    umma_commit(bar_tfull + 8 * acc);
                    if (++acc == 2) {
                        acc = 0;
                        acc_phase ^= 1;
                    }
                }
                if (!ok) break;
                umma_commit(bar_qempty);  // resident queries free once these MMAs are done
            }
            if (!ok && issued) {
                const uint32_t last = (stage + kStages - 1) % kStages;
                mbar_wait_drain(bar_empty + 8 * last, phase ^ (stage == 0 ? 1u : 0u), 20000000ull);
            }
        }
    } else if (warp >= 4) {
        // ---------------- epilogue: the best LR candidates per query ----------------
        // Thread = one query (TMEM lane). A value enters the reservoir when it beats
        // the admission threshold: while the reservoir fills, the query's published
        // lower bound (p.thr, raised by earlier items: any item's LR-th best is at most
        // the query's overall L-th best), afterwards the reservoir's worst entry. A
        // 32-value chunk in which no lane of the warp beats its threshold costs one max
        // and one vote.
        const int ew = warp - 4;
        const int quad = warp & 3;       // TMEM lane quadrant this warp may read
        const int rb = ew >> 2;          // query row block
        const bool active = rb < p.nrb;
        float* my_stage = reinterpret_cast<float*>(smem + stage_off) + (ew * 32 + lane) * 17;
        Reservoir<LR> res;
        uint32_t acc = 0, acc_phase = 0;
        bool ok = true;
        for (int item = blockIdx.x; item < n_items && ok; item += gridDim.x) {
            const int qb = item / p.n_sl, sl = item - qb * p.n_sl;
            const int t0 = (int)((long long)sl * p.n_rt / p.n_sl);
            const int t1 = (int)((long long)(sl + 1) * p.n_rt / p.n_sl);
            const int q = (qb * p.nrb + rb) * kRows + quad * 32 + lane;
            res.reset();
            // the largest float below the bound: values equal to the bound still enter
            float floor_s = -INFINITY;
            if (active && q < p.n_q_pad) {
                const float b = key_score(((volatile int*)p.thr)[q]);
                floor_s = b > -INFINITY ? nextafterf(b, -INFINITY) : -INFINITY;
            }
            for (int t = t0; t < t1; ++t) {
                if (!mbar_wait(bar_tfull + 8 * acc, acc_phase, p.err, VDB_ERR_TIMEOUT_TFULL,
                               abort_flag)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                if (active) {
                    const uint32_t taddr = tmem_base + ((uint32_t)(quad * 32) << 16) +
                                           acc * acc_cols + (uint32_t)(rb * kRows);
                    const int r0 = t * kRows;
                    const int valid = min(kRows, p.n_reg - r0);
#pragma unroll 1
                    for (int cb = 0; cb < kRows; cb += 64) {
                        // two 32-column loads in flight, one wait
                        uint32_t v[2][32];
                        __syncwarp();  // tcgen05.ld is warp-collective: reconverge first
                        tmem_ld_32x32b_x32_nowait(taddr + (uint32_t)cb, v[0]);
                        tmem_ld_32x32b_x32_nowait(taddr + (uint32_t)cb + 32u, v[1]);
                        tmem_wait_ld();
                        tmem_regs_ready(v[0]);
                        tmem_regs_ready(v[1]);
                        float thr = res.n < LR ? floor_s : fmaxf(floor_s, res.mn);
                        // strictly above: a later row with an equal score has a higher
                        // index, so it never displaces an earlier one
                        uint32_t mask[4] = {0u, 0u, 0u, 0u};
#pragma unroll
                        for (int i = 0; i < 64; ++i)
                            mask[i >> 4] |= (__uint_as_float(v[i >> 5][i & 31]) > thr &&
                                             cb + i < valid) ? (1u << (i & 15)) : 0u;
#pragma unroll
                        for (int h = 0; h < 4; ++h) {
                            uint32_t m = mask[h];
                            if (m == 0) continue;
                            // the rare lanes with candidates walk them in a rolled loop (one
                            // inlined insertion: an unrolled one per value made the
                            // epilogue's hot code too large for the instruction cache)
#pragma unroll
                            for (int i = 0; i < 16; ++i)
                                my_stage[i] = __uint_as_float(v[h >> 1][(h & 1) * 16 + i]);
#pragma unroll 1
                            for (; m; m &= m - 1) {
                                const int i = __ffs(m) - 1;
                                const float sv = my_stage[i];
                                if (sv > thr) {
                                    res.add(sv, r0 + cb + h * 16 + i);
                                    thr = res.n < LR ? floor_s : fmaxf(floor_s, res.mn);
                                }
                            }
                        }
                    }
                }
                tc_fence_before();
                mbar_arrive(bar_tempty + 8 * acc);
                if (++acc == 2) {
                    acc = 0;
                    acc_phase ^= 1;
                }
                // every 4 tiles: share this item's LR-th best with the query's other
                // items (running concurrently on other SMs) and take the best bound so far
                if (active && q < p.n_q && ((t - t0) & 3) == 3) {
                    if (res.n == LR) atomicMax(p.thr + q, score_key(res.mn));
                    const float b = key_score(((volatile int*)p.thr)[q]);
                    if (b > -INFINITY) floor_s = fmaxf(floor_s, nextafterf(b, -INFINITY));
                }
            }
            if (!ok || !active || q >= p.n_q) continue;
            // this item's LR-th best bounds the query's overall L-th best from below
            if (res.n == LR) atomicMax(p.thr + q, score_key(res.mn));
            if (p.seed) continue;
            const long long o = ((long long)sl * p.n_q_pad + q) * LR;
#pragma unroll
            for (int j = 0; j < LR; ++j) {
                p.part_s[o + j] = res.s[j];
                p.part_i[o + j] = res.i[j];
            }
        }
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        __syncwarp();
        tc_fence_after();
        tmem_dealloc(tmem_base, 2 * acc_cols < 256 ? 256 : 2 * acc_cols);
    }
}

// ---------------------------------------------------------------------------
// 3. merge the slices' candidates, rescore exactly, emit the top k
// ---------------------------------------------------------------------------
// Warp per query over LS candidates per slice. Candidates are ranked by (f16 score
// desc, index asc); the best L are rescored as dot(q, r) / (|q| |r|) in f64 from the f32 inputs, and the top k
// of those by (exact score desc, index asc) are written (-1 / -inf past n_reg).
__global__ void __launch_bounds__(256)
merge_rescore_kernel(const float* __restrict__ part_s, const int* __restrict__ part_i, int n_sl,
                     int n_q_pad, int LS, int L, const float* __restrict__ q,
                     const float* __restrict__ reg, int n_q, int dim,
                     const double* __restrict__ qn, const double* __restrict__ rn, int k,
                     int* __restrict__ out_idx, float* __restrict__ out_score) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int qq = blockIdx.x * 8 + warp;
    if (qq >= n_q) return;
    // this lane's candidates, sorted by (f16 score desc, index asc)
    float ls[kMaxL];
    int li[kMaxL];
    int n = 0;
    for (int e = lane; e < n_sl * LS; e += 32) {
        const int sl = e / LS, j = e - sl * LS;
        const long long o = ((long long)sl * n_q_pad + qq) * LS + j;
        const int i = part_i[o];
        if (i < 0) continue;
        const float s = part_s[o];
        if (n == L && !better(s, i, ls[L - 1], li[L - 1])) continue;
        int pos = n < L ? n : L - 1;
        while (pos > 0 && better(s, i, ls[pos - 1], li[pos - 1])) {
            ls[pos] = ls[pos - 1];
            li[pos] = li[pos - 1];
            --pos;
        }
        ls[pos] = s;
        li[pos] = i;
        if (n < L) ++n;
    }
    // the best L over the warp (L rounds of an arg-best over the lanes' heads), each
    // rescored exactly by the whole warp; kept sorted by (exact desc, index asc)
    const float* qrow = q + (long long)qq * dim;
    const double qnorm = qn[qq];
    float es[kMaxL];
    int ei[kMaxL];
    int m = 0, head = 0;
    for (int r = 0; r < L; ++r) {
        float bs = head < n ? ls[head] : -INFINITY;
        int bi = head < n ? li[head] : INT_MAX;
#pragma unroll
        for (int o = 16; o >= 1; o >>= 1) {
            const float os = __shfl_xor_sync(0xffffffffu, bs, o);
            const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
            if (better(os, oi, bs, bi)) {
                bs = os;
                bi = oi;
            }
        }
        if (bi == INT_MAX) break;
        if (head < n && li[head] == bi) ++head;
        const float* rrow = reg + (long long)bi * dim;
        double dot = 0.0;
        for (int d = lane; d < dim; d += 32) dot += (double)qrow[d] * (double)rrow[d];
#pragma unroll
        for (int o = 16; o >= 1; o >>= 1) dot += __shfl_xor_sync(0xffffffffu, dot, o);
        const double den = qnorm * rn[bi];
        const float es_new = den > 0.0 ? (float)(dot / den) : 0.0f;
        // insert into the exact list (identical on every lane)
        int pos = m;
        while (pos > 0 && better(es_new, bi, es[pos - 1], ei[pos - 1])) {
            es[pos] = es[pos - 1];
            ei[pos] = ei[pos - 1];
            --pos;
        }
        es[pos] = es_new;
        ei[pos] = bi;
        ++m;
    }
    if (lane == 0) {
        for (int j = 0; j < k; ++j) {
            out_idx[(long long)qq * k + j] = j < m ? ei[j] : -1;
            out_score[(long long)qq * k + j] = j < m ? es[j] : -INFINITY;
        }
    }
}

// ---------------------------------------------------------------------------
// CUDA-core path for dim > 512
// ---------------------------------------------------------------------------
constexpr int kTile = 128, kBK = 16;

__global__ void row_norm_kernel(const float* __restrict__ v, int n, int dim,
                                float* __restrict__ nrm) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    const float* r = v + (long long)i * dim;
    float s = 0.0f;
    for (int d = 0; d < dim; ++d) s = fmaf(r[d], r[d], s);
    nrm[i] = sqrtf(s);
}

// scores[q][r - r0] = dot(q, reg[r]) / (|q| |reg[r]|) (0 when a norm is 0), for
// registry rows [r0, r0 + nr) and queries [q0, q0 + nq).
__global__ void __launch_bounds__(256)
score_kernel(const float* __restrict__ q, int q0, int nq, const float* __restrict__ reg, int r0,
             int nr, int dim, const float* __restrict__ qn, const float* __restrict__ rn,
             float* __restrict__ scores) {
    __shared__ float As[kBK][kTile + 4];
    __shared__ float Bs[kBK][kTile + 4];
    const int qb = blockIdx.y * kTile, rb = blockIdx.x * kTile;
    const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;
    float acc[8][8];
#pragma unroll
    for (int i = 0; i < 8; ++i)
#pragma unroll
        for (int j = 0; j < 8; ++j) acc[i][j] = 0.0f;
    for (int k0 = 0; k0 < dim; k0 += kBK) {
        for (int e = threadIdx.x; e < kTile * kBK; e += 256) {
            const int row = e / kBK, kk = e - row * kBK;
            const int qq = qb + row, rr = rb + row, d = k0 + kk;
            As[kk][row] = (qq < nq && d < dim) ? q[(long long)(q0 + qq) * dim + d] : 0.0f;
            Bs[kk][row] = (rr < nr && d < dim) ? reg[(long long)(r0 + rr) * dim + d] : 0.0f;
        }
        __syncthreads();
#pragma unroll
        for (int kk = 0; kk < kBK; ++kk) {
            float a[8], b[8];
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                a[i] = As[kk][ty * 4 + i];
                a[4 + i] = As[kk][64 + ty * 4 + i];
                b[i] = Bs[kk][tx * 4 + i];
                b[4 + i] = Bs[kk][64 + tx * 4 + i];
            }
#pragma unroll
            for (int i = 0; i < 8; ++i)
#pragma unroll
                for (int j = 0; j < 8; ++j) acc[i][j] = fmaf(a[i], b[j], acc[i][j]);
        }
        __syncthreads();
    }
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const int qq = qb + (i < 4 ? ty * 4 + i : 64 + ty * 4 + i - 4);
        if (qq >= nq) continue;
        const float nq_ = qn[q0 + qq];
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const int rr = rb + (j < 4 ? tx * 4 + j : 64 + tx * 4 + j - 4);
            if (rr >= nr) continue;
            const float den = nq_ * rn[r0 + rr];
            scores[(long long)qq * nr + rr] = den > 0.0f ? acc[i][j] / den : 0.0f;
        }
    }
}

// Warp per query: merge scores[q][0..nr) (registry rows r0..) into the running top-k
// (valid entries first; the first chunk starts empty). NaN scores never enter.
__global__ void __launch_bounds__(256)
topk_kernel(const float* __restrict__ scores, int q0, int nq, int r0, int nr, int k, int first,
            int* __restrict__ out_idx, float* __restrict__ out_score) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int qi = blockIdx.x * 8 + warp;
    if (qi >= nq) return;
    const int qq = q0 + qi;
    float ls[kMaxK];
    int li[kMaxK];
    int n = 0;
    auto push = [&](float s, int i) {
        if (!(s >= -FLT_MAX)) return;  // NaN (and -inf) never enter the list
        if (n == k && !better(s, i, ls[k - 1], li[k - 1])) return;
        int pos = n < k ? n : k - 1;
        while (pos > 0 && better(s, i, ls[pos - 1], li[pos - 1])) {
            ls[pos] = ls[pos - 1];
            li[pos] = li[pos - 1];
            --pos;
        }
        ls[pos] = s;
        li[pos] = i;
        if (n < k) ++n;
    };
    const float* row = scores + (long long)qi * nr;
    for (int r = lane; r < nr; r += 32) push(row[r], r0 + r);
    if (!first && lane == 0) {
        for (int j = 0; j < k; ++j) {
            const int i = out_idx[(long long)qq * k + j];
            if (i >= 0) push(out_score[(long long)qq * k + j], i);
        }
    }
    int head = 0;
    for (int j = 0; j < k; ++j) {
        float bs = head < n ? ls[head] : -INFINITY;
        int bi = head < n ? li[head] : INT_MAX;
#pragma unroll
        for (int o = 16; o >= 1; o >>= 1) {
            const float os = __shfl_xor_sync(0xffffffffu, bs, o);
            const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
            if (better(os, oi, bs, bi)) {
                bs = os;
                bi = oi;
            }
        }
        if (head < n && li[head] == bi) ++head;
        if (lane == 0) {
            out_idx[(long long)qq * k + j] = bi == INT_MAX ? -1 : bi;
            out_score[(long long)qq * k + j] = bi == INT_MAX ? -INFINITY : bs;
        }
    }
}

int identify_cuda_cores(const float* q, int n_q, const float* reg, int n_reg, int dim, int k,
                        int* out_idx, float* out_score, cudaStream_t st) {
    // Score scratch bounded to 2^28 floats (1 GB): queries in chunks of at most 8192
    // and registry rows in chunks of (2^28 / query chunk), a multiple of 128.
    const int qc = std::min(n_q, 8192);
    long long chunk = (1LL << 28) / qc;
    chunk = std::max<long long>(kTile, std::min<long long>(chunk, 32768)) / kTile * kTile;
    chunk = std::min<long long>(chunk, n_reg);
    float* work = nullptr;
    const size_t bytes = sizeof(float) * ((size_t)n_q + n_reg + (size_t)qc * chunk);
    keep_async_pool();
    VDB_CHECK_CUDA(cudaMallocAsync(&work, bytes, st));
    float* qn = work;
    float* rn = qn + n_q;
    float* sc = rn + n_reg;
    row_norm_kernel<<<(n_q + 255) / 256, 256, 0, st>>>(q, n_q, dim, qn);
    row_norm_kernel<<<(n_reg + 255) / 256, 256, 0, st>>>(reg, n_reg, dim, rn);
    int rc = 0;
    for (int q0 = 0; q0 < n_q && rc == 0; q0 += qc) {
        const int nq = std::min(qc, n_q - q0);
        for (int r0 = 0; r0 < n_reg && rc == 0; r0 += (int)chunk) {
            const int nr = (int)std::min<long long>(chunk, n_reg - r0);
            const dim3 grid((nr + kTile - 1) / kTile, (nq + kTile - 1) / kTile);
            score_kernel<<<grid, 256, 0, st>>>(q, q0, nq, reg, r0, nr, dim, qn, rn, sc);
            topk_kernel<<<(nq + 7) / 8, 256, 0, st>>>(sc, q0, nq, r0, nr, k, r0 == 0 ? 1 : 0,
                                                      out_idx, out_score);
            if (cudaGetLastError() != cudaSuccess) rc = 1;
        }
    }
    cudaFreeAsync(work, st);
    if (rc) {
        set_error("vdb_identify: kernel launch failed");
        return 1;
    }
    return 0;
}

bool make_map_rows(CUtensorMap* m, const void* ptr, int dim_pad, long long rows) {
    cuuint64_t dims[2] = {(cuuint64_t)dim_pad, (cuuint64_t)rows};
    cuuint64_t strides[1] = {(cuuint64_t)dim_pad * 2};
    cuuint32_t box[2] = {(cuuint32_t)kKc, (cuuint32_t)kRows};
    cuuint32_t estr[2] = {1, 1};
    return encode_tiled_fn()(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void*>(ptr), dims,
                             strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                             CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

}  // namespace
}  // namespace vdb

using namespace vdb;

extern "C" int vdb_identify(const float* q, int n_q, const float* reg, int n_reg, int dim, int k,
                            int* out_idx, float* out_score, void* stream) {
    if (!q || !reg || !out_idx || !out_score) {
        set_error("vdb_identify: NULL argument");
        return 1;
    }
    if (n_q <= 0 || n_reg <= 0 || dim <= 0 || dim > 1024 || k <= 0 || k > kMaxK) {
        set_error("vdb_identify: need n_q, n_reg > 0, 0 < dim <= 1024, 0 < k <= 64");
        return 1;
    }
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    const int dim_pad = (dim + kKc - 1) / kKc * kKc;
    if (dim_pad > 512) return identify_cuda_cores(q, n_q, reg, n_reg, dim, k, out_idx, out_score, st);

    IdDev p{};
    p.nrb = dim_pad <= 256 ? 2 : 1;
    p.n_kc = dim_pad / kKc;
    p.n_q = n_q;
    p.n_reg = n_reg;
    p.n_rt = (n_reg + kRows - 1) / kRows;
    p.n_qb = (n_q + p.nrb * kRows - 1) / (p.nrb * kRows);
    p.n_q_pad = p.n_qb * p.nrb * kRows;
    // reservoir per query and item: 16 entries for k <= 8 (registers), else 72
    const int LR = k + kExtra <= 16 ? 16 : kMaxL;
    const int L_pool = std::min(k + kExtra, LR);
    p.L = LR;
    // Registry slices per query block: enough work items for every SM, choosing the
    // count whose last wave is fullest (an item = one query block x one slice).
    const int G = num_sms();
    int best = 1;
    double best_eff = -1.0;
    const int lo = std::max(1, std::min(p.n_rt, (2 * G + p.n_qb - 1) / p.n_qb));
    const int hi = std::max(lo, std::min(p.n_rt, (16 * G + p.n_qb - 1) / p.n_qb));
    for (int s = lo; s <= hi; ++s) {
        const long long items = (long long)p.n_qb * s;
        const long long waves = (items + G - 1) / G;
        const double eff = (double)items / (double)(waves * G);
        if (eff > best_eff + 1e-9) {
            best_eff = eff;
            best = s;
        }
    }
    p.n_sl = best;
    const long long n_reg_pad = (long long)p.n_rt * kRows;

    // workspace: f16 rows, f64 norms, per-slice candidate lists
    const size_t qh_b = (size_t)p.n_q_pad * dim_pad * 2, rh_b = (size_t)n_reg_pad * dim_pad * 2;
    const size_t nrm_b = sizeof(double) * ((size_t)n_q + (size_t)n_reg);
    const size_t part_n = (size_t)p.n_sl * p.n_q_pad * p.L;
    auto up = [](size_t b) { return (b + 255) / 256 * 256; };
    const size_t thr_b = sizeof(int) * (size_t)p.n_q_pad;
    const size_t bytes = up(qh_b) + up(rh_b) + up(nrm_b) + up(part_n * 4) * 2 + up(thr_b);
    uint8_t* work = nullptr;
    keep_async_pool();
    VDB_CHECK_CUDA(cudaMallocAsync(reinterpret_cast<void**>(&work), bytes, st));
    __half* qh = reinterpret_cast<__half*>(work);
    __half* rh = reinterpret_cast<__half*>(work + up(qh_b));
    double* qn = reinterpret_cast<double*>(work + up(qh_b) + up(rh_b));
    double* rn = qn + n_q;
    p.part_s = reinterpret_cast<float*>(work + up(qh_b) + up(rh_b) + up(nrm_b));
    p.part_i = reinterpret_cast<int*>(work + up(qh_b) + up(rh_b) + up(nrm_b) + up(part_n * 4));
    p.thr = reinterpret_cast<int*>(work + up(qh_b) + up(rh_b) + up(nrm_b) + 2 * up(part_n * 4));
    p.err = nullptr;

    int rc = 0;
    normalize_rows_kernel<<<(p.n_q_pad + 7) / 8, 256, 0, st>>>(q, n_q, p.n_q_pad, dim, dim_pad, qh,
                                                                qn, p.thr);
    normalize_rows_kernel<<<(int)((n_reg_pad + 7) / 8), 256, 0, st>>>(reg, n_reg, (int)n_reg_pad,
                                                                      dim, dim_pad, rh, rn, nullptr);
    CUtensorMap tq, tr;
    if (!make_map_rows(&tq, qh, dim_pad, p.n_q_pad) || !make_map_rows(&tr, rh, dim_pad, n_reg_pad)) {
        set_error("vdb_identify: cuTensorMapEncodeTiled failed");
        rc = 1;
    }
    if (!rc) {
        const uint32_t q_bytes = (uint32_t)p.nrb * p.n_kc * kChunkBytes;
        const size_t smem =
            1024 + q_bytes + kStages * kChunkBytes + kStageBytes + 8 * (2 * kStages + 6) + 16;
        auto kern = LR == 16 ? identify_tc_kernel<16> : identify_tc_kernel<kMaxL>;
        cudaError_t e = cudaSuccess;
        {
            // the shared-memory opt-in, once per device and kernel (the size is fixed)
            static std::mutex mu;
            static bool set[64][2] = {};
            int dev = 0;
            cudaGetDevice(&dev);
            std::lock_guard<std::mutex> lk(mu);
            const int kv = LR == 16 ? 0 : 1;
            if (dev < 0 || dev >= 64 || !set[dev][kv]) {
                e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)(1024 + 2 * 4 * kChunkBytes + kStages * kChunkBytes +
                                               kStageBytes + 8 * (2 * kStages + 6) + 16));
                if (e == cudaSuccess && dev >= 0 && dev < 64) set[dev][kv] = true;
            }
        }
        // Seed pass over the first 32 registry tiles (4096 rows, 8 slices of 4): raises
        // every query's admission bound before the full pass, so the full pass's items
        // start warm instead of admitting most values of their first tiles.
        if (e == cudaSuccess && p.n_rt >= 64) {
            IdDev ps = p;
            ps.seed = 1;
            ps.n_rt = 32;
            ps.n_sl = 8;
            // same reservoir size as the full pass: the bound must be an LR-th best
            kern<<<std::min(ps.n_qb * ps.n_sl, G), kThreads, smem, st>>>(tq, tr, ps);
            e = cudaGetLastError();
        }
        const int items = p.n_qb * p.n_sl;
        const int grid = std::min(items, G);
        if (e == cudaSuccess) {
            kern<<<grid, kThreads, smem, st>>>(tq, tr, p);
            e = cudaGetLastError();
        }
        if (e == cudaSuccess) {
            merge_rescore_kernel<<<(n_q + 7) / 8, 256, 0, st>>>(p.part_s, p.part_i, p.n_sl,
                                                                p.n_q_pad, p.L, L_pool, q, reg,
                                                                n_q, dim, qn, rn, k, out_idx,
                                                                out_score);
            e = cudaGetLastError();
        }
        if (e != cudaSuccess) {
            set_error(std::string("vdb_identify: ") + cudaGetErrorString(e));
            rc = 1;
        }
    }
    cudaFreeAsync(work, st);
    return rc;
}
