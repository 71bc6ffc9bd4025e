// Identify: top-k cosine search of query embeddings against a registry. The
// reference advertises identify (README.md:15,44,59) but has no implementation,
// so the semantics here are the ones the oracle (oracle/vd_oracle.c,
// vdo_identify) fixes: cosine = dot / (|q| |r|), top-k by descending score, and
// among equal scores the lower registry index first.
//
// Three kernels per registry chunk: row norms (once), a tiled f32 GEMM that writes
// the chunk's cosine scores [n_q][chunk] to scratch (128 x 128 tiles, 8 x 8 outputs
// per thread, each dot product accumulated with fmaf over the dimensions in order),
// and a warp-per-query top-k that merges the chunk into the running top-k. Scores
// are bitwise those of a sequential fmaf loop, and the top-k is the first k of the
// order (score descending, registry index ascending).
#include <algorithm>
#include <cfloat>
#include <climits>

#include "vdb_internal.h"
#include "vdb_ops.h"

namespace vdb {
namespace {

constexpr int kMaxK = 64;
constexpr int kTile = 128, kBK = 16;

// |v| per row: sqrt of an in-order fmaf sum of squares.
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
// registry rows [r0, r0 + nr).
__global__ void __launch_bounds__(256)
score_kernel(const float* __restrict__ q, int n_q, const float* __restrict__ reg, int r0, int nr,
             int dim, const float* __restrict__ qn, const float* __restrict__ rn,
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
        // 128 rows x 16 dims of each operand: 2048 floats, 8 per thread, transposed
        for (int e = threadIdx.x; e < kTile * kBK; e += 256) {
            const int row = e / kBK, kk = e - row * kBK;
            const int qq = qb + row, rr = rb + row, d = k0 + kk;
            As[kk][row] = (qq < n_q && d < dim) ? q[(long long)qq * dim + d] : 0.0f;
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
        if (qq >= n_q) continue;
        const float nq = qn[qq];
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const int rr = rb + (j < 4 ? tx * 4 + j : 64 + tx * 4 + j - 4);
            if (rr >= nr) continue;
            const float den = nq * rn[r0 + rr];
            scores[(long long)qq * nr + rr] = den > 0.0f ? acc[i][j] / den : 0.0f;
        }
    }
}

__device__ __forceinline__ bool better(float s, int i, float t, int j) {
    return s > t || (s == t && i < j);
}

// Warp per query: merge scores[q][0..nr) (registry rows r0..) into the running
// top-k in out_idx / out_score (valid entries first; the first chunk starts empty).
__global__ void __launch_bounds__(256)
topk_kernel(const float* __restrict__ scores, int n_q, int r0, int nr, int k, int first,
            int* __restrict__ out_idx, float* __restrict__ out_score) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int qq = blockIdx.x * 8 + warp;
    if (qq >= n_q) return;
    // this lane's candidates in registry order, kept sorted (score desc, index asc)
    float ls[kMaxK];
    int li[kMaxK];
    for (int j = 0; j < k; ++j) {
        ls[j] = -INFINITY;
        li[j] = INT_MAX;
    }
    int n = 0;
    auto push = [&](float s, int i) {
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
    const float* row = scores + (long long)qq * nr;
    for (int r = lane; r < nr; r += 32) push(row[r], r0 + r);
    if (!first && lane == 0) {
        for (int j = 0; j < k; ++j) {
            const int i = out_idx[(long long)qq * k + j];
            if (i >= 0) push(out_score[(long long)qq * k + j], i);
        }
    }
    // k rounds of a warp-wide arg-best over the lanes' heads
    int head = 0;
    for (int j = 0; j < k; ++j) {
        float s = head < n ? ls[head] : -INFINITY;
        int i = head < n ? li[head] : INT_MAX;
        float bs = s;
        int bi = i;
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
    // registry chunk: at most ~1 GB of f32 scores per pass
    long long chunk = (1LL << 28) / n_q;
    chunk = std::max<long long>(kTile, std::min<long long>(chunk, 32768)) / kTile * kTile;
    chunk = std::min<long long>(chunk, n_reg);
    float* work = nullptr;
    const size_t bytes = sizeof(float) * ((size_t)n_q + n_reg + (size_t)n_q * chunk);
    VDB_CHECK_CUDA(cudaMallocAsync(&work, bytes, st));
    float* qn = work;
    float* rn = qn + n_q;
    float* sc = rn + n_reg;
    row_norm_kernel<<<(n_q + 255) / 256, 256, 0, st>>>(q, n_q, dim, qn);
    row_norm_kernel<<<(n_reg + 255) / 256, 256, 0, st>>>(reg, n_reg, dim, rn);
    int rc = 0;
    for (int r0 = 0; r0 < n_reg && rc == 0; r0 += (int)chunk) {
        const int nr = (int)std::min<long long>(chunk, n_reg - r0);
        const dim3 grid((nr + kTile - 1) / kTile, (n_q + kTile - 1) / kTile);
        score_kernel<<<grid, 256, 0, st>>>(q, n_q, reg, r0, nr, dim, qn, rn, sc);
        topk_kernel<<<(n_q + 7) / 8, 256, 0, st>>>(sc, n_q, r0, nr, k, r0 == 0 ? 1 : 0, out_idx,
                                                   out_score);
        if (cudaGetLastError() != cudaSuccess) rc = 1;
    }
    cudaFreeAsync(work, st);
    if (rc) {
        set_error("vdb_identify: kernel launch failed");
        return 1;
    }
    return 0;
}
