// Identify: top-k cosine search of query embeddings against a registry. The
// reference advertises identify (README.md:15,44,59) but has no implementation,
// so the semantics here are the ones the oracle (oracle/vd_oracle.c,
// vdo_identify) fixes: cosine = dot / (|q| |r|), top-k by descending score, and
// among equal scores the lower registry index first.
//
// One CTA per tile of 32 queries streams the registry through shared memory in
// tiles of 32 rows; the 32x32 score tile is computed on CUDA cores in f32 and
// merged, in registry order, into a per-query sorted top-k list held in shared
// memory. The full n_q x n_reg score matrix is never materialised.
#include <cfloat>

#include "vdb_internal.h"
#include "vdb_ops.h"

namespace vdb {
namespace {

constexpr int kQT = 32;   // queries per CTA
constexpr int kRT = 32;   // registry rows per tile
constexpr int kMaxK = 64;

__global__ void __launch_bounds__(256)
identify_kernel(const float* __restrict__ q, int n_q, const float* __restrict__ reg, int n_reg,
                int dim, int k, int* __restrict__ out_idx, float* __restrict__ out_score) {
    extern __shared__ float sm[];
    const int ld = dim + 1;
    float* sq = sm;                        // [kQT][ld]
    float* sr = sq + kQT * ld;             // [kRT][ld]
    float* ssc = sr + kRT * ld;            // [kQT][kRT]
    float* qn = ssc + kQT * kRT;           // [kQT]
    float* rn = qn + kQT;                  // [kRT]
    float* tks = rn + kRT;                 // [kQT][k] scores
    int* tki = reinterpret_cast<int*>(tks + kQT * k);  // [kQT][k] indices
    int* tkn = tki + kQT * k;              // [kQT] fill counts

    const int q0 = blockIdx.x * kQT;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    for (int i = tid; i < kQT * dim; i += blockDim.x) {
        const int r = i / dim, d = i - r * dim;
        sq[r * ld + d] = (q0 + r < n_q) ? q[(long long)(q0 + r) * dim + d] : 0.0f;
    }
    if (tid < kQT) tkn[tid] = 0;
    __syncthreads();
    if (tid < kQT) {
        float s = 0.0f;
        for (int d = 0; d < dim; ++d) s = fmaf(sq[tid * ld + d], sq[tid * ld + d], s);
        qn[tid] = sqrtf(s);
    }
    const int my_q = tid >> 3, rg = tid & 7;
    for (int r0 = 0; r0 < n_reg; r0 += kRT) {
        __syncthreads();
        for (int i = tid; i < kRT * dim; i += blockDim.x) {
            const int r = i / dim, d = i - r * dim;
            sr[r * ld + d] = (r0 + r < n_reg) ? reg[(long long)(r0 + r) * dim + d] : 0.0f;
        }
        __syncthreads();
        if (tid < kRT) {
            float s = 0.0f;
            for (int d = 0; d < dim; ++d) s = fmaf(sr[tid * ld + d], sr[tid * ld + d], s);
            rn[tid] = sqrtf(s);
        }
        float acc[kRT / 8] = {0.0f, 0.0f, 0.0f, 0.0f};
        for (int d = 0; d < dim; ++d) {
            const float a = sq[my_q * ld + d];
#pragma unroll
            for (int j = 0; j < kRT / 8; ++j) acc[j] = fmaf(a, sr[(rg + 8 * j) * ld + d], acc[j]);
        }
        __syncthreads();
#pragma unroll
        for (int j = 0; j < kRT / 8; ++j) {
            const int r = rg + 8 * j;
            const float den = qn[my_q] * rn[r];
            ssc[my_q * kRT + r] = (r0 + r < n_reg) ? (den > 0.0f ? acc[j] / den : 0.0f) : -FLT_MAX;
        }
        __syncthreads();
        // merge this tile into each query's sorted top-k, in registry order
        for (int qq = warp; qq < kQT; qq += blockDim.x >> 5) {
            if (lane == 0 && q0 + qq < n_q) {
                float* ls = tks + qq * k;
                int* li = tki + qq * k;
                int nb = tkn[qq];
                for (int r = 0; r < kRT && r0 + r < n_reg; ++r) {
                    const float s = ssc[qq * kRT + r];
                    if (nb < k || s > ls[nb - 1]) {
                        int pos = nb < k ? nb : k - 1;
                        while (pos > 0 && ls[pos - 1] < s) {
                            ls[pos] = ls[pos - 1];
                            li[pos] = li[pos - 1];
                            --pos;
                        }
                        ls[pos] = s;
                        li[pos] = r0 + r;
                        if (nb < k) ++nb;
                    }
                }
                tkn[qq] = nb;
            }
        }
    }
    __syncthreads();
    for (int i = tid; i < kQT * k; i += blockDim.x) {
        const int qq = i / k, j = i - qq * k;
        if (q0 + qq >= n_q) continue;
        const bool have = j < tkn[qq];
        out_idx[(long long)(q0 + qq) * k + j] = have ? tki[qq * k + j] : -1;
        out_score[(long long)(q0 + qq) * k + j] = have ? tks[qq * k + j] : -INFINITY;
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
    const int ld = dim + 1;
    const size_t smem = sizeof(float) * ((size_t)(kQT + kRT) * ld + kQT * kRT + kQT + kRT +
                                         (size_t)kQT * k) +
                        sizeof(int) * ((size_t)kQT * k + kQT);
    VDB_CHECK_CUDA(cudaFuncSetAttribute(identify_kernel,
                                        cudaFuncAttributeMaxDynamicSharedMemorySize,
                                        (int)smem));
    identify_kernel<<<(n_q + kQT - 1) / kQT, 256, smem, static_cast<cudaStream_t>(stream)>>>(
        q, n_q, reg, n_reg, dim, k, out_idx, out_score);
    VDB_CHECK_CUDA(cudaGetLastError());
    return 0;
}
