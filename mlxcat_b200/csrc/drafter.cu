// drafter.cu -- batched prompt-lookup drafter, one CTA per row.
//
// Restates proposeSuffixTokens (BatchGenerator.swift:982-1010) and the gate
// canSpeculate / proposal limit (:877-892, :957-975) for every row at once:
//
//   for L = min(n, |ctx|-1) .. 1: the most recent start c with
//   c + L <= |ctx| - L and ctx[c, c+L) == ctx[|ctx|-L, |ctx|); proposal =
//   ctx[c+L, min(|ctx|, c+L+limit)).
//
// The nested scan becomes one pass: for every end position e the backward
// match length lcs(e) against the row's tail (capped at n) gives the longest
// admissible suffix at that end, smax(e) = min(lcs(e), |ctx|-1-e); the answer
// is the lexicographic maximum of (smax(e), e).  This is the same choice the
// reference's loops make (largest L first, then the latest start), in
// O(|ctx| * n) compares with no per-candidate allocation.
#include "common.cuh"
#include "kernels.h"

namespace mlxcat {

namespace {

constexpr int DTPB = 256;
constexpr int MAX_N = 64;   // tail tokens staged in shared memory

__global__ void draft_kernel(RowState rs, SpecParams sp, int32_t *__restrict__ vtok,
                             int32_t *__restrict__ count, int32_t *__restrict__ trow,
                             int32_t *__restrict__ tpos) {
    __shared__ int32_t tail[MAX_N];
    __shared__ unsigned long long red[DTPB / 32];
    __shared__ int n_active_sh;
    const int r = blockIdx.x;
    const int K1 = sp.k + 1;
    const int32_t *hist = rs.hist + (size_t)r * rs.hist_cap;
    const int L = rs.hist_len[r];
    const bool active = rs.active[r] != 0;

    if (threadIdx.x == 0) {
        int na = 0;
        for (int i = 0; i < rs.rows; ++i) na += rs.active[i] != 0;
        n_active_sh = na;
    }
    __syncthreads();

    const int remaining = rs.max_new[r] - rs.n_gen[r];
    bool gate = active && sp.enabled && sp.k > 0 && L >= sp.min_ctx && remaining > 1;
    if (sp.mode == 0)  // compat: width 1, greedy, no per-request seed (:959-972)
        gate = gate && n_active_sh == 1 && rs.temperature[r] == 0.0f && !rs.has_seed[r];
    const int limit = min(sp.k, remaining - 1);
    const int S = min(sp.n, L - 1);   // any n: tail positions past MAX_N come from global memory
    gate = gate && limit > 0 && S > 0;

    unsigned long long best = 0;
    if (gate) {
        for (int i = threadIdx.x; i < min(S, MAX_N); i += blockDim.x) tail[i] = hist[L - 1 - i];
        __syncthreads();
        const int32_t last = tail[0];
        for (int e = threadIdx.x; e <= L - 2; e += blockDim.x) {
            if (hist[e] != last) continue;
            int l = 1;
            while (l < S && e - l >= 0 && hist[e - l] == (l < MAX_N ? tail[l] : hist[L - 1 - l])) ++l;
            const int smax = min(l, L - 1 - e);
            if (smax >= 1) {
                const unsigned long long key = ((unsigned long long)smax << 32) | (unsigned)e;
                best = key > best ? key : best;
            }
        }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const unsigned long long v = __shfl_xor_sync(0xffffffffu, best, o);
        best = v > best ? v : best;
    }
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = best;
    __syncthreads();
    if (threadIdx.x == 0) {
        unsigned long long b = 0;
        for (int i = 0; i < DTPB / 32; ++i) b = red[i] > b ? red[i] : b;
        int cnt = 0;
        const int32_t cur = L > 0 ? hist[L - 1] : 0;
        int32_t *vt = vtok + (size_t)r * K1;
        vt[0] = cur;
        if (b != 0) {
            const int e = (int)(b & 0xffffffffu);
            const int start = e + 1;
            cnt = min(limit, L - start);
            for (int i = 0; i < cnt; ++i) vt[1 + i] = hist[start + i];
        }
        for (int i = cnt; i < sp.k; ++i) vt[1 + i] = cur;
        count[r] = cnt;
        const int kv = rs.kv_len[r];
        for (int j = 0; j < K1; ++j) {
            trow[r * K1 + j] = r;
            tpos[r * K1 + j] = kv + j;
        }
    }
}

}  // namespace

cudaError_t draft(const RowState &rs, const SpecParams &sp, int32_t *vtok, int32_t *count,
                  int32_t *trow, int32_t *tpos, cudaStream_t st) {
    if (sp.k < 0 || sp.n < 1) return cudaErrorInvalidValue;
    draft_kernel<<<rs.rows, DTPB, 0, st>>>(rs, sp, vtok, count, trow, tpos);
    return cudaGetLastError();
}

}  // namespace mlxcat
