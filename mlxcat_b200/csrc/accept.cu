// accept.cu -- fused acceptance + in-place rollback of the speculative step.
//
// Greedy rows restate the acceptance loop of BatchGenerator.swift:906-954:
//   COMPAT (mode 0): all-or-nothing; a sampled tool trigger or a mismatch
//     rejects the batch and the step emits the one token an ordinary decode
//     would (position 0's sample -- the verify forward computes position 0
//     exactly as the one-token decode does); EOS stops early.
//   PREFIX (mode 1): the matching prefix plus the correcting / bonus token.
// Temperature rows (extension, PREFIX mode) run single-draft rejection
// sampling on fixed-point distributions: P[i] = floor(2^24 e^((l_i - max)/T))
// over the top-p nucleus (Sampling.swift:847-858 rule, decided at T = 1 as the
// reference does before dividing by T, :504-523); draft d at position p
// survives iff floor(u_acc * S / 2^32) < P[d]; otherwise the residual
// (P without d) is sampled by inverse CDF in token order with u_samp; a fully
// accepted proposal samples the bonus token.  u_acc/u_samp come from the
// request's Philox stream at its generation index, so a row's tokens depend on
// its own seed and position only.  All sums are integer: bit-exact with the
// CPU restatement given the same logits.
//
// Commit: append emitted tokens to the history, advance n_gen, and set the KV
// length to old + emitted (the verify K/V past that point is dropped by
// length -- the in-place rollback), mark finished rows inactive.
#include "common.cuh"
#include "kernels.h"

namespace mlxcat {

namespace {

__device__ __forceinline__ bool is_eos(const RowState &rs, int r, int tok) {
    const int n = rs.n_eos[r];
    for (int i = 0; i < n && i < MLXCAT_MAX_EOS; ++i)
        if (rs.eos[r * MLXCAT_MAX_EOS + i] == tok) return true;
    return false;
}

__device__ void commit_row(const RowState &rs, int r, const int32_t *em, int n, int cnt,
                           bool rejected, int K1, StepOut out) {
    const int L = rs.hist_len[r];
    int32_t *h = rs.hist + (size_t)r * rs.hist_cap;
    for (int i = 0; i < n; ++i) {
        h[L + i] = em[i];
        out.tokens[r * K1 + i] = em[i];
    }
    rs.hist_len[r] = L + n;
    rs.kv_len[r] += n;
    const int g = rs.n_gen[r] + n;
    rs.n_gen[r] = g;
    out.n[r] = n;
    const bool fin = is_eos(rs, r, em[n - 1]) || g >= rs.max_new[r];
    out.finished[r] = fin;
    if (fin) rs.active[r] = 0;
    if (cnt > 0) {
        atomicAdd(&out.stats[0], (unsigned long long)cnt);
        atomicAdd(&out.stats[1], (unsigned long long)(n - 1));
        atomicAdd(&out.stats[2], 1ull);
        if (rejected) atomicAdd(&out.stats[3], 1ull);
    }
}

__global__ void accept_greedy_kernel(RowState rs, SpecParams sp, const int32_t *vtok,
                                     const int32_t *count, const int32_t *amax, StepOut out) {
    const int r = blockIdx.x * blockDim.x + threadIdx.x;
    if (r >= rs.rows) return;
    const int K1 = sp.k + 1;
    if (!rs.active[r]) {
        out.n[r] = 0;
        out.finished[r] = 0;
        return;
    }
    if (rs.temperature[r] != 0.0f) return;   // sampled rows: accept_sampled
    const int cnt = count[r];
    const int32_t *a = amax + r * K1;
    const int32_t *d = vtok + r * K1 + 1;
    const int trig = rs.trigger[r];
    int32_t em[17];
    int n = 0;
    bool rejected = false;
    if (sp.mode == 0) {
        bool ok = true;
        for (int p = 0; p <= cnt; ++p) {
            const int s = a[p];
            if (s == trig) { ok = false; break; }
            if (p < cnt && s != d[p]) { ok = false; break; }
            em[n++] = s;
            if (is_eos(rs, r, s)) break;
        }
        if (!ok) {
            rejected = cnt > 0;
            em[0] = a[0];
            n = 1;
        }
    } else {
        for (int p = 0; p <= cnt; ++p) {
            const int s = a[p];
            em[n++] = s;
            if (s == trig) { rejected = p < cnt; break; }
            if (p < cnt && s != d[p]) { rejected = true; break; }
            if (is_eos(rs, r, s)) break;
        }
    }
    commit_row(rs, r, em, n, cnt, rejected, K1, out);
}

// ---------------------------------------------------------------------------
// fixed-point distribution of one logits row (block of 1024 threads)
// ---------------------------------------------------------------------------
constexpr int STPB = 1024;
constexpr int NB = 2048;

struct DistSmem {
    unsigned long long mass[NB];
    unsigned int cnt[NB];
    unsigned long long scan[STPB / 32];
    unsigned long long red64[STPB / 32];
    float redf[STPB / 32];
    int sel;
    unsigned long long base;
};

__device__ float block_max_f(float v, DistSmem &sm) {
    v = warp_max(v);
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
    __syncthreads();
    if (lane == 0) sm.redf[w] = v;
    __syncthreads();
    float r = sm.redf[0];
    for (int i = 1; i < STPB / 32; ++i) r = fmaxf(r, sm.redf[i]);
    return r;
}

__device__ unsigned long long block_sum_u64(unsigned long long v, DistSmem &sm) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
    __syncthreads();
    if (lane == 0) sm.red64[w] = v;
    __syncthreads();
    unsigned long long r = 0;
    for (int i = 0; i < STPB / 32; ++i) r += sm.red64[i];
    return r;
}

// exclusive prefix over threads (thread order), returns this thread's prefix
__device__ unsigned long long block_excl_scan_u64(unsigned long long v, DistSmem &sm) {
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
    unsigned long long x = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const unsigned long long y = __shfl_up_sync(0xffffffffu, x, o);
        if (lane >= o) x += y;
    }
    __syncthreads();
    if (lane == 31) sm.scan[w] = x;
    __syncthreads();
    unsigned long long off = 0;
    for (int i = 0; i < w; ++i) off += sm.scan[i];
    return off + x - v;
}

// top-p threshold: lowest key whose strictly-higher mass A satisfies
// (A << 20) < S1 * tp, found MSB-first over 11/11/10-bit buckets.  S1, the
// total fixed-point mass of the row, is the sum of the first pass's histogram
// (integer sums: the same value as a separate pass over the row, without its
// exponentials).
__device__ uint32_t top_p_threshold(const float *l, int V, float m, uint64_t tp, DistSmem &sm) {
    uint32_t prefix = 0;
    unsigned long long base = 0, S1 = 0;
    const int shifts[3] = {21, 10, 0};
    const int widths[3] = {11, 11, 10};
    for (int pass = 0; pass < 3; ++pass) {
        const int sh = shifts[pass], nb = 1 << widths[pass];
        for (int b = threadIdx.x; b < NB; b += STPB) { sm.mass[b] = 0; sm.cnt[b] = 0; }
        if (threadIdx.x == 0) sm.sel = NB;
        __syncthreads();
        for (int i = threadIdx.x; i < V; i += STPB) {
            const uint32_t key = float_key(l[i]);
            const bool in = pass == 0 || (key >> (sh + widths[pass])) == prefix;
            if (in) {
                const int b = (int)((key >> sh) & (uint32_t)(nb - 1));
                const uint32_t P = fix24(det_exp_neg(__fadd_rn(l[i], -m)));
                // Logits cluster in a few buckets, so the lanes of a warp that
                // share a bucket add their masses first (integer sums: the same
                // totals in any order) and one of them updates the histogram.
                const unsigned grp = __match_any_sync(__activemask(), b);
                const unsigned sum = __reduce_add_sync(grp, P);   // < 32 * 2^24: no overflow
                if ((int)(__ffs(grp) - 1) == (threadIdx.x & 31)) {
                    if (sum) atomicAdd(&sm.mass[b], (unsigned long long)sum);
                    atomicAdd(&sm.cnt[b], (unsigned)__popc(grp));
                }
            }
        }
        __syncthreads();
        // thread j owns buckets 2047-2j, 2046-2j (descending)
        const int b_hi = NB - 1 - 2 * threadIdx.x, b_lo = b_hi - 1;
        const unsigned long long mh = sm.mass[b_hi], ml = sm.mass[b_lo];
        if (pass == 0) S1 = block_sum_u64(mh + ml, sm);
        const unsigned long long ex = block_excl_scan_u64(mh + ml, sm);
        const unsigned long long above_hi = base + ex, above_lo = base + ex + mh;
        int cand = NB;
        if (sm.cnt[b_lo] && ((above_lo << 20) < S1 * tp)) cand = b_lo;
        else if (sm.cnt[b_hi] && ((above_hi << 20) < S1 * tp)) cand = b_hi;
        if (cand < NB) atomicMin(&sm.sel, cand);
        __syncthreads();
        const int sel = sm.sel;
        // base for the next level: mass above the selected bucket
        if (threadIdx.x == 0) sm.base = 0;
        __syncthreads();
        if (sel < NB) {
            if (b_hi == sel) sm.base = above_hi;
            if (b_lo == sel) sm.base = above_lo;
        }
        __syncthreads();
        base = sm.base;
        prefix = (prefix << widths[pass]) | (uint32_t)sel;
        __syncthreads();
    }
    return prefix;
}

__device__ __forceinline__ uint32_t tempered_p(float li, float m, float T, uint32_t thr) {
    return float_key(li) >= thr ? fix24(det_exp_neg(__fdiv_rn(__fadd_rn(li, -m), T))) : 0u;
}

__device__ void dist_stats(const float *l, int V, float T, float top_p, int d, DistSmem &sm,
                           float *m_out, uint32_t *thr_out, unsigned long long *S_out,
                           unsigned long long *Pd_out) {
    float mx = -INFINITY;
    for (int i = threadIdx.x; i < V; i += STPB) mx = fmaxf(mx, l[i]);
    const float m = block_max_f(mx, sm);
    uint32_t thr = 0;
    if (top_p > 0.0f && top_p < 1.0f) {
        long long tp = (long long)rintf(__fmul_rn(top_p, 1048576.0f));
        tp = tp < 1 ? 1 : (tp > 1048576 ? 1048576 : tp);
        thr = top_p_threshold(l, V, m, (uint64_t)tp, sm);
    }
    unsigned long long s = 0;
    for (int i = threadIdx.x; i < V; i += STPB) s += tempered_p(l[i], m, T, thr);
    const unsigned long long S = block_sum_u64(s, sm);
    if (threadIdx.x == 0) {
        *m_out = m;
        *thr_out = thr;
        *S_out = S;
        *Pd_out = d >= 0 ? tempered_p(l[d], m, T, thr) : 0ull;
    }
}

// inverse CDF in token order over P (skipping `skip`); t < S' guaranteed
__device__ int block_pick(const float *l, int V, float m, float T, uint32_t thr, int skip,
                          unsigned long long t, DistSmem &sm) {
    const int per = (V + STPB - 1) / STPB;
    const int i0 = threadIdx.x * per, i1 = min(V, i0 + per);
    unsigned long long loc = 0;
    for (int i = i0; i < i1; ++i)
        if (i != skip) loc += tempered_p(l[i], m, T, thr);
    const unsigned long long pre = block_excl_scan_u64(loc, sm);
    if (threadIdx.x == 0) sm.sel = -1;
    __syncthreads();
    if (loc > 0 && pre <= t && t < pre + loc) {
        unsigned long long c = pre;
        for (int i = i0; i < i1; ++i) {
            if (i == skip) continue;
            c += tempered_p(l[i], m, T, thr);
            if (c > t) { sm.sel = i; break; }
        }
    }
    __syncthreads();
    return sm.sel;
}

__global__ void __launch_bounds__(STPB)
dist_stats_kernel(RowState rs, SpecParams sp, const int32_t *vtok, const int32_t *count,
                  const float *logits, int V, SampleScratch sc) {
    __shared__ DistSmem sm;
    const int r = blockIdx.x, p = blockIdx.y, K1 = sp.k + 1;
    if (!rs.active[r] || rs.temperature[r] == 0.0f || p > count[r]) return;
    const int idx = r * K1 + p;
    const int d = p < count[r] ? vtok[r * K1 + 1 + p] : -1;
    dist_stats(logits + (size_t)idx * V, V, rs.temperature[r], rs.top_p[r], d, sm, &sc.m[idx],
               &sc.thr[idx], &sc.S[idx], &sc.Pd[idx]);
}

__global__ void __launch_bounds__(STPB)
accept_sampled_kernel(RowState rs, SpecParams sp, const int32_t *vtok, const int32_t *count,
                      const float *logits, int V, SampleScratch sc, StepOut out) {
    __shared__ DistSmem sm;
    __shared__ int32_t em[17];
    __shared__ int n_sh, ppick, skip_sh, rej_sh;
    __shared__ unsigned long long t_sh;
    const int r = blockIdx.x, K1 = sp.k + 1;
    if (!rs.active[r] || rs.temperature[r] == 0.0f) return;
    const int cnt = count[r];
    if (threadIdx.x == 0) {
        const uint64_t seed = rs.seed[r];
        const uint64_t g0 = (uint64_t)rs.n_gen[r];
        const int trig = rs.trigger[r];
        int n = 0, pick_at = -1, skip = -1;
        bool rej = false;
        for (int p = 0; p <= cnt; ++p) {
            const int idx = r * K1 + p;
            if (p < cnt) {
                const int dd = vtok[r * K1 + 1 + p];
                const uint32_t ua = request_uniform(seed, g0 + p, 0);
                if (scale_u32(ua, sc.S[idx]) < sc.Pd[idx]) {
                    em[n++] = dd;
                    if (dd == trig) { rej = true; break; }
                    if (is_eos(rs, r, dd)) break;
                    continue;
                }
                pick_at = p; skip = dd; rej = true;
                break;
            }
            pick_at = p;   // bonus
        }
        n_sh = n;
        ppick = pick_at;
        skip_sh = skip;
        rej_sh = rej;
        if (pick_at >= 0) {
            const int idx = r * K1 + pick_at;
            const uint32_t us = request_uniform(seed, g0 + pick_at, 1);
            const unsigned long long S = sc.S[idx] - (skip >= 0 ? sc.Pd[idx] : 0ull);
            t_sh = scale_u32(us, S);
        }
    }
    __syncthreads();
    const int pick_at = ppick;
    if (pick_at >= 0) {
        const int idx = r * K1 + pick_at;
        const int tok = block_pick(logits + (size_t)idx * V, V, sc.m[idx], rs.temperature[r],
                                   sc.thr[idx], skip_sh, t_sh, sm);
        if (threadIdx.x == 0) em[n_sh++] = tok;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        int n = n_sh;
        // a picked trigger / EOS ends the step like any other sample
        commit_row(rs, r, em, n, cnt, rej_sh != 0, K1, out);
    }
}

__global__ void __launch_bounds__(STPB)
sample_first_kernel(RowState rs, int r, const float *logits, int V, const int32_t *amax,
                    SampleScratch sc, int32_t *out_token) {
    __shared__ DistSmem sm;
    __shared__ unsigned long long t_sh;
    int tok;
    if (rs.temperature[r] == 0.0f) {
        tok = amax[0];
    } else {
        dist_stats(logits, V, rs.temperature[r], rs.top_p[r], -1, sm, &sc.m[0], &sc.thr[0],
                   &sc.S[0], &sc.Pd[0]);
        __syncthreads();
        if (threadIdx.x == 0) t_sh = scale_u32(request_uniform(rs.seed[r], 0, 1), sc.S[0]);
        __syncthreads();
        tok = block_pick(logits, V, sc.m[0], rs.temperature[r], sc.thr[0], -1, t_sh, sm);
    }
    if (threadIdx.x == 0) {
        *out_token = tok;
        const int L = rs.hist_len[r];
        rs.hist[(size_t)r * rs.hist_cap + L] = tok;
        rs.hist_len[r] = L + 1;
        rs.n_gen[r] = 1;
        const bool fin = is_eos(rs, r, tok) || rs.max_new[r] <= 1;
        rs.active[r] = fin ? 0 : 1;
    }
}

}  // namespace

// Allowed-token masks of grammar-constrained rows (the device side of
// applyAllowedTokenMask, Sampling.swift:557-569): per verify token i with
// on[i] set, logits outside the allowed set become -inf; ids >= V are not
// tokens, and a set with no valid id leaves the row unchanged.
__global__ void token_mask_kernel(float *__restrict__ logits, int V, int W, const uint32_t *__restrict__ bits,
                                  const uint8_t *__restrict__ on) {
    const int i = blockIdx.x;
    if (!on[i]) return;
    const uint32_t *b = bits + (size_t)i * W;
    const uint32_t tail = (V & 31) ? (1u << (V & 31)) - 1u : 0xffffffffu;
    int any = 0;
    for (int w = threadIdx.x; w < W; w += blockDim.x) any |= (b[w] & (w == W - 1 ? tail : 0xffffffffu)) != 0u;
    if (!__syncthreads_or(any)) return;
    float *l = logits + (size_t)i * V;
    for (int v = threadIdx.x; v < V; v += blockDim.x)
        if (!((b[v >> 5] >> (v & 31)) & 1u)) l[v] = -INFINITY;
}

cudaError_t apply_token_masks(float *logits, int M, int V, const uint32_t *bits, const uint8_t *on,
                              cudaStream_t st) {
    if (M <= 0 || V <= 0 || !bits || !on) return cudaErrorInvalidValue;
    token_mask_kernel<<<M, 256, 0, st>>>(logits, V, (V + 31) / 32, bits, on);
    return cudaGetLastError();
}

cudaError_t accept_greedy(const RowState &rs, const SpecParams &sp, const int32_t *vtok,
                          const int32_t *count, const int32_t *amax, StepOut out,
                          cudaStream_t st) {
    if (sp.k > 16) return cudaErrorInvalidValue;
    accept_greedy_kernel<<<(rs.rows + 127) / 128, 128, 0, st>>>(rs, sp, vtok, count, amax, out);
    return cudaGetLastError();
}

cudaError_t accept_sampled(const RowState &rs, const SpecParams &sp, const int32_t *vtok,
                           const int32_t *count, const float *logits, int V, SampleScratch sc,
                           StepOut out, cudaStream_t st) {
    if (sp.k > 16) return cudaErrorInvalidValue;
    dim3 g1(rs.rows, sp.k + 1);
    dist_stats_kernel<<<g1, STPB, 0, st>>>(rs, sp, vtok, count, logits, V, sc);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return e;
    accept_sampled_kernel<<<rs.rows, STPB, 0, st>>>(rs, sp, vtok, count, logits, V, sc, out);
    return cudaGetLastError();
}

cudaError_t sample_first(const RowState &rs, int row, const float *logits, int V,
                         const int32_t *amax, SampleScratch sc, int32_t *out_token,
                         cudaStream_t st) {
    sample_first_kernel<<<1, STPB, 0, st>>>(rs, row, logits, V, amax, sc, out_token);
    return cudaGetLastError();
}

}  // namespace mlxcat
