// q4_tc.cu -- MLX affine 4-bit (group 64) linear on the 5th-generation tensor
// cores, with the split-K reduction and the consumer epilogue fused in.
//
//   y[m][n] = sum_k x[m][k] * (scale[n][k/64] * q[n][k] + bias[n][k/64])
//
// Replaces mlx-swift's quantizedMatmul (QuantizedLinear in mlx-swift-lm) on
// the verify forward (BatchGenerator.swift:900-904).  Weights stay in the MLX
// layout: packed uint32 [N][K/8] with the lowest nibble first, fp16 scales and
// biases [N][K/64].
//
// Swap-AB: the 128 weight rows of a CTA are the MMA's M dimension, the tokens
// of the verify batch (16..128) its N dimension.  One 256-wide k chunk per
// pipeline stage:
//
//   warp 16 (one lane)  TMA producer: weight tile [128 rows x 128 B] (128B
//                       swizzle) and the token tile [4 x NT x 64] (one 3-D box,
//                       128B swizzle) into a ring of shared-memory stages.
//   warps 0-15          dequantisers: warp w owns rows 32*(w%4).. and the
//                       64-wide quantisation group w/4 of the chunk; 32 bytes
//                       per thread from the staged tile, nibbles unpacked with
//                       the 0x6400 fp16 magic and dequantised in registers
//                       (hfma2 / hadd2), stored to tensor memory (tcgen05.st)
//                       as the MMA's A operand.
//   (persistent, one CTA per SM, stream-K: see unit_begin below)
//   warps 17-18 (lane0) MMA issuers: each issues half of the chunk's sixteen
//                       tcgen05.mma (M=128, N=NT, K=16, A from TMEM, B from
//                       shared memory) into its own fp32 accumulator in TMEM;
//                       one thread issues at most one MMA per ~65 cycles, two
//                       keep the tensor pipe fed at small N.
//
// Inside each 8-wide k block the unpack order is (0,4,1,5,2,6,3,7); the token
// operand is stored in that order and blocked by 64 features ([K/64][rows][64],
// see common.cuh: xblk) by its producers.
//
// A row block whose k range is shared by several CTAs: each writes its fp32
// partial to its slot; the last to finish (atomic ticket) sums the slots in
// slot order -- deterministic -- and runs the epilogue:
//   STORE   logits  out[m][n] = y
//   RESID   residual stream h[m][n] += y
//   SWIGLU  gate/up rows interleaved per 64 -> x_next[m][i] = silu(g) * u
//   QKV     per-head q/k RMSNorm (Qwen3), rotate-half RoPE, q to the query
//           buffer, k/v appended to the KV cache at each token's position
//
// Every mbarrier wait is bounded (tc.cuh); a timeout sets *err and the CTA
// drains its in-flight copies and MMAs (bounded) before freeing TMEM.
#include <cuda.h>
#include <cudaTypedefs.h>

#include "common.cuh"
#include "kernels.h"
#include "tc.cuh"

namespace mlxcat {

int q4_tc_pmax(int U, int G, int nc);

namespace {

constexpr int ROWS = 128;              // weight rows per CTA (MMA M)
constexpr int CHUNK = 256;             // k per pipeline stage
constexpr int DQ_WARPS = 16;           // dequant / epilogue warps
constexpr int DQ_THREADS = DQ_WARPS * 32;
constexpr int TMA_WARP = DQ_WARPS;
constexpr int MMA_WARP0 = DQ_WARPS + 1;
constexpr int ISSUERS = 2;
constexpr int THREADS = (DQ_WARPS + 1 + ISSUERS) * 32;
constexpr int A_COLS = CHUNK / 2;      // TMEM columns of one A stage (fp16 pairs)
constexpr int PF = 4;                  // chunks of scale/bias prefetch
constexpr int MAX_STAGES = 8;

enum ErrCode { ERR_FULL = 1, ERR_AFULL = 2, ERR_MMA = 3, ERR_DONE = 4 };

template <int NT>
struct Cfg {
    static constexpr int A_STAGES = NT <= 64 ? 3 : 2;
    static constexpr int DCOLS = NT <= 64 ? 64 : 128;        // columns per accumulator
    static constexpr int D_COL = A_STAGES * A_COLS;
    static constexpr int XBYTES = 4 * NT * 128;              // four 64-k boxes
    static constexpr int WBYTES = ROWS * 128;
    static constexpr int STAGE = XBYTES + WBYTES;
    static_assert(D_COL + ISSUERS * DCOLS <= 512, "TMEM budget");
};

__device__ __forceinline__ void named_bar_sync(int id, int n) {
    asm volatile("bar.sync %0, %1;\n" ::"r"(id), "r"(n) : "memory");
}

// named barrier over the dequant warps that also ORs a predicate across them
__device__ __forceinline__ bool named_bar_or(int id, int n, bool pred) {
    uint32_t r;
    asm volatile(
        "{\n\t.reg .pred p, q;\n\t"
        "setp.ne.u32 q, %3, 0;\n\t"
        "bar.red.or.pred p, %1, %2, q;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}\n"
        : "=r"(r)
        : "r"(id), "r"(n), "r"((uint32_t)pred)
        : "memory");
    return r != 0;
}

__device__ __forceinline__ uint32_t lop3_and_or(uint32_t a, uint32_t b, uint32_t c) {
    uint32_t d;
    asm("lop3.b32 %0, %1, %2, %3, 0xea;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}

// 8 nibbles of one word -> four fp16 pairs (n0,n4) (n1,n5) (n2,n6) (n3,n7),
// each = s*q + b.  lo pairs: (1024 + q) * s - 1024 s is exact before the one
// rounding of the fma; hi pairs come out as 1024 + 16 q and use s/16, -64 s.
__device__ __forceinline__ void dequant_word(uint32_t w, __half2 s1, __half2 m1, __half2 s16,
                                             __half2 m64, __half2 b2, uint32_t *out) {
    const uint32_t w8 = w >> 8;
    uint32_t v[4];
    v[0] = lop3_and_or(w, 0x000f000fu, 0x64006400u);
    v[1] = lop3_and_or(w, 0x00f000f0u, 0x64006400u);
    v[2] = lop3_and_or(w8, 0x000f000fu, 0x64006400u);
    v[3] = lop3_and_or(w8, 0x00f000f0u, 0x64006400u);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        const __half2 x = *reinterpret_cast<const __half2 *>(&v[j]);
        const __half2 qs = (j & 1) ? __hfma2(x, s16, m64) : __hfma2(x, s1, m1);
        const __half2 r = __hadd2(qs, b2);
        out[j] = *reinterpret_cast<const uint32_t *>(&r);
    }
}

struct Smem {
    uint64_t full[MAX_STAGES], mma_done[MAX_STAGES], a_full[3], d_free;
    uint32_t tmem_base;
    int abort_flag;
    int last_flag;
    float wsum[4][4][16];   // [token group][row quarter][token]
    float xch[4][ROWS * 16];   // epilogue exchange: [token group][row][token]
};

// Stream-K schedule: the flattened (row block, k chunk) units are split into
// gridDim.x contiguous, equal ranges, one per CTA (one CTA per SM).  A row
// block whose chunks span several CTAs is finished by the last of them.
__device__ __forceinline__ int unit_begin(int c, int U, int G) { return (int)(((long long)c * U) / G); }
__device__ __forceinline__ int unit_owner(int u, int U, int G) {
    int c = (int)(((long long)u * G) / U);
    while (c + 1 < G && unit_begin(c + 1, U, G) <= u) ++c;
    while (c > 0 && unit_begin(c, U, G) > u) --c;
    return c;
}

template <int NT>
__global__ void __launch_bounds__(THREADS, 1)
q4_tc_kernel(const __grid_constant__ CUtensorMap wmap, const __grid_constant__ CUtensorMap xmap,
             const __half *__restrict__ scales, const __half *__restrict__ biases, int N, int K,
             int M, int tok_base, int nblk, int nc, int U, int pmax, int stages, Q4Epilogue ep) {
    using C = Cfg<NT>;
    constexpr int PIECES = NT <= 64 ? 1 : 2;      // 16-token pieces per token group
    extern __shared__ __align__(1024) unsigned char smem_raw[];
    unsigned char *ring = reinterpret_cast<unsigned char *>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
    Smem &cs = *reinterpret_cast<Smem *>(ring + (size_t)stages * C::STAGE);

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int G = gridDim.x, cta = blockIdx.x;
    const int u0 = unit_begin(cta, U, G), u1 = unit_begin(cta + 1, U, G);
    const int n = u1 - u0;                        // chunks of this CTA
    const uint32_t ring_a = tc::smem_u32(ring);

    if (warp == TMA_WARP && lane == 0) {
        for (int s = 0; s < stages; ++s) {
            tc::mbar_init(tc::smem_u32(&cs.full[s]), 1);
            tc::mbar_init(tc::smem_u32(&cs.mma_done[s]), ISSUERS);
        }
        for (int a = 0; a < C::A_STAGES; ++a) tc::mbar_init(tc::smem_u32(&cs.a_full[a]), DQ_WARPS);
        tc::mbar_init(tc::smem_u32(&cs.d_free), DQ_WARPS);
        cs.abort_flag = 0;
        tc::fence_barrier_init();
        tc::prefetch_tmap(&wmap);
        tc::prefetch_tmap(&xmap);
    }
    if (warp == 0) tc::tmem_alloc(tc::smem_u32(&cs.tmem_base), 512);
    tc::fence_before_sync();
    __syncthreads();
    tc::fence_after_sync();
    const uint32_t tmem = cs.tmem_base;
    volatile int *abort_flag = &cs.abort_flag;

    if (warp == TMA_WARP) {
        if (lane == 0) {
            // ---------------- TMA producer ----------------
            int issued = 0;
            for (int i = 0; i < n && !*abort_flag; ++i) {
                const int s = i % stages;
                if (i >= stages) {
                    const int pc = i - stages;   // previous user of this stage
                    if (!tc::mbar_wait(tc::smem_u32(&cs.mma_done[s]), (pc / stages) & 1, ep.err, ERR_MMA)) {
                        *abort_flag = 1;
                        break;
                    }
                }
                const int u = u0 + i, b = u / nc, c = u - b * nc;
                const int tile = b / nblk, blk = b - tile * nblk;
                const uint32_t st = ring_a + (uint32_t)(s * C::STAGE);
                const uint32_t bar = tc::smem_u32(&cs.full[s]);
                tc::mbar_arrive_expect_tx(bar, C::STAGE);
                tc::tma_load_3d(st, &xmap, 0, tok_base + tile * NT, c * (CHUNK / 64), bar);
                tc::tma_load_2d(st + C::XBYTES, &wmap, c * (CHUNK / 2), blk * ROWS, bar);
                issued = i + 1;
            }
            if (*abort_flag) {
                // let every issued copy land before the CTA can exit
                for (int i = max(0, issued - stages); i < issued; ++i)
                    tc::mbar_wait(tc::smem_u32(&cs.full[i % stages]), (i / stages) & 1, nullptr, 0);
            }
        }
    } else if (warp >= MMA_WARP0) {
        if (lane == 0) {
            // ---------------- MMA issuer j: k steps [8j, 8j+8) of every chunk ----------------
            const int j = warp - MMA_WARP0;
            const uint32_t idesc = tc::idesc_f16_f32(ROWS, NT);
            const uint32_t dcol = tmem + C::D_COL + j * C::DCOLS;
            int done = 0, seg = 0;
            for (int i = 0; i < n && !*abort_flag; ++i) {
                const int u = u0 + i, c = u % nc;
                const bool first = i == 0 || c == 0;             // first chunk of a segment
                if (first && seg > 0) {
                    // the epilogue of the previous segment has read the accumulator
                    if (!tc::mbar_wait(tc::smem_u32(&cs.d_free), (seg - 1) & 1, ep.err, ERR_DONE)) {
                        *abort_flag = 1;
                        break;
                    }
                }
                const int s = i % stages, as = i % C::A_STAGES;
                if (!tc::mbar_wait(tc::smem_u32(&cs.full[s]), (i / stages) & 1, ep.err, ERR_FULL) ||
                    !tc::mbar_wait(tc::smem_u32(&cs.a_full[as]), (i / C::A_STAGES) & 1, ep.err, ERR_AFULL)) {
                    *abort_flag = 1;
                    break;
                }
                tc::fence_after_sync();
                const uint32_t xs = ring_a + (uint32_t)(s * C::STAGE);
#pragma unroll
                for (int kk = 8 * j; kk < 8 * j + 8; ++kk) {
                    const uint32_t baddr = xs + (uint32_t)((kk >> 2) * NT * 128 + (kk & 3) * 32);
                    tc::mma_ts_f16(dcol, tmem + as * A_COLS + kk * 8, tc::sdesc_k_sw128(baddr), idesc,
                                   (!first || kk > 8 * j) ? 1u : 0u);
                }
                tc::mma_commit(tc::smem_u32(&cs.mma_done[s]));
                done = i + 1;
                if (c == nc - 1 || i == n - 1) ++seg;
            }
            if (*abort_flag && done > 0) {
                const int pc = done - 1;   // committed MMAs must finish before TMEM is freed
                tc::mbar_wait(tc::smem_u32(&cs.mma_done[pc % stages]), (pc / stages) & 1, nullptr, 0);
            }
        }
    } else {
        // ------- dequant warps: rows 32*quarter.., quantisation group g of each chunk -------
        const int quarter = warp & 3, g = warp >> 2;
        const int r = quarter * 32 + lane;       // row within the block, 0..127
        const uint32_t lane_base = (uint32_t)(quarter * 32) << 16;
        const int KG = K / MLXCAT_GS;
        constexpr int GPC = CHUNK / MLXCAT_GS;   // groups per chunk
        // scale / bias of unit u for this thread's row and group; groups past K
        // (a half last chunk) read zero weights from TMA and use s = b = 0
        auto sb_of = [&](int u, __half &sv, __half &bv) {
            const int b = u / nc, c = u - b * nc, blk = b % nblk;
            const int grp = GPC * c + g;
            if (grp < KG) {
                const size_t o = (size_t)(blk * ROWS + r) * KG + grp;
                sv = scales[o];
                bv = biases[o];
            } else {
                sv = bv = __float2half(0.f);
            }
        };
        __half sc_pf[PF], bi_pf[PF];
#pragma unroll
        for (int p = 0; p < PF; ++p)
            if (p < n) sb_of(u0 + p, sc_pf[p], bi_pf[p]);
        const int sw = r & 7;                    // 128B swizzle of this row
        const int tg = g;                        // token group of this warp in the epilogue
        for (int i = 0; i < n; ++i) {
            const int u = u0 + i, b = u / nc, c = u - b * nc;
            const int s = i % stages, as = i % C::A_STAGES;
            const __half2 s1 = __half2half2(sc_pf[0]);
            const __half2 b2 = __half2half2(bi_pf[0]);
#pragma unroll
            for (int p = 0; p + 1 < PF; ++p) { sc_pf[p] = sc_pf[p + 1]; bi_pf[p] = bi_pf[p + 1]; }
            if (i + PF < n) sb_of(u + PF, sc_pf[PF - 1], bi_pf[PF - 1]);
            // after an abort every wait is skipped, but the warp still walks the
            // chunk sequence so that all dequant warps meet the same named barriers
            bool ok = !*abort_flag && tc::mbar_wait(tc::smem_u32(&cs.full[s]), (i / stages) & 1, ep.err, ERR_FULL);
            if (!ok) *abort_flag = 1;
            const unsigned char *wt = ring + (size_t)s * C::STAGE + C::XBYTES + r * 128;
            const uint4 w0 = *reinterpret_cast<const uint4 *>(wt + (((2 * g) ^ sw) << 4));
            const uint4 w1 = *reinterpret_cast<const uint4 *>(wt + (((2 * g + 1) ^ sw) << 4));
            const __half2 m1 = __hmul2(s1, __float2half2_rn(-1024.0f));
            const __half2 s16 = __hmul2(s1, __float2half2_rn(0.0625f));
            const __half2 m64 = __hmul2(s1, __float2half2_rn(-64.0f));
            uint32_t a[32];
            dequant_word(w0.x, s1, m1, s16, m64, b2, &a[0]);
            dequant_word(w0.y, s1, m1, s16, m64, b2, &a[4]);
            dequant_word(w0.z, s1, m1, s16, m64, b2, &a[8]);
            dequant_word(w0.w, s1, m1, s16, m64, b2, &a[12]);
            dequant_word(w1.x, s1, m1, s16, m64, b2, &a[16]);
            dequant_word(w1.y, s1, m1, s16, m64, b2, &a[20]);
            dequant_word(w1.z, s1, m1, s16, m64, b2, &a[24]);
            dequant_word(w1.w, s1, m1, s16, m64, b2, &a[28]);
            if (ok && i >= C::A_STAGES) {
                const int pc = i - C::A_STAGES;   // last chunk that used this A stage
                ok = tc::mbar_wait(tc::smem_u32(&cs.mma_done[pc % stages]), (pc / stages) & 1, ep.err, ERR_MMA);
                if (!ok) *abort_flag = 1;
            }
            if (!__any_sync(0xffffffffu, !ok || *abort_flag)) {
                const uint32_t ta = tmem + lane_base + (uint32_t)(as * A_COLS + g * 32);
                tc::tmem_st16(ta + 0, &a[0]);
                tc::tmem_st16(ta + 16, &a[16]);
                tc::tmem_wait_st();
                tc::fence_before_sync();
                __syncwarp();
                if (lane == 0) tc::mbar_arrive(tc::smem_u32(&cs.a_full[as]));
            } else {
                *abort_flag = 1;
            }

            if (c != nc - 1 && i != n - 1) continue;
            // ---------------- epilogue of the segment ending with this chunk ----------------
            const int seg_first_unit = max(u0, b * nc);
            const bool full = seg_first_unit == b * nc && c == nc - 1;
            const int tile = b / nblk, blk = b - tile * nblk;
            const int f = blk * ROWS + r;
            bool bad = *abort_flag != 0;
            if (!bad) bad = !tc::mbar_wait(tc::smem_u32(&cs.mma_done[s]), (i / stages) & 1, ep.err, ERR_DONE);
            if (named_bar_or(1, DQ_THREADS, bad)) { *abort_flag = 1; break; }
            tc::fence_after_sync();
            float acc[PIECES][16];
#pragma unroll
            for (int p = 0; p < PIECES; ++p) {
                const int cc = p * 64 + tg * 16;
                if (cc < NT) {   // warp-uniform
                    uint32_t v0[16], v1[16];
                    tc::tmem_ld16(tmem + lane_base + C::D_COL + cc, v0);
                    tc::tmem_ld16(tmem + lane_base + C::D_COL + C::DCOLS + cc, v1);
                    tc::tmem_wait_ld();
#pragma unroll
                    for (int q = 0; q < 16; ++q) acc[p][q] = __uint_as_float(v0[q]) + __uint_as_float(v1[q]);
                } else {
#pragma unroll
                    for (int q = 0; q < 16; ++q) acc[p][q] = 0.f;
                }
            }
            tc::fence_before_sync();
            __syncwarp();
            if (lane == 0) tc::mbar_arrive(tc::smem_u32(&cs.d_free));   // accumulator may be reused

            if (!full) {
                // partial block: slot of this CTA among the block's contributors
                const int first_owner = unit_owner(b * nc, U, G);
                const int ncontrib = unit_owner(b * nc + nc - 1, U, G) - first_owner + 1;
                float *pblk = ep.part + ((size_t)b * pmax) * ROWS * NT;
                float *mine = pblk + ((size_t)(cta - first_owner) * ROWS + r) * NT;
#pragma unroll
                for (int p = 0; p < PIECES; ++p) {
                    const int cc = p * 64 + tg * 16;
                    if (cc < NT) {
#pragma unroll
                        for (int q = 0; q < 16; q += 4)
                            *reinterpret_cast<float4 *>(mine + cc + q) =
                                make_float4(acc[p][q], acc[p][q + 1], acc[p][q + 2], acc[p][q + 3]);
                    }
                }
                __threadfence();
                named_bar_sync(1, DQ_THREADS);
                if (tid == 0) {
                    unsigned *ctr = ep.counters + b;
                    const unsigned prev = atomicAdd(ctr, 1u);
                    cs.last_flag = prev == (unsigned)(ncontrib - 1);
                    if (cs.last_flag) *ctr = 0u;   // ready for the next launch
                }
                named_bar_sync(1, DQ_THREADS);
                if (!cs.last_flag) continue;
                __threadfence();
#pragma unroll
                for (int p = 0; p < PIECES; ++p) {
                    const int cc = p * 64 + tg * 16;
#pragma unroll
                    for (int q = 0; q < 16; ++q) acc[p][q] = 0.f;
                    if (cc < NT) {
                        for (int sl = 0; sl < ncontrib; ++sl) {
                            const float *pp = pblk + ((size_t)sl * ROWS + r) * NT + cc;
#pragma unroll
                            for (int q = 0; q < 16; q += 4) {
                                const float4 t4 = __ldcg(reinterpret_cast<const float4 *>(pp + q));
                                acc[p][q] += t4.x; acc[p][q + 1] += t4.y; acc[p][q + 2] += t4.z; acc[p][q + 3] += t4.w;
                            }
                        }
                    }
                }
            }
            float *xch = cs.xch[tg];
#pragma unroll
            for (int p = 0; p < PIECES; ++p) {
                const int cc = p * 64 + tg * 16;
                const int m0 = tile * NT + cc;
                const int mlim = cc < NT ? max(0, min(16, M - m0)) : 0;   // valid tokens in this piece
                float *y = acc[p];
                if (ep.op == Q4Epilogue::STORE) {
#pragma unroll
                    for (int q = 0; q < 16; ++q)
                        if (q < mlim) ep.out[(size_t)(m0 + q) * ep.ldo + f] = y[q];
                } else if (ep.op == Q4Epilogue::RESID) {
#pragma unroll
                    for (int q = 0; q < 16; ++q)
                        if (q < mlim) ep.out[(size_t)(m0 + q) * ep.ldo + f] += y[q];
                } else if (ep.op == Q4Epilogue::SWIGLU) {
                    // rows [0,64) gate, [64,128) up of the same 64 outputs
                    if (r >= 64) {
#pragma unroll
                        for (int q = 0; q < 16; ++q) xch[(r - 64) * 16 + q] = y[q];
                    }
                    named_bar_sync(1, DQ_THREADS);
                    if (r < 64) {
                        const int oi = blk * 64 + r;
#pragma unroll
                        for (int q = 0; q < 16; ++q) {
                            if (q >= mlim) break;
                            const float gv = y[q], uv = xch[r * 16 + q];
                            const float av = gv / (1.0f + expf(-gv)) * uv;
                            ep.xout[xblk(m0 + q, oi, ep.ldx_rows)] = __float2half_rn(av);
                        }
                    }
                    named_bar_sync(1, DQ_THREADS);
                } else {   // QKV
                    const int D = ep.head_dim;
                    const int hh = f / D;      // head index in q|k|v order
                    const int d = f % D;
                    const bool is_q = hh < ep.n_heads, is_k = !is_q && hh < ep.n_heads + ep.n_kv;
                    const float *nw = is_q ? ep.q_norm : (is_k ? ep.k_norm : nullptr);
                    if (nw) {
                        // per-head sum of squares for each token: warp shuffles + smem
#pragma unroll
                        for (int q = 0; q < 16; ++q) {
                            const float t2 = warp_sum(y[q] * y[q]);
                            if (lane == q) cs.wsum[tg][quarter][q] = t2;
                        }
                    }
                    named_bar_sync(1, DQ_THREADS);
                    if (nw) {
                        const int wpk = D / 32, w0 = (quarter / wpk) * wpk;
#pragma unroll
                        for (int q = 0; q < 16; ++q) {
                            float ss = 0.f;
                            for (int ww = w0; ww < w0 + wpk; ++ww) ss += cs.wsum[tg][ww][q];
                            y[q] = y[q] * (1.0f / sqrtf(ss / (float)D + ep.eps)) * nw[d];
                        }
                    }
                    // rotate-half RoPE on q and k: partner row r +- D/2
#pragma unroll
                    for (int q = 0; q < 16; ++q) xch[r * 16 + q] = y[q];
                    named_bar_sync(1, DQ_THREADS);
                    if (is_q || is_k) {
                        const int half = D / 2;
                        const int pr = d < half ? r + half : r - half;
                        const float fr = ep.inv_freq[d % half];
#pragma unroll
                        for (int q = 0; q < 16; ++q) {
                            if (q >= mlim) break;
                            const float ang = __fmul_rn((float)ep.tpos[m0 + q], fr);
                            float sn, cn;
                            sincosf(ang, &sn, &cn);
                            const float pv = xch[pr * 16 + q];
                            y[q] = d < half ? y[q] * cn - pv * sn : pv * sn + y[q] * cn;
                        }
                    }
#pragma unroll
                    for (int q = 0; q < 16; ++q) {
                        if (q >= mlim) break;
                        const int m = m0 + q;
                        __half *dst;
                        if (is_q) {
                            dst = ep.qbuf + ((size_t)m * ep.n_heads + hh) * D;
                        } else {
                            const int kvh = is_k ? hh - ep.n_heads : hh - ep.n_heads - ep.n_kv;
                            dst = (is_k ? ep.kc : ep.vc) +
                                  (((size_t)ep.trow[m] * ep.n_kv + kvh) * ep.max_len + ep.tpos[m]) * D;
                        }
                        dst[d] = __float2half_rn(y[q]);
                    }
                    named_bar_sync(1, DQ_THREADS);
                }
            }
        }
    }
    tc::fence_before_sync();
    __syncthreads();
    if (warp == 0) {
        tc::fence_after_sync();
        tc::tmem_dealloc(tmem, 512);
    }
}

// ---------------------------------------------------------------------------
// host side: tensor maps and launch
// ---------------------------------------------------------------------------
PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    if (!fn) {
        cudaDriverEntryPointQueryResult q;
        void *p = nullptr;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    }
    return fn;
}

template <int NT>
int stages_for() {
    int s = (int)((227 * 1024 - 1024 - sizeof(Smem)) / Cfg<NT>::STAGE);
    return s < 2 ? 2 : (s > MAX_STAGES ? MAX_STAGES : s);
}

template <int NT>
size_t smem_for(int stages) {
    return 1024 + (size_t)stages * Cfg<NT>::STAGE + sizeof(Smem);
}

template <int NT>
cudaError_t launch_nt(const Q4WeightTC &w, const CUtensorMap &xmap, int M, int tok_base, int tiles,
                      int sm_count, const Q4Epilogue &ep, cudaStream_t st) {
    static bool attr[64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    const int stages = stages_for<NT>();
    const size_t sm = smem_for<NT>(stages);
    if (!attr[dev & 63]) {
        cudaError_t e = cudaFuncSetAttribute(q4_tc_kernel<NT>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm);
        if (e != cudaSuccess) return e;
        attr[dev & 63] = true;
    }
    const int nblk = w.N / ROWS, nc = (w.K + CHUNK - 1) / CHUNK;
    const int U = tiles * nblk * nc;
    const int G = U < sm_count ? U : sm_count;
    const int pmax = q4_tc_pmax(U, G, nc);
    if (pmax > 1 && (!ep.part || !ep.counters)) return cudaErrorInvalidValue;
    q4_tc_kernel<NT><<<G, THREADS, sm, st>>>(w.map, xmap, w.scales, w.biases, w.N, w.K, M, tok_base, nblk, nc,
                                             U, pmax, stages, ep);
    return cudaGetLastError();
}

}  // namespace

bool make_weight_map(Q4WeightTC &w) {
    auto fn = encode_fn();
    if (!fn) return false;
    const cuuint64_t dims[2] = {(cuuint64_t)(w.K / 2), (cuuint64_t)w.N};
    const cuuint64_t strides[1] = {(cuuint64_t)(w.K / 2)};
    const cuuint32_t box[2] = {128, ROWS};
    const cuuint32_t es[2] = {1, 1};
    return fn(&w.map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<uint32_t *>(w.wq), dims, strides, box, es,
              CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

int q4_tc_tile(int M) {
    const int nt = ((M + 15) / 16) * 16;
    return nt > 128 ? 128 : nt;
}

// most CTAs that share one row block (stream-K contributors)
int q4_tc_pmax(int U, int G, int nc) {
    // a CTA covers floor(U/G) or ceil(U/G) units; a block of nc units meets at most
    // ceil((nc - 1) / floor(U/G)) + 1 of them
    const int per = U / G > 0 ? U / G : 1;
    return (nc - 1 + per - 1) / per + 1;
}

size_t q4_tc_partial_floats(int N, int K, int M, int sm_count) {
    const int nt = q4_tc_tile(M);
    const int tiles = (M + nt - 1) / nt;
    const int nblk = N / ROWS, nc = (K + CHUNK - 1) / CHUNK;
    const int U = tiles * nblk * nc, G = U < sm_count ? U : sm_count;
    return (size_t)tiles * nblk * q4_tc_pmax(U, G, nc) * ROWS * nt;
}

size_t q4_tc_counters(int N, int M) {
    const int nt = q4_tc_tile(M);
    return (size_t)((M + nt - 1) / nt) * (N / ROWS);
}

cudaError_t q4_tc(const Q4WeightTC &w, const __half *x_blk, int ldx_rows, int tok_base, int M,
                  int sm_count, const Q4Epilogue &ep, cudaStream_t st) {
    if (w.N % ROWS || w.K % 128 || M <= 0 || tok_base + M > ldx_rows) return cudaErrorInvalidValue;
    auto fn = encode_fn();
    if (!fn) return cudaErrorNotSupported;
    const int nt = q4_tc_tile(M);
    const int tiles = (M + nt - 1) / nt;
    // token operand [K/64][ldx_rows][64] fp16 -> 3-D map (64, rows, K/64)
    CUtensorMap xmap;
    const cuuint64_t dims[3] = {64, (cuuint64_t)ldx_rows, (cuuint64_t)(w.K / 64)};   // boxes past K read 0
    const cuuint64_t strides[2] = {128, (cuuint64_t)ldx_rows * 128};
    const cuuint32_t box[3] = {64, (cuuint32_t)nt, CHUNK / 64};
    const cuuint32_t es[3] = {1, 1, 1};
    if (fn(&xmap, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, const_cast<__half *>(x_blk), dims, strides, box, es,
           CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
           CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
        return cudaErrorInvalidValue;
    switch (nt) {
    case 16: return launch_nt<16>(w, xmap, M, tok_base, tiles, sm_count, ep, st);
    case 32: return launch_nt<32>(w, xmap, M, tok_base, tiles, sm_count, ep, st);
    case 48: return launch_nt<48>(w, xmap, M, tok_base, tiles, sm_count, ep, st);
    case 64: return launch_nt<64>(w, xmap, M, tok_base, tiles, sm_count, ep, st);
    case 80: return launch_nt<80>(w, xmap, M, tok_base, tiles, sm_count, ep, st);
    case 96: return launch_nt<96>(w, xmap, M, tok_base, tiles, sm_count, ep, st);
    case 112: return launch_nt<112>(w, xmap, M, tok_base, tiles, sm_count, ep, st);
    default: return launch_nt<128>(w, xmap, M, tok_base, tiles, sm_count, ep, st);
    }
}

}  // namespace mlxcat
