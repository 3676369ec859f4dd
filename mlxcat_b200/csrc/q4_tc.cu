// q4_tc.cu -- MLX affine 4-bit (group 64) linear on the 5th-generation tensor
// cores, with the split-K reduction and the consumer epilogue fused in.
//
//   y[m][n] = sum_k x[m][k] * (scale[n][k/64] * q[n][k] + bias[n][k/64])
//
// Replaces mlx-swift's quantizedMatmul (QuantizedLinear in mlx-swift-lm) on
// the verify forward (BatchGenerator.swift:900-904).  The packed weights stay
// in the MLX layout (uint32 [N][K/8], lowest nibble first); scales and biases
// are re-packed once per weight into (scale, bias) fp16 pairs ordered
// [N/128][K/512][8 groups][128 rows] so that one bulk copy brings a unit's
// 4 KB of them next to its weight tile (pack_q4_sb below).
//
// Swap-AB: the 128 weight rows of a block are the MMA's M dimension, the
// tokens of the verify batch (a tile of 16..128, or 144..160 for the gate/up
// projection) its N dimension.  One tcgen05.mma of M=128, K=16 holds the
// tensor pipe for about 120 cycles whatever its N up to 128 (measured on
// B200), so 129..160 tokens of the gate/up projection run as one tile instead
// of two (the other projections keep two: measured slower as one).
//
// Schedule: persistent, one CTA per SM, stream-K over units of (128-row block
// x 512-wide k chunk); a block whose chunks span several CTAs is finished by
// the last of them (deterministic slot-ordered sum).  Within a unit the k
// range is processed as two 256-wide sub-chunks.
//
// Warp roles (20 warps):
//   warp 18 (one lane)  W producer: per unit one W stage = two TMA boxes of
//                       [128 rows x 128 B] (128B swizzle) + the unit's packed
//                       scale/bias (bulk copy); per 256-k half (one box) for
//                       tiles above 128 tokens, whose 80 KB x stages leave
//                       less room.  A W stage is released once the dequant
//                       warps have put its values into TMEM.
//   warp 19 (one lane)  x producer: per sub-chunk one x stage = the token tile
//                       [4 x NT x 64] fp16 (3-D box, 128B swizzle), released
//                       when the MMAs reading it have completed.  x stages and
//                       TMEM A buffers form one ring: sub-chunk j uses slot
//                       j % R of both, and one MMA-completion barrier per slot
//                       (one commit per issuer per sub-chunk) frees both.
//   warps 0-15          dequantisers: warp w owns rows 32*(w%4).. (its TMEM
//                       lane quarter) and 64-wide group g = w/4 of each
//                       sub-chunk: nibbles -> fp16 in registers (0x6400 magic,
//                       hfma2 / hadd2), tcgen05.st into TMEM (the MMA's A
//                       operand, a ring of three sub-chunk buffers for
//                       NT <= 64, two above), then a named-barrier arrive for
//                       the issuer of group g.
//   warps 16-17         MMA issuers (lane 0): issuer i waits on its named
//                       barrier, then issues tcgen05.mma (M=128, N=NT, K=16,
//                       A from TMEM, B from shared memory) for groups 2i, 2i+1
//                       into its own fp32 accumulator in TMEM.  Tiles above
//                       128 tokens have one issuer (one accumulator of NT
//                       columns: the TMEM holds no second one).
//
// Inside each 8-wide k block the unpack order is (0,4,1,5,2,6,3,7); the token
// operand is stored in that order and blocked by 64 features ([K/64][rows][64],
// see common.cuh: xblk) by its producers.
//
// Epilogue (dequant warps, after the last sub-chunk of a block segment):
//   STORE   logits  out[m][n] = y
//   RESID   residual stream h[m][n] += y
//   SWIGLU  gate/up rows interleaved per 64 -> x_next[m][i] = silu(g) * u
//   QKV     per-head q/k RMSNorm (Qwen3), rotate-half RoPE, q to the query
//           buffer, k/v appended to the KV cache at each token's position
//
// Every mbarrier wait is bounded (tc.cuh).  A timeout sets *err and an abort
// flag; from then on every role skips its waits and work but still walks the
// same sequence of named barriers, so no thread is left waiting on one, and
// the CTA drains its in-flight copies and MMAs (bounded) before freeing TMEM.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <algorithm>

#include "common.cuh"
#include "kernels.h"
#include "tc.cuh"

namespace mlxcat {

int q4_tc_pmax(int U, int G, int nc);

// the driver's tensor-map encoder, fetched once through the runtime
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

namespace {

constexpr int ROWS = 128;              // weight rows per block (MMA M)
constexpr int KU = 512;                // k per stream-K unit (one W stage)
constexpr int KS = 256;                // k per sub-chunk (one x stage, one A buffer)
constexpr int DQ_WARPS = 16;           // dequantising warps
constexpr int ISS_WARP0 = DQ_WARPS;    // issuer warps 16..17
constexpr int MAX_NI = 2;              // MMA issuer warps
constexpr int WP_WARP = DQ_WARPS + MAX_NI; // W producer
constexpr int XP_WARP = WP_WARP + 1;   // x producer
constexpr int EP_WARP0 = XP_WARP + 1;  // epilogue warps 20..23 (TMEM lane quarters 0..3)
constexpr int EP_THREADS = 128;
constexpr int THREADS = (EP_WARP0 + 4) * 32;
constexpr int A_COLS = KS / 2;         // TMEM columns of one A buffer (fp16 pairs)
constexpr int WBOX = ROWS * 128;       // one [128 rows x 128 B] weight box (256 k)
constexpr int SB_BYTES = 8 * ROWS * 4; // packed (scale, bias) of one unit
constexpr int MAX_SW = 4, MAX_AST = 3;
constexpr int MAX_NT = 160;            // widest token tile (gate/up projection)
constexpr int EPI_BAR = 9;             // named barrier of the epilogue warps (1..6: issuers)
constexpr int TAIL_BAR = 10;           // named barrier of the dequant warps' tail epilogue
constexpr int TAIL_THREADS = DQ_WARPS * 32;

enum ErrCode { ERR_WFULL = 1, ERR_XFULL = 2, ERR_MDONE = 3, ERR_XFREE = 4, ERR_WFREE = 5, ERR_DFREE = 6 };

template <int NT>
struct Cfg {
    static constexpr bool WIDE = NT > 128;                   // one accumulator of up to 160 columns
    static constexpr int NI = WIDE ? 1 : 2;                  // MMA issuers (one accumulator each)
    static constexpr int GPI = 4 / NI;                       // 64-k groups per issuer
    static constexpr int BAR_COUNT = 32 + 128 * GPI;         // issuer warp + its dequant warps
    // TMEM: ring of A buffers, then DSETS sets of NI fp32 accumulators.  With
    // two sets the MMAs of the next block segment run while the epilogue warps
    // read the previous one.
    static constexpr int DCOLS = NT <= 32 ? 32 : (NT <= 64 ? 64 : (NT <= 128 ? 128 : 256));
    static constexpr int DSETS = NT <= 64 ? 2 : 1;
    static constexpr int AST = NT <= 32 ? 3 : 2;             // ring slots: A buffers in TMEM = x stages
    static constexpr int D_COL = AST * A_COLS;
    static constexpr int XSTAGE = 4 * NT * 128;              // 256 k of NT tokens
    static constexpr int PIECES = NT / 16;                   // 16-token pieces of the epilogue
    // W: one stage per unit (two boxes + the unit's scale/bias), or per 256-k
    // half (one box + half of them) for the wide tile; two sub-chunks or one
    // read each
    static constexpr int WSTAGE = WIDE ? WBOX + SB_BYTES / 2 : 2 * WBOX + SB_BYTES;
    static_assert(D_COL + DSETS * NI * DCOLS <= 512, "TMEM budget");
    static_assert(NT % 16 == 0 && NT <= MAX_NT, "token tile");
};

__device__ __forceinline__ void named_bar_sync(int id, int n) {
    asm volatile("bar.sync %0, %1;\n" ::"r"(id), "r"(n) : "memory");
}
__device__ __forceinline__ void named_bar_arrive(int id, int n) {
    asm volatile("bar.arrive %0, %1;\n" ::"r"(id), "r"(n) : "memory");
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

__device__ __forceinline__ void bulk_load(uint32_t dst, const void *src, uint32_t bytes, uint32_t bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];\n"
                 ::"r"(dst), "l"(src), "r"(bytes), "r"(bar)
                 : "memory");
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

// the constants of one quantisation group, from its (scale, bias) pair
struct GroupConst {
    __half2 s1, m1, s16, m64, b2;
    __device__ __forceinline__ explicit GroupConst(uint32_t sb) {
        const __half2 sbh = *reinterpret_cast<const __half2 *>(&sb);
        s1 = __low2half2(sbh);
        b2 = __high2half2(sbh);
        m1 = __hmul2(s1, __float2half2_rn(-1024.0f));
        s16 = __hmul2(s1, __float2half2_rn(0.0625f));
        m64 = __hmul2(s1, __float2half2_rn(-64.0f));
    }
};

// 16 bytes (32 nibbles) of one row -> 16 fp16 pairs
__device__ __forceinline__ void dequant16(const uint4 &w, const GroupConst &k, uint32_t *a) {
    dequant_word(w.x, k.s1, k.m1, k.s16, k.m64, k.b2, &a[0]);
    dequant_word(w.y, k.s1, k.m1, k.s16, k.m64, k.b2, &a[4]);
    dequant_word(w.z, k.s1, k.m1, k.s16, k.m64, k.b2, &a[8]);
    dequant_word(w.w, k.s1, k.m1, k.s16, k.m64, k.b2, &a[12]);
}

struct Smem {
    uint64_t full_w[MAX_SW], w_free[MAX_SW], full_x[MAX_AST], mma_done[MAX_AST], d_full[2], d_free[2];
    uint32_t tmem_base;
    int abort_flag;
    int last_flag;
    float wsum[4][16];          // [row quarter][token of the piece]
    float xch[MAX_NT];          // epilogue warps: folded-norm scales; QKV tail: token rows / positions
    // the tail epilogue of the dequant warps (may overlap the epilogue warps)
    int last_flag2;
    float wsum2[4][4][16];      // [token group][row quarter][token]
    float xch2[2][ROWS * 16];   // [token group pair][row][token]
    float cscale[MAX_NT];       // folded RMSNorm: per-token column scale of the tail epilogue
    int cscale_tile;            // token tile whose scales the idle epilogue warps put in cscale
};

// Stream-K schedule: the flattened (row block, k unit) space is split into
// gridDim.x contiguous, equal ranges, one per CTA.
// (U * G < 2^32 for every launch: checked on the host)
__device__ __forceinline__ int unit_begin(int c, int U, int G) { return (int)(((uint32_t)c * (uint32_t)U) / (uint32_t)G); }
__device__ __forceinline__ int unit_owner(int u, int U, int G) {
    int c = (int)(((uint32_t)u * (uint32_t)G) / (uint32_t)U);
    while (c + 1 < G && unit_begin(c + 1, U, G) <= u) ++c;
    while (c > 0 && unit_begin(c, U, G) > u) --c;
    return c;
}

// Folded RMSNorm, consumer side: the token operand rows are fp16(h * w * s[m])
// with a pre-scale s (an earlier rstd of the same row); the accumulators of row m
// are multiplied by rstd(m) / s[m], rstd from the producer's per-block sums of
// squares (summed in block order).  Thread t0 of `stride` threads fills dst[t]
// for t = t0, t0 + stride, .. < NT, the x rows xrow0 + t (rows past the operand
// give 0).
__device__ __forceinline__ void fold_scale(const Q4Epilogue &ep, int K, int xrow0, int nrows, int t0, int stride,
                                           float *dst, int NT) {
    for (int t = t0; t < NT; t += stride) {
        const int m = xrow0 + t;
        float c = 0.f;
        if (t < nrows) {
            // 16 loads in flight per batch; summed in block order
            const float prev = __ldcg(ep.col_prev + m);
            const int nb = K / 128;
            float ss = 0.f;
            for (int b0 = 0; b0 < nb; b0 += 16) {
                float v[16];
#pragma unroll
                for (int k = 0; k < 16; ++k)
                    v[k] = b0 + k < nb ? __ldcg(ep.col_part + (size_t)(b0 + k) * ep.norm_rows + m) : 0.f;
#pragma unroll
                for (int k = 0; k < 16; ++k) ss += v[k];
            }
            const float r = 1.0f / sqrtf(ss / (float)K + ep.col_eps);
            if (ep.col_rstd) ep.col_rstd[m] = r;
            c = r / prev;
        }
        dst[t] = c;
    }
}

// Sums over the warp of sixteen per-lane values (one per token of a piece) in
// 16 shuffles instead of 16 x 5: at each of five butterfly steps a lane keeps
// the half of its tokens picked by one lane bit and adds the partner's copy of
// that half.  Returns the total of token (lane >> 1) & 15 (held by both lanes of
// a pair); the summation order is fixed.
__device__ __forceinline__ float warp_sum16(const float *v, int lane) {
    float a[8], b[4], c[2];
    const bool b4 = lane & 16, b3 = lane & 8, b2 = lane & 4, b1 = lane & 2;
#pragma unroll
    for (int i = 0; i < 8; ++i)
        a[i] = (b4 ? v[i + 8] : v[i]) + __shfl_xor_sync(0xffffffffu, b4 ? v[i] : v[i + 8], 16);
#pragma unroll
    for (int i = 0; i < 4; ++i)
        b[i] = (b3 ? a[i + 4] : a[i]) + __shfl_xor_sync(0xffffffffu, b3 ? a[i] : a[i + 4], 8);
#pragma unroll
    for (int i = 0; i < 2; ++i)
        c[i] = (b2 ? b[i + 2] : b[i]) + __shfl_xor_sync(0xffffffffu, b2 ? b[i] : b[i + 2], 4);
    float d = (b1 ? c[1] : c[0]) + __shfl_xor_sync(0xffffffffu, b1 ? c[0] : c[1], 2);
    return d + __shfl_xor_sync(0xffffffffu, d, 1);
}

// bounded wait that gives up at once after an abort
__device__ __forceinline__ bool wait_or_abort(uint32_t bar, uint32_t parity, volatile int *abort_flag, int *err,
                                              int code) {
    if (*abort_flag) return false;
    if (tc::mbar_wait(bar, parity, err, code)) return true;
    *abort_flag = 1;
    return false;
}

// STORE epilogue: feature f of tokens m0..m0+mlim-1, into out[m][f] or, when
// the projection scatters to peers (tensor parallel), into the owner's slot
__device__ __forceinline__ void store_rows(const Q4Epilogue &ep, int f, int m0, int mlim, const float *y) {
    float *o;
    size_t ld;
    if (ep.peers) {
        const int d = f / ep.peer_cols;
        o = reinterpret_cast<float *>(ep.peers[d] + ep.peer_off) + (f - d * ep.peer_cols);
        ld = (size_t)ep.peer_cols;
    } else {
        o = ep.out + f;
        ld = (size_t)ep.ldo;
    }
#pragma unroll
    for (int q = 0; q < 16; ++q)
        if (q < mlim) o[(size_t)(m0 + q) * ld] = y[q];
}

template <int NT, int OP>
__global__ void __launch_bounds__(THREADS, 1)
q4_tc_kernel(const __grid_constant__ CUtensorMap wmap, const __grid_constant__ CUtensorMap xmap,
             const uint32_t *__restrict__ sbp, int N, int K, int M, int tok_base, int nblk, int nc, int U,
             int pmax, int sw, Q4Epilogue ep) {
    using C = Cfg<NT>;
    // the epilogue warps take the non-last segments of the cheap epilogues; the
    // QKV and SWIGLU epilogues (norms, RoPE, exchanges) stay on sixteen warps
    constexpr bool EPW = OP == Q4Epilogue::STORE || OP == Q4Epilogue::RESID;
    extern __shared__ __align__(1024) unsigned char smem_raw[];
    unsigned char *wring = reinterpret_cast<unsigned char *>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
    unsigned char *xring = wring + (size_t)sw * C::WSTAGE;
    constexpr int R = C::AST;
    Smem &cs = *reinterpret_cast<Smem *>(xring + (size_t)R * C::XSTAGE);

    // The weights do not depend on the previous kernel: let the next launch be
    // scheduled early, and (launched with programmatic serialisation) start
    // streaming and dequantising weights before the previous kernel finishes;
    // only the token operand waits for it (griddep_wait in the x producer).
    griddep_launch_dependents();
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int G = gridDim.x, cta = blockIdx.x;
    const int u0 = unit_begin(cta, U, G), u1 = unit_begin(cta + 1, U, G);
    const int n = u1 - u0;                        // units of this CTA
    const int nsub = 2 * n;                       // sub-chunks of this CTA

    if (warp == WP_WARP && lane == 0) {
        for (int s = 0; s < sw; ++s) {
            tc::mbar_init(tc::smem_u32(&cs.full_w[s]), 1);
            tc::mbar_init(tc::smem_u32(&cs.w_free[s]), DQ_WARPS);
        }
        for (int r = 0; r < R; ++r) {
            tc::mbar_init(tc::smem_u32(&cs.full_x[r]), 1);
            tc::mbar_init(tc::smem_u32(&cs.mma_done[r]), C::NI);
        }
        for (int d = 0; d < C::DSETS; ++d) {
            tc::mbar_init(tc::smem_u32(&cs.d_full[d]), C::NI);
            tc::mbar_init(tc::smem_u32(&cs.d_free[d]), EPW ? 4 : DQ_WARPS);
        }
        cs.abort_flag = 0;
        cs.cscale_tile = -1;
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

    if (warp == WP_WARP) {
        if (lane == 0) {
            // ------- W producer: one stage per unit (per 256-k half: wide tile) -------
            constexpr int HALVES = C::WIDE ? 2 : 1;      // W stages per unit
            int issued = 0;
            int b = u0 / nc, c = u0 - b * nc;
            for (int i = 0; i < n * HALVES && !*abort_flag; ++i) {
                const int hh = HALVES == 2 ? (i & 1) : 0, blk = b % nblk;
                const int s = i % sw;
                if (i >= sw && !wait_or_abort(tc::smem_u32(&cs.w_free[s]), ((i - sw) / sw) & 1, abort_flag, ep.err,
                                              ERR_WFREE))
                    break;
                const uint32_t st = tc::smem_u32(wring + (size_t)s * C::WSTAGE);
                const uint32_t bar = tc::smem_u32(&cs.full_w[s]);
                const uint32_t *sbu = sbp + (size_t)(blk * nc + c) * (8 * ROWS);
                tc::mbar_arrive_expect_tx(bar, C::WSTAGE);
                if constexpr (C::WIDE) {
                    tc::tma_load_2d(st, &wmap, c * (KU / 2) + hh * (KS / 2), blk * ROWS, bar);
                    bulk_load(st + WBOX, sbu + hh * (4 * ROWS), SB_BYTES / 2, bar);
                } else {
                    tc::tma_load_2d(st, &wmap, c * (KU / 2), blk * ROWS, bar);
                    tc::tma_load_2d(st + WBOX, &wmap, c * (KU / 2) + KS / 2, blk * ROWS, bar);
                    bulk_load(st + 2 * WBOX, sbu, SB_BYTES, bar);
                }
                issued = i + 1;
                if (hh == HALVES - 1 && ++c == nc) { c = 0; ++b; }
            }
            if (*abort_flag)   // let every issued copy land before the CTA can exit
                for (int i = max(0, issued - sw); i < issued; ++i)
                    tc::mbar_wait(tc::smem_u32(&cs.full_w[i % sw]), (i / sw) & 1, nullptr, 0);
        }
    } else if (warp == XP_WARP) {
        if (lane == 0) {
            // ---------------- x producer: one stage per sub-chunk ----------------
            griddep_wait();   // the token operand is the previous kernel's output
            int issued = 0;
            int b = u0 / nc, c = u0 - b * nc;
            for (int j = 0; j < nsub && !*abort_flag; ++j) {
                const int h = j & 1, tile = b / nblk;
                const int xs = j % R;
                if (j >= R && !wait_or_abort(tc::smem_u32(&cs.mma_done[xs]), ((j - R) / R) & 1, abort_flag,
                                             ep.err, ERR_XFREE))
                    break;
                const uint32_t bar = tc::smem_u32(&cs.full_x[xs]);
                tc::mbar_arrive_expect_tx(bar, C::XSTAGE);
                tc::tma_load_3d(tc::smem_u32(xring + (size_t)xs * C::XSTAGE), &xmap, 0, tok_base + tile * NT,
                                c * (KU / 64) + h * (KS / 64), bar);
                issued = j + 1;
                if (h == 1 && ++c == nc) { c = 0; ++b; }
            }
            if (*abort_flag)
                for (int j = max(0, issued - R); j < issued; ++j)
                    tc::mbar_wait(tc::smem_u32(&cs.full_x[j % R]), (j / R) & 1, nullptr, 0);
        }
    } else if (warp >= ISS_WARP0 && warp < ISS_WARP0 + MAX_NI) {
        const int is = warp - ISS_WARP0;
        if (is < C::NI) {
            // ---------------- MMA issuer `is`: groups [is*GPI, (is+1)*GPI) ----------------
            constexpr uint32_t idesc = tc::idesc_f16_f32(ROWS, NT);
            const uint64_t bdesc0 = tc::sdesc_k_sw128(tc::smem_u32(xring));   // slot r: + r * XSTAGE
            int c = u0 % nc, seg = 0, last = -1, dset = 0;
            for (int j = 0; j < nsub; ++j) {
                const int h = j & 1, as = j % R;
                const bool first = h == 0 && (j == 0 || c == 0);   // first sub-chunk of a block segment
                const bool seg_end = h == 1 && (c == nc - 1 || j == nsub - 1);
                if (first && seg >= C::DSETS && lane == 0)   // the epilogue has read this accumulator set
                    wait_or_abort(tc::smem_u32(&cs.d_free[dset]), ((seg - C::DSETS) / C::DSETS) & 1, abort_flag,
                                  ep.err, ERR_DFREE);
                __syncwarp();
                named_bar_sync(1 + is * MAX_AST + as, C::BAR_COUNT);
                if (lane == 0) {
                    if (wait_or_abort(tc::smem_u32(&cs.full_x[as]), (j / R) & 1, abort_flag, ep.err, ERR_XFULL)) {
                        tc::fence_after_sync();
                        const uint32_t dcol = tmem + C::D_COL + (dset * C::NI + is) * C::DCOLS;
                        const uint64_t bdesc = bdesc0 + (uint64_t)(as * (C::XSTAGE >> 4));
#pragma unroll
                        for (int gg = 0; gg < C::GPI; ++gg) {
                            const int grp = is * C::GPI + gg;
#pragma unroll
                            for (int q = 0; q < 4; ++q) {
                                const int kk = grp * 4 + q;             // k step of 16 inside the sub-chunk
                                const uint32_t boff = (uint32_t)(grp * NT * 128 + q * 32);
                                tc::mma_ts_f16(dcol, tmem + as * A_COLS + kk * 8, bdesc + (boff >> 4), idesc,
                                               (first && gg == 0 && q == 0) ? 0u : 1u);
                            }
                        }
                        tc::mma_commit(tc::smem_u32(&cs.mma_done[as]));   // frees A buffer and x stage
                        if (seg_end) tc::mma_commit(tc::smem_u32(&cs.d_full[dset]));   // segment complete
                        last = j;
                    }
                }
                __syncwarp();
                if (seg_end) {
                    ++seg;
                    if (++dset == C::DSETS) dset = 0;
                }
                if (h == 1 && ++c == nc) c = 0;
            }
            if (lane == 0 && last >= 0)   // committed MMAs must finish before TMEM is freed
                tc::mbar_wait(tc::smem_u32(&cs.mma_done[last % R]), (last / R) & 1, nullptr, 0);
        }
    } else if (warp < DQ_WARPS) {
        // ------- dequant warps: rows 32*quarter.., group g of each sub-chunk -------
        const int quarter = warp & 3, g = warp >> 2;
        const int r = quarter * 32 + lane;       // row within the block, 0..127
        const int is = g / C::GPI;               // issuer of this group
        const uint32_t lane_base = (uint32_t)(quarter * 32) << 16;
        const int sw8 = r & 7;                   // 128B swizzle of this row
        int ctile = -1;                          // token tile whose folded-norm scales are in cs.cscale
        // epilogue of one block segment by the sixteen dequantising warps
        auto seg_epilogue = [&](const int ub, const int lseg, const bool release) {
            constexpr int PIECES = NT <= 64 ? 1 : (NT <= 128 ? 2 : 3);   // 16-token pieces per token group
            const int tg = g;                             // token group of this warp
            const int ldset = lseg % C::DSETS;
            const int seg_first_unit = max(u0, ub * nc), seg_last_unit = min(u1 - 1, ub * nc + nc - 1);
            const bool full = seg_first_unit == ub * nc && seg_last_unit == ub * nc + nc - 1;
            const int tile = ub / nblk, blk = ub - tile * nblk;
            const int f = blk * ROWS + r;
            if constexpr (OP == Q4Epilogue::RESID) {
                // the residual rows this thread will update: into L1 while the
                // partials are exchanged
#pragma unroll
                for (int p = 0; p < PIECES; ++p) {
                    const int cc = p * 64 + tg * 16, m0 = tile * NT + cc;
                    const int mlim = cc < NT ? max(0, min(16, M - m0)) : 0;
#pragma unroll
                    for (int q = 0; q < 16; ++q)
                        if (q < mlim) asm volatile("prefetch.global.L1 [%0];" ::"l"(ep.out + (size_t)(m0 + q) * ep.ldo + f));
                }
            }
            bool bad = *abort_flag != 0;
            if (lane == 0 && !bad)
                bad = !wait_or_abort(tc::smem_u32(&cs.d_full[ldset]), (lseg / C::DSETS) & 1, abort_flag, ep.err,
                                     ERR_DFREE);
            bad = __shfl_sync(0xffffffffu, bad, 0);
            if (named_bar_or(TAIL_BAR, TAIL_THREADS, bad)) { *abort_flag = 1; return; }
            tc::fence_after_sync();
            {
            float acc[PIECES][16];
#pragma unroll
            for (int p = 0; p < PIECES; ++p) {
                const int cc = p * 64 + tg * 16;
#pragma unroll
                for (int q = 0; q < 16; ++q) acc[p][q] = 0.f;
                if (cc < NT) {   // warp-uniform
#pragma unroll
                    for (int d = 0; d < C::NI; ++d) {
                        uint32_t v[16];
                        tc::tmem_ld16(tmem + lane_base + C::D_COL + (ldset * C::NI + d) * C::DCOLS + cc, v);
                        tc::tmem_wait_ld();
#pragma unroll
                        for (int q = 0; q < 16; ++q) acc[p][q] += __uint_as_float(v[q]);
                    }
                }
            }
            if (release) {   // accumulators read: the issuers may reuse this set
                tc::fence_before_sync();
                __syncwarp();
                if (lane == 0) tc::mbar_arrive(tc::smem_u32(&cs.d_free[ldset]));
            }

            if (!full) {
                // partial block: slot of this CTA among the block's contributors.
                // Partials are stored [slot][token][row] so that a warp (32
                // consecutive rows) reads and writes 128 contiguous bytes.
                const int first_owner = unit_owner(ub * nc, U, G);
                const int ncontrib = unit_owner(ub * nc + nc - 1, U, G) - first_owner + 1;
                float *pblk = ep.part + (size_t)ub * pmax * NT * ROWS;
                float *mine = pblk + (size_t)(cta - first_owner) * NT * ROWS + r;
#pragma unroll
                for (int p = 0; p < PIECES; ++p) {
                    const int cc = p * 64 + tg * 16;
                    if (cc < NT) {
#pragma unroll
                        for (int q = 0; q < 16; ++q) mine[(size_t)(cc + q) * ROWS] = acc[p][q];
                    }
                }
                // the CTA barrier orders every thread's partial stores before thread
                // 0's gpu-scope fence (fences are cumulative), which orders them
                // before the ticket; the last contributor fences again before the
                // barrier that releases its readers
                named_bar_sync(TAIL_BAR, TAIL_THREADS);
                if (tid == 0) {
                    unsigned *ctr = ep.counters + ub;
                    __threadfence();
                    const unsigned prev = atomicAdd(ctr, 1u);
                    const int last = prev == (unsigned)(ncontrib - 1);
                    if (last) {
                        *ctr = 0u;   // ready for the next launch
                        __threadfence();
                    }
                    cs.last_flag2 = last;
                }
                named_bar_sync(TAIL_BAR, TAIL_THREADS);
                if (!cs.last_flag2) return;
#pragma unroll
                for (int p = 0; p < PIECES; ++p) {
                    const int cc = p * 64 + tg * 16;
#pragma unroll
                    for (int q = 0; q < 16; ++q) acc[p][q] = 0.f;
                    if (cc < NT) {
                        // slots are summed in slot order; the loads of a batch of slots
                        // are issued together so their L2 latencies overlap
                        const float *pp = pblk + (size_t)cc * ROWS + r;
                        const size_t slot_stride = (size_t)NT * ROWS;
                        constexpr int BATCH = PIECES == 1 ? 2 : 1;
                        for (int sl = 0; sl < ncontrib; sl += BATCH) {
                            float t[BATCH][16];
#pragma unroll
                            for (int k = 0; k < BATCH; ++k)
#pragma unroll
                                for (int q = 0; q < 16; ++q)
                                    t[k][q] = sl + k < ncontrib ? __ldcg(pp + (sl + k) * slot_stride + (size_t)q * ROWS) : 0.f;
#pragma unroll
                            for (int k = 0; k < BATCH; ++k) {
                                if (sl + k >= ncontrib) break;
#pragma unroll
                                for (int q = 0; q < 16; ++q) acc[p][q] += t[k][q];
                            }
                        }
                    }
                }
            }
            if (ep.col_part && ctile != tile) {   // folded RMSNorm of the token operand
                bool have = false;
                if constexpr (!EPW) {
                    // the idle epilogue warps computed the first tile's scales during
                    // the main loop (bounded wait for their flag)
                    if (tid == 0) {
                        const uint64_t t0 = tc::global_ns();
                        while (*reinterpret_cast<volatile int *>(&cs.cscale_tile) < 0)
                            if (tc::global_ns() - t0 > tc::WAIT_LIMIT_NS) {
                                if (ep.err) atomicExch(ep.err, ERR_DFREE);
                                break;
                            }
                    }
                    named_bar_sync(TAIL_BAR, TAIL_THREADS);
                    have = *reinterpret_cast<volatile int *>(&cs.cscale_tile) == tile;
                }
                if (!have) {
                    griddep_wait();
                    fold_scale(ep, K, tok_base + tile * NT, max(0, min(NT, M - tile * NT)), tid, TAIL_THREADS, cs.cscale, NT);
                    named_bar_sync(TAIL_BAR, TAIL_THREADS);
                }
                ctile = tile;
            }
#pragma unroll
            for (int p = 0; p < PIECES; ++p) {
                const int cc = p * 64 + tg * 16;
                const int m0 = tile * NT + cc;
                const int mlim = cc < NT ? max(0, min(16, M - m0)) : 0;   // valid tokens in this piece
                float *y = acc[p];
                if (ep.col_part) {
#pragma unroll
                    for (int q = 0; q < 16; ++q) y[q] *= cs.cscale[cc + q];
                }
                if constexpr (OP == Q4Epilogue::STORE) {
                    store_rows(ep, f, m0, mlim, y);
                } else if constexpr (OP == Q4Epilogue::RESID) {
                    // every load of the piece is issued before its first store (the
                    // compiler cannot tell the pointers apart, so interleaving would
                    // serialise one L2 round trip per token)
#pragma unroll
                    for (int q = 0; q < 16; ++q) y[q] = q < mlim ? y[q] + ep.out[(size_t)(m0 + q) * ep.ldo + f] : 0.f;
                    if (!ep.norm_w) {
#pragma unroll
                        for (int q = 0; q < 16; ++q)
                            if (q < mlim) ep.out[(size_t)(m0 + q) * ep.ldo + f] = y[q];
                    } else {
                        // updated residual, the next linear's operand fp16(h * w * s), and
                        // this block's sum of squares per token
                        const float nw = ep.norm_w[f];
                        float sv[16];
#pragma unroll
                        for (int q = 0; q < 16; ++q) sv[q] = q < mlim ? __ldcg(ep.norm_scale + m0 + q) : 0.f;
                        float sq[16];
#pragma unroll
                        for (int q = 0; q < 16; ++q) {
                            const float v = y[q];
                            if (q < mlim) {
                                ep.out[(size_t)(m0 + q) * ep.ldo + f] = v;
                                ep.xout[xblk(m0 + q, f, ep.ldx_rows)] = __float2half_rn(v * nw * sv[q]);
                            }
                            sq[q] = v * v;
                        }
                        const float t2 = warp_sum16(sq, lane);
                        if (!(lane & 1)) cs.wsum2[tg][quarter][(lane >> 1) & 15] = t2;
                        named_bar_sync(TAIL_BAR, TAIL_THREADS);
                        if (tid < 64) {
                            const int tg2 = tid >> 4, q = tid & 15, cc2 = p * 64 + tg2 * 16;
                            const int m = tile * NT + cc2 + q;
                            if (cc2 < NT && m < M)
                                ep.norm_part[(size_t)blk * ep.norm_rows + m] =
                                    cs.wsum2[tg2][0][q] + cs.wsum2[tg2][1][q] + cs.wsum2[tg2][2][q] + cs.wsum2[tg2][3][q];
                        }
                        named_bar_sync(TAIL_BAR, TAIL_THREADS);
                    }
                } else if constexpr (OP == Q4Epilogue::SWIGLU) {
                    // rows [0,64) gate, [64,128) up of the same 64 outputs; token
                    // groups exchange through the buffer in two rounds of two
#pragma unroll
                    for (int ph = 0; ph < 2; ++ph) {
                        float *xch = cs.xch2[tg & 1];
                        const bool mine = (tg >> 1) == ph;
                        if (mine && r >= 64) {
#pragma unroll
                            for (int q = 0; q < 16; ++q) xch[(r - 64) * 16 + q] = y[q];
                        }
                        named_bar_sync(TAIL_BAR, TAIL_THREADS);
                        if (mine && r < 64) {
                            const int oi = blk * 64 + r;
#pragma unroll
                            for (int q = 0; q < 16; ++q) {
                                if (q >= mlim) break;
                                const float gv = y[q], uv = xch[r * 16 + q];
                                const float av = gv / (1.0f + expf(-gv)) * uv;
                                ep.xout[xblk(m0 + q, oi, ep.ldx_rows)] = __float2half_rn(av);
                            }
                        }
                        named_bar_sync(TAIL_BAR, TAIL_THREADS);
                    }
                } else {   // QKV
                    const int D = ep.head_dim;
                    const int hh = f / D;      // head index in q|k|v order
                    const int d = f % D;
                    const bool is_q = hh < ep.n_heads, is_k = !is_q && hh < ep.n_heads + ep.n_kv;
                    const float *nw = is_q ? ep.q_norm : (is_k ? ep.k_norm : nullptr);
                    const float nwd = nw ? nw[d] : 1.f;   // issued early: its latency overlaps the sums
                    // cache row and position of the piece's tokens, staged once in shared
                    // memory (the epilogue-warp buffer cs.xch is idle for QKV): the
                    // stores below then wait on no global loads
                    int *tok_pos = reinterpret_cast<int *>(cs.xch), *tok_row = tok_pos + 64;
                    if (tid < 64) {
                        const int tg2 = tid >> 4, q = tid & 15, cc2 = p * 64 + tg2 * 16;
                        const int m = tile * NT + cc2 + q;
                        const bool ok = cc2 < NT && m < M;
                        tok_pos[tid] = ok ? ep.tpos[m] : 0;
                        tok_row[tid] = ok ? ep.trow[m] : 0;
                    }
                    if (nw) {
                        // per-head sum of squares for each token: warp shuffles + smem
                        float sq[16];
#pragma unroll
                        for (int q = 0; q < 16; ++q) sq[q] = y[q] * y[q];
                        const float t2 = warp_sum16(sq, lane);
                        if (!(lane & 1)) cs.wsum2[tg][quarter][(lane >> 1) & 15] = t2;
                    }
                    named_bar_sync(TAIL_BAR, TAIL_THREADS);
                    if (ep.q_norm || ep.k_norm) {
                        // one thread per (token group, head of the block, token) turns the
                        // head's sum of squares into its rstd, kept in the head's first
                        // quarter slot; the head's rows then only multiply
                        const int wpk = D / 32, hpb = 4 / wpk;   // quarters per head, heads per block
                        if (tid < 4 * hpb * 16) {
                            const int tg2 = tid / (hpb * 16), hq = (tid / 16) % hpb, q = tid & 15;
                            float ss = 0.f;
                            for (int ww = hq * wpk; ww < hq * wpk + wpk; ++ww) ss += cs.wsum2[tg2][ww][q];
                            cs.wsum2[tg2][hq * wpk][q] = 1.0f / sqrtf(ss / (float)D + ep.eps);
                        }
                        named_bar_sync(TAIL_BAR, TAIL_THREADS);
                    }
                    if (nw) {
                        const int w0 = (quarter / (D / 32)) * (D / 32);
#pragma unroll
                        for (int q = 0; q < 16; ++q) y[q] = y[q] * cs.wsum2[tg][w0][q] * nwd;
                    }
                    // rotate-half RoPE on q and k: partner row r +- D/2, exchanged
                    // through the buffer in two rounds of two token groups
#pragma unroll
                    for (int ph = 0; ph < 2; ++ph) {
                        float *xch = cs.xch2[tg & 1];
                        const bool mine = (tg >> 1) == ph;
                        if (mine) {
#pragma unroll
                            for (int q = 0; q < 16; ++q) xch[r * 16 + q] = y[q];
                        }
                        named_bar_sync(TAIL_BAR, TAIL_THREADS);
                        if (mine && (is_q || is_k)) {
                            const int half = D / 2;
                            const int pr = d < half ? r + half : r - half;
#pragma unroll
                            for (int q = 0; q < 16; ++q) {
                                if (q >= mlim) break;
                                const float2 csn = ep.rope[(size_t)tok_pos[tg * 16 + q] * half + d % half];
                                const float sn = csn.y, cn = csn.x;
                                const float pv = xch[pr * 16 + q];
                                y[q] = d < half ? y[q] * cn - pv * sn : pv * sn + y[q] * cn;
                            }
                        }
                        named_bar_sync(TAIL_BAR, TAIL_THREADS);
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
                                  (((size_t)tok_row[tg * 16 + q] * ep.n_kv + kvh) * ep.max_len + tok_pos[tg * 16 + q]) * D;
                        }
                        dst[d] = __float2half_rn(y[q]);
                    }
                }
            }
            }
        };
        int b = u0 / nc, c = u0 - b * nc, seg = 0;
        int s = 0, wpar = 0;            // W stage of the current unit and its phase parity
        int as = 0;                     // ring slot (A buffer, x stage) of the current sub-chunk
        uint32_t mpar = 0;              // per slot: parity of its next MMA-completion wait
        const uint32_t lane_col = lane_base + (uint32_t)(g * 32);
        const int sw_off = (((2 * g) ^ sw8) << 4), sw_off1 = (((2 * g + 1) ^ sw8) << 4);
        for (int j = 0; j < nsub; ++j) {
            const int h = j & 1;
            // the W stage of this sub-chunk: half h of the unit's stage, or a stage of
            // its own for the wide tile
            const bool stage_first = C::WIDE || h == 0, stage_last = C::WIDE || h == 1;
            const unsigned char *wst = wring + (size_t)s * C::WSTAGE;
            bool ok = true;
            if (stage_first) {
                if (lane == 0) ok = wait_or_abort(tc::smem_u32(&cs.full_w[s]), wpar, abort_flag, ep.err, ERR_WFULL);
                ok = __shfl_sync(0xffffffffu, ok, 0);
            }
            const unsigned char *wt = wst + (C::WIDE ? 0 : h * WBOX) + r * 128;
            const uint4 w0 = *reinterpret_cast<const uint4 *>(wt + sw_off);
            const uint4 w1 = *reinterpret_cast<const uint4 *>(wt + sw_off1);
            const uint32_t *sbs = reinterpret_cast<const uint32_t *>(wst + (C::WIDE ? WBOX : 2 * WBOX));
            const uint32_t sbv = sbs[((C::WIDE ? 0 : h * 4) + g) * ROWS + r];
            const int s_read = s;           // released once its values are in TMEM
            if (stage_last && ++s == sw) { s = 0; wpar ^= 1; }
            if (j >= R) {   // the MMAs that last read this A buffer have completed
                if (lane == 0)
                    ok = ok && wait_or_abort(tc::smem_u32(&cs.mma_done[as]), (mpar >> as) & 1, abort_flag, ep.err,
                                             ERR_MDONE);
                mpar ^= 1u << as;
                ok = __shfl_sync(0xffffffffu, ok, 0);
                tc::fence_after_sync();
            }
            if (ok) {
                const GroupConst kc(sbv);
                const uint32_t ta = tmem + lane_col + (uint32_t)(as * A_COLS);
                uint32_t a[16];
                dequant16(w0, kc, a);
                tc::tmem_st16(ta + 0, a);
                dequant16(w1, kc, a);
                tc::tmem_st16(ta + 16, a);
                tc::tmem_wait_st();
            }
            if (stage_last) {
                // the stage goes back to the producer only once the values read
                // from it are in TMEM: handing it back right after the loads were
                // issued let the next TMA write race them
                __syncwarp();
                if (lane == 0) tc::mbar_arrive(tc::smem_u32(&cs.w_free[s_read]));
            }
            tc::fence_before_sync();
            named_bar_arrive(1 + is * MAX_AST + as, C::BAR_COUNT);
            if (++as == R) as = 0;

            const int ub = b, uc = c;            // block / unit of this sub-chunk
            if (h == 1 && ++c == nc) { c = 0; ++b; }
            if (h != 1 || (uc != nc - 1 && j != nsub - 1)) continue;
            // end of a block segment: the epilogue warps take the non-last ones of
            // the cheap epilogues; everything else is done here
            const bool last_seg = j == nsub - 1;
            if (!(EPW && !last_seg)) seg_epilogue(ub, seg, !last_seg);
            ++seg;
        }
    } else if (!EPW && warp >= EP_WARP0) {
        // idle in QKV and SWIGLU: the folded-norm scales of the first token tile,
        // computed while the main loop runs (the tail epilogue picks them up)
        if (ep.col_part) {
            const int et = tid - EP_WARP0 * 32;
            const int tile0 = u0 / (nblk * nc);
            griddep_wait();   // the sums of squares come from the previous kernel
            fold_scale(ep, K, tok_base + tile0 * NT, max(0, min(NT, M - tile0 * NT)), et, EP_THREADS, cs.cscale, NT);
            named_bar_sync(EPI_BAR, EP_THREADS);
            if (et == 0) {
                __threadfence_block();
                *reinterpret_cast<volatile int *>(&cs.cscale_tile) = tile0;
            }
        }
    } else if (EPW && warp >= EP_WARP0) {
        // ---------------- epilogue warps: one thread per row, all tokens ----------------
        const int quarter = warp & 3;
        const int r = quarter * 32 + lane;
        const int etid = tid - EP_WARP0 * 32;    // 0..127
        const uint32_t lane_base = (uint32_t)(quarter * 32) << 16;
        int seg = 0, dset = 0;
        int ctile = -1;                          // token tile whose folded-norm scales are in cs.xch
        for (int ub = u0 / nc; ub < (u1 - 1) / nc; ++ub, ++seg) {   // all but the last segment
            const int seg_first_unit = max(u0, ub * nc), seg_last_unit = min(u1 - 1, ub * nc + nc - 1);
            const bool full = seg_first_unit == ub * nc && seg_last_unit == ub * nc + nc - 1;
            const int tile = ub / nblk, blk = ub - tile * nblk;
            const int f = blk * ROWS + r;
            bool bad = *abort_flag != 0;
            if (lane == 0 && !bad)
                bad = !wait_or_abort(tc::smem_u32(&cs.d_full[dset]), (seg / C::DSETS) & 1, abort_flag, ep.err,
                                     ERR_DFREE);
            bad = __shfl_sync(0xffffffffu, bad, 0);
            const bool skip = named_bar_or(EPI_BAR, EP_THREADS, bad);
            if (skip) *abort_flag = 1;
            tc::fence_after_sync();
            const uint32_t dbase = tmem + lane_base + C::D_COL + dset * C::NI * C::DCOLS;
            // the accumulators of piece p (16 tokens), summed over the issuers
            auto load_piece = [&](int p, float *y) {
#pragma unroll
                for (int q = 0; q < 16; ++q) y[q] = 0.f;
#pragma unroll
                for (int d = 0; d < C::NI; ++d) {
                    uint32_t v[16];
                    tc::tmem_ld16(dbase + d * C::DCOLS + p * 16, v);
                    tc::tmem_wait_ld();
#pragma unroll
                    for (int q = 0; q < 16; ++q) y[q] += __uint_as_float(v[q]);
                }
            };
            float *pblk = nullptr;
            int ncontrib = 1, last = 1;
            if (!skip && !full) {
                // partial block: slot of this CTA among the block's contributors,
                // stored [slot][token][row] (a warp writes 128 contiguous bytes)
                const int first_owner = unit_owner(ub * nc, U, G);
                ncontrib = unit_owner(ub * nc + nc - 1, U, G) - first_owner + 1;
                pblk = ep.part + (size_t)ub * pmax * NT * ROWS;
                float *mine = pblk + (size_t)(cta - first_owner) * NT * ROWS + r;
                for (int p = 0; p < C::PIECES; ++p) {
                    float y[16];
                    load_piece(p, y);
#pragma unroll
                    for (int q = 0; q < 16; ++q) mine[(size_t)(p * 16 + q) * ROWS] = y[q];
                }
            }
            if (!skip && !full) {
                tc::fence_before_sync();
                __syncwarp();
                if (lane == 0) tc::mbar_arrive(tc::smem_u32(&cs.d_free[dset]));   // accumulators read
                // the barrier orders every thread's partial stores before thread 0's
                // gpu-scope fence (fences are cumulative), which orders them before
                // the ticket; the last contributor fences again before releasing its
                // readers
                named_bar_sync(EPI_BAR, EP_THREADS);
                if (etid == 0) {
                    unsigned *ctr = ep.counters + ub;
                    __threadfence();
                    const unsigned prev = atomicAdd(ctr, 1u);
                    const int lst = prev == (unsigned)(ncontrib - 1);
                    if (lst) {
                        *ctr = 0u;   // ready for the next launch
                        __threadfence();
                    }
                    cs.last_flag = lst;
                }
                named_bar_sync(EPI_BAR, EP_THREADS);
                last = cs.last_flag;
            }
            if (!skip && last) {
                if (ep.col_part && ctile != tile) {   // folded RMSNorm of the token operand (STORE only)
                    griddep_wait();
                    fold_scale(ep, K, tok_base + tile * NT, max(0, min(NT, M - tile * NT)), etid, EP_THREADS, cs.xch, NT);
                    named_bar_sync(EPI_BAR, EP_THREADS);
                    ctile = tile;
                }
                for (int p = 0; p < C::PIECES; ++p) {
                    float y[16];
                    if (full) {
                        load_piece(p, y);
                        if (p == C::PIECES - 1) {   // accumulators read: the issuers may reuse them
                            tc::fence_before_sync();
                            __syncwarp();
                            if (lane == 0) tc::mbar_arrive(tc::smem_u32(&cs.d_free[dset]));
                        }
                    } else {
                        // slots summed in slot order, two slots' loads in flight
#pragma unroll
                        for (int q = 0; q < 16; ++q) y[q] = 0.f;
                        const float *pp = pblk + (size_t)(p * 16) * ROWS + r;
                        const size_t slot_stride = (size_t)NT * ROWS;
                        for (int sl = 0; sl < ncontrib; sl += 2) {
                            float t[2][16];
#pragma unroll
                            for (int k = 0; k < 2; ++k)
#pragma unroll
                                for (int q = 0; q < 16; ++q)
                                    t[k][q] = sl + k < ncontrib ? __ldcg(pp + (sl + k) * slot_stride + (size_t)q * ROWS) : 0.f;
#pragma unroll
                            for (int k = 0; k < 2; ++k) {
                                if (sl + k >= ncontrib) break;
#pragma unroll
                                for (int q = 0; q < 16; ++q) y[q] += t[k][q];
                            }
                        }
                    }
                    const int m0 = tile * NT + p * 16;
                    const int mlim = max(0, min(16, M - m0));   // valid tokens in this piece
                    if (ep.col_part) {
#pragma unroll
                        for (int q = 0; q < 16; ++q) y[q] *= cs.xch[p * 16 + q];
                    }
                    if constexpr (OP == Q4Epilogue::STORE) {
                        store_rows(ep, f, m0, mlim, y);
                    } else if constexpr (OP == Q4Epilogue::RESID) {
                        // loads of the piece before its stores (see the tail epilogue)
#pragma unroll
                        for (int q = 0; q < 16; ++q) y[q] = q < mlim ? y[q] + ep.out[(size_t)(m0 + q) * ep.ldo + f] : 0.f;
                        if (!ep.norm_w) {
#pragma unroll
                            for (int q = 0; q < 16; ++q)
                                if (q < mlim) ep.out[(size_t)(m0 + q) * ep.ldo + f] = y[q];
                        } else {
                            // updated residual, the next linear's operand fp16(h * w * s), and
                            // this block's sum of squares per token
                            const float nw = ep.norm_w[f];
                            float sv[16];
#pragma unroll
                            for (int q = 0; q < 16; ++q) sv[q] = q < mlim ? __ldcg(ep.norm_scale + m0 + q) : 0.f;
                            float sq[16];
#pragma unroll
                            for (int q = 0; q < 16; ++q) {
                                const float v = y[q];
                                if (q < mlim) {
                                    ep.out[(size_t)(m0 + q) * ep.ldo + f] = v;
                                    ep.xout[xblk(m0 + q, f, ep.ldx_rows)] = __float2half_rn(v * nw * sv[q]);
                                }
                                sq[q] = v * v;
                            }
                            const float t2 = warp_sum16(sq, lane);
                            if (!(lane & 1)) cs.wsum[quarter][(lane >> 1) & 15] = t2;
                            named_bar_sync(EPI_BAR, EP_THREADS);
                            if (etid < mlim)
                                ep.norm_part[(size_t)blk * ep.norm_rows + m0 + etid] =
                                    cs.wsum[0][etid] + cs.wsum[1][etid] + cs.wsum[2][etid] + cs.wsum[3][etid];
                            named_bar_sync(EPI_BAR, EP_THREADS);
                        }
                    }
                }
            } else if (!skip && full) {
                // unreachable: a full block always has last = 1
            }
            if (skip && lane == 0) {
                // keep the issuers' accumulator waits balanced after an abort
            }
            if (++dset == C::DSETS) dset = 0;
        }
    }
    if (OP == Q4Epilogue::STORE && ep.peers) __threadfence_system();   // this thread's peer stores
    tc::fence_before_sync();
    __syncthreads();
    if (warp == 0) {
        tc::fence_after_sync();
        tc::tmem_dealloc(tmem, 512);
    }
    if (OP == Q4Epilogue::STORE && ep.peers && tid == 0 && atomicAdd(ep.peer_ctr, 1u) == (unsigned)G - 1) {
        // every CTA's partial sums are stored: flag every owner
        *ep.peer_ctr = 0u;
        __threadfence_system();
        const unsigned flag = *ep.peer_flag * 512u + (unsigned)ep.peer_call + 1u;
        for (int d = 0; d < ep.peer_n; ++d)
            tc::st_release_sys(reinterpret_cast<unsigned *>(ep.peers[d] + ep.peer_flag_off), flag);
    }
}

// (scale, bias) fp16 pairs of rows blk*128.. and groups 8c.. of unit (blk, c):
// sbp[((blk * nc + c) * 8 + gi) * 128 + r]; groups past K are zero
__global__ void pack_sb_kernel(const __half *__restrict__ scales, const __half *__restrict__ biases, int N, int K,
                               uint32_t *__restrict__ sbp) {
    const int KG = K / MLXCAT_GS, nc = (K + KU - 1) / KU;
    const long long total = (long long)N * nc * 8;
    for (long long t = (long long)blockIdx.x * blockDim.x + threadIdx.x; t < total;
         t += (long long)gridDim.x * blockDim.x) {
        const int r = (int)(t % ROWS);
        const long long rest = t / ROWS;
        const int gi = (int)(rest % 8);
        const long long bc = rest / 8;
        const int c = (int)(bc % nc), blk = (int)(bc / nc);
        const int row = blk * ROWS + r, grp = c * 8 + gi;
        __half2 v = __halves2half2(__float2half(0.f), __float2half(0.f));
        if (grp < KG) v = __halves2half2(scales[(size_t)row * KG + grp], biases[(size_t)row * KG + grp]);
        sbp[t] = *reinterpret_cast<uint32_t *>(&v);
    }
}

// ---------------------------------------------------------------------------
// host side: tensor maps and launch
// ---------------------------------------------------------------------------

constexpr size_t SMEM_LIMIT = 227 * 1024;

template <int NT>
size_t smem_for(int sw) {
    return 1024 + (size_t)sw * Cfg<NT>::WSTAGE + (size_t)Cfg<NT>::AST * Cfg<NT>::XSTAGE + sizeof(Smem);
}

// deepest W ring that fits the shared memory of one CTA
template <int NT>
int stages_for() {
    for (int sw = MAX_SW; sw > 2; --sw)
        if (smem_for<NT>(sw) <= SMEM_LIMIT) return sw;
    return 2;
}

template <int NT, int OP>
cudaError_t launch_op(const Q4WeightTC &w, const CUtensorMap &xmap, int M, int tok_base, int tiles,
                      int sm_count, const Q4Epilogue &ep, cudaStream_t st) {
    static bool attr[64] = {};   // per instantiation
    int dev = 0;
    cudaGetDevice(&dev);
    static_assert(1024 + 2 * Cfg<NT>::WSTAGE + Cfg<NT>::AST * Cfg<NT>::XSTAGE + sizeof(Smem) <= SMEM_LIMIT,
                  "two W stages, the x ring and the CTA state must fit one CTA's shared memory");
    const int sw = stages_for<NT>();
    const size_t sm = smem_for<NT>(sw);
    if (sm > SMEM_LIMIT) return cudaErrorInvalidConfiguration;
    if (!attr[dev & 63]) {
        cudaError_t e = cudaFuncSetAttribute(q4_tc_kernel<NT, OP>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm);
        if (e != cudaSuccess) return e;
        attr[dev & 63] = true;
    }
    const int nblk = w.N / ROWS, nc = (w.K + KU - 1) / KU;
    const int U = tiles * nblk * nc;
    const int G = U < sm_count ? U : sm_count;
    const int pmax = q4_tc_pmax(U, G, nc);
    if (pmax > 1 && (!ep.part || !ep.counters)) return cudaErrorInvalidValue;
    if ((unsigned long long)U * (unsigned long long)(G + 1) >= (1ull << 32)) return cudaErrorInvalidValue;
    if (OP == Q4Epilogue::RESID && ep.norm_w &&
        (!ep.xout || !ep.norm_scale || !ep.norm_part || tok_base != 0 || M > ep.ldx_rows || M > ep.norm_rows))
        return cudaErrorInvalidValue;
    if (ep.col_part && (!ep.col_prev || w.K % 128 || tok_base + M > ep.norm_rows)) return cudaErrorInvalidValue;
    // the QKV epilogue keeps every head inside one 128-row block
    if (OP == Q4Epilogue::QKV && (ep.head_dim < 32 || ROWS % ep.head_dim)) return cudaErrorInvalidValue;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(G);
    cfg.blockDim = dim3(THREADS);
    cfg.dynamicSmemBytes = sm;
    cfg.stream = st;
    cudaLaunchAttribute attr1[1];
    attr1[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr1[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr1;
    cfg.numAttrs = ep.pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, q4_tc_kernel<NT, OP>, w.map, xmap, w.sbp, w.N, w.K, M, tok_base, nblk, nc, U, pmax,
                              sw, ep);
}

template <int NT>
cudaError_t launch_nt(const Q4WeightTC &w, const CUtensorMap &xmap, int M, int tok_base, int tiles,
                      int sm_count, const Q4Epilogue &ep, cudaStream_t st) {
    switch (ep.op) {
    case Q4Epilogue::STORE: return launch_op<NT, Q4Epilogue::STORE>(w, xmap, M, tok_base, tiles, sm_count, ep, st);
    case Q4Epilogue::RESID: return launch_op<NT, Q4Epilogue::RESID>(w, xmap, M, tok_base, tiles, sm_count, ep, st);
    case Q4Epilogue::SWIGLU: return launch_op<NT, Q4Epilogue::SWIGLU>(w, xmap, M, tok_base, tiles, sm_count, ep, st);
    case Q4Epilogue::QKV: return launch_op<NT, Q4Epilogue::QKV>(w, xmap, M, tok_base, tiles, sm_count, ep, st);
    default: return cudaErrorInvalidValue;
    }
}

}  // namespace

bool make_weight_map(Q4WeightTC &w) {
    auto fn = encode_fn();
    if (!fn) return false;
    const cuuint64_t dims[2] = {(cuuint64_t)(w.K / 2), (cuuint64_t)w.N};   // boxes past K read 0
    const cuuint64_t strides[1] = {(cuuint64_t)(w.K / 2)};
    const cuuint32_t box[2] = {128, ROWS};
    const cuuint32_t es[2] = {1, 1};
    return fn(&w.map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<uint32_t *>(w.wq), dims, strides, box, es,
              CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

size_t q4_sbp_words(int N, int K) { return (size_t)N * ((K + KU - 1) / KU) * 8; }

cudaError_t pack_q4_sb(const __half *scales, const __half *biases, int N, int K, uint32_t *sbp, cudaStream_t st) {
    if (N % ROWS || K % MLXCAT_GS || !scales || !biases || !sbp) return cudaErrorInvalidValue;
    const long long total = (long long)q4_sbp_words(N, K);
    const int threads = 256;
    const long long want = (total + threads - 1) / threads;
    const unsigned blocks = (unsigned)(want < 4096 ? want : 4096);
    pack_sb_kernel<<<blocks, threads, 0, st>>>(scales, biases, N, K, sbp);
    return cudaGetLastError();
}

// token tile of the two-issuer launches: the fewest tiles of at most 128
// tokens, split evenly (M = 160 -> two tiles of 80, not 128 + 32 padded to
// 128: the token-operand loads and the epilogue scale with the tile width)
int q4_tc_tile(int M) {
    const int tiles = (M + 127) / 128;
    const int per = (M + tiles - 1) / tiles;
    return ((per + 15) / 16) * 16;
}

// token tile of one launch: the gate/up projection (SWIGLU epilogue) runs
// 129..160 tokens as one tile (one pass of its 117 M weights instead of two;
// its kernel span 75 -> 60 us at the Llama-3-8B verify shape), the other
// projections as two (one wide tile measured slower for them)
int q4_tc_launch_tile(int M, int op) {
    if (op == Q4Epilogue::SWIGLU && M > 128 && M <= MAX_NT) return ((M + 15) / 16) * 16;
    return q4_tc_tile(M);
}

// most CTAs that share one row block (stream-K contributors)
int q4_tc_pmax(int U, int G, int nc) {
    // a CTA covers floor(U/G) or ceil(U/G) units; a block of nc units meets at most
    // ceil((nc - 1) / floor(U/G)) + 1 of them
    const int per = U / G > 0 ? U / G : 1;
    return (nc - 1 + per - 1) / per + 1;
}

// split-K partials / tickets of a launch: enough for either tiling of M
size_t q4_tc_partial_floats(int N, int K, int M, int sm_count) {
    size_t most = 0;
    for (const int nt : {q4_tc_tile(M), q4_tc_launch_tile(M, Q4Epilogue::SWIGLU)}) {
        const int tiles = (M + nt - 1) / nt;
        const int nblk = N / ROWS, nc = (K + KU - 1) / KU;
        const int U = tiles * nblk * nc, G = U < sm_count ? U : sm_count;
        most = std::max(most, (size_t)tiles * nblk * q4_tc_pmax(U, G, nc) * ROWS * nt);
    }
    return most;
}

size_t q4_tc_counters(int N, int M) {
    const int nt = q4_tc_tile(M);   // the one-tile launch has fewer blocks to count
    return (size_t)((M + nt - 1) / nt) * (N / ROWS);
}

cudaError_t q4_tc(const Q4WeightTC &w, const __half *x_blk, int ldx_rows, int tok_base, int M,
                  int sm_count, const Q4Epilogue &ep, cudaStream_t st) {
    if (w.N % ROWS || w.K % 128 || M <= 0 || tok_base + M > ldx_rows || !w.sbp) return cudaErrorInvalidValue;
    auto fn = encode_fn();
    if (!fn) return cudaErrorNotSupported;
    const int nt = q4_tc_launch_tile(M, ep.op);
    const int tiles = (M + nt - 1) / nt;
    // token operand [K/64][ldx_rows][64] fp16 -> 3-D map (64, rows, K/64)
    CUtensorMap xmap;
    const cuuint64_t dims[3] = {64, (cuuint64_t)ldx_rows, (cuuint64_t)(w.K / 64)};   // boxes past K read 0
    const cuuint64_t strides[2] = {128, (cuuint64_t)ldx_rows * 128};
    const cuuint32_t box[3] = {64, (cuuint32_t)nt, KS / 64};
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
    case 128: return launch_nt<128>(w, xmap, M, tok_base, tiles, sm_count, ep, st);
    case 144: return launch_op<144, Q4Epilogue::SWIGLU>(w, xmap, M, tok_base, tiles, sm_count, ep, st);
    case 160: return launch_op<160, Q4Epilogue::SWIGLU>(w, xmap, M, tok_base, tiles, sm_count, ep, st);
    default: return cudaErrorInvalidValue;
    }
}

}  // namespace mlxcat
