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
// of the verify batch (16..128) its N dimension.
//
//   warp 4 (one lane)   TMA: weight tile [128 rows x 64 B] (64B swizzle) and
//                       token tile [NT x 128 k] (128B swizzle) per 128-k chunk
//                       into a ring of shared-memory stages; then issues the
//                       eight tcgen05.mma (M=128, N=NT, K=16) of the chunk with
//                       A from tensor memory and B from shared memory, and
//                       commits them to the stage's mbarrier.
//   warps 0-3           one weight row per thread: 64 bytes from the staged
//                       tile, nibbles unpacked with the 0x6400 fp16 magic and
//                       dequantised in registers (hfma2 / hadd2), stored into
//                       tensor memory (tcgen05.st, two A stages) as the MMA's
//                       A operand; afterwards the epilogue reads the fp32
//                       accumulator back with tcgen05.ld.
//
// Inside each 8-wide k block the unpack order is (0,4,1,5,2,6,3,7); the token
// operand is stored in the same order by its producers (common.cuh: perm8).
//
// Split-K across CTAs (grid.y): each CTA writes its fp32 partial; the last CTA
// of a feature block (atomic ticket) sums all partials in split order --
// deterministic -- and runs the epilogue:
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

namespace {

constexpr int ROWS = 128;          // weight rows per CTA (MMA M)
constexpr int CHUNK = 128;         // k per pipeline stage
constexpr int DQ_THREADS = 128;    // dequant / epilogue warps 0-3
constexpr int THREADS = 160;       // + producer / MMA warp
constexpr int A_COLS = 64;         // TMEM columns of one A stage (128 k fp16)
constexpr int D_COL = 2 * A_COLS;  // accumulator columns start

enum ErrCode { ERR_FULL = 1, ERR_AFULL = 2, ERR_MMA = 3, ERR_DONE = 4 };

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
    uint64_t full[8], mma_done[8], a_full[2];
    uint32_t tmem_base;
    int abort_flag;
    int last_flag;
    float wsum[4][32];
};

template <int NT>
__global__ void __launch_bounds__(THREADS, 1)
q4_tc_kernel(const __grid_constant__ CUtensorMap wmap, const __grid_constant__ CUtensorMap xmap,
             const __half *__restrict__ scales, const __half *__restrict__ biases, int N, int K,
             int M, int cps, int stages, Q4Epilogue ep) {
    extern __shared__ __align__(1024) unsigned char smem_raw[];
    // 1024-byte aligned stage ring; control block after it
    unsigned char *ring = reinterpret_cast<unsigned char *>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
    constexpr int XBYTES = 2 * NT * 128;                 // two 64-k boxes
    constexpr int STAGE = XBYTES + ROWS * 64;            // + weight tile
    Smem &cs = *reinterpret_cast<Smem *>(ring + (size_t)stages * STAGE);

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int blk = blockIdx.x, split = blockIdx.y, tile = blockIdx.z;
    const int nchunks = K / CHUNK;
    const int c_begin = split * cps;
    const int n = min(nchunks, c_begin + cps) - c_begin;
    const int tok0 = tile * NT;
    const uint32_t ring_a = tc::smem_u32(ring);

    if (warp == 4 && lane == 0) {
        for (int s = 0; s < stages; ++s) {
            tc::mbar_init(tc::smem_u32(&cs.full[s]), 1);
            tc::mbar_init(tc::smem_u32(&cs.mma_done[s]), 1);
        }
        tc::mbar_init(tc::smem_u32(&cs.a_full[0]), 4);
        tc::mbar_init(tc::smem_u32(&cs.a_full[1]), 4);
        cs.abort_flag = 0;
        tc::fence_barrier_init();
        tc::prefetch_tmap(&wmap);
        tc::prefetch_tmap(&xmap);
    }
    if (warp == 0) tc::tmem_alloc(tc::smem_u32(&cs.tmem_base), 256);
    tc::fence_before_sync();
    __syncthreads();
    tc::fence_after_sync();
    const uint32_t tmem = cs.tmem_base;
    volatile int *abort_flag = &cs.abort_flag;

    if (warp == 4) {
        if (lane == 0) {
            // ---------------- producer + MMA issuer ----------------
            const uint32_t idesc = tc::idesc_f16_f32(ROWS, NT);
            auto issue = [&](int i) {
                const int s = i % stages;
                const uint32_t st = ring_a + (uint32_t)(s * STAGE);
                const uint32_t bar = tc::smem_u32(&cs.full[s]);
                tc::mbar_arrive_expect_tx(bar, STAGE);
                const int kc = (c_begin + i) * CHUNK;
                tc::tma_load_2d(st, &xmap, kc, tok0, bar);
                tc::tma_load_2d(st + NT * 128, &xmap, kc + 64, tok0, bar);
                tc::tma_load_2d(st + XBYTES, &wmap, kc / 2, blk * ROWS, bar);
            };
            int issued = 0;
            for (; issued < min(stages - 1, n); ++issued) issue(issued);
            int done = 0;   // chunks whose MMAs were committed
            for (int i = 0; i < n && !*abort_flag; ++i) {
                const int s = i % stages, ts = i & 1;
                if (!tc::mbar_wait(tc::smem_u32(&cs.full[s]), (i / stages) & 1, ep.err, ERR_FULL) ||
                    !tc::mbar_wait(tc::smem_u32(&cs.a_full[ts]), (i >> 1) & 1, ep.err, ERR_AFULL)) {
                    *abort_flag = 1;
                    break;
                }
                tc::fence_after_sync();
                const uint32_t xs = ring_a + (uint32_t)(s * STAGE);
#pragma unroll
                for (int kk = 0; kk < CHUNK / 16; ++kk) {
                    const uint32_t baddr = xs + (uint32_t)((kk >> 2) * NT * 128 + (kk & 3) * 32);
                    tc::mma_ts_f16(tmem + D_COL, tmem + ts * A_COLS + kk * 8, tc::sdesc_k_sw128(baddr), idesc,
                                   (i > 0 || kk > 0) ? 1u : 0u);
                }
                tc::mma_commit(tc::smem_u32(&cs.mma_done[s]));
                done = i + 1;
                // refill: chunk j reuses the stage of chunk j - stages = i - 1
                const int j = i + stages - 1;
                if (j < n) {
                    if (j >= stages) {
                        const int pc = j - stages;
                        if (!tc::mbar_wait(tc::smem_u32(&cs.mma_done[pc % stages]), (pc / stages) & 1,
                                           ep.err, ERR_MMA)) { *abort_flag = 1; break; }
                    }
                    issue(j);
                    issued = j + 1;
                }
            }
            if (*abort_flag) {
                // drain: every issued copy lands, every committed MMA completes
                for (int i = done; i < issued; ++i)
                    tc::mbar_wait(tc::smem_u32(&cs.full[i % stages]), (i / stages) & 1, nullptr, 0);
                if (done > 0) {
                    const int pc = done - 1;
                    tc::mbar_wait(tc::smem_u32(&cs.mma_done[pc % stages]), (pc / stages) & 1, nullptr, 0);
                }
            }
        }
    } else {
        // ---------------- dequant warps: one weight row per thread ----------------
        const int r = tid;                       // 0..127
        const int f = blk * ROWS + r;
        const uint32_t lane_base = (uint32_t)(warp * 32) << 16;
        const size_t KG = (size_t)K / MLXCAT_GS;
        const __half2 *srow = reinterpret_cast<const __half2 *>(scales + (size_t)f * KG);
        const __half2 *brow = reinterpret_cast<const __half2 *>(biases + (size_t)f * KG);
        __half2 sc_next = srow[c_begin], bi_next = brow[c_begin];
        for (int i = 0; i < n; ++i) {
            const int s = i % stages, ts = i & 1;
            const __half2 sc = sc_next, bi = bi_next;
            if (i + 1 < n) { sc_next = srow[c_begin + i + 1]; bi_next = brow[c_begin + i + 1]; }
            bool ok = tc::mbar_wait(tc::smem_u32(&cs.full[s]), (i / stages) & 1, ep.err, ERR_FULL);
            if (!ok) *abort_flag = 1;
            uint4 w[4];
            const unsigned char *wt = ring + (size_t)s * STAGE + XBYTES + r * 64;
#pragma unroll
            for (int j = 0; j < 4; ++j)
                w[j] = *reinterpret_cast<const uint4 *>(wt + ((j ^ ((r >> 1) & 3)) << 4));
            uint32_t a[64];
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                // words 0..7 of the chunk belong to group 2c, 8..15 to 2c+1
                const __half2 s1 = (j < 2) ? __low2half2(sc) : __high2half2(sc);
                const __half2 b2 = (j < 2) ? __low2half2(bi) : __high2half2(bi);
                const __half2 m1 = __hmul2(s1, __float2half2_rn(-1024.0f));
                const __half2 s16 = __hmul2(s1, __float2half2_rn(0.0625f));
                const __half2 m64 = __hmul2(s1, __float2half2_rn(-64.0f));
                dequant_word(w[j].x, s1, m1, s16, m64, b2, &a[16 * j + 0]);
                dequant_word(w[j].y, s1, m1, s16, m64, b2, &a[16 * j + 4]);
                dequant_word(w[j].z, s1, m1, s16, m64, b2, &a[16 * j + 8]);
                dequant_word(w[j].w, s1, m1, s16, m64, b2, &a[16 * j + 12]);
            }
            if (ok && i >= 2) {
                const int pc = i - 2;   // last chunk that used this A stage
                ok = tc::mbar_wait(tc::smem_u32(&cs.mma_done[pc % stages]), (pc / stages) & 1, ep.err, ERR_MMA);
                if (!ok) *abort_flag = 1;
            }
            if (__any_sync(0xffffffffu, !ok || *abort_flag)) { *abort_flag = 1; break; }
            const uint32_t ta = tmem + lane_base + (uint32_t)(ts * A_COLS);
            tc::tmem_st16(ta + 0, &a[0]);
            tc::tmem_st16(ta + 16, &a[16]);
            tc::tmem_st16(ta + 32, &a[32]);
            tc::tmem_st16(ta + 48, &a[48]);
            tc::tmem_wait_st();
            tc::fence_before_sync();
            __syncwarp();
            if (lane == 0) tc::mbar_arrive(tc::smem_u32(&cs.a_full[ts]));
        }
        // ---------------- epilogue ----------------
        // every dequant thread waits for the last commit; the decision to run
        // the epilogue is made uniform across the four warps by a reducing barrier
        bool bad = *abort_flag != 0;
        if (!bad) {
            const int pc = n - 1;
            bad = !tc::mbar_wait(tc::smem_u32(&cs.mma_done[pc % stages]), (pc / stages) & 1, ep.err, ERR_DONE);
        }
        const bool ok = !named_bar_or(1, DQ_THREADS, bad);
        if (ok) {
            tc::fence_after_sync();
            const int splits = gridDim.y;
            const int nblk = gridDim.x;
            float *part = ep.part + (((size_t)tile * splits) * N) * NT;   // [split][N][NT] of this tile
            bool last = true;
            if (splits > 1) {
                float *mine = part + ((size_t)split * N + f) * NT;
#pragma unroll
                for (int c = 0; c < NT; c += 16) {
                    uint32_t v[16];
                    tc::tmem_ld16(tmem + lane_base + D_COL + c, v);
                    tc::tmem_wait_ld();
#pragma unroll
                    for (int q = 0; q < 16; q += 4)
                        *reinterpret_cast<float4 *>(mine + c + q) =
                            make_float4(__uint_as_float(v[q]), __uint_as_float(v[q + 1]),
                                        __uint_as_float(v[q + 2]), __uint_as_float(v[q + 3]));
                }
                __threadfence();
                named_bar_sync(1, DQ_THREADS);
                if (tid == 0) {
                    unsigned *ctr = ep.counters + (size_t)tile * nblk + blk;
                    const unsigned prev = atomicAdd(ctr, 1u);
                    cs.last_flag = prev == (unsigned)(splits - 1);
                    if (cs.last_flag) *ctr = 0u;   // ready for the next launch
                }
                named_bar_sync(1, DQ_THREADS);
                last = cs.last_flag != 0;
                if (last) __threadfence();
            }
            if (last) {
                float *xch = reinterpret_cast<float *>(ring);   // [128][16] exchange (stages are idle)
                for (int c = 0; c < NT; c += 16) {
                    float y[16];
                    if (splits > 1) {
#pragma unroll
                        for (int q = 0; q < 16; ++q) y[q] = 0.f;
                        for (int s = 0; s < splits; ++s) {
                            const float *p = part + ((size_t)s * N + f) * NT + c;
#pragma unroll
                            for (int q = 0; q < 16; q += 4) {
                                const float4 t4 = *reinterpret_cast<const float4 *>(p + q);
                                y[q] += t4.x; y[q + 1] += t4.y; y[q + 2] += t4.z; y[q + 3] += t4.w;
                            }
                        }
                    } else {
                        uint32_t v[16];
                        tc::tmem_ld16(tmem + lane_base + D_COL + c, v);
                        tc::tmem_wait_ld();
#pragma unroll
                        for (int q = 0; q < 16; ++q) y[q] = __uint_as_float(v[q]);
                    }
                    const int m0 = tok0 + c;
                    if (ep.op == Q4Epilogue::STORE) {
                        for (int q = 0; q < 16; ++q)
                            if (m0 + q < M) ep.out[(size_t)(m0 + q) * ep.ldo + f] = y[q];
                    } else if (ep.op == Q4Epilogue::RESID) {
                        for (int q = 0; q < 16; ++q)
                            if (m0 + q < M) ep.out[(size_t)(m0 + q) * ep.ldo + f] += y[q];
                    } else if (ep.op == Q4Epilogue::SWIGLU) {
                        // rows [0,64) gate, [64,128) up of the same 64 outputs
                        if (r >= 64)
                            for (int q = 0; q < 16; ++q) xch[(r - 64) * 16 + q] = y[q];
                        named_bar_sync(1, DQ_THREADS);
                        if (r < 64) {
                            const int oi = blk * 64 + r;
                            for (int q = 0; q < 16; ++q) {
                                if (m0 + q >= M) break;
                                const float g = y[q], u = xch[r * 16 + q];
                                const float a = g / (1.0f + expf(-g)) * u;
                                ep.xout[(size_t)(m0 + q) * ep.ldx + perm8(oi)] = __float2half_rn(a);
                            }
                        }
                        named_bar_sync(1, DQ_THREADS);
                    } else {   // QKV
                        const int D = ep.head_dim;
                        const int hh = (blk * ROWS + r) / D;      // head index in q|k|v order
                        const int d = (blk * ROWS + r) % D;
                        const bool is_q = hh < ep.n_heads, is_k = !is_q && hh < ep.n_heads + ep.n_kv;
                        const float *nw = is_q ? ep.q_norm : (is_k ? ep.k_norm : nullptr);
                        if (nw) {
                            // per-head sum of squares for each token: warp shuffles + smem
                            for (int q = 0; q < 16; ++q) {
                                const float t2 = warp_sum(y[q] * y[q]);
                                if (lane == q) cs.wsum[warp][q] = t2;
                            }
                        }
                        named_bar_sync(1, DQ_THREADS);
                        if (nw) {
                            const int wpk = D / 32, w0 = (warp / wpk) * wpk;
                            for (int q = 0; q < 16; ++q) {
                                float ss = 0.f;
                                for (int ww = w0; ww < w0 + wpk; ++ww) ss += cs.wsum[ww][q];
                                y[q] = y[q] * (1.0f / sqrtf(ss / (float)D + ep.eps)) * nw[d];
                            }
                        }
                        // rotate-half RoPE on q and k: partner row r +- D/2
                        for (int q = 0; q < 16; ++q) xch[r * 16 + q] = y[q];
                        named_bar_sync(1, DQ_THREADS);
                        if (is_q || is_k) {
                            const int half = D / 2;
                            const int pr = d < half ? r + half : r - half;
                            const float fr = ep.inv_freq[d % half];
                            for (int q = 0; q < 16; ++q) {
                                if (m0 + q >= M) break;
                                const float ang = __fmul_rn((float)ep.tpos[m0 + q], fr);
                                float sn, cn;
                                sincosf(ang, &sn, &cn);
                                const float pv = xch[pr * 16 + q];
                                y[q] = d < half ? y[q] * cn - pv * sn : pv * sn + y[q] * cn;
                            }
                        }
                        for (int q = 0; q < 16; ++q) {
                            const int m = m0 + q;
                            if (m >= M) break;
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
    }
    tc::fence_before_sync();
    __syncthreads();
    if (warp == 0) {
        tc::fence_after_sync();
        tc::tmem_dealloc(tmem, 256);
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
    constexpr int stage = 2 * NT * 128 + ROWS * 64;
    int s = (100 * 1024) / stage;
    return s < 2 ? 2 : (s > 6 ? 6 : s);
}

template <int NT>
size_t smem_for(int stages) {
    return 1024 + (size_t)stages * (2 * NT * 128 + ROWS * 64) + sizeof(Smem);
}

template <int NT>
cudaError_t launch_nt(const Q4WeightTC &w, const CUtensorMap &xmap, int M, int splits, int tiles,
                      const Q4Epilogue &ep, cudaStream_t st) {
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
    const int nchunks = w.K / CHUNK;
    const int cps = (nchunks + splits - 1) / splits;
    dim3 grid(w.N / ROWS, splits, tiles);
    q4_tc_kernel<NT><<<grid, THREADS, sm, st>>>(w.map, xmap, w.scales, w.biases, w.N, w.K, M, cps, stages, ep);
    return cudaGetLastError();
}

}  // namespace

bool make_weight_map(Q4WeightTC &w) {
    auto fn = encode_fn();
    if (!fn) return false;
    const cuuint64_t dims[2] = {(cuuint64_t)(w.K / 2), (cuuint64_t)w.N};
    const cuuint64_t strides[1] = {(cuuint64_t)(w.K / 2)};
    const cuuint32_t box[2] = {64, ROWS};
    const cuuint32_t es[2] = {1, 1};
    return fn(&w.map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<uint32_t *>(w.wq), dims, strides, box, es,
              CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_64B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

int q4_tc_tile(int M) {
    const int nt = ((M + 15) / 16) * 16;
    return nt > 128 ? 128 : nt;
}

int q4_tc_splits(int N, int K, int M, int sm_count) {
    const int nt = q4_tc_tile(M);
    const int tiles = (M + nt - 1) / nt;
    const int ctas = N / ROWS * tiles;
    const int nchunks = K / CHUNK;
    // 1 CTA per SM fits comfortably; aim for >= 1 wave, >= 4 chunks per split
    int s = 1;
    while (ctas * s < sm_count && nchunks / (s * 2) >= 4) s *= 2;
    const int cps = (nchunks + s - 1) / s;
    return (nchunks + cps - 1) / cps;
}

size_t q4_tc_partial_floats(int N, int K, int M, int sm_count) {
    const int nt = q4_tc_tile(M);
    const int tiles = (M + nt - 1) / nt;
    const int s = q4_tc_splits(N, K, M, sm_count);
    return s > 1 ? (size_t)tiles * s * N * nt : 0;
}

size_t q4_tc_counters(int N, int M) {
    const int nt = q4_tc_tile(M);
    return (size_t)((M + nt - 1) / nt) * (N / ROWS);
}

cudaError_t q4_tc(const Q4WeightTC &w, const __half *x_perm8, int M, int sm_count, const Q4Epilogue &ep,
                  cudaStream_t st) {
    if (w.N % ROWS || w.K % CHUNK || M <= 0) return cudaErrorInvalidValue;
    auto fn = encode_fn();
    if (!fn) return cudaErrorNotSupported;
    const int nt = q4_tc_tile(M);
    const int tiles = (M + nt - 1) / nt;
    const int splits = q4_tc_splits(w.N, w.K, M, sm_count);
    if (splits > 1 && (!ep.part || !ep.counters)) return cudaErrorInvalidValue;
    CUtensorMap xmap;
    const cuuint64_t dims[2] = {(cuuint64_t)w.K, (cuuint64_t)M};
    const cuuint64_t strides[1] = {(cuuint64_t)w.K * 2};
    const cuuint32_t box[2] = {64, (cuuint32_t)nt};
    const cuuint32_t es[2] = {1, 1};
    if (fn(&xmap, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<__half *>(x_perm8), dims, strides, box, es,
           CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
           CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
        return cudaErrorInvalidValue;
    switch (nt) {
    case 16: return launch_nt<16>(w, xmap, M, splits, tiles, ep, st);
    case 32: return launch_nt<32>(w, xmap, M, splits, tiles, ep, st);
    case 48: return launch_nt<48>(w, xmap, M, splits, tiles, ep, st);
    case 64: return launch_nt<64>(w, xmap, M, splits, tiles, ep, st);
    case 80: return launch_nt<80>(w, xmap, M, splits, tiles, ep, st);
    case 96: return launch_nt<96>(w, xmap, M, splits, tiles, ep, st);
    case 112: return launch_nt<112>(w, xmap, M, splits, tiles, ep, st);
    default: return launch_nt<128>(w, xmap, M, splits, tiles, ep, st);
    }
}

}  // namespace mlxcat
