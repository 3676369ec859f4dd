// gemm_tc.cu -- dense fp16 GEMM on the 5th-generation tensor cores, the
// prefill path's linears:
//
//   Y[m][n] = sum_k X[m][k] * W[n][k]      (fp16 operands, fp32 accumulation)
//
// Prompt prefill (Scheduler.completeAdmission -> the model forward over the
// prompt, Scheduler.swift:599-668) runs the same q4 linears as the verify
// step at M = hundreds to thousands of tokens.  There the contraction is
// dense (2*M flops per weight), so each q4 weight is dequantised once per
// forward chunk into fp16 [N][K] (dequant_q4 below: HBM-bound, a few percent
// of the GEMM at M = 2048) and both operands stream through shared memory by
// TMA, 128-byte swizzled.
//
// Tile: 128 weight rows (the MMA's M) x BN tokens (its N, 256), k in steps of
// 64 (one 128-byte row per operand row and stage); the plain-store GEMMs take
// two 128-row blocks per tile (see GTile).  Persistent CTAs walk the
// tiles with the token tile fastest, so CTAs running at the same time share a
// weight block and each weight byte comes from HBM about once; the
// activations stay in L2.
//
// Warp roles (6 warps, one CTA per SM):
//   warp 0, lane 0    TMA producer: A (weights) and B (tokens) of one k step
//                     into a GSTAGES-deep ring, completion counted on full[s].
//   warp 1, lane 0    MMA issuer: 4 x tcgen05.mma kind::f16 (M=128, N=BN,
//                     K=16, A and B from shared memory) per stage into one of
//                     two fp32 accumulators in TMEM; a commit frees the stage,
//                     another publishes the finished tile.  Two accumulators
//                     let the epilogue of one tile overlap the next tile's MMAs.
//   warps 2-5         epilogue: each reads its TMEM lane quarter (32 weight
//                     rows) with tcgen05.ld, 16 token columns at a time, and
//                     stores 32 consecutive outputs per token.
//
// Epilogues: STORE (fp32), ADD (fp32 residual stream += y: the O and down
// projections; every output element has one writer, no split-K), SWIGLU
// (the fused gate/up matrix interleaves 64 gate and the matching 64 up rows
// per 128-row tile, so lanes 0-63 and 64-127 of a tile pair up through shared
// memory; out fp16 silu(g) * u).
//
// Every wait is bounded (tc.cuh: 2 s).  A timeout sets *err and an abort flag
// in shared memory after which every role stops; the producer then waits
// (bounded) for the copies it issued and the issuer for its last commit, so
// the CTA leaves no copy or MMA in flight before TMEM is freed.
#include <cuda.h>
#include <cudaTypedefs.h>

#include "common.cuh"
#include "kernels.h"
#include "tc.cuh"

namespace mlxcat {

PFN_cuTensorMapEncodeTiled_v12000 encode_fn();

namespace {

constexpr int GM = 128;        // weight rows per row block (the MMA's M)
constexpr int GBN = 256;       // tokens per tile
constexpr int GK = 64;         // k per stage
constexpr int GSTAGES = 4;     // stages of a one-block tile (3 of a two-block tile)
constexpr int G_THREADS = 192;
constexpr int A_BYTES = GM * GK * 2;           // 16 KB per row block
constexpr int B_BYTES = GBN * GK * 2;          // 32 KB

// Tiles of RB row blocks (RB = 1: 128 x 256, two accumulator sets so a tile's
// epilogue overlaps the next tile's MMAs; RB = 2: 256 x 256, the two blocks'
// MMAs share each token stage -- a third fewer operand bytes per FLOP -- with
// one accumulator set of 2 x 256 TMEM columns).
template <int RB> struct GTile {
    static constexpr int ROWS = GM * RB;
    static constexpr int STAGES = RB == 1 ? 4 : 3;
    static constexpr int STAGE = RB * A_BYTES + B_BYTES;
    static constexpr int SETS = 2 / RB;
};
constexpr int EPI_BAR = 1;                     // named barrier of the 4 epilogue warps
constexpr int SWG_COLS = 16;                   // token columns per epilogue step

enum GemmErr { GE_FULL = 11, GE_EMPTY = 12, GE_DFULL = 13, GE_DEMPTY = 14 };

struct GemmBars {
    unsigned long long full[GSTAGES], empty[GSTAGES], dfull[2], dempty[2];
    uint32_t tmem;
    int abort;
    float up[64][SWG_COLS + 1];   // SWIGLU: up-row values of one 16-column step
};

__device__ __forceinline__ void mma_ss_f16(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                           uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}\n"
        ::"r"(d_tmem), "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
}

// bounded wait that gives up at once when another role has aborted
__device__ __forceinline__ bool gwait(uint32_t bar, uint32_t parity, volatile int *abort, int *err, int code) {
    if (*abort) return false;
    if (tc::mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = tc::global_ns();
    for (;;) {
        if (tc::mbar_try_wait(bar, parity)) return true;
        if (*abort) return false;
        if (tc::global_ns() - t0 > tc::WAIT_LIMIT_NS) {
            *abort = 1;
            if (err) atomicExch(err, code);
            return false;
        }
    }
}

__device__ __forceinline__ void named_sync(int id, int n) {
    asm volatile("bar.sync %0, %1;\n" ::"r"(id), "r"(n) : "memory");
}

// named barrier that also ORs a predicate over the participating threads
__device__ __forceinline__ bool named_sync_or(int id, int n, bool pred) {
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

template <int EPI, int RB>
__global__ void __launch_bounds__(G_THREADS, 1)
gemm_tc_kernel(const __grid_constant__ CUtensorMap wmap, const __grid_constant__ CUtensorMap xmap, int N, int M,
               int K, void *out, int ldo, int *err) {
    using T = GTile<RB>;
    constexpr int NS = T::STAGES, STAGE_BYTES = T::STAGE, SETS = T::SETS;
    // token rows of one B box: the whole 256-row tile, or M when the operand is
    // shorter (the stage's remaining rows then hold stale data, which only
    // feeds accumulator columns >= M that are never stored)
    const uint32_t stage_tx = RB * A_BYTES + (uint32_t)(M < GBN ? M : GBN) * GK * 2;
    extern __shared__ __align__(1024) unsigned char gsm_raw[];
    unsigned char *ring = reinterpret_cast<unsigned char *>(
        (reinterpret_cast<uintptr_t>(gsm_raw) + 1023) & ~(uintptr_t)1023);
    GemmBars &gb = *reinterpret_cast<GemmBars *>(ring + NS * STAGE_BYTES);
    volatile int *abort = &gb.abort;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int mt = (M + GBN - 1) / GBN, tiles = (N / T::ROWS) * mt, nk = K / GK;

    if (threadIdx.x == 0) {
        for (int s = 0; s < NS; ++s) {
            tc::mbar_init(tc::smem_u32(&gb.full[s]), 1);
            tc::mbar_init(tc::smem_u32(&gb.empty[s]), 1);
        }
        for (int a = 0; a < SETS; ++a) {
            tc::mbar_init(tc::smem_u32(&gb.dfull[a]), 1);
            tc::mbar_init(tc::smem_u32(&gb.dempty[a]), 4);
        }
        gb.abort = 0;
        tc::fence_barrier_init();
        tc::prefetch_tmap(&wmap);
        tc::prefetch_tmap(&xmap);
    }
    if (warp == 1) tc::tmem_alloc(tc::smem_u32(&gb.tmem), 2 * GBN);   // two 256-column accumulators
    tc::fence_before_sync();
    __syncthreads();
    tc::fence_after_sync();
    const uint32_t tmem = gb.tmem;

    if (warp == 0) {
        if (lane == 0) {
            // ---------------- TMA producer ----------------
            int it = 0;
            for (int t = blockIdx.x; t < tiles && !*abort; t += gridDim.x) {
                const int n0 = (t / mt) * T::ROWS, m0 = (t % mt) * GBN;
                for (int kb = 0; kb < nk; ++kb, ++it) {
                    const int s = it % NS;
                    if (!gwait(tc::smem_u32(&gb.empty[s]), ((it / NS) & 1) ^ 1, abort, err, GE_EMPTY)) break;
                    const uint32_t bar = tc::smem_u32(&gb.full[s]);
                    unsigned char *st = ring + (size_t)s * STAGE_BYTES;
                    tc::mbar_arrive_expect_tx(bar, stage_tx);
#pragma unroll
                    for (int rb = 0; rb < RB; ++rb)
                        tc::tma_load_2d(tc::smem_u32(st + rb * A_BYTES), &wmap, kb * GK, n0 + rb * GM, bar);
                    tc::tma_load_2d(tc::smem_u32(st + RB * A_BYTES), &xmap, kb * GK, m0, bar);
                }
            }
            if (*abort)   // copies issued must land before the CTA's shared memory is released
                for (int j = it - NS > 0 ? it - NS : 0; j < it; ++j)
                    tc::mbar_wait(tc::smem_u32(&gb.full[j % NS]), (j / NS) & 1, nullptr, 0);
        }
    } else if (warp == 1) {
        if (lane == 0) {
            // ---------------- MMA issuer ----------------
            constexpr uint32_t idesc = tc::idesc_f16_f32(GM, GBN);
            int it = 0, lt = 0, last = -1;
            for (int t = blockIdx.x; t < tiles && !*abort; t += gridDim.x, ++lt) {
                const int a = lt % SETS;
                if (!gwait(tc::smem_u32(&gb.dempty[a]), ((lt / SETS) & 1) ^ 1, abort, err, GE_DEMPTY)) break;
                tc::fence_after_sync();
                const uint32_t dcol = tmem + a * RB * GBN;   // row block rb accumulates at dcol + rb * GBN
                bool ok = true;
                for (int kb = 0; kb < nk; ++kb, ++it) {
                    const int s = it % NS;
                    if (!gwait(tc::smem_u32(&gb.full[s]), (it / NS) & 1, abort, err, GE_FULL)) { ok = false; break; }
                    tc::fence_after_sync();
                    const uint32_t sa = tc::smem_u32(ring + (size_t)s * STAGE_BYTES);
                    const uint64_t bd = tc::sdesc_k_sw128(sa + RB * A_BYTES);
#pragma unroll
                    for (int q = 0; q < GK / 16; ++q)   // +32 bytes per 16-element k step
#pragma unroll
                        for (int rb = 0; rb < RB; ++rb)
                            mma_ss_f16(dcol + rb * GBN, tc::sdesc_k_sw128(sa + rb * A_BYTES) + 2 * q, bd + 2 * q, idesc,
                                       (kb | q) ? 1u : 0u);
                    tc::mma_commit(tc::smem_u32(&gb.empty[s]));   // stage free once these MMAs finish
                    last = it;
                }
                if (!ok) break;
                tc::mma_commit(tc::smem_u32(&gb.dfull[a]));       // tile complete
            }
            if (*abort && last >= 0)   // MMAs in flight read shared memory and write TMEM
                tc::mbar_wait(tc::smem_u32(&gb.empty[last % NS]), (last / NS) & 1, nullptr, 0);
        }
    } else {
        // ---------------- epilogue: warps 2..5, TMEM lane quarter warp % 4 ----------------
        const int q = warp & 3;
        const int row = q * 32 + lane;   // weight row inside the tile
        int lt = 0;
        for (int t = blockIdx.x; t < tiles; t += gridDim.x, ++lt) {
            const int a = lt % SETS;
            const int m0 = (t % mt) * GBN;
            bool failed = !gwait(tc::smem_u32(&gb.dfull[a]), (lt / SETS) & 1, abort, err, GE_DFULL);
            // the SwiGLU steps pair warps through named barriers: all four leave together
            if (EPI == GEMM_SWIGLU) failed = named_sync_or(EPI_BAR, 128, failed);
            if (failed) break;
            tc::fence_after_sync();
            const int ncols = min(GBN, M - m0);
            for (int rb = 0; rb < RB; ++rb) {
            const int n0 = (t / mt) * T::ROWS + rb * GM;
            const uint32_t tbase = tmem + ((uint32_t)(q * 32) << 16) + (a * RB + rb) * GBN;
            for (int c = 0; c < GBN / SWG_COLS; ++c) {
                if (c * SWG_COLS >= ncols) break;
                uint32_t v[16];
                tc::tmem_ld16(tbase + c * SWG_COLS, v);
                tc::tmem_wait_ld();
                const int mb = m0 + c * SWG_COLS;
                if (EPI == GEMM_STORE) {
                    float *o = static_cast<float *>(out);
#pragma unroll
                    for (int j = 0; j < 16; ++j)
                        if (mb + j < M) o[(size_t)(mb + j) * ldo + n0 + row] = __uint_as_float(v[j]);
                } else if (EPI == GEMM_ADD) {
                    float *o = static_cast<float *>(out);
#pragma unroll
                    for (int j = 0; j < 16; ++j)
                        if (mb + j < M) {
                            float *p = o + (size_t)(mb + j) * ldo + n0 + row;
                            *p = __fadd_rn(*p, __uint_as_float(v[j]));
                        }
                } else {   // SWIGLU: quarters 2, 3 hold the up rows of quarters 0, 1
                    if (q >= 2)
#pragma unroll
                        for (int j = 0; j < 16; ++j) gb.up[row - 64][j] = __uint_as_float(v[j]);
                    named_sync(EPI_BAR, 128);
                    if (q < 2) {
                        __half *o = static_cast<__half *>(out);
                        const int i = (n0 / GM) * 64 + row;   // output feature
#pragma unroll
                        for (int j = 0; j < 16; ++j)
                            if (mb + j < M) {
                                const float g = __uint_as_float(v[j]), u = gb.up[row][j];
                                o[(size_t)(mb + j) * ldo + i] = __float2half_rn(g / (1.0f + __expf(-g)) * u);
                            }
                    }
                    named_sync(EPI_BAR, 128);
                }
            }
            }
            tc::fence_before_sync();
            __syncwarp();
            if (lane == 0) tc::mbar_arrive(tc::smem_u32(&gb.dempty[a]));
        }
    }
    tc::fence_before_sync();
    __syncthreads();
    tc::fence_after_sync();
    if (warp == 1) tc::tmem_dealloc(tmem, 2 * GBN);
}

// w[n][k] = scale * q + bias in fp16 (the q4 kernels' dequantisation: hfma of
// fp16 q, scale and bias), one packed word (8 weights) per thread
__global__ void dequant_q4_kernel(const uint32_t *__restrict__ wq, const __half *__restrict__ sc,
                                  const __half *__restrict__ bi, int N, int K, __half *__restrict__ w) {
    const size_t words = (size_t)N * (K / 8);
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < words; i += (size_t)gridDim.x * blockDim.x) {
        const size_t n = i / (K / 8), kw = i - n * (K / 8);
        const size_t g = n * (K / MLXCAT_GS) + kw * 8 / MLXCAT_GS;
        const __half s = sc[g], b = bi[g];
        const uint32_t word = __ldg(wq + i);
        __align__(16) __half o[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) o[j] = __hfma(__uint2half_rn((word >> (4 * j)) & 0xfu), s, b);
        *reinterpret_cast<uint4 *>(w + i * 8) = *reinterpret_cast<const uint4 *>(o);
    }
}

bool make_map_2d(CUtensorMap *map, const __half *p, int inner, int outer, int box_outer) {
    auto fn = encode_fn();
    if (!fn) return false;
    const cuuint64_t dims[2] = {(cuuint64_t)inner, (cuuint64_t)outer};
    const cuuint64_t strides[1] = {(cuuint64_t)inner * 2};
    const cuuint32_t box[2] = {GK, (cuuint32_t)box_outer};
    const cuuint32_t es[2] = {1, 1};
    return fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<__half *>(p), dims, strides, box, es,
              CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <int RB>
size_t gemm_smem() { return 1024 + (size_t)GTile<RB>::STAGES * GTile<RB>::STAGE + sizeof(GemmBars); }

}  // namespace

cudaError_t dequant_q4(const Q4Weight &w, __half *out, cudaStream_t st) {
    if (w.K % 64 || !w.wq || !out) return cudaErrorInvalidValue;
    const size_t words = (size_t)w.N * (w.K / 8);
    const size_t want = (words + 255) / 256;
    dequant_q4_kernel<<<(unsigned)(want < 8192 ? want : 8192), 256, 0, st>>>(w.wq, w.scales, w.biases, w.N, w.K, out);
    return cudaGetLastError();
}

cudaError_t gemm_tc(const __half *w, int N, int K, const __half *x, int M, int epi, void *out, int ldo,
                    int sm_count, int *err, cudaStream_t st) {
    if (N % GM || K % GK || M <= 0 || !w || !x || !out) return cudaErrorInvalidValue;
    if (epi == GEMM_SWIGLU && ldo < N / 2) return cudaErrorInvalidValue;
    if (epi != GEMM_SWIGLU && ldo < N) return cudaErrorInvalidValue;
    CUtensorMap wmap, xmap;
    if (!make_map_2d(&wmap, w, K, N, GM) || !make_map_2d(&xmap, x, K, M, M < GBN ? M : GBN))
        return cudaErrorInvalidValue;
    // Two-block tiles for the plain store, where the rows allow them and the token
    // tiles are full: 1.18 -> 1.36 PFLOP/s on the prefill's QKV / O / down shapes.
    // The SwiGLU epilogue (exchange through shared memory, exponentials) is too
    // long to run unoverlapped after every tile (0.81 -> 1.13 ms per gate/up
    // launch at 4096 tokens), so it keeps the double-buffered one-block tiles.
    const bool two = epi == GEMM_STORE && N % (2 * GM) == 0 && M >= GBN;
    const int tiles = (N / (two ? 2 * GM : GM)) * ((M + GBN - 1) / GBN);
    const int grid = tiles < sm_count ? tiles : sm_count;
    auto launch = [&](auto kern, size_t smem) -> cudaError_t {
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return e;
        kern<<<grid, G_THREADS, smem, st>>>(wmap, xmap, N, M, K, out, ldo, err);
        return cudaGetLastError();
    };
    if (two) return launch(gemm_tc_kernel<GEMM_STORE, 2>, gemm_smem<2>());
    switch (epi) {
    case GEMM_STORE: return launch(gemm_tc_kernel<GEMM_STORE, 1>, gemm_smem<1>());
    case GEMM_ADD: return launch(gemm_tc_kernel<GEMM_ADD, 1>, gemm_smem<1>());
    case GEMM_SWIGLU: return launch(gemm_tc_kernel<GEMM_SWIGLU, 1>, gemm_smem<1>());
    default: return cudaErrorInvalidValue;
    }
}

}  // namespace mlxcat
