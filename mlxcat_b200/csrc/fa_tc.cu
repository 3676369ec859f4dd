// fa_tc.cu -- causal attention of the prompt prefill on the 5th-generation
// tensor cores (head_dim 128).
//
// Replaces MLXFast.scaledDotProductAttention with the causal mask over one
// prompt chunk of one row (the admission prefill, Scheduler.swift:599-668):
// query token i of the chunk sits at position s0 + i and sees keys 0..s0+i of
// the row's cache (earlier chunks included).
//
// CTA = (128-query tile, query head).  Keys stream in blocks of 128 through two
// K and two V stages (TMA, 128-byte swizzle), each fed by its own producer
// thread.  Per key block j (buffer b = j & 1):
//   S_j  = Q K_j^T            tcgen05.mma, A = Q and B = K_j from shared memory
//                              (both K-major), S into TMEM buffer b
//   P_j  = exp2(S_j*c - m)    eight softmax warps, two per query row (TMEM lane),
//                              each taking 64 of the block's 128 keys; the
//                              running max m moves only when a row's max grows
//                              by more than 8 (log2 units), so P <= 256 fits
//                              fp16 and O rarely needs rescaling.  P goes back
//                              into TMEM as fp16 key pairs over the first 64
//                              columns of S buffer b.
//   O   += P_j V_j            tcgen05.mma with A = P_j from TMEM and B = V_j
//                              read in place from its TMA tile as an MN-major
//                              operand (keys along K, features along N); O
//                              [query][feature] accumulates in TMEM.
// When a row's max moved, its two softmax threads scale that row of O (once
// the product of block j - 1 is in) before P_j is handed to the issuer; they
// finally write O / l as fp16 [token][head * 128 + d].  (An earlier layout
// computed O^T = V^T P^T with V^T copied into TMEM by four more warps; that copy
// set the pace of every key block.)
//
// Warps: 0 TMA producer (Q, K), 1 MMA issuer, 2 TMEM allocation, 3 TMA
// producer (V), 4-11 softmax and epilogue (keys 0-63 in warps 4-7, 64-127 in
// warps 8-11; the two halves of a row exchange their partial max through
// shared memory).  The softmax is the critical path: exp2 runs as ex2.approx
// (fp16 P).  Every wait is bounded; a timeout sets *err and an abort flag after
// which every role skips its work, the producers wait for their copies and the
// issuer for everything it committed, and the CTA frees TMEM.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <cmath>

#include "common.cuh"
#include "kernels.h"
#include "tc.cuh"

namespace mlxcat {

PFN_cuTensorMapEncodeTiled_v12000 encode_fn();

namespace {

constexpr int FD = 128;                 // head_dim
constexpr int BQ = 128;                 // queries per CTA (MMA M of both products)
constexpr int BKEYS = 128;              // keys per block
constexpr int BOX = 128 * 128;          // one [128 rows x 128 B] swizzled box
constexpr int TILE = 2 * BOX;           // 128 rows x 256 B (head_dim 128, two boxes)
constexpr int F_THREADS = 384;
constexpr int SM_WARP0 = 4;
constexpr int PAIR_BAR0 = 1;            // 1..4: the two softmax warps of one lane quarter
constexpr uint32_t COL_S = 0, COL_O = 256;   // S (and P over it): 2 x 128 columns, O: 128 columns

enum FaErr { FE_Q = 31, FE_K = 32, FE_V = 33, FE_FREE = 34, FE_SFULL = 35, FE_P = 37, FE_PV = 39 };

// Block j uses buffer j & 1 of every double-buffered resource (K and V stages,
// S / P in TMEM, partial maxima) and the barriers of that buffer, so a role may
// run one block ahead of another without a barrier phase being overtaken.
struct FaBars {
    unsigned long long q_full, k_full[2], k_free[2], v_full[2], v_free[2], s_full[2], p_full[2], pv_done[2], fin;
    float pmax[2][2][BQ];    // per block parity, per key half: partial row max
    float lsum[2][BQ];       // per key half
    uint32_t tmem;
    int abort;
};

constexpr size_t SMEM_Q = 0, SMEM_K = TILE, SMEM_V = 3 * TILE, SMEM_BARS = 5 * TILE;
constexpr size_t FA_SMEM = 1024 + SMEM_BARS + sizeof(FaBars);
static_assert(FA_SMEM <= 227 * 1024, "Q and two K and two V tiles must fit one CTA");

// Q: [tokens][Hq * 128] fp16 (the prefill's query buffer); K, V: one layer's
// cache viewed as [(row * Hkv + kvh) * max_len + key][128]; out: [tokens][Hq * 128].
__global__ void __launch_bounds__(F_THREADS, 1)
fa_prefill_kernel(const __grid_constant__ CUtensorMap qmap, const __grid_constant__ CUtensorMap kmap,
                  const __grid_constant__ CUtensorMap vmap, int n, int s0, int row, int Hq, int Hkv, int max_len,
                  float scale_log2, __half *__restrict__ out, int *err) {
    extern __shared__ __align__(1024) unsigned char fsm_raw[];
    unsigned char *sm = reinterpret_cast<unsigned char *>((reinterpret_cast<uintptr_t>(fsm_raw) + 1023) &
                                                          ~(uintptr_t)1023);
    FaBars &fb = *reinterpret_cast<FaBars *>(sm + SMEM_BARS);
    volatile int *abort = &fb.abort;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    // longest tiles (furthest into the prompt) first
    const int qt = gridDim.x - 1 - blockIdx.x, h = blockIdx.y, kvh = h / (Hq / Hkv);
    const int q0 = qt * BQ, nq = min(BQ, n - q0), qp0 = s0 + q0;   // first query position
    const int nb = (qp0 + nq - 1) / BKEYS + 1;                        // key blocks
    const int kv_row0 = (row * Hkv + kvh) * max_len;

    if (threadIdx.x == 0) {
        tc::mbar_init(tc::smem_u32(&fb.q_full), 1);
        for (int s = 0; s < 2; ++s) {
            tc::mbar_init(tc::smem_u32(&fb.k_full[s]), 1);
            tc::mbar_init(tc::smem_u32(&fb.k_free[s]), 1);    // the S product's commit
            tc::mbar_init(tc::smem_u32(&fb.v_full[s]), 1);
            tc::mbar_init(tc::smem_u32(&fb.v_free[s]), 1);    // the O product's commit
            tc::mbar_init(tc::smem_u32(&fb.s_full[s]), 1);
            tc::mbar_init(tc::smem_u32(&fb.p_full[s]), 8);    // the eight softmax warps
            tc::mbar_init(tc::smem_u32(&fb.pv_done[s]), 1);
        }
        tc::mbar_init(tc::smem_u32(&fb.fin), 1);
        fb.abort = 0;
        tc::fence_barrier_init();
        tc::prefetch_tmap(&qmap);
        tc::prefetch_tmap(&kmap);
        tc::prefetch_tmap(&vmap);
    }
    if (warp == 2) tc::tmem_alloc(tc::smem_u32(&fb.tmem), 512);
    tc::fence_before_sync();
    __syncthreads();
    tc::fence_after_sync();
    const uint32_t tmem = fb.tmem;
    griddep_wait();   // the queries and the chunk's keys come from the previous kernel

    if (warp == 0 || warp == 3) {
        if (lane == 0) {
            // ---------------- TMA producers: warp 0 Q and K, warp 3 V ----------------
            const bool kp = warp == 0;
            if (kp) {
                const uint32_t qb = tc::smem_u32(&fb.q_full);
                tc::mbar_arrive_expect_tx(qb, TILE);
                tc::tma_load_2d(tc::smem_u32(sm + SMEM_Q), &qmap, h * FD, q0, qb);
                tc::tma_load_2d(tc::smem_u32(sm + SMEM_Q + BOX), &qmap, h * FD + 64, q0, qb);
            }
            const CUtensorMap *map = kp ? &kmap : &vmap;
            unsigned long long *full = kp ? fb.k_full : fb.v_full, *freed = kp ? fb.k_free : fb.v_free;
            unsigned char *stage0 = sm + (kp ? SMEM_K : SMEM_V);
            int issued = 0;
            for (int j = 0; j < nb && !*abort; ++j) {
                const int y = kv_row0 + j * BKEYS, b = j & 1;
                // stage b was last read by the product of block j - 2
                if (j >= 2 && !tc::mbar_wait_abort(tc::smem_u32(&freed[b]), ((j - 2) >> 1) & 1, abort, err, FE_FREE)) break;
                const uint32_t bar = tc::smem_u32(&full[b]), st = tc::smem_u32(stage0 + b * TILE);
                tc::mbar_arrive_expect_tx(bar, TILE);
                tc::tma_load_2d(st, map, 0, y, bar);
                tc::tma_load_2d(st + BOX, map, 64, y, bar);
                issued = j + 1;
            }
            // copies in flight must land before the CTA's shared memory is released
            if (kp) tc::mbar_wait(tc::smem_u32(&fb.q_full), 0, nullptr, 0);
            for (int i = issued >= 2 ? issued - 2 : 0; i < issued; ++i)
                tc::mbar_wait(tc::smem_u32(&full[i & 1]), (i >> 1) & 1, nullptr, 0);
        }
    } else if (warp == 1) {
        if (lane == 0) {
            // ---------------- MMA issuer ----------------
            constexpr uint32_t idesc_s = tc::idesc_f16_f32(128, 128);
            constexpr uint32_t idesc_pv = tc::idesc_f16_f32(128, 128) | (1u << 16);   // B (V) MN-major
            const uint32_t qa = tc::smem_u32(sm + SMEM_Q);
            bool ok = tc::mbar_wait_abort(tc::smem_u32(&fb.q_full), 0, abort, err, FE_Q);
            auto issue_s = [&](int j) -> bool {
                const int b = j & 1;
                if (!tc::mbar_wait_abort(tc::smem_u32(&fb.k_full[b]), (j >> 1) & 1, abort, err, FE_K)) return false;
                // S buffer b holds P_{j-2} until the product of block j - 2 has read it
                if (j >= 2 && !tc::mbar_wait_abort(tc::smem_u32(&fb.pv_done[b]), ((j - 2) >> 1) & 1, abort, err, FE_PV))
                    return false;
                tc::fence_after_sync();
                const uint32_t ka = tc::smem_u32(sm + SMEM_K + b * TILE);
#pragma unroll
                for (int kk = 0; kk < FD / 16; ++kk) {   // 16 features per step: box kk/4, +32 B per step
                    const uint32_t off = (uint32_t)((kk >> 2) * BOX + (kk & 3) * 32);
                    tc::mma_ss_f16(tmem + COL_S + b * 128, tc::sdesc_k_sw128(qa + off), tc::sdesc_k_sw128(ka + off), idesc_s,
                           kk ? 1u : 0u);
                }
                tc::mma_commit(tc::smem_u32(&fb.s_full[b]));
                tc::mma_commit(tc::smem_u32(&fb.k_free[b]));   // K stage b read
                return true;
            };
            if (ok) ok = issue_s(0);
            for (int j = 0; j < nb && ok; ++j) {
                const int b = j & 1;
                if (j + 1 < nb && !issue_s(j + 1)) break;
                if (!tc::mbar_wait_abort(tc::smem_u32(&fb.p_full[b]), (j >> 1) & 1, abort, err, FE_P)) break;
                if (!tc::mbar_wait_abort(tc::smem_u32(&fb.v_full[b]), (j >> 1) & 1, abort, err, FE_V)) break;
                tc::fence_after_sync();
                const uint32_t va = tc::smem_u32(sm + SMEM_V + b * TILE);
#pragma unroll
                for (int kk = 0; kk < BKEYS / 16; ++kk)   // 16 keys per step: 8 TMEM columns of P, 2048 B of V
                    tc::mma_ts_f16(tmem + COL_O, tmem + COL_S + b * 128 + kk * 8, tc::sdesc_mn_sw128(va + kk * 2048, BOX),
                                   idesc_pv, (j | kk) ? 1u : 0u);
                tc::mma_commit(tc::smem_u32(&fb.pv_done[b]));
                tc::mma_commit(tc::smem_u32(&fb.v_free[b]));   // V stage b read
            }
            // every product issued must finish before TMEM is freed
            tc::mma_commit(tc::smem_u32(&fb.fin));
            tc::mbar_wait(tc::smem_u32(&fb.fin), 0, nullptr, 0);
        }
    } else if (warp >= SM_WARP0) {
        // ---------------- softmax and epilogue: thread = (query row, key half) ----------------
        const int quarter = warp & 3, half = (warp - SM_WARP0) >> 2;
        const int q = quarter * 32 + lane;
        const uint32_t lane_base = (uint32_t)(quarter * 32) << 16;
        const int qpos = qp0 + q;
        const bool qvalid = q < nq;
        float m_used = -INFINITY, l = 0.f;
        bool ok = true;
        for (int j = 0; j < nb; ++j) {
            const int b = j & 1;
            ok = tc::mbar_wait_abort(tc::smem_u32(&fb.s_full[b]), (j >> 1) & 1, abort, err, FE_SFULL);
            ok = __shfl_sync(0xffffffffu, ok, 0);
            // this half's 64 scores of row q
            uint32_t v[64];
            const int lim = qvalid ? qpos - j * BKEYS - half * 64 : -1;   // columns 0..lim visible
            float mx = -INFINITY;
            if (ok) {
                tc::fence_after_sync();
                tc::tmem_ld32(tmem + lane_base + COL_S + b * 128 + half * 64, v);
                tc::tmem_ld32(tmem + lane_base + COL_S + b * 128 + half * 64 + 32, v + 32);
                tc::tmem_wait_ld();
                if (lim >= 63) {
#pragma unroll
                    for (int i = 0; i < 64; ++i) mx = fmaxf(mx, __uint_as_float(v[i]));
                } else {
#pragma unroll
                    for (int i = 0; i < 64; ++i)
                        if (i <= lim) mx = fmaxf(mx, __uint_as_float(v[i]));
                }
                fb.pmax[b][half][q] = mx;
            }
            // the two halves of the row meet here (both have read their scores before
            // either writes P over them); both leave together on an abort
            tc::fence_before_sync();
            ok = !tc::bar_sync_or(PAIR_BAR0 + quarter, 64, !ok);
            if (!ok) break;
            tc::fence_after_sync();
            mx = fmaxf(fb.pmax[b][0][q], fb.pmax[b][1][q]) * scale_log2;
            float alpha = 1.f;
            if (mx > m_used + 8.f) {   // the row's max moved: rescale l and O
                alpha = m_used == -INFINITY ? 0.f : exp2f(m_used - mx);
                m_used = mx;
            }
            // P = exp2(S c - m) as fp16 key pairs into columns half*32.. of S buffer b.
            // A half with every key visible (all but the diagonal blocks) skips the mask;
            // l sums the fp32 values (their fp16 rounding errors average out in l).
            const bool live = m_used != -INFINITY;
            const float nm = -m_used;
            float sum = 0.f;
            uint32_t pk[32];
            if (live && lim >= 63) {
#pragma unroll
                for (int i = 0; i < 32; ++i) {
                    const float p0 = tc::ex2_approx(fmaf(__uint_as_float(v[2 * i]), scale_log2, nm));
                    const float p1 = tc::ex2_approx(fmaf(__uint_as_float(v[2 * i + 1]), scale_log2, nm));
                    sum += p0 + p1;
                    const __half2 hp = __floats2half2_rn(p0, p1);
                    pk[i] = *reinterpret_cast<const uint32_t *>(&hp);
                }
            } else {
#pragma unroll
                for (int i = 0; i < 32; ++i) {
                    const int c0 = 2 * i;
                    const float p0 = (live && c0 <= lim) ? tc::ex2_approx(fmaf(__uint_as_float(v[c0]), scale_log2, nm)) : 0.f;
                    const float p1 = (live && c0 + 1 <= lim) ? tc::ex2_approx(fmaf(__uint_as_float(v[c0 + 1]), scale_log2, nm)) : 0.f;
                    sum += p0 + p1;
                    const __half2 hp = __floats2half2_rn(p0, p1);
                    pk[i] = *reinterpret_cast<const uint32_t *>(&hp);
                }
            }
            tc::tmem_st32(tmem + lane_base + COL_S + b * 128 + half * 32, pk);
            l = l * alpha + sum;
            // a row whose max moved scales its O (this half's 64 features) once the
            // product of block j - 1 is in; the product of block j waits for p_full
            if (__any_sync(0xffffffffu, alpha != 1.f && j > 0)) {
                bool okp = true;
                if (lane == 0) okp = tc::mbar_wait_abort(tc::smem_u32(&fb.pv_done[b ^ 1]), ((j - 1) >> 1) & 1, abort, err, FE_PV);
                okp = __shfl_sync(0xffffffffu, okp, 0);
                if (okp) {
                    tc::fence_after_sync();
#pragma unroll 1
                    for (int c = 0; c < 4; ++c) {
                        uint32_t o[16];
                        tc::tmem_ld16(tmem + lane_base + COL_O + half * 64 + c * 16, o);
                        tc::tmem_wait_ld();
#pragma unroll
                        for (int i = 0; i < 16; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * alpha);
                        tc::tmem_st16(tmem + lane_base + COL_O + half * 64 + c * 16, o);
                    }
                }
            }
            tc::tmem_wait_st();
            tc::fence_before_sync();
            __syncwarp();
            if (lane == 0) tc::mbar_arrive(tc::smem_u32(&fb.p_full[b]));
        }
        // epilogue: O / l of row q, this half's 64 features, once the last product is in
        fb.lsum[half][q] = l;
        if (ok && lane == 0) ok = tc::mbar_wait_abort(tc::smem_u32(&fb.pv_done[(nb - 1) & 1]), ((nb - 1) >> 1) & 1, abort, err, FE_PV);
        ok = __shfl_sync(0xffffffffu, ok, 0);
        ok = !tc::bar_sync_or(PAIR_BAR0 + quarter, 64, !ok) && !*abort;
        if (ok) {
            tc::fence_after_sync();
            const float lq = fb.lsum[0][q] + fb.lsum[1][q];
            const float inv = lq > 0.f ? 1.f / lq : 0.f;
            __half *o = out + (size_t)(q0 + q) * Hq * FD + h * FD + half * 64;
#pragma unroll 1
            for (int c = 0; c < 2; ++c) {
                uint32_t acc[32];
                tc::tmem_ld32(tmem + lane_base + COL_O + half * 64 + c * 32, acc);
                tc::tmem_wait_ld();
                uint32_t hv[16];
#pragma unroll
                for (int i = 0; i < 16; ++i) {
                    const __half2 h2 = __floats2half2_rn(__uint_as_float(acc[2 * i]) * inv,
                                                         __uint_as_float(acc[2 * i + 1]) * inv);
                    hv[i] = *reinterpret_cast<const uint32_t *>(&h2);
                }
                if (qvalid) {
                    uint4 *dst = reinterpret_cast<uint4 *>(o + c * 32);
#pragma unroll
                    for (int i = 0; i < 4; ++i) dst[i] = make_uint4(hv[4 * i], hv[4 * i + 1], hv[4 * i + 2], hv[4 * i + 3]);
                }
            }
        }
    }
    tc::fence_before_sync();
    __syncthreads();
    if (warp == 2) {
        tc::fence_after_sync();
        tc::tmem_dealloc(tmem, 512);
    }
}

bool map2d(CUtensorMap *m, const void *base, uint64_t inner, uint64_t rows, uint64_t row_bytes) {
    auto fn = encode_fn();
    if (!fn) return false;
    const cuuint64_t dims[2] = {inner, rows};
    const cuuint64_t strides[1] = {row_bytes};
    const cuuint32_t box[2] = {64, 128};
    const cuuint32_t es[2] = {1, 1};
    return fn(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void *>(base), dims, strides, box, es,
              CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

}  // namespace

bool fa_prefill_supported(int head_dim) { return head_dim == FD; }

cudaError_t fa_prefill(const __half *q, int q_rows, const KVLayer &kv, int rows, int row, int s0, int n, int Hq,
                       int Hkv, int D, __half *out, int *err, cudaStream_t st) {
    if (D != FD || n <= 0 || n > q_rows || Hq % Hkv || row < 0 || row >= rows || s0 < 0 || s0 + n > kv.max_len ||
        !err)
        return cudaErrorInvalidValue;
    CUtensorMap qm, km, vm;
    const uint64_t kv_rows = (uint64_t)rows * Hkv * kv.max_len;
    if (!map2d(&qm, q, (uint64_t)Hq * FD, (uint64_t)q_rows, (uint64_t)Hq * FD * 2) ||
        !map2d(&km, kv.k, FD, kv_rows, FD * 2) || !map2d(&vm, kv.v, FD, kv_rows, FD * 2))
        return cudaErrorInvalidValue;
    static bool attr[64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (!attr[dev & 63]) {
        const cudaError_t e = cudaFuncSetAttribute(fa_prefill_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                   (int)FA_SMEM);
        if (e != cudaSuccess) return e;
        attr[dev & 63] = true;
    }
    const float scale_log2 = 1.4426950408889634f / sqrtf((float)FD);
    const dim3 grid((unsigned)((n + BQ - 1) / BQ), (unsigned)Hq);
    fa_prefill_kernel<<<grid, F_THREADS, FA_SMEM, st>>>(qm, km, vm, n, s0, row, Hq, Hkv, kv.max_len, scale_log2,
                                                        out, err);
    return cudaGetLastError();
}

}  // namespace mlxcat
