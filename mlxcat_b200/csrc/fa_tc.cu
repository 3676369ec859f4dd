// fa_tc.cu -- causal attention of the prompt prefill on the 5th-generation
// tensor cores (head_dim 128).
//
// Replaces MLXFast.scaledDotProductAttention with the causal mask over one
// prompt chunk of one row (the admission prefill, Scheduler.swift:599-668):
// query token i of the chunk sits at position s0 + i and sees keys 0..s0+i of
// the row's cache (earlier chunks included).
//
// CTA = (128-query tile, query head).  Keys stream in blocks of 128 through a
// two-stage TMA ring (K and V of the head's kv head, 128-byte swizzle).  Per
// key block j:
//   S_j  = Q K_j^T            tcgen05.mma, A = Q tile and B = K tile from shared
//                              memory (both K-major), S in TMEM (two buffers, so
//                              S_{j+1} is computed while S_j is in the softmax)
//   P_j  = exp2(S_j*c - m)    four softmax warps, thread = query row (TMEM lane):
//                              the running max m moves only when a row's max
//                              grows by more than 8 (log2 units), so P <= 256
//                              fits fp16 and O rarely needs rescaling; P is
//                              stored row-major into shared memory with the
//                              128-byte swizzle (the MMA's K-major B operand)
//   O^T += V_j^T P_j^T         tcgen05.mma with A = V_j^T in TMEM: four warps,
//                              thread = feature d (TMEM lane), read V_j column d
//                              out of the swizzled tile and store it as fp16
//                              key pairs; O^T [d][query] accumulates in TMEM
// so every shared-memory operand is K-major.  When some row's max moved, the
// V warps scale the O^T columns of those rows by alpha before the next
// product.  The V warps then write O^T / l as fp16 [token][head * 128 + d].
//
// Warps: 0 TMA producer, 1 MMA issuer, 2 TMEM allocation, 4-7 softmax,
// 8-11 V^T / rescale / epilogue (warp w owns TMEM lanes 32 * (w % 4)..).
// Every wait is bounded; a timeout sets *err and an abort flag after which
// every role skips its work, the producer waits for its copies and the issuer
// for its last commit, and the CTA frees TMEM.
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
constexpr int BQ = 128;                 // queries per CTA (MMA M of Q K^T, N of V^T P^T)
constexpr int BKEYS = 128;              // keys per block
constexpr int BOX = 128 * 128;          // one [128 rows x 128 B] swizzled box
constexpr int TILE = 2 * BOX;           // 128 rows x 256 B (head_dim 128, two boxes)
constexpr int F_THREADS = 384;
constexpr int SM_WARP0 = 4, VT_WARP0 = 8;
constexpr int EPI_BAR = 1;              // softmax + V warps, before the epilogue
constexpr uint32_t COL_S = 0, COL_O = 256, COL_VT = 384;

enum FaErr { FE_Q = 31, FE_K = 32, FE_V = 33, FE_FREE = 34, FE_SFULL = 35, FE_SFREE = 36, FE_P = 37, FE_VT = 38,
             FE_PV = 39 };

struct FaBars {
    unsigned long long q_full, k_full[2], v_full[2], kv_free[2], s_full[2], s_free[2], p_full, vt_full, pv_done;
    float alpha[BQ];
    float lsum[BQ];
    int rescale[2][4];       // per block parity, per softmax warp: some row's max moved
    uint32_t tmem;
    int abort;
};

constexpr size_t SMEM_Q = 0, SMEM_K = TILE, SMEM_V = 3 * TILE, SMEM_P = 5 * TILE, SMEM_BARS = 6 * TILE;
constexpr size_t FA_SMEM = 1024 + SMEM_BARS + sizeof(FaBars);

__device__ __forceinline__ void mma_ss(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                       uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}\n"
        ::"r"(d_tmem), "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
}

__device__ __forceinline__ bool fwait(uint32_t bar, uint32_t parity, volatile int *abort, int *err, int code) {
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

// byte offset of (row r, byte b) inside a 1024-aligned [rows x 128 B] box with the 128-byte swizzle
__device__ __forceinline__ uint32_t sw128(int r, int b) {
    return (uint32_t)(r * 128 + ((((b >> 4) ^ (r & 7)) << 4) | (b & 15)));
}

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
            tc::mbar_init(tc::smem_u32(&fb.v_full[s]), 1);
            tc::mbar_init(tc::smem_u32(&fb.kv_free[s]), 1 + 4);   // the S MMA's commit + the four V warps
            tc::mbar_init(tc::smem_u32(&fb.s_full[s]), 1);
            tc::mbar_init(tc::smem_u32(&fb.s_free[s]), 4);
        }
        tc::mbar_init(tc::smem_u32(&fb.p_full), 4);
        tc::mbar_init(tc::smem_u32(&fb.vt_full), 4);
        tc::mbar_init(tc::smem_u32(&fb.pv_done), 1);
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

    if (warp == 0) {
        if (lane == 0) {
            // ---------------- TMA producer ----------------
            int issued = 0;
            const uint32_t qb = tc::smem_u32(&fb.q_full);
            tc::mbar_arrive_expect_tx(qb, TILE);
            tc::tma_load_2d(tc::smem_u32(sm + SMEM_Q), &qmap, h * FD, q0, qb);
            tc::tma_load_2d(tc::smem_u32(sm + SMEM_Q + BOX), &qmap, h * FD + 64, q0, qb);
            for (int j = 0; j < nb && !*abort; ++j) {
                const int s = j & 1;
                if (j >= 2 && !fwait(tc::smem_u32(&fb.kv_free[s]), ((j - 2) >> 1) & 1, abort, err, FE_FREE)) break;
                const int y = kv_row0 + j * BKEYS;
                const uint32_t kb = tc::smem_u32(&fb.k_full[s]), vb = tc::smem_u32(&fb.v_full[s]);
                tc::mbar_arrive_expect_tx(kb, TILE);
                tc::tma_load_2d(tc::smem_u32(sm + SMEM_K + s * TILE), &kmap, 0, y, kb);
                tc::tma_load_2d(tc::smem_u32(sm + SMEM_K + s * TILE + BOX), &kmap, 64, y, kb);
                tc::mbar_arrive_expect_tx(vb, TILE);
                tc::tma_load_2d(tc::smem_u32(sm + SMEM_V + s * TILE), &vmap, 0, y, vb);
                tc::tma_load_2d(tc::smem_u32(sm + SMEM_V + s * TILE + BOX), &vmap, 64, y, vb);
                issued = j + 1;
            }
            // copies in flight must land before the CTA's shared memory is released
            tc::mbar_wait(tc::smem_u32(&fb.q_full), 0, nullptr, 0);
            for (int j = issued - 2 > 0 ? issued - 2 : 0; j < issued; ++j) {
                tc::mbar_wait(tc::smem_u32(&fb.k_full[j & 1]), (j >> 1) & 1, nullptr, 0);
                tc::mbar_wait(tc::smem_u32(&fb.v_full[j & 1]), (j >> 1) & 1, nullptr, 0);
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {
            // ---------------- MMA issuer ----------------
            constexpr uint32_t idesc = tc::idesc_f16_f32(128, 128);
            const uint32_t qa = tc::smem_u32(sm + SMEM_Q), pa = tc::smem_u32(sm + SMEM_P);
            bool ok = fwait(tc::smem_u32(&fb.q_full), 0, abort, err, FE_Q);
            int committed = 0;   // PV products committed
            auto issue_s = [&](int j) -> bool {
                const int s = j & 1;
                if (!fwait(tc::smem_u32(&fb.k_full[s]), (j >> 1) & 1, abort, err, FE_K)) return false;
                if (j >= 2 && !fwait(tc::smem_u32(&fb.s_free[s]), ((j - 2) >> 1) & 1, abort, err, FE_SFREE))
                    return false;
                tc::fence_after_sync();
                const uint32_t ka = tc::smem_u32(sm + SMEM_K + s * TILE);
#pragma unroll
                for (int kk = 0; kk < FD / 16; ++kk) {   // 16 features per step: box kk/4, +32 B per step
                    const uint32_t off = (uint32_t)((kk >> 2) * BOX + (kk & 3) * 32);
                    mma_ss(tmem + COL_S + s * 128, tc::sdesc_k_sw128(qa + off), tc::sdesc_k_sw128(ka + off), idesc,
                           kk ? 1u : 0u);
                }
                tc::mma_commit(tc::smem_u32(&fb.s_full[s]));
                tc::mma_commit(tc::smem_u32(&fb.kv_free[s]));   // K read (the V warps arrive for V)
                return true;
            };
            if (ok) ok = issue_s(0);
            for (int j = 0; j < nb && ok; ++j) {
                if (j + 1 < nb && !issue_s(j + 1)) break;
                if (!fwait(tc::smem_u32(&fb.p_full), j & 1, abort, err, FE_P)) break;
                if (!fwait(tc::smem_u32(&fb.vt_full), j & 1, abort, err, FE_VT)) break;
                tc::fence_after_sync();
#pragma unroll
                for (int kk = 0; kk < BKEYS / 16; ++kk) {   // 16 keys per step: 8 TMEM columns of V^T
                    const uint32_t off = (uint32_t)((kk >> 2) * BOX + (kk & 3) * 32);
                    tc::mma_ts_f16(tmem + COL_O, tmem + COL_VT + kk * 8, tc::sdesc_k_sw128(pa + off), idesc,
                                   (j | kk) ? 1u : 0u);
                }
                tc::mma_commit(tc::smem_u32(&fb.pv_done));
                committed = j + 1;
            }
            // the MMAs issued must finish before TMEM is freed
            if (committed > 0) tc::mbar_wait(tc::smem_u32(&fb.pv_done), (committed - 1) & 1, nullptr, 0);
        }
    } else if (warp >= SM_WARP0 && warp < SM_WARP0 + 4) {
        // ---------------- softmax: thread = query row ----------------
        const int q = (warp - SM_WARP0) * 32 + lane;
        const uint32_t lane_base = (uint32_t)((warp & 3) * 32) << 16;
        const int qpos = qp0 + q;
        const bool qvalid = q < nq;
        float m_used = -INFINITY, l = 0.f;
        unsigned char *prow = sm + SMEM_P;
        for (int j = 0; j < nb; ++j) {
            const int s = j & 1;
            bool ok = fwait(tc::smem_u32(&fb.s_full[s]), (j >> 1) & 1, abort, err, FE_SFULL);
            ok = __shfl_sync(0xffffffffu, ok, 0);
            if (!ok) break;
            tc::fence_after_sync();
            const uint32_t sc = tmem + lane_base + COL_S + s * 128;
            const int k0 = j * BKEYS;
            const int lim = qvalid ? qpos - k0 : -1;   // columns 0..lim are visible keys
            float mx = -INFINITY;
#pragma unroll
            for (int c = 0; c < 8; ++c) {
                uint32_t v[16];
                tc::tmem_ld16(sc + c * 16, v);
                tc::tmem_wait_ld();
#pragma unroll
                for (int i = 0; i < 16; ++i)
                    if (c * 16 + i <= lim) mx = fmaxf(mx, __uint_as_float(v[i]));
            }
            mx *= scale_log2;
            float alpha = 1.f;
            if (mx > m_used + 8.f) {   // the row's max moved: rescale l (and O, by the V warps)
                alpha = m_used == -INFINITY ? 0.f : exp2f(m_used - mx);
                m_used = mx;
            }
            // P is single-buffered: the previous product must have read it
            if (j >= 1) {
                ok = fwait(tc::smem_u32(&fb.pv_done), (j - 1) & 1, abort, err, FE_PV);
                ok = __shfl_sync(0xffffffffu, ok, 0);
                if (!ok) break;
            }
            float sum = 0.f;
#pragma unroll
            for (int c = 0; c < 8; ++c) {
                uint32_t v[16];
                tc::tmem_ld16(sc + c * 16, v);
                tc::tmem_wait_ld();
                uint32_t pk[8];
#pragma unroll
                for (int i = 0; i < 8; ++i) {
                    const int c0 = c * 16 + 2 * i;
                    const float p0 = (c0 <= lim && m_used != -INFINITY)
                                         ? exp2f(__uint_as_float(v[2 * i]) * scale_log2 - m_used) : 0.f;
                    const float p1 = (c0 + 1 <= lim && m_used != -INFINITY)
                                         ? exp2f(__uint_as_float(v[2 * i + 1]) * scale_log2 - m_used) : 0.f;
                    const __half2 hp = __floats2half2_rn(p0, p1);
                    sum += __low2float(hp) + __high2float(hp);   // l sums what the product uses
                    pk[i] = *reinterpret_cast<const uint32_t *>(&hp);
                }
                // keys c*16 .. c*16+15 of row q: box (c/4), bytes (c%4)*32 .. +31 (two 16-byte chunks)
                unsigned char *bx = prow + (c >> 2) * BOX;
                const int b0 = (c & 3) * 32;
                *reinterpret_cast<uint4 *>(bx + sw128(q, b0)) = make_uint4(pk[0], pk[1], pk[2], pk[3]);
                *reinterpret_cast<uint4 *>(bx + sw128(q, b0 + 16)) = make_uint4(pk[4], pk[5], pk[6], pk[7]);
            }
            l = l * alpha + sum;
            fb.alpha[q] = alpha;
            const int moved = __any_sync(0xffffffffu, alpha != 1.f && j > 0);
            if (lane == 0) fb.rescale[s][warp - SM_WARP0] = moved;
            tc::fence_before_sync();
            tc::fence_proxy_async_smem();   // P (generic stores) visible to the tensor core
            __syncwarp();
            if (lane == 0) {
                tc::mbar_arrive(tc::smem_u32(&fb.s_free[s]));
                tc::mbar_arrive(tc::smem_u32(&fb.p_full));
            }
        }
        fb.lsum[q] = l;
        named_sync(EPI_BAR, 256);
    } else if (warp >= VT_WARP0) {
        // ---------------- V^T into TMEM, O rescale, epilogue: thread = feature d ----------------
        const int d = (warp - VT_WARP0) * 32 + lane;
        const uint32_t lane_base = (uint32_t)((warp & 3) * 32) << 16;
        const int vbox = d >> 6, vb = (d & 63) * 2;   // V[key][d]: box, byte within the 128-byte row
        bool ok = true;
        for (int j = 0; j < nb && ok; ++j) {
            const int s = j & 1;
            ok = fwait(tc::smem_u32(&fb.v_full[s]), (j >> 1) & 1, abort, err, FE_V);
            if (ok && j >= 1) ok = fwait(tc::smem_u32(&fb.pv_done), (j - 1) & 1, abort, err, FE_PV);
            ok = __shfl_sync(0xffffffffu, ok, 0);
            if (!ok) break;
            tc::fence_after_sync();
            const unsigned char *vt = sm + SMEM_V + s * TILE + vbox * BOX;
#pragma unroll
            for (int cp = 0; cp < 4; ++cp) {   // 32 keys -> 16 TMEM columns of key pairs
                uint32_t r[16];
#pragma unroll
                for (int i = 0; i < 16; ++i) {
                    const int key = cp * 32 + 2 * i;
                    const uint16_t a = *reinterpret_cast<const uint16_t *>(vt + sw128(key, vb));
                    const uint16_t b = *reinterpret_cast<const uint16_t *>(vt + sw128(key + 1, vb));
                    r[i] = (uint32_t)a | ((uint32_t)b << 16);
                }
                tc::tmem_st16(tmem + lane_base + COL_VT + cp * 16, r);
            }
            __syncwarp();
            if (lane == 0) tc::mbar_arrive(tc::smem_u32(&fb.kv_free[s]));   // V read
            // the softmax of block j decides whether O^T must be rescaled first
            ok = fwait(tc::smem_u32(&fb.p_full), j & 1, abort, err, FE_P);
            ok = __shfl_sync(0xffffffffu, ok, 0);
            if (!ok) break;
            if (fb.rescale[s][0] | fb.rescale[s][1] | fb.rescale[s][2] | fb.rescale[s][3]) {
#pragma unroll 1
                for (int c = 0; c < 8; ++c) {
                    uint32_t v[16];
                    tc::tmem_ld16(tmem + lane_base + COL_O + c * 16, v);
                    tc::tmem_wait_ld();
#pragma unroll
                    for (int i = 0; i < 16; ++i) v[i] = __float_as_uint(__uint_as_float(v[i]) * fb.alpha[c * 16 + i]);
                    tc::tmem_st16(tmem + lane_base + COL_O + c * 16, v);
                }
            }
            tc::tmem_wait_st();
            tc::fence_before_sync();
            __syncwarp();
            if (lane == 0) tc::mbar_arrive(tc::smem_u32(&fb.vt_full));
        }
        if (ok && nb > 0) ok = fwait(tc::smem_u32(&fb.pv_done), (nb - 1) & 1, abort, err, FE_PV);
        named_sync(EPI_BAR, 256);
        ok = __shfl_sync(0xffffffffu, ok, 0) && !*abort;
        if (ok) {
            tc::fence_after_sync();
            __half *o = out + (size_t)q0 * Hq * FD + h * FD + d;
#pragma unroll 1
            for (int c = 0; c < 8; ++c) {
                uint32_t v[16];
                tc::tmem_ld16(tmem + lane_base + COL_O + c * 16, v);
                tc::tmem_wait_ld();
#pragma unroll
                for (int i = 0; i < 16; ++i) {
                    const int q = c * 16 + i;
                    const float lq = fb.lsum[q];
                    if (q < nq) o[(size_t)q * Hq * FD] = __float2half_rn(lq > 0.f ? __uint_as_float(v[i]) / lq : 0.f);
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
