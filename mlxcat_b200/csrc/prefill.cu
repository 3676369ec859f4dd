// prefill.cu -- the per-token kernels of the dense prefill path, between the
// tcgen05 GEMMs of gemm_tc.cu.  Activations are row-major ([tokens][features]),
// the layout the GEMM's TMA maps read.
//
// Model math is the verify forward's (mlx-swift-lm Llama / Qwen3 blocks, run
// by the reference's admission prefill, Scheduler.swift:670-1016): embedding,
// pre-norm RMSNorm, q|k|v with per-head q/k RMSNorm (Qwen3) and rotate-half
// RoPE from the cache's (cos, sin) table, K/V appended to the cache at each
// token's position.  The SwiGLU is fused into the gate/up GEMM's epilogue; the
// residual adds after the O and down projections into the RMSNorm that
// follows them (pf_add_rmsnorm_kernel: the GEMM stores its output at full
// rate, the add is two streamed passes over the row).
#include "common.cuh"
#include "kernels.h"

namespace mlxcat {

namespace {

constexpr int PF_TPB = 256;

__device__ __forceinline__ float pf_block_sum(float v, float *sh) {
    v = warp_sum(v);
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
    __syncthreads();
    if (lane == 0) sh[w] = v;
    __syncthreads();
    float r = 0.f;
    for (int i = 0; i < (int)(blockDim.x >> 5); ++i) r += sh[i];
    return r;
}

// h[m][k] = scale * q + bias of the embedding row of tok[m] (as embed_norm)
__global__ void pf_embed_kernel(const uint32_t *__restrict__ wq, const __half *__restrict__ sc,
                                const __half *__restrict__ bi, int H, const int32_t *__restrict__ tok,
                                float *__restrict__ h) {
    const int m = blockIdx.x, t = tok[m];
    const uint32_t *row = wq + (size_t)t * (H / 8);
    for (int w = threadIdx.x; w < H / 8; w += blockDim.x) {
        const uint32_t word = row[w];
        const int grp = (w * 8) / MLXCAT_GS;
        const float s = __half2float(sc[(size_t)t * (H / MLXCAT_GS) + grp]);
        const float b = __half2float(bi[(size_t)t * (H / MLXCAT_GS) + grp]);
        for (int i = 0; i < 8; ++i) h[(size_t)m * H + w * 8 + i] = s * (float)((word >> (4 * i)) & 0xfu) + b;
    }
}

// x[m] = fp16(h[m] * rstd * w), rstd = 1/sqrt(mean(h^2) + eps); one CTA per token
__global__ void pf_rmsnorm_kernel(const float *__restrict__ h, int H, const float *__restrict__ nw, float eps,
                                  __half *__restrict__ x) {
    __shared__ float sh[32];
    const int m = blockIdx.x;
    const float *hm = h + (size_t)m * H;
    float ss = 0.f;
    for (int k = threadIdx.x; k < H; k += blockDim.x) ss += hm[k] * hm[k];
    ss = pf_block_sum(ss, sh);
    const float r = 1.0f / sqrtf(ss / (float)H + eps);
    for (int k = threadIdx.x; k < H; k += blockDim.x) x[(size_t)m * H + k] = __float2half_rn(hm[k] * r * nw[k]);
}

// The residual step after the O and down projections: h[m] += y[m] (the
// projection's fp32 output), then x[m] = fp16(h[m] * rstd * w).  One CTA per
// token, 16-byte accesses; the second pass re-reads the row just written (L1).
__global__ void pf_add_rmsnorm_kernel(float *__restrict__ h, const float *__restrict__ y, int H,
                                      const float *__restrict__ nw, float eps, __half *__restrict__ x) {
    __shared__ float sh[32];
    const int m = blockIdx.x, H4 = H / 4;
    float4 *hm = reinterpret_cast<float4 *>(h + (size_t)m * H);
    const float4 *ym = reinterpret_cast<const float4 *>(y + (size_t)m * H);
    float ss = 0.f;
    for (int k = threadIdx.x; k < H4; k += blockDim.x) {
        float4 a = hm[k];
        const float4 b = ym[k];
        a.x += b.x; a.y += b.y; a.z += b.z; a.w += b.w;
        hm[k] = a;
        ss += a.x * a.x + a.y * a.y + a.z * a.z + a.w * a.w;
    }
    ss = pf_block_sum(ss, sh);
    const float r = 1.0f / sqrtf(ss / (float)H + eps);
    const float4 *w4 = reinterpret_cast<const float4 *>(nw);
    uint2 *xm = reinterpret_cast<uint2 *>(x + (size_t)m * H);
    for (int k = threadIdx.x; k < H4; k += blockDim.x) {
        const float4 a = hm[k], w = w4[k];
        __half2 lo = __floats2half2_rn(a.x * r * w.x, a.y * r * w.y), hi = __floats2half2_rn(a.z * r * w.z, a.w * r * w.w);
        uint2 o;
        o.x = *reinterpret_cast<uint32_t *>(&lo);
        o.y = *reinterpret_cast<uint32_t *>(&hi);
        xm[k] = o;
    }
}

// q|k|v rows of one token: per-head q/k RMSNorm, RoPE, q -> qbuf [m][Hq][D],
// k/v -> the cache at (row, pos).  One CTA per token, one warp per head; lane
// owns the rotate-half pairs (i, i + D/2), i = lane + 32 p.
__global__ void pf_qkv_kernel(const float *__restrict__ y, int n_heads, int n_kv, int D,
                              const float *__restrict__ q_norm, const float *__restrict__ k_norm, float eps,
                              const float2 *__restrict__ rope, int row, const int32_t *__restrict__ tpos,
                              __half *__restrict__ qbuf, __half *__restrict__ kc, __half *__restrict__ vc,
                              int max_len) {
    const int m = blockIdx.x;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nwarps = blockDim.x >> 5;
    const int N = (n_heads + 2 * n_kv) * D, half = D / 2, pos = tpos[m];
    constexpr int PP = 4;   // pairs per lane (D <= 256)
    for (int hh = warp; hh < n_heads + 2 * n_kv; hh += nwarps) {
        const bool is_q = hh < n_heads, is_k = !is_q && hh < n_heads + n_kv;
        const float *src = y + (size_t)m * N + (size_t)hh * D;
        float a[PP], b[PP], ss = 0.f;
#pragma unroll
        for (int p = 0; p < PP; ++p) {
            const int i = lane + 32 * p;
            a[p] = i < half ? src[i] : 0.f;
            b[p] = i < half ? src[i + half] : 0.f;
            ss += a[p] * a[p] + b[p] * b[p];
        }
        if (is_q || is_k) {
            const float *nw = is_q ? q_norm : k_norm;
            float r = 1.f;
            if (nw) r = 1.0f / sqrtf(warp_sum(ss) / (float)D + eps);
#pragma unroll
            for (int p = 0; p < PP; ++p) {
                const int i = lane + 32 * p;
                if (i < half) {
                    float x0 = a[p], x1 = b[p];
                    if (nw) { x0 = x0 * r * nw[i]; x1 = x1 * r * nw[i + half]; }
                    const float2 cs = rope[(size_t)pos * half + i];
                    a[p] = x0 * cs.x - x1 * cs.y;
                    b[p] = x1 * cs.x + x0 * cs.y;
                }
            }
        }
        __half *dst;
        if (is_q) {
            dst = qbuf + ((size_t)m * n_heads + hh) * D;
        } else {
            const int kvh = is_k ? hh - n_heads : hh - n_heads - n_kv;
            dst = (is_k ? kc : vc) + (((size_t)row * n_kv + kvh) * max_len + pos) * D;
        }
#pragma unroll
        for (int p = 0; p < PP; ++p) {
            const int i = lane + 32 * p;
            if (i < half) {
                dst[i] = __float2half_rn(a[p]);
                dst[i + half] = __float2half_rn(b[p]);
            }
        }
    }
}

__global__ void pf_rows_kernel(int32_t *trow, int32_t *tpos, int row, int s0, int n) {
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
        trow[i] = row;
        tpos[i] = s0 + i;
    }
}

// one token's row-major fp16 features into row 0 of the blocked operand layout
__global__ void pf_to_blocked_kernel(const __half *__restrict__ x, int K, __half *__restrict__ xb, int ldx_rows) {
    for (int k = blockIdx.x * blockDim.x + threadIdx.x; k < K; k += gridDim.x * blockDim.x)
        xb[xblk(0, k, ldx_rows)] = x[k];
}

}  // namespace

cudaError_t prefill_embed(const Q4Weight &embed, const int32_t *tok, int n, float *h, cudaStream_t st) {
    pf_embed_kernel<<<n, PF_TPB, 0, st>>>(embed.wq, embed.scales, embed.biases, embed.K, tok, h);
    return cudaGetLastError();
}

cudaError_t prefill_rmsnorm(const float *h, int n, int H, const float *w, float eps, __half *x, cudaStream_t st) {
    pf_rmsnorm_kernel<<<n, PF_TPB, 0, st>>>(h, H, w, eps, x);
    return cudaGetLastError();
}

cudaError_t prefill_add_rmsnorm(float *h, const float *y, int n, int H, const float *w, float eps, __half *x,
                                cudaStream_t st) {
    if (H % 4) return cudaErrorInvalidValue;
    pf_add_rmsnorm_kernel<<<n, PF_TPB, 0, st>>>(h, y, H, w, eps, x);
    return cudaGetLastError();
}

cudaError_t prefill_qkv(const float *y, int n, int n_heads, int n_kv, int D, const float *q_norm,
                        const float *k_norm, float eps, const float2 *rope, int row, const int32_t *tpos,
                        __half *qbuf, KVLayer kv, cudaStream_t st) {
    if (D > 256 || (D & 1)) return cudaErrorInvalidValue;
    pf_qkv_kernel<<<n, PF_TPB, 0, st>>>(y, n_heads, n_kv, D, q_norm, k_norm, eps, rope, row, tpos, qbuf, kv.k,
                                        kv.v, kv.max_len);
    return cudaGetLastError();
}

cudaError_t prefill_rows(int32_t *trow, int32_t *tpos, int row, int s0, int n, cudaStream_t st) {
    pf_rows_kernel<<<(n + PF_TPB - 1) / PF_TPB, PF_TPB, 0, st>>>(trow, tpos, row, s0, n);
    return cudaGetLastError();
}

cudaError_t prefill_to_blocked(const __half *x, int K, __half *xb, int ldx_rows, cudaStream_t st) {
    pf_to_blocked_kernel<<<(K + PF_TPB - 1) / PF_TPB, PF_TPB, 0, st>>>(x, K, xb, ldx_rows);
    return cudaGetLastError();
}

}  // namespace mlxcat
