// fused.cu -- per-token kernels around the q4 linears of the verify forward:
// embedding + first RMSNorm, the blocked activation layout, the RoPE table,
// argmax, and the table model used as the reference's fake LanguageModel.
// (The norms, q/k/v epilogue and SwiGLU between the linears are fused into
// the q4 linear's epilogues, q4_tc.cu.)
//
// Model math follows mlx-swift-lm's Llama / Qwen3 blocks as used on the
// verify forward (BatchGenerator.swift:900-904): pre-norm residual blocks,
// rotate-half RoPE, GQA, SwiGLU.
#include "common.cuh"
#include "kernels.h"

namespace mlxcat {

namespace {

constexpr int TPB = 256;

__device__ __forceinline__ float block_sum(float v, float *sh) {
    v = warp_sum(v);
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
    __syncthreads();
    if (lane == 0) sh[w] = v;
    __syncthreads();
    float r = 0.f;
    const int nw = blockDim.x >> 5;
    for (int i = 0; i < nw; ++i) r += sh[i];
    return r;
}

__global__ void embed_norm_kernel(const uint32_t *__restrict__ wq, const __half *__restrict__ sc,
                                  const __half *__restrict__ bi, int H, const int32_t *tok,
                                  const float *__restrict__ nw, float eps, float *__restrict__ h,
                                  __half *__restrict__ xn, int ldx_rows, float *__restrict__ rstd_out) {
    __shared__ float sh[32];
    const int m = blockIdx.x;
    const int t = tok[m];
    const uint32_t *row = wq + (size_t)t * (H / 8);
    float *hm = h + (size_t)m * H;
    float ss = 0.f;
    for (int w = threadIdx.x; w < H / 8; w += blockDim.x) {
        const uint32_t word = row[w];
        const int grp = (w * 8) / MLXCAT_GS;
        const float s = __half2float(sc[(size_t)t * (H / MLXCAT_GS) + grp]);
        const float b = __half2float(bi[(size_t)t * (H / MLXCAT_GS) + grp]);
        for (int i = 0; i < 8; ++i) {
            const float v = s * (float)((word >> (4 * i)) & 0xfu) + b;
            hm[w * 8 + i] = v;
            ss += v * v;
        }
    }
    ss = block_sum(ss, sh);
    const float r = 1.0f / sqrtf(ss / (float)H + eps);
    if (rstd_out && threadIdx.x == 0) rstd_out[m] = r;
    for (int w = threadIdx.x; w < H / 8; w += blockDim.x)
        for (int i = 0; i < 8; ++i) {
            const int k = w * 8 + i;
            xn[xblk(m, k, ldx_rows)] = __float2half_rn(hm[k] * r * nw[k]);
        }
}

__global__ void permute_kernel(const __half *__restrict__ x, __half *__restrict__ y, int M, int K) {
    const size_t n = (size_t)M * K;
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
         i += (size_t)gridDim.x * blockDim.x) {
        const int m = (int)(i / K), k = (int)(i - (size_t)m * K);
        y[xblk(m, k, M)] = x[i];
    }
}

// max value, lowest index on ties (MLX argMax returns the first maximum)
// Row argmax as a 64-bit key: (order-preserving float bits, ~index), so the
// largest key is the largest logit and, among equal logits, the lowest index.
__device__ __forceinline__ unsigned long long argmax_key(float v, int i) {
    return ((unsigned long long)float_key(v) << 32) | (unsigned long long)(0xffffffffu - (uint32_t)i);
}

__device__ __forceinline__ unsigned long long block_max_u64(unsigned long long v, unsigned long long *sh) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const unsigned long long t = __shfl_xor_sync(0xffffffffu, v, o);
        v = t > v ? t : v;
    }
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
    if (lane == 0) sh[w] = v;
    __syncthreads();
    if (w == 0) {
        v = lane < (int)(blockDim.x >> 5) ? sh[lane] : 0ull;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const unsigned long long t = __shfl_xor_sync(0xffffffffu, v, o);
            v = t > v ? t : v;
        }
    }
    return v;   // valid in thread 0
}

// best key of logits[lo, hi) of one row (float4 loads when the row is 16-byte aligned)
__device__ __forceinline__ unsigned long long range_best(const float *l, int lo, int hi, bool vec) {
    unsigned long long best = 0;
    if (vec) {
        const int lo4 = (lo + 3) & ~3, hi4 = hi & ~3;
        for (int i = lo + threadIdx.x; i < min(lo4, hi); i += blockDim.x) {
            const unsigned long long k = argmax_key(l[i], i);
            best = k > best ? k : best;
        }
        for (int i = lo4 + 4 * threadIdx.x; i < hi4; i += 4 * blockDim.x) {
            const float4 v = __ldg(reinterpret_cast<const float4 *>(l + i));
            unsigned long long k = argmax_key(v.x, i);     best = k > best ? k : best;
            k = argmax_key(v.y, i + 1); best = k > best ? k : best;
            k = argmax_key(v.z, i + 2); best = k > best ? k : best;
            k = argmax_key(v.w, i + 3); best = k > best ? k : best;
        }
        for (int i = max(hi4, lo4) + threadIdx.x; i < hi; i += blockDim.x) {
            const unsigned long long k = argmax_key(l[i], i);
            best = k > best ? k : best;
        }
    } else {
        for (int i = lo + threadIdx.x; i < hi; i += blockDim.x) {
            const unsigned long long k = argmax_key(l[i], i);
            best = k > best ? k : best;
        }
    }
    return best;
}

// one CTA per row
__global__ void argmax_kernel(const float *__restrict__ logits, int V, int32_t *out) {
    __shared__ unsigned long long sh[32];
    const int m = blockIdx.x;
    const float *l = logits + (size_t)m * V;
    const bool vec = (V & 3) == 0 && (reinterpret_cast<uintptr_t>(logits) & 15) == 0;
    const unsigned long long b = block_max_u64(range_best(l, 0, V, vec), sh);
    if (threadIdx.x == 0) out[m] = (int32_t)(0xffffffffu - (uint32_t)(b & 0xffffffffull));
}

// S CTAs per row; the last CTA of a row (ticket) reduces the S partial keys
// (max is order-independent, so the result does not depend on timing)
__global__ void argmax_split_kernel(const float *__restrict__ logits, int V, int S,
                                    unsigned long long *__restrict__ part, unsigned *__restrict__ ctr,
                                    int32_t *out) {
    __shared__ unsigned long long sh[32];
    __shared__ int last;
    const int s = blockIdx.x, m = blockIdx.y;
    const float *l = logits + (size_t)m * V;
    const bool vec = (V & 3) == 0 && (reinterpret_cast<uintptr_t>(logits) & 15) == 0;
    const int chunk = ((V + S - 1) / S + 3) & ~3;
    const int lo = min(V, s * chunk), hi = min(V, lo + chunk);
    const unsigned long long b = block_max_u64(range_best(l, lo, hi, vec), sh);
    if (threadIdx.x == 0) {
        part[(size_t)m * S + s] = b;
        __threadfence();
        const unsigned prev = atomicAdd(ctr + m, 1u);
        last = prev == (unsigned)(S - 1);
        if (last) {
            ctr[m] = 0u;   // ready for the next launch
            __threadfence();
            unsigned long long best = 0;
            for (int i = 0; i < S; ++i) {
                const unsigned long long k = __ldcg(part + (size_t)m * S + i);
                best = k > best ? k : best;
            }
            out[m] = (int32_t)(0xffffffffu - (uint32_t)(best & 0xffffffffull));
        }
    }
}

__global__ void table_logits_kernel(const int32_t *next, const int32_t *tok, int V, float *logits) {
    const int m = blockIdx.y;
    const int nt = next[tok[m]];
    for (int v = blockIdx.x * blockDim.x + threadIdx.x; v < V; v += gridDim.x * blockDim.x)
        logits[(size_t)m * V + v] = v == nt ? 20.0f : -20.0f;
}

}  // namespace

cudaError_t embed_norm(const Q4Weight &embed, const int32_t *tok, int M, const float *norm_w,
                       float eps, float *h, __half *xn, int ldx_rows, cudaStream_t st, float *rstd_out) {
    embed_norm_kernel<<<M, TPB, 0, st>>>(embed.wq, embed.scales, embed.biases, embed.K, tok,
                                         norm_w, eps, h, xn, ldx_rows, rstd_out);
    return cudaGetLastError();
}

cudaError_t permute_activations(const __half *x, __half *x_perm, int M, int K, cudaStream_t st) {
    if (K % 64) return cudaErrorInvalidValue;
    const size_t n = (size_t)M * K;
    const int blocks = (int)((n + TPB - 1) / TPB < 4096 ? (n + TPB - 1) / TPB : 4096);
    permute_kernel<<<blocks > 0 ? blocks : 1, TPB, 0, st>>>(x, x_perm, M, K);
    return cudaGetLastError();
}

__global__ void rope_table_kernel(const float *__restrict__ inv_freq, int half, int max_len, float2 *tab) {
    const long long n = (long long)max_len * half;
    for (long long t = (long long)blockIdx.x * blockDim.x + threadIdx.x; t < n; t += (long long)gridDim.x * blockDim.x) {
        const int p = (int)(t / half), i = (int)(t - (long long)p * half);
        float sn, cn;
        sincosf(__fmul_rn((float)p, inv_freq[i]), &sn, &cn);
        tab[t] = make_float2(cn, sn);
    }
}

cudaError_t rope_table(const float *inv_freq, int half, int max_len, float2 *tab, cudaStream_t st) {
    const long long n = (long long)max_len * half;
    const long long b = (n + TPB - 1) / TPB;
    rope_table_kernel<<<(unsigned)(b < 4096 ? (b ? b : 1) : 4096), TPB, 0, st>>>(inv_freq, half, max_len, tab);
    return cudaGetLastError();
}

size_t argmax_scratch_words(int M) { return (size_t)M * ARGMAX_SPLITS; }

cudaError_t argmax_rows(const float *logits, int M, int V, int32_t *out, cudaStream_t st,
                        unsigned long long *part, unsigned *ctr) {
    if (part && ctr && V >= 4096 * ARGMAX_SPLITS / 8) {
        argmax_split_kernel<<<dim3(ARGMAX_SPLITS, M), 256, 0, st>>>(logits, V, ARGMAX_SPLITS, part, ctr, out);
    } else {
        argmax_kernel<<<M, 1024, 0, st>>>(logits, V, out);
    }
    return cudaGetLastError();
}

cudaError_t table_logits(const int32_t *next, const int32_t *tok, int M, int V, float *logits,
                         cudaStream_t st) {
    dim3 grid((V + TPB - 1) / TPB < 64 ? (V + TPB - 1) / TPB : 64, M);
    table_logits_kernel<<<grid, TPB, 0, st>>>(next, tok, V, logits);
    return cudaGetLastError();
}

}  // namespace mlxcat
