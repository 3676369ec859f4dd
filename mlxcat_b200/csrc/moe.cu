// moe.cu -- sparse MoE MLP of Qwen3-MoE-shape models on the verify forward.
//
// Replaces the SwitchGLU block of mlx-swift-lm's Qwen3-MoE model (un-vendored,
// dcfa3aa1), which the verify forward of BatchGenerator.swift:900 runs in every
// layer of such a model:
//   logits = x . Wr^T (bf16 router, logits kept bf16), p = softmax(logits),
//   top-k experts (ties to the lower index), weights renormalised over the k,
//   y = sum_j w_j * down_e(silu(gate_e(x)) * up_e(x)).
//
// Kernels (one verify step touches every expert, so the experts' q4 weights
// stream from HBM once per layer like a dense MLP's):
//   moe_route_kernel    bf16 router GEMV + softmax + top-k for RT tokens per CTA;
//                       appends each (token, slot) assignment to its expert's
//                       list (atomic slot, fixed capacity = token rows).
//   moe_expert_kernel   grouped q4 linear: CTA = (128-row tile, expert); the
//                       expert's assignments are the columns.  Weights stay in
//                       the MLX SwitchGLU layout, [E][out][in/8] per projection,
//                       and are the A operand of mma.m16n8k16 (dequantised in registers from
//                       coalesced 16-byte loads), tokens the B operand in groups
//                       of 8 -- a ~20-token expert wastes at most 7 columns.
//                       GATEUP: one tile = 64 gate rows + the matching 64 up
//                       rows, SwiGLU epilogue into the down projection's
//                       blocked operand.  DOWN: output scaled by the routing
//                       weight, fp32 per assignment.
//   moe_combine_kernel  h += sum_j y_j in selection order (deterministic); the
//                       next linear's operand fp16(h * w * s) and per-128-block
//                       sums of squares (the folded RMSNorm of the dense path).
#include <cuda_bf16.h>

#include "common.cuh"
#include "kernels.h"

namespace mlxcat {

namespace {

constexpr int RT = 4;                 // tokens per router CTA
constexpr int ROUTE_THREADS = 256;
constexpr int EX_THREADS = 128;       // 4 warps x 32 weight rows
constexpr int EX_ROWS = 128;
constexpr int EX_TOK = 32;            // assignments per pass (4 n8 tiles)
constexpr int COMBINE_THREADS = 256;

__device__ __forceinline__ uint4 ldg_stream16(const void *p) {
    uint4 r;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];\n"
                 : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
                 : "l"(p));
    return r;
}

__device__ __forceinline__ uint32_t dq2(uint32_t w, int shift, __half2 s2, __half2 b2) {
    // nibbles (shift/4, shift/4 + 4) as fp16 1024 + q, then q * scale + bias
    uint32_t v = ((w >> shift) & 0x000f000fu) | 0x64006400u;
    __half2 q = __hsub2(*reinterpret_cast<const __half2 *>(&v),
                        __halves2half2(__ushort_as_half(0x6400), __ushort_as_half(0x6400)));
    __half2 r = __hfma2(q, s2, b2);
    return *reinterpret_cast<uint32_t *>(&r);
}

__device__ __forceinline__ void mma16816(float *c, uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                         uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
        "{%8,%9}, {%0,%1,%2,%3};\n"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

__device__ __forceinline__ float bf16_round(float x) {
    return __bfloat162float(__float2bfloat16_rn(x));
}

// ---------------------------------------------------------------------------
// router + top-k
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(ROUTE_THREADS)
moe_route_kernel(MoERouteArgs a) {
    extern __shared__ float rsm[];
    float *xs = rsm;                       // [RT][H]
    float *ls = rsm + (size_t)RT * a.H;    // [RT][E]
    __shared__ float sc[RT];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int m0 = blockIdx.x * RT;
    const int H = a.H, E = a.E;
    if (tid < RT) {
        const int m = m0 + tid;
        float s = 0.f;
        if (m < a.M && !a.col_part) {
            s = 1.f;   // operand already normalised
            a.tok_scale[m] = s;
        } else if (m < a.M) {
            // folded RMSNorm of the operand: rstd from the producer's block sums
            float ss = 0.f;
            for (int b = 0; b < H / 128; ++b) ss += __ldcg(a.col_part + (size_t)b * a.norm_rows + m);
            const float r = 1.0f / sqrtf(ss / (float)H + a.eps);
            a.col_rstd[m] = r;
            s = r / __ldcg(a.col_prev + m);
            a.tok_scale[m] = s;
        }
        sc[tid] = s;
    }
    for (int i = tid; i < RT * H; i += ROUTE_THREADS) {
        const int t = i / H, k = i - t * H, m = m0 + t;
        xs[i] = m < a.M ? __half2float(a.x[xblk(m, k, a.ldx_rows)]) : 0.f;
    }
    __syncthreads();
    // logits: warp w takes experts w, w+8, ...; lanes split k in 8-wide slices
    for (int e = warp; e < E; e += ROUTE_THREADS / 32) {
        float acc[RT];
#pragma unroll
        for (int t = 0; t < RT; ++t) acc[t] = 0.f;
        const __nv_bfloat16 *wr = a.wr + (size_t)e * H;
        for (int k0 = lane * 8; k0 < H; k0 += 256) {
            const uint4 wv = *reinterpret_cast<const uint4 *>(wr + k0);
            const __nv_bfloat162 *w2 = reinterpret_cast<const __nv_bfloat162 *>(&wv);
            float w[8];
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const float2 f = __bfloat1622float2(w2[i]);
                w[2 * i] = f.x;
                w[2 * i + 1] = f.y;
            }
#pragma unroll
            for (int t = 0; t < RT; ++t) {
                const float4 x0 = *reinterpret_cast<const float4 *>(xs + t * H + k0);
                const float4 x1 = *reinterpret_cast<const float4 *>(xs + t * H + k0 + 4);
                acc[t] += x0.x * w[0] + x0.y * w[1] + x0.z * w[2] + x0.w * w[3] +
                          x1.x * w[4] + x1.y * w[5] + x1.z * w[6] + x1.w * w[7];
            }
        }
#pragma unroll
        for (int t = 0; t < RT; ++t) {
            const float v = warp_sum(acc[t]);
            if (lane == 0) ls[t * E + e] = bf16_round(v * sc[t]);
        }
    }
    __syncthreads();
    // softmax + top-k: warp t routes token m0 + t; lane holds experts lane + 32 i
    if (warp < RT && m0 + warp < a.M) {
        const int m = m0 + warp;
        const int per = E / 32;
        float l[8], p[8];
        bool used[8];
        float mx = -INFINITY;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            l[i] = i < per ? ls[warp * E + lane + 32 * i] : -INFINITY;
            used[i] = i >= per;
            mx = fmaxf(mx, l[i]);
        }
        mx = warp_max(mx);
        float den = 0.f;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            p[i] = i < per ? expf(l[i] - mx) : 0.f;
            den += p[i];
        }
        den = warp_sum(den);
        float sel = 0.f;
        float wsel = 0.f;   // lane j keeps the weight of pick j
        int isel = 0;
        for (int j = 0; j < a.TK; ++j) {
            // lane's best unused (largest logit, then lowest index)
            float bv = -INFINITY;
            int bi = 0x7fffffff;
#pragma unroll
            for (int i = 0; i < 8; ++i)
                if (!used[i] && (l[i] > bv || (l[i] == bv && lane + 32 * i < bi))) { bv = l[i]; bi = lane + 32 * i; }
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) {
                const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
                const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
                if (ov > bv || (ov == bv && oi < bi)) { bv = ov; bi = oi; }
            }
            const int owner = bi & 31, slot = bi >> 5;
            float pw = 0.f;
#pragma unroll
            for (int i = 0; i < 8; ++i)
                if (lane == owner && i == slot) { used[i] = true; pw = p[i] / den; }
            pw = __shfl_sync(0xffffffffu, pw, owner);
            sel += pw;
            if (lane == j) { wsel = pw; isel = bi; }
        }
        if (lane < a.TK) {
            const float w = a.norm_topk ? wsel / sel : wsel;
            const int asg = m * a.TK + lane;
            a.topk_w[asg] = w;
            a.topk_id[asg] = isel;
            const int s = atomicAdd(a.exp_count + isel, 1);
            a.exp_list[(size_t)isel * a.list_cap + s] = asg;
        }
    }
}

// ---------------------------------------------------------------------------
// grouped expert q4 linear
// ---------------------------------------------------------------------------
template <int EPI>
__global__ void __launch_bounds__(EX_THREADS)
moe_expert_kernel(MoEExpertArgs a) {
    __shared__ float up_s[64][EX_TOK + 1];
    __shared__ int asg_s[EX_TOK];
    __shared__ float sc_s[EX_TOK];
    const int e = blockIdx.y, tile = blockIdx.x;
    const int cnt = __ldcg(a.exp_count + e);
    if (cnt == 0) return;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int g = lane >> 2, t = lane & 3;
    const int K = a.K, KW = K / 8, KG = K / 64, nch = K / 128;
    // weight rows of this warp: GATEUP tiles hold 64 gate rows (warps 0, 1) and
    // the 64 up rows of the same outputs (warps 2, 3); DOWN tiles 128 rows
    const bool upper = EPI == 0 && warp >= 2;
    const uint32_t *wq = upper ? a.wq2 : a.wq;
    const __half *sc_base = upper ? a.scales2 : a.scales, *bi_base = upper ? a.biases2 : a.biases;
    const size_t row0 = (size_t)e * a.N + (EPI == 0 ? (size_t)tile * 64 + (warp & 1) * 32
                                                    : (size_t)tile * EX_ROWS + warp * 32);
    // this thread's four weight rows: mt * 16 + h * 8 + g
    const uint4 *wp[2][2];
    const __half *sp[2][2], *bp[2][2];
#pragma unroll
    for (int mt = 0; mt < 2; ++mt)
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            const size_t r = row0 + mt * 16 + h * 8 + g;
            wp[mt][h] = reinterpret_cast<const uint4 *>(wq + r * KW) + t;
            sp[mt][h] = sc_base + r * KG + (t >> 1);
            bp[mt][h] = bi_base + r * KG + (t >> 1);
        }

    for (int tok0 = 0; tok0 < cnt; tok0 += EX_TOK) {
        const int ntile = min(4, (cnt - tok0 + 7) >> 3);
        __syncthreads();   // previous pass's epilogue done with the shared arrays
        if (tid < EX_TOK) {
            const int s = tok0 + tid;
            const int asg = s < cnt ? __ldcg(a.exp_list + (size_t)e * a.list_cap + s) : -1;
            asg_s[tid] = asg;
            if (EPI == 0) sc_s[tid] = asg >= 0 ? __ldcg(a.tok_scale + asg / a.x_div) : 0.f;
            else sc_s[tid] = asg >= 0 ? __ldcg(a.topk_w + asg) : 0.f;
        }
        __syncthreads();
        // operand rows of the B fragments this thread feeds (token g of each n8 tile)
        const __half *xr[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            int asg = asg_s[min(8 * j + g, EX_TOK - 1)];
            if (asg < 0) asg = asg_s[0];
            xr[j] = a.x + (size_t)(asg / a.x_div) * 64 + ((32 * t) & 63);
        }
        float acc[2][4][4];
#pragma unroll
        for (int mt = 0; mt < 2; ++mt)
#pragma unroll
            for (int j = 0; j < 4; ++j)
#pragma unroll
                for (int r = 0; r < 4; ++r) acc[mt][j][r] = 0.f;

        uint4 wcur[2][2];
#pragma unroll
        for (int mt = 0; mt < 2; ++mt)
#pragma unroll
            for (int h = 0; h < 2; ++h) wcur[mt][h] = ldg_stream16(wp[mt][h]);
        for (int c = 0; c < nch; ++c) {
            uint4 wnext[2][2];
            if (c + 1 < nch) {
#pragma unroll
                for (int mt = 0; mt < 2; ++mt)
#pragma unroll
                    for (int h = 0; h < 2; ++h) wnext[mt][h] = ldg_stream16(wp[mt][h] + (size_t)(c + 1) * 4);
            }
            __half2 s2[2][2], b2[2][2];
#pragma unroll
            for (int mt = 0; mt < 2; ++mt)
#pragma unroll
                for (int h = 0; h < 2; ++h) {
                    s2[mt][h] = __half2half2(sp[mt][h][2 * c]);
                    b2[mt][h] = __half2half2(bp[mt][h][2 * c]);
                }
            // 64-wide k block of this thread's 32 k: (128c + 32t) / 64
            const size_t xoff = (size_t)(2 * c + (t >> 1)) * a.ldx_rows * 64;
#pragma unroll
            for (int s = 0; s < 4; ++s) {
                uint4 xv[4];
#pragma unroll
                for (int j = 0; j < 4; ++j)
                    if (j < ntile) xv[j] = *reinterpret_cast<const uint4 *>(xr[j] + xoff + 8 * s);
                uint32_t p[2][2][4];
#pragma unroll
                for (int mt = 0; mt < 2; ++mt)
#pragma unroll
                    for (int h = 0; h < 2; ++h) {
                        const uint32_t w = (&wcur[mt][h].x)[s];
                        p[mt][h][0] = dq2(w, 0, s2[mt][h], b2[mt][h]);
                        p[mt][h][1] = dq2(w, 4, s2[mt][h], b2[mt][h]);
                        p[mt][h][2] = dq2(w, 8, s2[mt][h], b2[mt][h]);
                        p[mt][h][3] = dq2(w, 12, s2[mt][h], b2[mt][h]);
                    }
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    if (j < ntile) {
#pragma unroll
                        for (int mt = 0; mt < 2; ++mt) {
                            mma16816(acc[mt][j], p[mt][0][0], p[mt][1][0], p[mt][0][1], p[mt][1][1], xv[j].x, xv[j].y);
                            mma16816(acc[mt][j], p[mt][0][2], p[mt][1][2], p[mt][0][3], p[mt][1][3], xv[j].z, xv[j].w);
                        }
                    }
                }
            }
            if (c + 1 < nch) {
#pragma unroll
                for (int mt = 0; mt < 2; ++mt)
#pragma unroll
                    for (int h = 0; h < 2; ++h) wcur[mt][h] = wnext[mt][h];
            }
        }

        // accumulator (mt, j, r): weight row warp*32 + mt*16 + g + 8*(r>>1),
        // assignment column 8j + 2t + (r&1)
        if (EPI == 0) {
            if (warp >= 2) {
#pragma unroll
                for (int mt = 0; mt < 2; ++mt)
#pragma unroll
                    for (int j = 0; j < 4; ++j)
#pragma unroll
                        for (int r = 0; r < 4; ++r)
                            up_s[(warp - 2) * 32 + mt * 16 + g + 8 * (r >> 1)][8 * j + 2 * t + (r & 1)] = acc[mt][j][r];
            }
            __syncthreads();
            if (warp < 2) {
#pragma unroll
                for (int mt = 0; mt < 2; ++mt)
#pragma unroll
                    for (int j = 0; j < 4; ++j)
#pragma unroll
                        for (int r = 0; r < 4; ++r) {
                            const int row = warp * 32 + mt * 16 + g + 8 * (r >> 1);   // 0..63
                            const int col = 8 * j + 2 * t + (r & 1);
                            const int asg = asg_s[col];
                            if (j < ntile && asg >= 0) {
                                const float s = sc_s[col];
                                const float gv = acc[mt][j][r] * s, uv = up_s[row][col] * s;
                                const float act = gv / (1.0f + expf(-gv)) * uv;
                                const int o = tile * 64 + row;
                                a.act[xblk(asg, o, a.act_rows)] = __float2half_rn(act);
                            }
                        }
            }
        } else {
#pragma unroll
            for (int mt = 0; mt < 2; ++mt)
#pragma unroll
                for (int j = 0; j < 4; ++j)
#pragma unroll
                    for (int r = 0; r < 4; ++r) {
                        const int row = tile * EX_ROWS + warp * 32 + mt * 16 + g + 8 * (r >> 1);
                        const int col = 8 * j + 2 * t + (r & 1);
                        const int asg = asg_s[col];
                        if (j < ntile && asg >= 0) a.y[(size_t)asg * a.N + row] = acc[mt][j][r] * sc_s[col];
                    }
        }
    }
}

// ---------------------------------------------------------------------------
// combine + folded RMSNorm producer
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(COMBINE_THREADS)
moe_combine_kernel(MoECombineArgs a) {
    __shared__ float wsum[64];   // per 32-feature slice (H <= 2048 per pass of 256 x 8)
    const int m = blockIdx.x, tid = threadIdx.x, lane = tid & 31;
    const int H = a.H;
    const float s = a.norm_w ? __ldcg(a.norm_scale + m) : 0.f;
    for (int base = 0; base < H; base += 2048) {
        const int span = min(2048, H - base);
        for (int i = tid; i < span; i += COMBINE_THREADS) {
            const int f = base + i;
            float v = a.h[(size_t)m * H + f];
            for (int j = 0; j < a.TK; ++j) v += __ldcg(a.y + ((size_t)m * a.TK + j) * H + f);
            a.h[(size_t)m * H + f] = v;
            if (a.norm_w) {
                a.xout[xblk(m, f, a.ldx_rows)] = __float2half_rn(v * a.norm_w[f] * s);
                const float q = warp_sum(v * v);
                if (lane == 0) wsum[i >> 5] = q;
            }
        }
        if (a.norm_w) {
            __syncthreads();
            if (tid < span / 128) {
                const int b = tid;
                a.norm_part[(size_t)(base / 128 + b) * a.norm_rows + m] =
                    wsum[4 * b] + wsum[4 * b + 1] + wsum[4 * b + 2] + wsum[4 * b + 3];
            }
            __syncthreads();
        }
    }
}

__global__ void router_synth_kernel(uint64_t seed, uint32_t tensor_id, float stddev, int E, int H,
                                    __nv_bfloat16 *w) {
    const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= (long long)E * H) return;
    w[i] = __float2bfloat16_rn(__fmul_rn(det_normal(seed, tensor_id, (uint64_t)i), stddev));
}

}  // namespace

size_t moe_route_smem(int H, int E) { return sizeof(float) * (size_t)RT * (H + E); }

cudaError_t moe_route(const MoERouteArgs &a, cudaStream_t st) {
    if (a.E % 32 || a.E > 256 || a.TK < 1 || a.TK > 8 || a.TK > a.E || a.H % 256 || a.M <= 0)
        return cudaErrorInvalidValue;
    const size_t sm = moe_route_smem(a.H, a.E);
    if (sm > 48 * 1024) {
        cudaError_t e = cudaFuncSetAttribute(moe_route_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm);
        if (e != cudaSuccess) return e;
    }
    moe_route_kernel<<<(a.M + RT - 1) / RT, ROUTE_THREADS, sm, st>>>(a);
    return cudaGetLastError();
}

cudaError_t moe_expert(const MoEExpertArgs &a, int epi, cudaStream_t st) {
    if (a.K % 128 || a.E <= 0 || (epi == 0 ? a.N % 64 || !a.wq2 : a.N % EX_ROWS)) return cudaErrorInvalidValue;
    dim3 grid(epi == 0 ? a.N / 64 : a.N / EX_ROWS, a.E);
    if (epi == 0) moe_expert_kernel<0><<<grid, EX_THREADS, 0, st>>>(a);
    else moe_expert_kernel<1><<<grid, EX_THREADS, 0, st>>>(a);
    return cudaGetLastError();
}

cudaError_t moe_combine(const MoECombineArgs &a, cudaStream_t st) {
    if (a.H % 128 || a.M <= 0) return cudaErrorInvalidValue;
    moe_combine_kernel<<<a.M, COMBINE_THREADS, 0, st>>>(a);
    return cudaGetLastError();
}

cudaError_t router_synth(uint64_t seed, uint32_t tensor_id, float stddev, int E, int H, void *w, cudaStream_t st) {
    const long long n = (long long)E * H;
    router_synth_kernel<<<(unsigned)((n + 255) / 256), 256, 0, st>>>(seed, tensor_id, stddev, E, H,
                                                                     static_cast<__nv_bfloat16 *>(w));
    return cudaGetLastError();
}

}  // namespace mlxcat
