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
//   moe_logits_kernel   bf16 router GEMV, 4 tokens x 4 experts per warp, logits
//                       rounded to bf16;
//   moe_topk_kernel     softmax + top-k, one warp per token; appends each
//                       (token, slot) assignment to its expert's list (atomic
//                       slot, fixed capacity = token rows).
//   moe_expert_kernel   grouped q4 linear: CTA = (128-row tile, expert); the
//                       expert's assignments are the columns.  Weights stay in
//                       the MLX SwitchGLU layout, [E][out][in/8] per projection,
//                       and are the A operand of mma.m16n8k16 (dequantised in
//                       registers from coalesced 16-byte loads), tokens the B operand in groups
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

// The four nibble pairs (i, i + 4) of one packed word with one shift: the pairs
// at bits 0-3 / 16-19 take the 0x6400 magic (fp16 1024 + q); the pairs at bits
// 4-7 / 20-23 take the 0x5400 magic (fp16 64.0, whose unit in the last place is
// 1/16, so mantissa bits 4-7 hold exactly 64 + q); the other two pairs the same
// from w >> 8.  Each pair then becomes q * scale + bias.
__device__ __forceinline__ void dq_word(uint32_t w, __half2 s2, __half2 b2, uint32_t out[4]) {
    const uint32_t hi = w >> 8;
    uint32_t v[4] = {(w & 0x000f000fu) | 0x64006400u, (w & 0x00f000f0u) | 0x54005400u,
                     (hi & 0x000f000fu) | 0x64006400u, (hi & 0x00f000f0u) | 0x54005400u};
    const __half2 k1024 = __halves2half2(__ushort_as_half(0x6400), __ushort_as_half(0x6400));
    const __half2 k64 = __halves2half2(__ushort_as_half(0x5400), __ushort_as_half(0x5400));
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const __half2 q = __hsub2(*reinterpret_cast<const __half2 *>(&v[i]), (i & 1) ? k64 : k1024);
        const __half2 r = __hfma2(q, s2, b2);
        out[i] = *reinterpret_cast<const uint32_t *>(&r);
    }
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
// router logits: warp = 4 tokens x 4 experts, lanes split k in 8-wide blocks;
// CTA = 8 warps = 32 experts of 4 tokens (grid: token groups x E/32)
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(ROUTE_THREADS)
moe_logits_kernel(MoERouteArgs a) {
    __shared__ float sc[RT];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int m0 = blockIdx.x * RT;
    const int H = a.H, E = a.E;
    if (tid < RT) {
        const int m = m0 + tid;
        float s = 0.f;
        if (m < a.M && !a.col_part) {
            s = 1.f;   // operand already normalised
        } else if (m < a.M) {
            // folded RMSNorm of the operand: rstd from the producer's block sums
            float ss = 0.f;
            for (int b = 0; b < H / 128; ++b) ss += __ldcg(a.col_part + (size_t)b * a.norm_rows + m);
            const float r = 1.0f / sqrtf(ss / (float)H + a.eps);
            if (blockIdx.y == 0) a.col_rstd[m] = r;
            s = r / __ldcg(a.col_prev + m);
        }
        if (m < a.M && blockIdx.y == 0) a.tok_scale[m] = s;
        sc[tid] = s;
    }
    __syncthreads();
    const int e0 = (blockIdx.y * (ROUTE_THREADS / 32) + warp) * 4;
    float acc[RT][4];
#pragma unroll
    for (int t = 0; t < RT; ++t)
#pragma unroll
        for (int q = 0; q < 4; ++q) acc[t][q] = 0.f;
    for (int b = lane; b < H / 8; b += 32) {
        // operand 8-block b of each token, perm8 order (k0, k0+4, k0+1, k0+5, ...)
        float xv[RT][8];
#pragma unroll
        for (int t = 0; t < RT; ++t) {
            const int m = m0 + t;
            uint4 u = make_uint4(0, 0, 0, 0);
            if (m < a.M)
                u = *reinterpret_cast<const uint4 *>(a.x + ((size_t)(b >> 3) * a.ldx_rows + m) * 64 + (b & 7) * 8);
            const __half2 *h2 = reinterpret_cast<const __half2 *>(&u);
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const float2 f = __half22float2(h2[i]);
                xv[t][2 * i] = f.x;       // natural k0 + i
                xv[t][2 * i + 1] = f.y;   // natural k0 + i + 4
            }
        }
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            const uint4 wv = *reinterpret_cast<const uint4 *>(a.wr + (size_t)(e0 + q) * H + 8 * b);
            const __nv_bfloat162 *w2 = reinterpret_cast<const __nv_bfloat162 *>(&wv);
            float w[8];
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const float2 f = __bfloat1622float2(w2[i]);
                w[2 * i] = f.x;
                w[2 * i + 1] = f.y;
            }
            // pinned arithmetic (no contraction): d = sum_i (x[k0+i] w[k0+i] + x[k0+i+4] w[k0+i+4]),
            // lane accumulator += d; lanes then summed by the xor butterfly 16, 8, 4, 2, 1.
            // The CPU restatement repeats exactly this order, so the bf16 logits are
            // bit-identical for the same operand.
#pragma unroll
            for (int t = 0; t < RT; ++t) {
                float d = 0.f;
#pragma unroll
                for (int i = 0; i < 4; ++i)
                    d = __fadd_rn(d, __fadd_rn(__fmul_rn(xv[t][2 * i], w[i]), __fmul_rn(xv[t][2 * i + 1], w[i + 4])));
                acc[t][q] = __fadd_rn(acc[t][q], d);
            }
        }
    }
#pragma unroll
    for (int t = 0; t < RT; ++t)
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            const float v = warp_sum(acc[t][q]);
            if (lane == 0 && m0 + t < a.M) a.logits[(size_t)(m0 + t) * E + e0 + q] = bf16_round(__fmul_rn(v, sc[t]));
        }
}

// ---------------------------------------------------------------------------
// softmax + top-k: one warp per token; lane holds experts lane + 32 i
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(ROUTE_THREADS)
moe_topk_kernel(MoERouteArgs a) {
    const int lane = threadIdx.x & 31;
    const int m = blockIdx.x * (ROUTE_THREADS / 32) + (threadIdx.x >> 5);
    if (m >= a.M) return;
    const int E = a.E, per = E / 32;
    float l[8], p[8];
    bool used[8];
    float mx = -INFINITY;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        l[i] = i < per ? __ldcg(a.logits + (size_t)m * E + lane + 32 * i) : -INFINITY;
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
                        dq_word(w, s2[mt][h], b2[mt][h], p[mt][h]);
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
// combine + folded RMSNorm producer: thread = 8 consecutive features (two
// 16-byte loads per source row), 16 threads = one 128-feature norm block
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(COMBINE_THREADS)
moe_combine_kernel(MoECombineArgs a) {
    const int m = blockIdx.x, tid = threadIdx.x, lane = tid & 31;
    const int H = a.H, tk = a.TK;
    const float s = a.norm_w ? __ldcg(a.norm_scale + m) : 0.f;
    for (int base = 0; base < H; base += 8 * COMBINE_THREADS) {
        const int f0 = base + 8 * tid;
        const bool on = f0 < H;
        float v[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
        if (on) {
            float4 *hp = reinterpret_cast<float4 *>(a.h + (size_t)m * H + f0);
            float4 y[16];
#pragma unroll
            for (int j = 0; j < 8; ++j)
                if (j < tk) {
                    const float4 *yp = reinterpret_cast<const float4 *>(a.y + ((size_t)m * tk + j) * H + f0);
                    y[2 * j] = __ldcg(yp);
                    y[2 * j + 1] = __ldcg(yp + 1);
                }
            const float4 h0 = hp[0], h1 = hp[1];
            v[0] = h0.x; v[1] = h0.y; v[2] = h0.z; v[3] = h0.w;
            v[4] = h1.x; v[5] = h1.y; v[6] = h1.z; v[7] = h1.w;
#pragma unroll
            for (int j = 0; j < 8; ++j)
                if (j < tk) {   // selection order
                    v[0] += y[2 * j].x; v[1] += y[2 * j].y; v[2] += y[2 * j].z; v[3] += y[2 * j].w;
                    v[4] += y[2 * j + 1].x; v[5] += y[2 * j + 1].y; v[6] += y[2 * j + 1].z; v[7] += y[2 * j + 1].w;
                }
            hp[0] = make_float4(v[0], v[1], v[2], v[3]);
            hp[1] = make_float4(v[4], v[5], v[6], v[7]);
        }
        if (a.norm_w) {
            float sq = 0.f;
            if (on) {
                __align__(16) __half o[8];
#pragma unroll
                for (int i = 0; i < 8; ++i) {
                    o[perm8(i)] = __float2half_rn(v[i] * a.norm_w[f0 + i] * s);
                    sq += v[i] * v[i];
                }
                *reinterpret_cast<uint4 *>(a.xout + xblk(m, f0, a.ldx_rows)) = *reinterpret_cast<const uint4 *>(o);
            }
#pragma unroll
            for (int o = 8; o > 0; o >>= 1) sq += __shfl_xor_sync(0xffffffffu, sq, o);
            if (on && (lane & 15) == 0) a.norm_part[(size_t)(f0 / 128) * a.norm_rows + m] = sq;
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

cudaError_t moe_route(const MoERouteArgs &a, cudaStream_t st) {
    if (a.E % 32 || a.E > 256 || a.TK < 1 || a.TK > 8 || a.TK > a.E || a.H % 256 || a.M <= 0 || !a.logits)
        return cudaErrorInvalidValue;
    moe_logits_kernel<<<dim3((a.M + RT - 1) / RT, a.E / 32), ROUTE_THREADS, 0, st>>>(a);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return e;
    moe_topk_kernel<<<(a.M + ROUTE_THREADS / 32 - 1) / (ROUTE_THREADS / 32), ROUTE_THREADS, 0, st>>>(a);
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
    if (a.H % 128 || a.M <= 0 || a.TK < 1 || a.TK > 8) return cudaErrorInvalidValue;
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
