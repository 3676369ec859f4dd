// q4_linear.cu -- MLX affine 4-bit (group 64) linear for small token counts.
//
//   y[s][m][n] = sum_{k in split s} x[m][k] * (scale[n][k/64] * q[n][k] + bias[n][k/64])
//
// Replaces mlx-swift's quantizedMatmul (QuantizedLinear in mlx-swift-lm) on
// the verify forward (BatchGenerator.swift:900-904).  Weights stay in the MLX
// layout: packed uint32 [N][K/8] with the lowest nibble first, fp16 scales and
// biases [N][K/64].
//
// Design (HBM-bound stream of weights, tokens on the tensor core):
//   * CTA = 8 warps = 4 feature warps x 2 k-halves; a feature warp owns
//     32 output features (4 n8 tiles), the two k-halves take alternate
//     128-wide chunks and are summed through shared memory at the end.
//   * Each thread streams one 16-byte (32-nibble) load per n8 tile per chunk:
//     coalesced 128-bit loads of whole 64-byte row segments, prefetched one
//     chunk ahead in registers.
//   * Nibbles are unpacked with the 0x6400 fp16 magic (lop3), made exact
//     integers with one hsub2 and dequantised with one hfma2 per pair, and fed
//     as the B operand (k16 x n8) of mma.m16n8k16; tokens are the A operand
//     (m16 tiles), staged in shared memory from the permuted activation layout
//     (common.cuh: xperm) so a plain ldmatrix.x4 matches the unpack order.
//   * Split-K across CTAs (grid.y) writes fp32 partials; the consumer kernel
//     sums the splits in a fixed order (deterministic, no atomics).
#include "common.cuh"
#include "kernels.h"

namespace mlxcat {

namespace {

constexpr int NT = 4;              // n8 tiles per feature warp
constexpr int FWARPS = 4;          // feature warps per CTA
constexpr int THREADS = 256;       // FWARPS x 2 k-halves
constexpr int FEAT_PER_CTA = FWARPS * NT * 8;   // 128
constexpr int CHUNK = 128;         // k per chunk
constexpr int SUB = 512;           // k per staged activation sub-block
constexpr int XPITCH = SUB + 8;    // halves; +16 B breaks ldmatrix bank conflicts

__device__ __forceinline__ uint32_t lop3_and_or(uint32_t a, uint32_t b, uint32_t c) {
    uint32_t d;
    asm("lop3.b32 %0, %1, %2, %3, 0xea;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}

__device__ __forceinline__ uint32_t dq_pair(uint32_t w, int shift, __half2 s2, __half2 b2) {
    const uint32_t v = lop3_and_or(w >> shift, 0x000f000fu, 0x64006400u);
    __half2 q = __hsub2(*reinterpret_cast<const __half2 *>(&v),
                        __halves2half2(__ushort_as_half(0x6400), __ushort_as_half(0x6400)));
    __half2 r = __hfma2(q, s2, b2);
    return *reinterpret_cast<uint32_t *>(&r);
}

__device__ __forceinline__ void mma16816(float *c, const uint32_t *a, uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
        "{%8,%9}, {%0,%1,%2,%3};\n"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

__device__ __forceinline__ void ldmatrix_x4(uint32_t *d, uint32_t saddr) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];\n"
                 : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
                 : "r"(saddr));
}

__device__ __forceinline__ void cp_async16(uint32_t saddr, const void *g, int src_bytes) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(saddr), "l"(g),
                 "r"(src_bytes));
}
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;\n" ::); }

__device__ __forceinline__ uint4 ldg_stream(const uint4 *p) {
    uint4 r;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];\n"
                 : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
                 : "l"(p));
    return r;
}

template <int MT>
__global__ void __launch_bounds__(THREADS, 2)
q4_linear_kernel(const uint32_t *__restrict__ wq, const __half *__restrict__ scales,
                 const __half *__restrict__ biases, int N, int K,
                 const __half *__restrict__ x, int M, int ldx, int chunks_per_split,
                 float *__restrict__ out) {
    extern __shared__ __align__(16) unsigned char smem[];
    __half *xs = reinterpret_cast<__half *>(smem);

    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int fw = warp & (FWARPS - 1), kh = warp >> 2;
    const int g = lane >> 2, t = lane & 3;
    const int split = blockIdx.y;
    const int tok0 = blockIdx.z * (MT * 16);
    const int nchunks = K / CHUNK;
    const int c_begin = split * chunks_per_split;
    const int c_end = min(nchunks, c_begin + chunks_per_split);
    const int f_base = blockIdx.x * FEAT_PER_CTA + fw * (NT * 8);
    const int KW = K / 8, KG = K / MLXCAT_GS;

    float acc[MT][NT][4];
#pragma unroll
    for (int i = 0; i < MT; ++i)
#pragma unroll
        for (int j = 0; j < NT; ++j)
#pragma unroll
            for (int r = 0; r < 4; ++r) acc[i][j][r] = 0.f;

    // weight row pointers for this thread: feature f_base + 8j + g, words at 4t
    const uint4 *wrow[NT];
#pragma unroll
    for (int j = 0; j < NT; ++j)
        wrow[j] = reinterpret_cast<const uint4 *>(wq + (size_t)(f_base + 8 * j + g) * KW) + t;

    // first chunk handled by this warp
    int c = c_begin + kh;
    uint4 wcur[NT];
    if (c < c_end) {
#pragma unroll
        for (int j = 0; j < NT; ++j) wcur[j] = ldg_stream(wrow[j] + (size_t)c * 4);
    }

    const uint32_t xs_base = (uint32_t)__cvta_generic_to_shared(xs);
    const int rows = MT * 16;

    for (int sb0 = c_begin; sb0 < c_end; sb0 += SUB / CHUNK) {
        const int sb_chunks = min(SUB / CHUNK, c_end - sb0);
        __syncthreads();
        // stage activations [rows][sb_chunks*128] (already permuted per 128-block)
        {
            const int vec_per_row = sb_chunks * CHUNK / 8;
            const int total = rows * vec_per_row;
            for (int v = threadIdx.x; v < total; v += THREADS) {
                const int r = v / vec_per_row, cv = v - r * vec_per_row;
                const int tok = tok0 + r;
                const __half *src = x + (size_t)min(tok, M - 1) * ldx + (size_t)sb0 * CHUNK + cv * 8;
                cp_async16(xs_base + (uint32_t)(r * XPITCH + cv * 8) * 2, src, tok < M ? 16 : 0);
            }
            cp_async_wait_all();
        }
        __syncthreads();

        for (; c < sb0 + sb_chunks; c += 2) {
            // prefetch the next chunk this warp will process
            const int cn = c + 2;
            uint4 wnext[NT];
            if (cn < c_end) {
#pragma unroll
                for (int j = 0; j < NT; ++j) wnext[j] = ldg_stream(wrow[j] + (size_t)cn * 4);
            }
            // group of this thread's 32 k: (c*128 + 32t)/64
            const int grp = c * 2 + (t >> 1);
            __half2 s2[NT], b2[NT];
#pragma unroll
            for (int j = 0; j < NT; ++j) {
                const size_t o = (size_t)(f_base + 8 * j + g) * KG + grp;
                s2[j] = __half2half2(scales[o]);
                b2[j] = __half2half2(biases[o]);
            }
            const int kc = (c - sb0) * CHUNK;   // chunk offset inside the staged block
#pragma unroll
            for (int i = 0; i < 4; ++i) {          // word i of the 16-byte load
                uint32_t bf[NT][4];
#pragma unroll
                for (int j = 0; j < NT; ++j) {
                    const uint32_t w = (&wcur[j].x)[i];
                    bf[j][0] = dq_pair(w, 0, s2[j], b2[j]);
                    bf[j][1] = dq_pair(w, 4, s2[j], b2[j]);
                    bf[j][2] = dq_pair(w, 8, s2[j], b2[j]);
                    bf[j][3] = dq_pair(w, 12, s2[j], b2[j]);
                }
#pragma unroll
                for (int e = 0; e < 2; ++e) {
                    const int s = 2 * i + e;
#pragma unroll
                    for (int mt = 0; mt < MT; ++mt) {
                        // matrix mi = lane/8: tokens +8*(mi&1), half h = mi>>1
                        const int mi = lane >> 3, rr = lane & 7;
                        const int row = mt * 16 + (mi & 1) * 8 + rr;
                        const uint32_t addr =
                            xs_base + (uint32_t)(row * XPITCH + kc + (s * 2 + (mi >> 1)) * 8) * 2;
                        uint32_t a[4];
                        ldmatrix_x4(a, addr);
#pragma unroll
                        for (int j = 0; j < NT; ++j) mma16816(acc[mt][j], a, bf[j][2 * e], bf[j][2 * e + 1]);
                    }
                }
            }
            if (cn < c_end) {
#pragma unroll
                for (int j = 0; j < NT; ++j) wcur[j] = wnext[j];
            }
        }
    }

    // sum the two k-halves through shared memory
    __syncthreads();
    float *red = reinterpret_cast<float *>(smem);
    constexpr int NR = MT * NT * 4;
    if (kh == 1) {
#pragma unroll
        for (int mt = 0; mt < MT; ++mt)
#pragma unroll
            for (int j = 0; j < NT; ++j)
#pragma unroll
                for (int r = 0; r < 4; ++r)
                    red[((fw * NR) + (mt * NT + j) * 4 + r) * 32 + lane] = acc[mt][j][r];
    }
    __syncthreads();
    if (kh == 0) {
        float *o = out + (size_t)split * M * N;
#pragma unroll
        for (int mt = 0; mt < MT; ++mt)
#pragma unroll
            for (int j = 0; j < NT; ++j) {
                float v[4];
#pragma unroll
                for (int r = 0; r < 4; ++r)
                    v[r] = acc[mt][j][r] + red[((fw * NR) + (mt * NT + j) * 4 + r) * 32 + lane];
                const int f = f_base + 8 * j + 2 * t;
                const int m0 = tok0 + mt * 16 + g;
                if (m0 < M) *reinterpret_cast<float2 *>(o + (size_t)m0 * N + f) = make_float2(v[0], v[1]);
                if (m0 + 8 < M)
                    *reinterpret_cast<float2 *>(o + (size_t)(m0 + 8) * N + f) = make_float2(v[2], v[3]);
            }
    }
}

template <int MT>
size_t smem_bytes() {
    const size_t xsb = (size_t)MT * 16 * XPITCH * 2;
    const size_t red = (size_t)FWARPS * MT * NT * 4 * 32 * 4;
    return xsb > red ? xsb : red;
}

template <int MT>
cudaError_t launch_mt(const Q4Weight &w, const __half *x, int M, int ldx, int splits, float *out,
                      cudaStream_t st) {
    static bool attr_set[64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    const size_t sm = smem_bytes<MT>();
    if (!attr_set[dev & 63]) {
        cudaError_t e = cudaFuncSetAttribute(q4_linear_kernel<MT>,
                                             cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm);
        if (e != cudaSuccess) return e;
        attr_set[dev & 63] = true;
    }
    const int nchunks = w.K / CHUNK;
    const int cps = (nchunks + splits - 1) / splits;
    const int real_splits = (nchunks + cps - 1) / cps;
    dim3 grid(w.N / FEAT_PER_CTA, real_splits, (M + MT * 16 - 1) / (MT * 16));
    q4_linear_kernel<MT><<<grid, THREADS, sm, st>>>(w.wq, w.scales, w.biases, w.N, w.K, x, M, ldx,
                                                    cps, out);
    return cudaGetLastError();
}

}  // namespace

int q4_linear_splits(int N, int K, int M, int sm_count) {
    // enough CTAs to cover ~2 waves of 148 SMs, each split >= 2 chunks per k-half
    const int ctas = N / FEAT_PER_CTA * ((M + 63) / 64);
    const int nchunks = K / CHUNK;
    int s = 1;
    while (ctas * s < 2 * sm_count && nchunks / (s * 2) >= 4) s *= 2;
    return s;
}

int q4_linear_real_splits(int K, int splits) {
    const int nchunks = K / CHUNK;
    const int cps = (nchunks + splits - 1) / splits;
    return (nchunks + cps - 1) / cps;
}

cudaError_t q4_linear(const Q4Weight &w, const __half *x, int M, int ldx, int splits, float *out,
                      cudaStream_t st) {
    if (w.N % FEAT_PER_CTA != 0 || w.K % CHUNK != 0 || M <= 0) return cudaErrorInvalidValue;
    // token tiles of up to 64 rows per grid.z slice
    if (M <= 16) return launch_mt<1>(w, x, M, ldx, splits, out, st);
    if (M <= 32) return launch_mt<2>(w, x, M, ldx, splits, out, st);
    if (M <= 48) return launch_mt<3>(w, x, M, ldx, splits, out, st);
    return launch_mt<4>(w, x, M, ldx, splits, out, st);
}

}  // namespace mlxcat
