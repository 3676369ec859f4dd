// common.cuh -- shared device helpers for the mlxcat_b200 kernels (sm_100a).
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#define MLXCAT_GS 64          // MLX affine group size
#define MLXCAT_MAX_EOS 8

namespace mlxcat {

// ---------------------------------------------------------------------------
// Deterministic arithmetic.  Every operation is an explicitly rounded
// intrinsic so nvcc cannot contract or reorder; the CPU oracle compiles the
// same sequence with -ffp-contract=off and gets identical bits.
// ---------------------------------------------------------------------------
__host__ __device__ __forceinline__ void philox4x32_10(uint32_t c0, uint32_t c1, uint32_t c2,
                                                       uint32_t c3, uint32_t k0, uint32_t k1,
                                                       uint32_t out[4]) {
    // Philox4x32-10, Salmon et al., SC'11.
#pragma unroll
    for (int r = 0; r < 10; ++r) {
        const uint64_t p0 = (uint64_t)0xD2511F53u * c0;
        const uint64_t p1 = (uint64_t)0xCD9E8D57u * c2;
        const uint32_t hi0 = (uint32_t)(p0 >> 32), lo0 = (uint32_t)p0;
        const uint32_t hi1 = (uint32_t)(p1 >> 32), lo1 = (uint32_t)p1;
        c0 = hi1 ^ c1 ^ k0;
        c1 = lo1;
        c2 = hi0 ^ c3 ^ k1;
        c3 = lo0;
        k0 += 0x9E3779B9u;
        k1 += 0xBB67AE85u;
    }
    out[0] = c0; out[1] = c1; out[2] = c2; out[3] = c3;
}

// Uniform stream of one request: key = its seed, counter = (generation index,
// purpose).  purpose 0: draft-acceptance uniform, 1: sampling uniform.
__device__ __forceinline__ uint32_t request_uniform(uint64_t seed, uint64_t gen_index,
                                                    uint32_t purpose) {
    uint32_t r[4];
    philox4x32_10((uint32_t)gen_index, (uint32_t)(gen_index >> 32), purpose, 0u,
                  (uint32_t)seed, (uint32_t)(seed >> 32), r);
    return r[0];
}

// e^x for x <= 0: Cody-Waite reduction by ln2 (fdlibm's hi/lo split) and the
// degree-7 Taylor polynomial of e^r on |r| <= ln2/2.
__device__ __forceinline__ float det_exp_neg(float x) {
    if (!(x > -87.0f)) return 0.0f;
    if (x > 0.0f) x = 0.0f;
    const float n = rintf(__fmul_rn(x, 1.44269504f));
    float r = __fmaf_rn(-n, 6.9314575195e-01f, x);
    r = __fmaf_rn(-n, 1.4286067653e-06f, r);
    float p = 1.0f / 5040.0f;
    p = __fmaf_rn(p, r, 1.0f / 720.0f);
    p = __fmaf_rn(p, r, 1.0f / 120.0f);
    p = __fmaf_rn(p, r, 1.0f / 24.0f);
    p = __fmaf_rn(p, r, 1.0f / 6.0f);
    p = __fmaf_rn(p, r, 0.5f);
    p = __fmaf_rn(p, r, 1.0f);
    p = __fmaf_rn(p, r, 1.0f);
    const float scale = __uint_as_float((uint32_t)((int)n + 127) << 23);
    return __fmul_rn(p, scale);
}

// log x for normal x > 0: x = m 2^e with m in [sqrt(1/2), sqrt(2)),
// log m = 2 atanh(f), f = (m-1)/(m+1), odd series to f^9.
__device__ __forceinline__ float det_log(float x) {
    const uint32_t b = __float_as_uint(x);
    int e = (int)((b >> 23) & 0xffu) - 127;
    float m = __uint_as_float((b & 0x7fffffu) | 0x3f800000u);
    if (m > 1.41421356f) { m = __fmul_rn(m, 0.5f); e += 1; }
    const float f = __fdiv_rn(__fadd_rn(m, -1.0f), __fadd_rn(m, 1.0f));
    const float f2 = __fmul_rn(f, f);
    float p = 2.0f / 9.0f;
    p = __fmaf_rn(p, f2, 2.0f / 7.0f);
    p = __fmaf_rn(p, f2, 2.0f / 5.0f);
    p = __fmaf_rn(p, f2, 2.0f / 3.0f);
    p = __fmaf_rn(p, f2, 2.0f);
    const float lm = __fmul_rn(p, f);
    const float fe = (float)e;
    return __fmaf_rn(fe, 6.9314575195e-01f, __fmaf_rn(fe, 1.4286067653e-06f, lm));
}

// Normal variate for weight synthesis: Marsaglia polar method on the Philox
// stream (key = weight seed, counter = (element index, tensor id, attempt)).
__device__ __forceinline__ float det_normal(uint64_t seed, uint32_t tensor_id, uint64_t index) {
    for (uint32_t a = 0; a < 8; ++a) {
        uint32_t r[4];
        philox4x32_10((uint32_t)index, (uint32_t)(index >> 32), tensor_id, a, (uint32_t)seed,
                      (uint32_t)(seed >> 32), r);
#pragma unroll
        for (int p = 0; p < 2; ++p) {
            const float u1 = __fadd_rn(__fmul_rn((float)(r[2 * p] >> 8), 1.1920928955078125e-07f), -1.0f);
            const float u2 = __fadd_rn(__fmul_rn((float)(r[2 * p + 1] >> 8), 1.1920928955078125e-07f), -1.0f);
            const float s = __fadd_rn(__fmul_rn(u1, u1), __fmul_rn(u2, u2));
            if (s < 1.0f && s > 0.0f) {
                const float t = __fdiv_rn(__fmul_rn(-2.0f, det_log(s)), s);
                return __fmul_rn(u1, __fsqrt_rn(t));
            }
        }
    }
    return 0.0f;
}

// Fixed-point probability: e in [0,1] at 2^24 resolution, truncated.
__device__ __forceinline__ uint32_t fix24(float e) { return __float2uint_rz(__fmul_rn(e, 16777216.0f)); }

// floor(u * S / 2^32) exactly, S < 2^64
__host__ __device__ __forceinline__ uint64_t scale_u32(uint32_t u, uint64_t S) {
    return (uint64_t)u * (S >> 32) + (((uint64_t)u * (S & 0xffffffffull)) >> 32);
}

// Monotone map float -> uint32 (larger float -> larger key).
__device__ __forceinline__ uint32_t float_key(float f) {
    const uint32_t u = __float_as_uint(f);
    return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

// Programmatic dependent launch: a kernel launched with programmatic stream
// serialisation may start while its predecessor still runs; it must call
// griddep_wait() before touching anything the predecessor writes.  A
// predecessor calls griddep_launch_dependents() to let that happen early.
__device__ __forceinline__ void griddep_wait() { asm volatile("griddepcontrol.wait;\n" ::: "memory"); }
__device__ __forceinline__ void griddep_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;\n" ::); }

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

// ---------------------------------------------------------------------------
// Activation layout for the q4 linear's token operand.  Inside every block of
// 128 input features the fp16 values are stored permuted so that a plain
// ldmatrix.x4 yields the mma.m16n8k16 A fragment in the order the weight
// nibbles are unpacked (see q4_linear.cu).  Natural index k = 32t + 8i + 2e +
// h + 4j  (t,i in [0,4), e,h,j in [0,2)) is stored at ((2i+e)*2 + h)*8 + 2t + j.
// ---------------------------------------------------------------------------
__host__ __device__ __forceinline__ int xperm(int k) {
    const int blk = k & ~127, r = k & 127;
    const int t = r >> 5, i = (r >> 3) & 3, w = r & 7;
    const int e = (w >> 1) & 1, h = w & 1, j = (w >> 2) & 1;
    return blk + (((2 * i + e) * 2 + h) * 8 + 2 * t + j);
}

// Token-operand layout of the tensor-core q4 linear: inside every block of 8
// features the fp16 values are stored in the order (0,4,1,5,2,6,3,7) -- the
// order in which the kernel unpacks the nibbles of one packed weight word.
__host__ __device__ __forceinline__ int perm8(int k) {
    return (k & ~7) | (((k & 3) << 1) | ((k >> 2) & 1));
}

// Token operand of the tensor-core q4 linear in memory: blocked by 64
// features, [K/64][rows][64] fp16, perm8 order inside each 8-block, so one
// 3-D TMA box fetches a [256 k x tokens] tile.  Element (m, k) of a buffer
// with `rows` token rows:
__host__ __device__ __forceinline__ size_t xblk(int m, int k, int rows) {
    return ((size_t)(k >> 6) * rows + m) * 64 + perm8(k & 63);
}

}  // namespace mlxcat
