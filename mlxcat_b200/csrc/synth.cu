// synth.cu -- seeded synthetic weights, quantised to MLX affine q4 on device.
//
// Each thread produces one 64-wide group: 64 normals N(0, std) from the Philox
// stream (element index n*K + k, tensor id), then the min/max affine
// quantizer: scale = fp16((max-min)/15), bias = fp16(min),
// q = clamp(rint((w - bias)/scale), 0, 15), nibbles packed lowest first.
// Bit-identical with the CPU restatement (orc_q4_synth).  Logical row n is
// written to row (n / rgroup) * rstride + n % rgroup + row_offset of the
// destination (fused matrices: contiguous q|k|v, gate/up interleaved per 64).
// A tensor-parallel slice (rows row_base.., columns col_base.. of a tensor with
// k_total columns) draws the same stream elements as the full tensor, so each
// rank's slice is bit-identical with that part of the full tensor.
#include "common.cuh"
#include "kernels.h"

namespace mlxcat {

__global__ void synth_q4_kernel(uint64_t seed, uint32_t tensor_id, float stddev, int N, int K,
                                uint32_t *__restrict__ wq, __half *__restrict__ scales,
                                __half *__restrict__ biases, int row_offset, int rgroup,
                                int rstride, int row_base, int col_base, int k_total) {
    const int G = K / MLXCAT_GS;
    const long long gid = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (gid >= (long long)N * G) return;
    const int n = (int)(gid / G), grp = (int)(gid - (long long)n * G);
    float w[MLXCAT_GS];
    float mn = 0.f, mx = 0.f;
    for (int i = 0; i < MLXCAT_GS; ++i) {
        const uint64_t idx = (uint64_t)(row_base + n) * (uint64_t)k_total +
                             (uint64_t)(col_base + grp * MLXCAT_GS + i);
        w[i] = __fmul_rn(det_normal(seed, tensor_id, idx), stddev);
        if (i == 0 || w[i] < mn) mn = w[i];
        if (i == 0 || w[i] > mx) mx = w[i];
    }
    const float sc = __fdiv_rn(__fadd_rn(mx, -mn), 15.0f);
    const __half sh = __float2half_rn(sc);
    const float sf = __half2float(sh);
    const __half bh = __float2half_rn(mn);
    const float bf = __half2float(bh);
    const int orow = (n / rgroup) * rstride + (n % rgroup) + row_offset;
    uint32_t *dst = wq + (size_t)orow * (K / 8) + grp * (MLXCAT_GS / 8);
    for (int j = 0; j < MLXCAT_GS / 8; ++j) {
        uint32_t word = 0;
        for (int b = 0; b < 8; ++b) {
            int q = 0;
            if (sf > 0.0f) {
                q = __float2int_rn(__fdiv_rn(__fadd_rn(w[j * 8 + b], -bf), sf));
                q = q < 0 ? 0 : (q > 15 ? 15 : q);
            }
            word |= (uint32_t)q << (4 * b);
        }
        dst[j] = word;
    }
    scales[(size_t)orow * G + grp] = sh;
    biases[(size_t)orow * G + grp] = bh;
}

cudaError_t synth_q4(uint64_t seed, uint32_t tensor_id, float stddev, int N, int K,
                     uint32_t *wq, __half *scales, __half *biases, int row_offset,
                     cudaStream_t st, int rgroup, int rstride, int row_base, int col_base, int k_total) {
    if (rgroup <= 0) { rgroup = N; rstride = 0; }
    if (k_total <= 0) k_total = K;
    if (col_base % MLXCAT_GS || col_base + K > k_total) return cudaErrorInvalidValue;
    const long long groups = (long long)N * (K / MLXCAT_GS);
    const int threads = 128;
    const long long blocks = (groups + threads - 1) / threads;
    synth_q4_kernel<<<(unsigned)blocks, threads, 0, st>>>(seed, tensor_id, stddev, N, K, wq,
                                                          scales, biases, row_offset, rgroup, rstride,
                                                          row_base, col_base, k_total);
    return cudaGetLastError();
}

}  // namespace mlxcat
