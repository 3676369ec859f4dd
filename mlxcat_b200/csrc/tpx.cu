// tpx.cu -- the tensor-parallel allreduce of the verify forward over NVLink
// peer memory, fused with the row-split projections (the Llama-3-70B
// configuration at 2/4/8 GPUs).
//
// Every row-split projection (O, down) ends in an allreduce of its fp32
// partial sums y_p [M][H].  Here it is a two-shot exchange over the caches'
// mapped regions (the same CUDA IPC regions as expert parallelism):
//   scatter   the q4 kernel's STORE epilogue writes each finished 128-feature
//             block straight into the region of the rank that owns those
//             features (owner = feature / (H/N)), slot [source], so the
//             partial sums cross NVLink while the other blocks are still
//             being computed; the kernel's last CTA then release-flags every
//             owner (q4_tc.cu, Q4Epilogue::peers).
//   reduce    the owner waits for every source's flag, sums the N slots of its
//             H/N features in rank order (fp32: every rank gets the same bits),
//             and stores the sums into every rank's gather buffer; its last
//             CTA release-flags every rank.
//   wait      each rank waits for every owner's flag; the residual step reads
//             the gathered [M][H] sums.
// Two buffer sets alternate by call (call = 2 * layer + {0: O, 1: down}).  A
// rank writes a set for call c + 2 only after its own call c + 1 finished,
// which needs every owner's reduce of c + 1, which follows that owner's reads
// of call c: a set is never overwritten while it is read.  Each flag holds
// epoch * 512 + call + 1 (epoch = forwards run so far).  Every wait is bounded.
#include <algorithm>

#include "common.cuh"
#include "kernels.h"
#include "tc.cuh"

namespace mlxcat {

namespace {

constexpr uint64_t TPX_WAIT_NS = 10000000000ull;   // 10 s: a peer may still be launching its step graph

__device__ __forceinline__ unsigned tpx_flag(const TpxArgs &a) { return *a.epoch * 512u + (unsigned)a.call + 1u; }

template <typename T>
__device__ __forceinline__ T *at(char *base, size_t off) {
    return reinterpret_cast<T *>(base + off);
}

// owner side: wait for the N scatter flags, sum the slots of this rank's
// features, store the sums into every rank's gather buffer, flag every rank
__global__ void __launch_bounds__(256) tpx_reduce_kernel(TpxArgs a, int M) {
    const TpxLayout &L = a.layout;
    char *mine = a.peers[a.me];
    if (threadIdx.x < a.N)
        tc::peer_flag_wait(at<unsigned>(mine, L.scat_flag) + a.set * a.N + threadIdx.x, tpx_flag(a), a.err, 23,
                           TPX_WAIT_NS);
    __syncthreads();
    __threadfence_system();
    const int cols = a.H / a.N, c4 = cols / 4;
    const float4 *scat = reinterpret_cast<const float4 *>(at<float>(mine, L.scat) + (size_t)a.set * a.N * a.mcap * cols);
    const size_t slot = (size_t)a.mcap * c4;   // float4s per source slot
    const int n = M * c4;
    if (!*reinterpret_cast<volatile int *>(a.err)) {
        for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
            const int m = i / c4, c = i - m * c4;
            float4 s = scat[(size_t)m * c4 + c];
            for (int src = 1; src < a.N; ++src) {
                const float4 t = scat[src * slot + (size_t)m * c4 + c];
                s.x += t.x; s.y += t.y; s.z += t.z; s.w += t.w;
            }
            const size_t dst = ((size_t)a.set * a.mcap + m) * a.H + (size_t)a.me * cols + 4 * c;
            for (int d = 0; d < a.N; ++d) *reinterpret_cast<float4 *>(at<float>(a.peers[d], L.gath) + dst) = s;
        }
    }
    __threadfence_system();
    __syncthreads();
    if (threadIdx.x == 0 && atomicAdd(a.done, 1u) == gridDim.x - 1) {
        *a.done = 0;
        __threadfence_system();
        const unsigned flag = tpx_flag(a);
        for (int d = 0; d < a.N; ++d) tc::st_release_sys(at<unsigned>(a.peers[d], L.gath_flag) + a.set * a.N + a.me, flag);
    }
}

__global__ void tpx_wait_kernel(TpxArgs a) {
    if (threadIdx.x < a.N)
        tc::peer_flag_wait(at<unsigned>(a.peers[a.me], a.layout.gath_flag) + a.set * a.N + threadIdx.x, tpx_flag(a),
                           a.err, 24, TPX_WAIT_NS);
    __syncthreads();
    __threadfence_system();
}

}  // namespace

TpxLayout tpx_layout(int N, int mcap, int H) {
    TpxLayout L;
    size_t off = 0;
    auto take = [&](size_t bytes) {
        const size_t o = off;
        off += (bytes + 255) & ~(size_t)255;
        return o;
    };
    L.scat = take((size_t)2 * mcap * H * 4);          // [set][src][mcap][H/N] fp32
    L.scat_flag = take((size_t)2 * N * sizeof(unsigned));
    L.gath = take((size_t)2 * mcap * H * 4);          // [set][mcap][H] fp32
    L.gath_flag = take((size_t)2 * N * sizeof(unsigned));
    L.total = off;
    return L;
}

void tpx_scatter_epilogue(const TpxArgs &a, Q4Epilogue &e) {
    const int cols = a.H / a.N;
    e.peers = a.peers;
    e.peer_n = a.N;
    e.peer_cols = cols;
    e.peer_off = a.layout.scat + (((size_t)a.set * a.N + a.me) * a.mcap) * cols * 4;
    e.peer_flag_off = a.layout.scat_flag + ((size_t)a.set * a.N + a.me) * sizeof(unsigned);
    e.peer_flag = a.epoch;
    e.peer_call = a.call;
    e.peer_ctr = a.sig;
}

cudaError_t tpx_reduce(const TpxArgs &a, int M, int sm_count, cudaStream_t st) {
    if (M <= 0 || M > a.mcap || a.H % (4 * a.N)) return cudaErrorInvalidValue;
    const int n = M * (a.H / a.N / 4);
    const int blocks = std::max(1, std::min((n + 255) / 256, sm_count));
    tpx_reduce_kernel<<<blocks, 256, 0, st>>>(a, M);
    return cudaGetLastError();
}

cudaError_t tpx_wait(const TpxArgs &a, cudaStream_t st) {
    tpx_wait_kernel<<<1, 32, 0, st>>>(a);
    return cudaGetLastError();
}

const float *tpx_gathered(const TpxArgs &a, const char *own_region) {
    return reinterpret_cast<const float *>(own_region + a.layout.gath) + (size_t)a.set * a.mcap * a.H;
}

}  // namespace mlxcat
