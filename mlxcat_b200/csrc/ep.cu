// ep.cu -- expert-parallel exchange of the sparse MoE MLP over NVLink peer
// memory (the Qwen3-30B-A3B configuration at 2/4/8 GPUs: experts split
// E/N per GPU, rows data-parallel).
//
// Every rank's cache exports one device region (CUDA IPC) that the other ranks
// map.  Per MoE layer (two buffer sets, alternating by layer):
//   dispatch   each routed assignment's operand row (fp16, the blocked layout
//              the expert kernels read, [H/64][N*cap][64]) and {local expert,
//              norm scale, routing weight, source assignment} are stored by the
//              SOURCE straight into the owner's receive slab at row
//              source*cap + slot: only routed rows cross NVLink.  The last CTA
//              then stores the per-owner row counts and, after a system fence,
//              a release flag (forward epoch x layer) into every owner.
//   wait       the owner polls its flags (acquire, bounded) -- one per source.
//   experts    the owner runs its experts over the received rows (moe.cu).
//   return     the owner stores each result row (fp32, already scaled by the
//              routing weight: exactly what the one-GPU combine reads) straight
//              into the source's return buffer at the source's assignment
//              index, then flags every source.
//   wait       the source waits for every owner's flag; the unchanged combine
//              reads the return buffer in assignment order.
// Buffer capacity per (source, owner) is the cache's token capacity x top_k
// (checked equal on every rank when the caches connect), so no count has to
// be known on the host and the whole exchange stays inside the captured step
// graph.  Ordering: a source reaches layer l+2 (the same buffer set as l) only
// after every owner returned layer l+1, which each owner does only after its
// layer-l reads are done, so a set is never overwritten while it is read.
// Every wait is bounded (EP_WAIT_NS, longer than the pipeline waits inside a
// kernel because a peer may still be instantiating or launching its step
// graph); a timeout sets the cache's device error flag (code 21: dispatch,
// 22: return), and later waits then return at once.
#include <algorithm>

#include "common.cuh"
#include "kernels.h"
#include "tc.cuh"

namespace mlxcat {

namespace {

using tc::ld_acquire_sys;
using tc::st_release_sys;

constexpr uint64_t EP_WAIT_NS = 10000000000ull;   // 10 s

__device__ __forceinline__ unsigned ep_flag(const EpArgs &a) { return *a.epoch * 256u + (unsigned)a.layer + 1u; }

template <typename T>
__device__ __forceinline__ T *at(char *base, size_t off) {
    return reinterpret_cast<T *>(base + off);
}

// one warp per assignment of this rank's tokens
__global__ void ep_dispatch_kernel(EpArgs a, const int32_t *__restrict__ topk_id, const float *__restrict__ topk_w,
                                   const float *__restrict__ tok_scale, const __half *__restrict__ x, int ldx_rows,
                                   int n) {
    const int asg = blockIdx.x * 8 + (threadIdx.x >> 5), lane = threadIdx.x & 31;
    const EpLayout &L = a.layout;
    if (asg < n) {
        const int m = asg / a.TK, e = topk_id[asg], d = e / a.epr;
        int slot = 0;
        if (lane == 0) slot = atomicAdd(a.lcount + d, 1);
        slot = __shfl_sync(0xffffffffu, slot, 0);
        char *peer = a.peers[d];
        const size_t row = ((size_t)a.set * a.N + a.me) * a.cap + slot;   // metadata row
        if (lane == 0) {
            EpMeta mt;
            mt.expert = e - d * a.epr;
            mt.scale = tok_scale[m];
            mt.weight = topk_w[asg];
            mt.pad = asg;   // the source's assignment index, where the result goes back
            at<EpMeta>(peer, L.recv_meta)[row] = mt;
        }
        // the token's operand row, 16 bytes at a time, from this rank's blocked
        // layout (ldx_rows rows) into the owner's (N * cap rows)
        const size_t rows = (size_t)a.N * a.cap, r = (size_t)a.me * a.cap + slot;
        __half *dst = at<__half>(peer, L.recv_x) + (size_t)a.set * rows * a.H;
        for (int b = lane; b < a.H / 8; b += 32)
            *reinterpret_cast<uint4 *>(dst + ((size_t)(b >> 3) * rows + r) * 64 + (b & 7) * 8) =
                *reinterpret_cast<const uint4 *>(x + ((size_t)(b >> 3) * ldx_rows + m) * 64 + (b & 7) * 8);
    }
    __threadfence_system();   // this CTA's peer stores, before the arrival below
    __syncthreads();
    if (threadIdx.x == 0 && atomicAdd(a.done, 1u) == gridDim.x - 1) {
        // last CTA: every row is stored; counts, then the flags, into every owner
        __threadfence_system();
        const unsigned flag = ep_flag(a);
        for (int d = 0; d < a.N; ++d)
            at<int>(a.peers[d], L.recv_count)[a.set * a.N + a.me] = atomicAdd(a.lcount + d, 0);
        __threadfence_system();
        for (int d = 0; d < a.N; ++d) {
            st_release_sys(at<unsigned>(a.peers[d], L.recv_flag) + a.set * a.N + a.me, flag);
            a.lcount[d] = 0;
        }
        *a.done = 0;
    }
}

// poll the flags[set][0..N) of this rank's region until each holds the
// current flag value (bounded)
__global__ void ep_wait_kernel(EpArgs a, size_t flag_off, int code) {
    const int t = threadIdx.x;
    if (t < a.N) tc::peer_flag_wait(at<unsigned>(a.peers[a.me], flag_off) + a.set * a.N + t, ep_flag(a), a.err, code,
                                    EP_WAIT_NS);
    __syncthreads();
    __threadfence_system();
}

// per-local-expert lists over the received rows (row = src * cap + slot)
__global__ void ep_lists_kernel(EpArgs a, int *__restrict__ exp_count, int32_t *__restrict__ exp_list,
                                float *__restrict__ row_scale, float *__restrict__ row_weight) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= a.N * a.cap) return;
    char *mine = a.peers[a.me];
    const int src = i / a.cap, slot = i - src * a.cap;
    if (slot >= at<int>(mine, a.layout.recv_count)[a.set * a.N + src]) return;
    const EpMeta mt = at<EpMeta>(mine, a.layout.recv_meta)[(size_t)a.set * a.N * a.cap + i];
    const int s = atomicAdd(exp_count + mt.expert, 1);
    exp_list[(size_t)mt.expert * a.N * a.cap + s] = i;
    row_scale[i] = mt.scale;
    row_weight[i] = mt.weight;
}

// owner: each received row's scaled expert output (fp32) back to its source
__global__ void ep_return_kernel(EpArgs a, const float *__restrict__ ys) {
    const int i = blockIdx.x * 8 + (threadIdx.x >> 5), lane = threadIdx.x & 31;
    const EpLayout &L = a.layout;
    char *mine = a.peers[a.me];
    if (i < a.N * a.cap) {
        const int src = i / a.cap, slot = i - src * a.cap;
        if (slot < at<int>(mine, L.recv_count)[a.set * a.N + src]) {
            const int asg = at<EpMeta>(mine, L.recv_meta)[(size_t)a.set * a.N * a.cap + i].pad;
            float4 *dst = reinterpret_cast<float4 *>(at<float>(a.peers[src], L.ret_y) + ((size_t)a.set * a.cap + asg) * a.H);
            const float4 *y = reinterpret_cast<const float4 *>(ys + (size_t)i * a.H);
            for (int b = lane; b < a.H / 4; b += 32) dst[b] = y[b];
        }
    }
    __threadfence_system();
    __syncthreads();
    if (threadIdx.x == 0 && atomicAdd(a.done, 1u) == gridDim.x - 1) {
        __threadfence_system();
        const unsigned flag = ep_flag(a);
        for (int s = 0; s < a.N; ++s) st_release_sys(at<unsigned>(a.peers[s], L.ret_flag) + a.set * a.N + a.me, flag);
        *a.done = 0;
    }
}

__global__ void ep_begin_kernel(unsigned *epoch) { *epoch += 1u; }

}  // namespace

EpLayout ep_layout(int N, int cap, int H) {
    EpLayout L;
    size_t off = 0;
    auto take = [&](size_t bytes) {
        const size_t o = off;
        off += (bytes + 255) & ~(size_t)255;
        return o;
    };
    L.recv_x = take((size_t)2 * N * cap * H * 2);      // [set][H/64][N*cap][64] fp16
    L.recv_meta = take((size_t)2 * N * cap * sizeof(EpMeta));
    L.recv_count = take((size_t)2 * N * sizeof(int));
    L.recv_flag = take((size_t)2 * N * sizeof(unsigned));
    L.ret_y = take((size_t)2 * cap * H * 4);           // [set][cap][H] fp32
    L.ret_flag = take((size_t)2 * N * sizeof(unsigned));
    L.total = off;
    return L;
}

cudaError_t ep_begin(unsigned *epoch, cudaStream_t st) {
    ep_begin_kernel<<<1, 1, 0, st>>>(epoch);
    return cudaGetLastError();
}

cudaError_t ep_dispatch(const EpArgs &a, const int32_t *topk_id, const float *topk_w, const float *tok_scale,
                        const __half *x_blk, int ldx_rows, int n, cudaStream_t st) {
    if (n <= 0 || n > a.cap || a.H % 64) return cudaErrorInvalidValue;
    ep_dispatch_kernel<<<(n + 7) / 8, 256, 0, st>>>(a, topk_id, topk_w, tok_scale, x_blk, ldx_rows, n);
    return cudaGetLastError();
}

cudaError_t ep_wait_dispatch(const EpArgs &a, cudaStream_t st) {
    ep_wait_kernel<<<1, 32, 0, st>>>(a, a.layout.recv_flag, 21);
    return cudaGetLastError();
}

cudaError_t ep_lists(const EpArgs &a, int *exp_count, int32_t *exp_list, float *row_scale, float *row_weight,
                     cudaStream_t st) {
    const int rows = a.N * a.cap;
    ep_lists_kernel<<<(rows + 255) / 256, 256, 0, st>>>(a, exp_count, exp_list, row_scale, row_weight);
    return cudaGetLastError();
}

cudaError_t ep_return(const EpArgs &a, const float *ys, cudaStream_t st) {
    if (a.H % 4) return cudaErrorInvalidValue;
    const int rows = a.N * a.cap;
    ep_return_kernel<<<(rows + 7) / 8, 256, 0, st>>>(a, ys);
    return cudaGetLastError();
}

cudaError_t ep_wait_return(const EpArgs &a, cudaStream_t st) {
    ep_wait_kernel<<<1, 32, 0, st>>>(a, a.layout.ret_flag, 22);
    return cudaGetLastError();
}

const float *ep_returned(const EpArgs &a, const char *own_region) {
    return reinterpret_cast<const float *>(own_region + a.layout.ret_y) + (size_t)a.set * a.cap * a.H;
}

const __half *ep_received(const EpArgs &a, const char *own_region) {
    return reinterpret_cast<const __half *>(own_region + a.layout.recv_x) + (size_t)a.set * a.N * a.cap * a.H;
}

}  // namespace mlxcat
