// attention.cu -- GQA decode attention for the verify forward.
//
// Replaces MLXFast.scaledDotProductAttention with the additive causal mask of
// BatchCache.swift:379-400 / CausalMask.swift:4-28 on the (k+1)-token verify
// step.  The cache is right-ragged: row r holds positions [0, len_r) and the
// mask comes from the per-token position alone (query at position p sees keys
// 0..p), so no left padding and no zeroed slots are ever read.
//
// Work item = (token group, kv head, key split, key half).  A token group is
// the qg consecutive verify tokens of one row; all G = Hq/Hkv query heads of
// the kv head and all qg tokens form the MMA M dimension (qg*G <= 16*QT), so
// every K/V tile fetched from HBM is used by every query of the group.
// K/V tiles of 32 keys go through a 3-deep cp.async ring in shared memory
// (small tiles keep several CTAs per SM, so enough loads are in flight); each
// of the two warps per query tile takes 16 keys of a tile (its own online
// softmax).  Partials (m, l, O) go to scratch; attention_combine merges them.
#include <algorithm>

#include "common.cuh"
#include "kernels.h"

namespace mlxcat {

namespace {

constexpr int KB = 32;       // keys per staged block
constexpr int KSTAGES = 3;   // cp.async ring depth (blocks in flight)

__device__ __forceinline__ void mma16816(float *c, const uint32_t *a, uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
        "{%8,%9}, {%0,%1,%2,%3};\n"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
__device__ __forceinline__ void ldsm_x4(uint32_t *d, uint32_t a) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];\n"
                 : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3]) : "r"(a));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t *d, uint32_t a) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];\n"
                 : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3]) : "r"(a));
}
__device__ __forceinline__ void cp16(uint32_t s, const void *g, int bytes) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(s), "l"(g), "r"(bytes));
}
__device__ __forceinline__ void cp_commit() { asm volatile("cp.async.commit_group;\n" ::); }
template <int N>
__device__ __forceinline__ void cp_wait() { asm volatile("cp.async.wait_group %0;\n" ::"n"(N)); }

__device__ __forceinline__ uint32_t pack_h2(float a, float b) {
    __half2 h = __floats2half2_rn(a, b);
    return *reinterpret_cast<uint32_t *>(&h);
}

template <int QT, int D>
__global__ void __launch_bounds__(QT * 64, 8 / QT)
attn_kernel(const __half *__restrict__ qbuf, const __half *__restrict__ kc,
            const __half *__restrict__ vc, int max_len, const int32_t *__restrict__ trow,
            const int32_t *__restrict__ tpos, int M, int qg, int Hq, int Hkv, int key_chunk,
            int splits, float scale_log2, float *__restrict__ o_part, float *__restrict__ ml_part,
            int early_kv, __half *__restrict__ direct_out) {
    constexpr int QROWS = QT * 16;
    constexpr int PITCH = D + 8;               // halves
    constexpr int NTHREADS = QT * 64;
    extern __shared__ __align__(16) unsigned char smem[];
    // The query tile is read into registers once, before the last V stage is
    // first filled, so when it fits that stage it lives there (52 KB instead of
    // 61 KB per CTA at 32 query rows: four CTAs per SM instead of three).
    constexpr bool QALIAS = QROWS <= KB;
    __half *ks = reinterpret_cast<__half *>(smem) + (QALIAS ? 0 : QROWS * PITCH);   // [KSTAGES][KB][PITCH]
    __half *vs = ks + KSTAGES * KB * PITCH;                                       // [KSTAGES][KB][PITCH]
    __half *qs = QALIAS ? vs + (KSTAGES - 1) * KB * PITCH : reinterpret_cast<__half *>(smem);   // [QROWS][PITCH]
    constexpr int KPW = KB / 2;                                     // keys per warp per block
    constexpr int NU = KPW / 16, NN = KPW / 8;

    griddep_launch_dependents();   // the combine pass may be scheduled
    // Inside the verify forward (early_kv) token rows and positions are inputs of
    // the forward and keys below the row's first position in this launch were
    // written by earlier forwards, so they are read before waiting for the
    // previous kernel (the QKV projection), which writes only the queries and the
    // new keys.  Otherwise everything waits for the previous kernel.
    if (!early_kv) griddep_wait();
    // direct_out (one key split, prefill): the groups furthest into the prompt
    // see the most keys, so they are scheduled first
    const int grp = direct_out ? gridDim.x - 1 - blockIdx.x : blockIdx.x, h = blockIdx.y, s = blockIdx.z;
    const int G = Hq / Hkv;
    const int t0 = grp * qg;
    const int ntok = min(qg, M - t0);
    const int NQ = ntok * G;
    const int row = trow[t0], pos0 = tpos[t0];
    const int kend = pos0 + ntok;
    const int kb = s * key_chunk, ke = min(kend, kb + key_chunk);
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int mt = warp >> 1, kh = warp & 1;
    const int g = lane >> 2, t = lane & 3;

    const size_t item = ((size_t)grp * Hkv + h) * splits + s;
    float *op = o_part + item * QROWS * D;
    float *mlp = ml_part + item * QROWS * 2;

    if (kb >= ke) {
        griddep_wait();   // the previous launch's combine may still read this scratch
        for (int i = threadIdx.x; i < QROWS * 2; i += NTHREADS) mlp[i] = (i & 1) ? 0.f : -INFINITY;
        return;
    }
    // first position of this row written by this launch (prefill puts several
    // groups of one row in a launch)
    int new_lo = pos0;
    for (int gg = 0; gg * qg < M; ++gg)
        if (trow[gg * qg] == row) new_lo = min(new_lo, tpos[gg * qg]);

    const __half *kbase = kc + ((size_t)row * Hkv + h) * max_len * D;
    const __half *vbase = vc + ((size_t)row * Hkv + h) * max_len * D;
    const uint32_t qs_a = (uint32_t)__cvta_generic_to_shared(qs);
    const uint32_t ks_a = (uint32_t)__cvta_generic_to_shared(ks);
    const uint32_t vs_a = (uint32_t)__cvta_generic_to_shared(vs);

    // stage Q: row qi = j*G + gh -> token t0+j, head h*G+gh
    auto stage_q = [&]() {
        for (int v = threadIdx.x; v < QROWS * (D / 8); v += NTHREADS) {
            const int qi = v / (D / 8), c8 = v - qi * (D / 8);
            const int j = qi / G, gh = qi - j * G;
            const bool ok = qi < NQ;
            const __half *src = qbuf + ((size_t)(ok ? t0 + j : t0) * Hq + h * G + (ok ? gh : 0)) * D + c8 * 8;
            cp16(qs_a + (uint32_t)(qi * PITCH + c8 * 8) * 2, src, ok ? 16 : 0);
        }
    };
    auto stage_kv = [&](int blk, int buf) {
        const int key0 = kb + blk * KB;
        for (int v = threadIdx.x; v < KB * (D / 8); v += NTHREADS) {
            const int kr = v / (D / 8), c8 = v - kr * (D / 8);
            const int key = key0 + kr;
            const bool ok = key < ke;
            const size_t off = (size_t)(ok ? key : kb) * D + c8 * 8;
            const uint32_t so = (uint32_t)((buf * KB + kr) * PITCH + c8 * 8) * 2;
            cp16(ks_a + so, kbase + off, ok ? 16 : 0);
            cp16(vs_a + so, vbase + off, ok ? 16 : 0);
        }
    };
    const int nblk = (ke - kb + KB - 1) / KB;
    // prologue: the first blocks, those holding only older keys before the wait
    // (they join the first cp.async group, with Q and block 0)
    bool pre[KSTAGES - 1];
#pragma unroll
    for (int p = 0; p < KSTAGES - 1; ++p) {
        pre[p] = early_kv && p < nblk && kb + (p + 1) * KB <= new_lo;
        if (pre[p]) stage_kv(p, p);
    }
    griddep_wait();                // queries and the new K/V come from the previous kernel
    stage_q();
#pragma unroll
    for (int p = 0; p < KSTAGES - 1; ++p) {
        if (p < nblk && !pre[p]) stage_kv(p, p);
        cp_commit();
    }

    uint32_t qf[D / 16][4];
    auto load_q = [&]() {
#pragma unroll
        for (int ks16 = 0; ks16 < D / 16; ++ks16) {
            const int mi = lane >> 3, rr = lane & 7;
            const int qr = mt * 16 + (mi & 1) * 8 + rr;
            ldsm_x4(qf[ks16], qs_a + (uint32_t)(qr * PITCH + ks16 * 16 + (mi >> 1) * 8) * 2);
        }
    };
    if (QALIAS) {   // Q (first cp.async group) into registers before its stage is reused
        cp_wait<KSTAGES - 2>();
        __syncthreads();
        load_q();
        __syncthreads();
    }
    float o[D / 8][4];
#pragma unroll
    for (int i = 0; i < D / 8; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
    float m_r[2] = {-INFINITY, -INFINITY}, l_r[2] = {0.f, 0.f};
    // query row -> allowed key limit (inclusive): pos0 + token index
    const int qrow0 = mt * 16 + g, qrow1 = qrow0 + 8;
    const int lim0 = qrow0 < NQ ? pos0 + qrow0 / G : -1;
    const int lim1 = qrow1 < NQ ? pos0 + qrow1 / G : -1;

    for (int b = 0; b < nblk; ++b) {
        if (b + KSTAGES - 1 < nblk) stage_kv(b + KSTAGES - 1, (b + KSTAGES - 1) % KSTAGES);
        cp_commit();
        cp_wait<KSTAGES - 1>();
        __syncthreads();
        if (!QALIAS && b == 0) load_q();
        const int buf = b % KSTAGES;
        const int key_base = kb + b * KB + kh * KPW;
        // S = Q K^T over this warp's KPW keys (NN n8 tiles)
        float sc[NN][4];
#pragma unroll
        for (int n = 0; n < NN; ++n) sc[n][0] = sc[n][1] = sc[n][2] = sc[n][3] = 0.f;
#pragma unroll
        for (int ks16 = 0; ks16 < D / 16; ++ks16) {
#pragma unroll
            for (int u = 0; u < NU; ++u) {
                const int mi = lane >> 3, rr = lane & 7;
                const int kr = kh * KPW + u * 16 + (mi >> 1) * 8 + rr;
                uint32_t bb[4];
                ldsm_x4(bb, ks_a + (uint32_t)((buf * KB + kr) * PITCH + ks16 * 16 + (mi & 1) * 8) * 2);
                mma16816(sc[2 * u], qf[ks16], bb[0], bb[1]);
                mma16816(sc[2 * u + 1], qf[ks16], bb[2], bb[3]);
            }
        }
        // Mask only where a key can lie past a query's position: the causal
        // corner and the zero-filled keys past kend (both beyond pos0).  Rows
        // past NQ (zero queries) are never written.
        if (key_base + KPW - 1 > pos0) {
#pragma unroll
            for (int n = 0; n < NN; ++n)
#pragma unroll
                for (int c = 0; c < 4; ++c) {
                    const int key = key_base + n * 8 + 2 * t + (c & 1);
                    const int lim = c < 2 ? lim0 : lim1;
                    if (!(key <= lim && key < ke)) sc[n][c] = -INFINITY;
                }
        }
        float mx[2] = {-INFINITY, -INFINITY};
#pragma unroll
        for (int n = 0; n < NN; ++n)
#pragma unroll
            for (int c = 0; c < 4; ++c) mx[c >> 1] = fmaxf(mx[c >> 1], sc[n][c]);
        // Online softmax in log2 units, z = s * scale_log2.  The running
        // reference m_r is raised only when a row's block max exceeds it by more
        // than 8 (then every row of the warp is rescaled), so exp2(z - m_r) <= 256
        // fits the fp16 P operand and most blocks skip the O rescale.
        bool raise = false;
#pragma unroll
        for (int rI = 0; rI < 2; ++rI) {
            mx[rI] = fmaxf(mx[rI], __shfl_xor_sync(0xffffffffu, mx[rI], 1));
            mx[rI] = fmaxf(mx[rI], __shfl_xor_sync(0xffffffffu, mx[rI], 2));
            mx[rI] *= scale_log2;
            raise |= mx[rI] > m_r[rI] + 8.f;
        }
        if (__any_sync(0xffffffffu, raise)) {
#pragma unroll
            for (int rI = 0; rI < 2; ++rI) {
                const float mn = fmaxf(m_r[rI], mx[rI]);
                const float alpha = (mn == -INFINITY || m_r[rI] == -INFINITY) ? 0.f : exp2f(m_r[rI] - mn);
                m_r[rI] = mn;
                l_r[rI] *= alpha;
#pragma unroll
                for (int i = 0; i < D / 8; ++i) { o[i][2 * rI] *= alpha; o[i][2 * rI + 1] *= alpha; }
            }
        }
        const float nm0 = m_r[0] == -INFINITY ? 0.f : -m_r[0];
        const float nm1 = m_r[1] == -INFINITY ? 0.f : -m_r[1];
        uint32_t pa[NU][4];
#pragma unroll
        for (int n = 0; n < NN; ++n) {
            float p[4];
#pragma unroll
            for (int c = 0; c < 4; ++c) {
                p[c] = exp2f(fmaf(sc[n][c], scale_log2, c < 2 ? nm0 : nm1));
                l_r[c >> 1] += p[c];
            }
            const int u = n >> 1;
            if ((n & 1) == 0) { pa[u][0] = pack_h2(p[0], p[1]); pa[u][1] = pack_h2(p[2], p[3]); }
            else { pa[u][2] = pack_h2(p[0], p[1]); pa[u][3] = pack_h2(p[2], p[3]); }
        }
        // O += P V
#pragma unroll
        for (int u = 0; u < NU; ++u) {
#pragma unroll
            for (int dv = 0; dv < D / 16; ++dv) {
                const int mi = lane >> 3, rr = lane & 7;
                const int kr = kh * KPW + u * 16 + (mi & 1) * 8 + rr;
                uint32_t bb[4];
                ldsm_x4_t(bb, vs_a + (uint32_t)((buf * KB + kr) * PITCH + dv * 16 + (mi >> 1) * 8) * 2);
                mma16816(o[2 * dv], pa[u], bb[0], bb[1]);
                mma16816(o[2 * dv + 1], pa[u], bb[2], bb[3]);
            }
        }
        __syncthreads();
    }
    cp_wait<0>();
    __syncthreads();   // K/V tiles no longer read: reuse shared memory for the merge

#pragma unroll
    for (int rI = 0; rI < 2; ++rI) {
        l_r[rI] += __shfl_xor_sync(0xffffffffu, l_r[rI], 1);
        l_r[rI] += __shfl_xor_sync(0xffffffffu, l_r[rI], 2);
    }
    // merge the two key halves of this split inside the CTA
    float *o_s = reinterpret_cast<float *>(smem);          // [QROWS][D]
    float *ml_s = o_s + QROWS * D;                          // [QROWS][2]
    if (kh == 1) {
#pragma unroll
        for (int i = 0; i < D / 8; ++i) {
            const int d = i * 8 + 2 * t;
            *reinterpret_cast<float2 *>(o_s + qrow0 * D + d) = make_float2(o[i][0], o[i][1]);
            *reinterpret_cast<float2 *>(o_s + qrow1 * D + d) = make_float2(o[i][2], o[i][3]);
        }
        if (t == 0) {
            ml_s[qrow0 * 2] = m_r[0]; ml_s[qrow0 * 2 + 1] = l_r[0];
            ml_s[qrow1 * 2] = m_r[1]; ml_s[qrow1 * 2 + 1] = l_r[1];
        }
    }
    __syncthreads();
    if (kh == 0 && direct_out) {
        // one split: this CTA holds every key of the group, so it writes the
        // normalised output itself (natural layout [M][Hq*D]); no combine pass
        const int rws[2] = {qrow0, qrow1};
        const int KO = Hq * D;
#pragma unroll
        for (int rI = 0; rI < 2; ++rI) {
            const int qi = rws[rI];
            if (qi >= NQ) continue;
            const float m1 = ml_s[qi * 2], l1 = ml_s[qi * 2 + 1];
            const float mm = fmaxf(m_r[rI], m1);
            const float a0 = m_r[rI] == -INFINITY ? 0.f : exp2f(m_r[rI] - mm);
            const float a1 = m1 == -INFINITY ? 0.f : exp2f(m1 - mm);
            const float den = a0 * l_r[rI] + a1 * l1;
            const float inv = den > 0.f ? 1.0f / den : 0.f;
            const int j = qi / G, gh = qi - j * G;
            __half *dst = direct_out + (size_t)(t0 + j) * KO + (size_t)(h * G + gh) * D;
#pragma unroll
            for (int i = 0; i < D / 8; ++i) {
                const int d = i * 8 + 2 * t;
                const float2 x = *reinterpret_cast<const float2 *>(o_s + qi * D + d);
                const float v0 = (a0 * o[i][2 * rI] + a1 * x.x) * inv, v1 = (a0 * o[i][2 * rI + 1] + a1 * x.y) * inv;
                *reinterpret_cast<__half2 *>(dst + d) = __floats2half2_rn(v0, v1);
            }
        }
    } else if (kh == 0) {
        float a0[2], a1[2];
        const int rws[2] = {qrow0, qrow1};
#pragma unroll
        for (int rI = 0; rI < 2; ++rI) {
            const float m1 = ml_s[rws[rI] * 2], l1 = ml_s[rws[rI] * 2 + 1];
            const float mm = fmaxf(m_r[rI], m1);
            a0[rI] = m_r[rI] == -INFINITY ? 0.f : exp2f(m_r[rI] - mm);
            a1[rI] = m1 == -INFINITY ? 0.f : exp2f(m1 - mm);
            if (t == 0) {
                mlp[rws[rI] * 2] = mm;
                mlp[rws[rI] * 2 + 1] = a0[rI] * l_r[rI] + a1[rI] * l1;
            }
        }
#pragma unroll
        for (int i = 0; i < D / 8; ++i) {
            const int d = i * 8 + 2 * t;
            const float2 x0 = *reinterpret_cast<const float2 *>(o_s + qrow0 * D + d);
            const float2 x1 = *reinterpret_cast<const float2 *>(o_s + qrow1 * D + d);
            *reinterpret_cast<float2 *>(op + (size_t)qrow0 * D + d) =
                make_float2(a0[0] * o[i][0] + a1[0] * x0.x, a0[0] * o[i][1] + a1[0] * x0.y);
            *reinterpret_cast<float2 *>(op + (size_t)qrow1 * D + d) =
                make_float2(a0[1] * o[i][2] + a1[1] * x1.x, a0[1] * o[i][3] + a1[1] * x1.y);
        }
    }
}

// merge the split partials of one (group, kv head): thread = 8 consecutive
// features of one query row (16-byte loads of each split, one 16-byte store);
// per feature the same two-level merge as a plain loop over the splits
template <int QT>
__global__ void attn_combine_kernel(const float *__restrict__ o_part, const float *__restrict__ ml_part,
                                    int M, int qg, int Hq, int Hkv, int D, int splits,
                                    __half *__restrict__ out, int permuted, int out_rows) {
    constexpr int QROWS = QT * 16;
    griddep_launch_dependents();   // the output projection may start prefetching its weights
    griddep_wait();                // the split partials come from the split pass
    const int grp = blockIdx.x, h = blockIdx.y;
    const int G = Hq / Hkv;
    const int t0 = grp * qg;
    const int ntok = min(qg, M - t0);
    const int NQ = ntok * G;
    const int P = splits, DC = D / 8;
    const size_t it0 = ((size_t)grp * Hkv + h) * P;
    const int KO = Hq * D;
    for (int w = threadIdx.x; w < NQ * DC; w += blockDim.x) {
        const int qi = w / DC, d0 = (w - qi * DC) * 8;
        // splits in batches of PB whose loads are all issued before any is used
        // (one L2 round trip per batch); a running max rescales across batches,
        // and with P <= PB the sums are exactly the two-pass ones
        constexpr int PB = 8;
        float num[8], den = 0.f, mrun = -INFINITY;
#pragma unroll
        for (int i = 0; i < 8; ++i) num[i] = 0.f;
        for (int p0 = 0; p0 < P; p0 += PB) {
            float m[PB], l[PB];
            float4 va[PB], vb[PB];
#pragma unroll
            for (int k = 0; k < PB; ++k) {
                m[k] = -INFINITY; l[k] = 0.f;
                va[k] = vb[k] = make_float4(0.f, 0.f, 0.f, 0.f);
                if (p0 + k < P) {
                    const size_t item = it0 + p0 + k;
                    const float2 ml = *reinterpret_cast<const float2 *>(ml_part + (item * QROWS + qi) * 2);
                    m[k] = ml.x; l[k] = ml.y;
                    const float4 *src = reinterpret_cast<const float4 *>(o_part + (item * QROWS + qi) * D + d0);
                    va[k] = src[0];
                    vb[k] = src[1];
                }
            }
            float mb = mrun;
#pragma unroll
            for (int k = 0; k < PB; ++k) mb = fmaxf(mb, m[k]);
            if (mb == -INFINITY) continue;
            if (mrun != -INFINITY && mrun != mb) {
                const float a = exp2f(mrun - mb);
#pragma unroll
                for (int i = 0; i < 8; ++i) num[i] *= a;
                den *= a;
            }
#pragma unroll
            for (int k = 0; k < PB; ++k) {
                if (m[k] == -INFINITY) continue;
                const float wk = exp2f(m[k] - mb);
                den += wk * l[k];
                num[0] += wk * va[k].x; num[1] += wk * va[k].y; num[2] += wk * va[k].z; num[3] += wk * va[k].w;
                num[4] += wk * vb[k].x; num[5] += wk * vb[k].y; num[6] += wk * vb[k].z; num[7] += wk * vb[k].w;
            }
            mrun = mb;
        }
        // 8 features inside one 64-feature block; the blocked operand layout keeps
        // them in perm8 order, so feature i goes to slot perm8(i) of the 16 bytes
        __align__(16) __half r[8];
#pragma unroll
        for (int i = 0; i < 8; ++i)
            r[permuted ? perm8(i) : i] = __float2half_rn(den > 0.f ? num[i] / den : 0.f);
        const int j = qi / G, gh = qi - j * G;
        const int k0 = (h * G + gh) * D + d0;
        __half *dst = permuted ? out + xblk(t0 + j, k0, out_rows) : out + (size_t)(t0 + j) * KO + k0;
        *reinterpret_cast<uint4 *>(dst) = *reinterpret_cast<const uint4 *>(r);
    }
}

template <int QT, int D>
cudaError_t launch_attn(const __half *qbuf, KVLayer kv, const int32_t *trow, const int32_t *tpos,
                        int M, int qg, int Hq, int Hkv, int key_chunk, int splits,
                        AttnScratch sc, __half *out, bool permuted, int out_rows, bool early_kv, cudaStream_t st) {
    constexpr int PITCH = D + 8;
    const size_t smem = std::max((size_t)((QT * 16 <= KB ? 0 : QT * 16) + 2 * KSTAGES * KB) * PITCH * 2,
                                 (size_t)QT * 16 * (D + 2) * 4);   // K/V ring (+ Q), then the split merge
    static bool attr[64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (!attr[dev & 63]) {
        cudaError_t e = cudaFuncSetAttribute(attn_kernel<QT, D>,
                                             cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return e;
        attr[dev & 63] = true;
    }
    const int groups = (M + qg - 1) / qg;
    dim3 grid(groups, Hkv, splits);
    const float scale_log2 = 1.4426950408889634f / sqrtf((float)D);
    // one key split and a natural-layout output: the split pass normalises and
    // writes the output itself
    __half *direct = splits == 1 && !permuted ? out : nullptr;
    cudaError_t e = launch_pdl(attn_kernel<QT, D>, grid, dim3(QT * 64), smem, st, qbuf, kv.k, kv.v, kv.max_len,
                               trow, tpos, M, qg, Hq, Hkv, key_chunk, splits, scale_log2, sc.o, sc.ml,
                               early_kv ? 1 : 0, direct);
    if (e != cudaSuccess || direct) return e;
    dim3 g2(groups, Hkv);
    const int cthreads = std::min(512, QT * 16 * (D / 8));
    return launch_pdl(attn_combine_kernel<QT>, g2, dim3(cthreads), 0, st, (const float *)sc.o, (const float *)sc.ml,
                      M, qg, Hq, Hkv, D, splits, out, permuted ? 1 : 0, out_rows);
}

}  // namespace

int attention_qrows(int qg, int n_heads, int n_kv) {
    const int nq = qg * (n_heads / n_kv);
    return nq <= 16 ? 16 : (nq <= 32 ? 32 : 64);
}

int attention_max_splits(int max_len, int key_chunk) { return (max_len + key_chunk - 1) / key_chunk; }

size_t attention_scratch_items(int groups, int n_kv, int splits) {
    return (size_t)groups * n_kv * splits;
}

cudaError_t attention(const __half *qbuf, KVLayer kv, const int32_t *trow, const int32_t *tpos,
                      int M, int qg, int n_heads, int n_kv, int D, int key_chunk, int splits,
                      AttnScratch scratch, __half *out, bool permuted_out, int out_rows,
                      cudaStream_t st, bool early_kv) {
    if (key_chunk % KB || n_heads % n_kv) return cudaErrorInvalidValue;
    const int nq = qg * (n_heads / n_kv);
    const int groups = (M + qg - 1) / qg;
    if (attention_scratch_items(groups, n_kv, splits) > scratch.items) return cudaErrorInvalidValue;
    if (D == 128) {
        if (nq <= 16) return launch_attn<1, 128>(qbuf, kv, trow, tpos, M, qg, n_heads, n_kv, key_chunk, splits, scratch, out, permuted_out, out_rows, early_kv, st);
        if (nq <= 32) return launch_attn<2, 128>(qbuf, kv, trow, tpos, M, qg, n_heads, n_kv, key_chunk, splits, scratch, out, permuted_out, out_rows, early_kv, st);
        if (nq <= 64) return launch_attn<4, 128>(qbuf, kv, trow, tpos, M, qg, n_heads, n_kv, key_chunk, splits, scratch, out, permuted_out, out_rows, early_kv, st);
    } else if (D == 64) {
        if (nq <= 16) return launch_attn<1, 64>(qbuf, kv, trow, tpos, M, qg, n_heads, n_kv, key_chunk, splits, scratch, out, permuted_out, out_rows, early_kv, st);
        if (nq <= 32) return launch_attn<2, 64>(qbuf, kv, trow, tpos, M, qg, n_heads, n_kv, key_chunk, splits, scratch, out, permuted_out, out_rows, early_kv, st);
        if (nq <= 64) return launch_attn<4, 64>(qbuf, kv, trow, tpos, M, qg, n_heads, n_kv, key_chunk, splits, scratch, out, permuted_out, out_rows, early_kv, st);
    }
    return cudaErrorInvalidValue;
}

}  // namespace mlxcat
