// kernels.h -- internal launch interface of the mlxcat_b200 CUDA kernels.
// Everything here is device-pointer based and stream ordered; the C ABI in
// include/mlxcat_cuda.h sits on top.
#pragma once

#include <utility>

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace mlxcat {

// Launch with programmatic stream serialisation: the kernel may start while
// its predecessor on the stream is still running; it must call griddep_wait()
// (common.cuh) before reading anything the predecessor writes.
template <typename... KArgs, typename... Args>
inline cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                              Args &&...args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = at;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}


// One MLX affine-q4 matrix [N][K]: packed words, fp16 scales and biases.
struct Q4Weight {
    const uint32_t *wq = nullptr;
    const __half *scales = nullptr;
    const __half *biases = nullptr;
    int N = 0, K = 0;
};

// ---- weight synthesis (seeded N(0, std) then affine q4, bit-exact with the
//      CPU restatement) ------------------------------------------------------
// row_base / col_base / k_total: the slice [row_base.., col_base..] of a tensor
// with k_total columns (tensor-parallel shards); defaults give the whole tensor
cudaError_t synth_q4(uint64_t seed, uint32_t tensor_id, float stddev, int N, int K,
                     uint32_t *wq, __half *scales, __half *biases, int row_offset,
                     cudaStream_t st, int rgroup = 0, int rstride = 0, int row_base = 0,
                     int col_base = 0, int k_total = 0);

// ---- q4 linear on tcgen05 (TMA + TMEM) with fused split-K and epilogue ------
}  // namespace mlxcat
#include <cuda.h>
namespace mlxcat {
struct Q4WeightTC {
    const uint32_t *wq = nullptr;
    const __half *scales = nullptr;
    const __half *biases = nullptr;
    const uint32_t *sbp = nullptr;   // (scale, bias) pairs re-packed by pack_q4_sb
    int N = 0, K = 0;
    CUtensorMap map;          // 2-D TMA map over the packed words (bytes x rows)
};
struct Q4Epilogue {
    enum Op { STORE = 0, RESID = 1, SWIGLU = 2, QKV = 3 };
    int op = STORE;
    int pdl = 0;              // launch with programmatic stream serialisation
    float *out = nullptr;     // STORE: [M][ldo] fp32; RESID: residual stream [M][ldo]
    int ldo = 0;
    __half *xout = nullptr;   // SWIGLU: next activations, blocked token layout (xblk)
    int ldx_rows = 0;         // token rows of xout
    // QKV
    __half *qbuf = nullptr, *kc = nullptr, *vc = nullptr;
    int max_len = 0, n_heads = 0, n_kv = 0, head_dim = 0;
    const float *q_norm = nullptr, *k_norm = nullptr, *inv_freq = nullptr;
    const float2 *rope = nullptr;   // QKV: (cos, sin) of pos * inv_freq[i], [max_len][head_dim/2]
    float eps = 0.f;
    const int32_t *trow = nullptr, *tpos = nullptr;
    // split-K
    float *part = nullptr;
    unsigned *counters = nullptr;
    int *err = nullptr;
    // Folded RMSNorm.  Producer (RESID with norm_w): besides h += y it writes the
    // next linear's operand xout = fp16(h * norm_w * norm_scale[m]) (blocked,
    // ldx_rows rows) and the per-block sums of squares of h.  The pre-scale is an
    // earlier rstd of the same row, which keeps the operand in fp16 range.
    const float *norm_w = nullptr;
    const float *norm_scale = nullptr;   // [rows]
    float *norm_part = nullptr;          // [N/128][norm_rows]
    int norm_rows = 0;                   // token rows of the sums-of-squares scratch
    // Consumer (any op): accumulators of operand row m are multiplied by
    // rstd(m) / col_prev[m], rstd = 1/sqrt(sum_b col_part[b][m] / K + col_eps);
    // rstd is also written to col_rstd when set.
    const float *col_part = nullptr;     // [K/128][norm_rows]
    const float *col_prev = nullptr;     // [rows] the producer's pre-scale
    float *col_rstd = nullptr;
    float col_eps = 0.f;
    // STORE into peer memory (the tensor-parallel scatter, tpx.cu): feature f of
    // token m goes to peers[f / peer_cols] + peer_off + (m * peer_cols + f % peer_cols) * 4
    // bytes; once every CTA has stored, the last one writes *peer_flag * 512 +
    // peer_call + 1 to the word at peer_flag_off of every peer's region (release)
    char *const *peers = nullptr;
    size_t peer_off = 0, peer_flag_off = 0;
    int peer_n = 0, peer_cols = 0, peer_call = 0;
    const unsigned *peer_flag = nullptr;   // the forward's epoch (device)
    unsigned *peer_ctr = nullptr;          // CTA arrivals (zero between launches)
};
// (cos, sin) of p * inv_freq[i] for every position p < max_len and i < half
cudaError_t rope_table(const float *inv_freq, int half, int max_len, float2 *tab, cudaStream_t st);
bool make_weight_map(Q4WeightTC &w);
// words of the re-packed (scale, bias) pairs of an N x K weight, and the packer
size_t q4_sbp_words(int N, int K);
cudaError_t pack_q4_sb(const __half *scales, const __half *biases, int N, int K, uint32_t *sbp, cudaStream_t st);
int q4_tc_tile(int M);
size_t q4_tc_partial_floats(int N, int K, int M, int sm_count);
size_t q4_tc_counters(int N, int M);
// tokens [tok_base, tok_base + M) of the blocked operand x_blk ([K/64][ldx_rows][64]);
// output rows are 0..M-1
cudaError_t q4_tc(const Q4WeightTC &w, const __half *x_blk, int ldx_rows, int tok_base, int M,
                  int sm_count, const Q4Epilogue &ep, cudaStream_t st);

// ---- dense fp16 GEMM on tcgen05 (gemm_tc.cu): the prefill path's linears ----
// out[m][n] from y[m][n] = sum_k x[m][k] w[n][k]; w fp16 [N][K], x fp16 [M][K]
// (row-major, K % 64 == 0, N % 128 == 0).  GEMM_STORE: fp32 out[m*ldo + n];
// GEMM_ADD: fp32 out[m*ldo + n] += y; GEMM_SWIGLU: w is the fused gate/up
// matrix (64 gate rows then the matching 64 up rows per 128-row block), fp16
// out[m*ldo + i] = silu(g_i) * u_i.  err: device flag set when a wait timed out.
enum GemmEpi { GEMM_STORE = 0, GEMM_ADD = 1, GEMM_SWIGLU = 2 };
cudaError_t gemm_tc(const __half *w, int N, int K, const __half *x, int M, int epi, void *out, int ldo,
                    int sm_count, int *err, cudaStream_t st);
// fp16 [N][K] = scale * q + bias of an MLX affine q4 matrix (hfma in fp16, as
// the q4 kernels dequantise)
cudaError_t dequant_q4(const Q4Weight &w, __half *out, cudaStream_t st);

// ---- activation layout helpers --------------------------------------------
// natural [M][K] fp16 -> blocked token layout with M rows
cudaError_t permute_activations(const __half *x, __half *x_blk, int M, int K, cudaStream_t st);

// ---- per-token fused kernels ------------------------------------------------
// h = dequant(embed[tok]);  xn = rmsnorm(h) * w   (xn permuted fp16)
// rstd_out (optional): the per-token 1/sqrt(mean(h^2) + eps) of the normalisation
cudaError_t embed_norm(const Q4Weight &embed, const int32_t *tok, int M, const float *norm_w,
                       float eps, float *h, __half *xn, int ldx_rows, cudaStream_t st,
                       float *rstd_out = nullptr);
// one layer of the KV cache
struct KVLayer {
    __half *k = nullptr, *v = nullptr;   // [rows][n_kv][max_len][D]
    int max_len = 0;
};

// ---- prefill attention on tcgen05 (fa_tc.cu) ---------------------------------
// Causal attention of n prompt tokens of cache row `row` at positions s0..s0+n-1
// over keys 0..s0+n-1: q [q_rows >= n][Hq * D] fp16, out [n][Hq * D] fp16.
bool fa_prefill_supported(int head_dim);
cudaError_t fa_prefill(const __half *q, int q_rows, const KVLayer &kv, int rows, int row, int s0, int n, int Hq,
                       int Hkv, int D, __half *out, int *err, cudaStream_t st);

// ---- dense prefill path (prefill.cu): row-major activations around gemm_tc ----
// h[m] = dequantised embedding row of tok[m]
cudaError_t prefill_embed(const Q4Weight &embed, const int32_t *tok, int n, float *h, cudaStream_t st);
// x[m] = fp16(h[m] * rstd(h[m]) * w)
cudaError_t prefill_rmsnorm(const float *h, int n, int H, const float *w, float eps, __half *x, cudaStream_t st);
// h += y, then x = fp16(rmsnorm(h) * w) (the residual step after O and down)
cudaError_t prefill_add_rmsnorm(float *h, const float *y, int n, int H, const float *w, float eps, __half *x,
                                cudaStream_t st);
// y [n][(Hq + 2 Hkv) D] fp32 -> q/k norm (optional), RoPE from the (cos, sin)
// table; q to qbuf [n][Hq][D], k/v to the cache of `row` at tpos[m]
cudaError_t prefill_qkv(const float *y, int n, int n_heads, int n_kv, int D, const float *q_norm,
                        const float *k_norm, float eps, const float2 *rope, int row, const int32_t *tpos,
                        __half *qbuf, KVLayer kv, cudaStream_t st);
// trow[i] = row, tpos[i] = s0 + i for i < n
cudaError_t prefill_rows(int32_t *trow, int32_t *tpos, int row, int s0, int n, cudaStream_t st);
// row-major fp16 features of one token -> row 0 of the blocked operand layout
cudaError_t prefill_to_blocked(const __half *x, int K, __half *xb, int ldx_rows, cudaStream_t st);
// ---- sparse MoE MLP (moe.cu) -------------------------------------------------
// router GEMV (bf16 weights) + softmax + top-k; assignment a = m * TK + j of
// token m's j-th expert is appended to exp_list[expert][slot] (exp_count must
// start at zero; list_cap >= M).  The operand is the folded-RMSNorm MLP input:
// the scale rstd/col_prev of each token goes to tok_scale and rstd to col_rstd.
struct MoERouteArgs {
    const __half *x = nullptr;      // blocked operand [H/64][ldx_rows][64]
    int ldx_rows = 0;
    int M = 0, H = 0, E = 0, TK = 0, norm_topk = 1;
    const __nv_bfloat16 *wr = nullptr;   // [E][H]
    const float *col_part = nullptr, *col_prev = nullptr;
    float *col_rstd = nullptr;
    int norm_rows = 0;
    float eps = 0.f;
    float *tok_scale = nullptr;     // [M]
    int32_t *topk_id = nullptr;     // [M*TK]
    float *topk_w = nullptr;        // [M*TK]
    int *exp_count = nullptr;       // [E]
    int32_t *exp_list = nullptr;    // [E][list_cap]
    int list_cap = 0;
    float *logits = nullptr;        // scratch [M][E]
};
// grouped expert linear over all E experts of one layer: weights [E][N][K/8]
// (+ scales/biases [E][N][K/64]), the MLX SwitchGLU layout.  epi 0: gate (wq)
// and up (wq2) projections, act = silu(g)*u in the blocked layout
// [N/64][act_rows][64] per assignment; epi 1: y[assignment][N] fp32 scaled by
// the routing weight.  Operand row of assignment a: a / x_div.  A route
// without col_part treats the operand as already normalised (scale 1).
struct MoEExpertArgs {
    const uint32_t *wq = nullptr, *wq2 = nullptr;
    const __half *scales = nullptr, *biases = nullptr, *scales2 = nullptr, *biases2 = nullptr;
    int N = 0, K = 0, E = 0;
    const __half *x = nullptr;
    int ldx_rows = 0, x_div = 1;
    const int *exp_count = nullptr;
    const int32_t *exp_list = nullptr;
    int list_cap = 0;
    const float *tok_scale = nullptr;   // epi 0: per operand row
    const float *topk_w = nullptr;      // epi 1: per assignment
    __half *act = nullptr;
    int act_rows = 0;
    float *y = nullptr;
};
// h[m] += sum_j y[m*TK + j] (selection order); with norm_w also the next
// linear's operand fp16(h * norm_w * norm_scale[m]) and per-128-block sums of
// squares of h (the residual epilogue of the dense path)
struct MoECombineArgs {
    float *h = nullptr;
    const float *y = nullptr;
    int M = 0, H = 0, TK = 0;
    const float *norm_w = nullptr, *norm_scale = nullptr;
    __half *xout = nullptr;
    int ldx_rows = 0;
    float *norm_part = nullptr;
    int norm_rows = 0;
};
cudaError_t moe_route(const MoERouteArgs &a, cudaStream_t st);
cudaError_t moe_expert(const MoEExpertArgs &a, int epi, cudaStream_t st);
cudaError_t moe_combine(const MoECombineArgs &a, cudaStream_t st);
// bf16 router weights N(0, stddev) from the weight stream (bit-identical with
// the CPU restatement's orc_router_synth)
cudaError_t router_synth(uint64_t seed, uint32_t tensor_id, float stddev, int E, int H, void *w,
                         cudaStream_t st);

// ---- tensor parallelism (tp.cu): NCCL opened at run time; error strings or nullptr
bool tp_available();
const char *tp_unique_id(uint8_t *out128);
const char *tp_connect(void **comm, const uint8_t *id128, int nranks, int rank);
const char *tp_allreduce_sum(void *comm, float *buf, size_t n, cudaStream_t st);
void tp_destroy(void *comm);

// ---- expert parallel MoE over NVLink peer memory (ep.cu) ---------------------
// Per-assignment metadata stored into the owner's receive slab.
struct EpMeta {
    int expert;      // the owner's local expert index
    float scale;     // folded-norm scale of the token
    float weight;    // routing weight
    int pad;         // the source's assignment index (where the result goes back)
};
// Byte offsets inside each rank's exported region (two buffer sets, by layer parity):
// recv_x [2][H/64][N*cap][64] fp16, recv_meta [2][N][cap], recv_count [2][N],
// recv_flag [2][N], ret_y [2][cap][H] fp32, ret_flag [2][N].
struct EpLayout {
    size_t recv_x = 0, recv_meta = 0, recv_count = 0, recv_flag = 0, ret_y = 0, ret_flag = 0, total = 0;
};
EpLayout ep_layout(int N, int cap, int H);
struct EpArgs {
    char *const *peers = nullptr;   // device array [N]: every rank's mapped region (own included)
    EpLayout layout;
    int N = 0, me = 0, cap = 0, H = 0, TK = 0, epr = 0, set = 0, layer = 0;
    const unsigned *epoch = nullptr;  // forwards run so far (device)
    int *lcount = nullptr;            // [N] rows dispatched per owner (zero between layers)
    unsigned *done = nullptr;         // CTA arrival counter (zero between kernels)
    int *err = nullptr;               // device error flag (wait timeouts)
};
cudaError_t ep_begin(unsigned *epoch, cudaStream_t st);
cudaError_t ep_dispatch(const EpArgs &a, const int32_t *topk_id, const float *topk_w, const float *tok_scale,
                        const __half *x_blk, int ldx_rows, int n, cudaStream_t st);
cudaError_t ep_wait_dispatch(const EpArgs &a, cudaStream_t st);
// owner side: per-local-expert lists over the received rows (row = src*cap + slot)
cudaError_t ep_lists(const EpArgs &a, int *exp_count, int32_t *exp_list, float *row_scale, float *row_weight,
                     cudaStream_t st);
cudaError_t ep_return(const EpArgs &a, const float *ys, cudaStream_t st);
// source side: wait for every owner's returned rows
cudaError_t ep_wait_return(const EpArgs &a, cudaStream_t st);
// this layer's buffer set inside this rank's own region: the returned rows
// [cap][H] fp32 in assignment order, the received operand rows [H/64][N*cap][64]
const float *ep_returned(const EpArgs &a, const char *own_region);
const __half *ep_received(const EpArgs &a, const char *own_region);

// ---- tensor-parallel allreduce over peer memory (tpx.cu) --------------------
// Byte offsets inside each rank's exported region (two buffer sets, by call parity):
// scat [2][N][mcap][H/N] fp32, scat_flag [2][N], gath [2][mcap][H] fp32, gath_flag [2][N].
struct TpxLayout {
    size_t scat = 0, scat_flag = 0, gath = 0, gath_flag = 0, total = 0;
};
TpxLayout tpx_layout(int N, int mcap, int H);
struct TpxArgs {
    char *const *peers = nullptr;   // device array [N]: every rank's mapped region (own included)
    TpxLayout layout;
    int N = 0, me = 0, mcap = 0, H = 0, set = 0, call = 0;
    const unsigned *epoch = nullptr;  // forwards run so far (device)
    unsigned *done = nullptr;         // reduce kernel's CTA arrivals (zero between kernels)
    unsigned *sig = nullptr;          // scatter (q4 kernel) CTA arrivals
    int *err = nullptr;
};
// the STORE epilogue fields that make a row-split projection scatter its partial sums
void tpx_scatter_epilogue(const TpxArgs &a, Q4Epilogue &e);
cudaError_t tpx_reduce(const TpxArgs &a, int M, int sm_count, cudaStream_t st);
cudaError_t tpx_wait(const TpxArgs &a, cudaStream_t st);
const float *tpx_gathered(const TpxArgs &a, const char *own_region);

// ---- decode attention (split-K over keys, GQA) -----------------------------
// Tokens come in groups of `qg` consecutive positions of one row (the verify
// tokens of a row, or a slice of a prompt).  Output fp16, permuted, [M][Hq*D].
struct AttnScratch {
    float *o = nullptr;     // [groups*n_kv*splits][QMAX][D]
    float *ml = nullptr;    // [groups*n_kv*splits][QMAX][2]
    size_t items = 0;
};
int attention_max_splits(int max_len, int key_chunk);
size_t attention_scratch_items(int groups, int n_kv, int splits);
int attention_qrows(int qg, int n_heads, int n_kv);
cudaError_t attention(const __half *qbuf, KVLayer kv, const int32_t *trow, const int32_t *tpos,
                      int M, int qg, int n_heads, int n_kv, int D, int key_chunk, int splits,
                      AttnScratch scratch, __half *out, bool permuted_out, int out_rows,
                      cudaStream_t st, bool early_kv = false);
// early_kv: the launch follows the QKV projection of the same forward, so cached
// keys older than the launch's tokens may be read before waiting for it

// ---- lm head / sampling ----------------------------------------------------
// argmax of each row of logits [M][V]; with scratch (part: argmax_scratch_words(M)
// u64, ctr: M u32 that start at zero and are left at zero) the rows are split
// over ARGMAX_SPLITS CTAs each
constexpr int ARGMAX_SPLITS = 16;
size_t argmax_scratch_words(int M);
cudaError_t argmax_rows(const float *logits, int M, int V, int32_t *out, cudaStream_t st,
                        unsigned long long *part = nullptr, unsigned *ctr = nullptr);

// ---- drafter ----------------------------------------------------------------
struct RowState {
    int32_t *hist;        // [rows][hist_cap]
    int32_t *hist_len;    // [rows]
    int32_t *kv_len;      // [rows]
    int32_t *n_gen;       // [rows]
    int32_t *max_new;     // [rows]
    int32_t *active;      // [rows]
    float *temperature;   // [rows]
    float *top_p;         // [rows]
    uint64_t *seed;       // [rows]
    int32_t *has_seed;    // [rows]
    int32_t *eos;         // [rows][8]
    int32_t *n_eos;       // [rows]
    int32_t *trigger;     // [rows]
    int hist_cap;
    int rows;
};
struct SpecParams {
    int mode, enabled, k, n, min_ctx;
};
// vtok[r][0..k]: current token then drafts (padding repeats the current
// token); count[r]; tokens' row/position descriptors for the forward.
cudaError_t draft(const RowState &rs, const SpecParams &sp, int32_t *vtok, int32_t *count,
                  int32_t *trow, int32_t *tpos, cudaStream_t st);

// greedy acceptance + in-place rollback (history append, kv_len, n_gen,
// finish).  amax: [rows][k+1] argmax per verify position.
struct StepOut {
    int32_t *tokens;        // [rows][k+1]
    int32_t *n;             // [rows]
    int32_t *finished;      // [rows]
    unsigned long long *stats;  // [4] proposed, accepted, proposal_batches, rejected
};
cudaError_t accept_greedy(const RowState &rs, const SpecParams &sp, const int32_t *vtok,
                          const int32_t *count, const int32_t *amax, StepOut out,
                          cudaStream_t st);
// sampling rows (temperature > 0): single-draft rejection sampling from the
// row's seeded uniforms; greedy rows are left to accept_greedy.
struct SampleScratch {
    float *m;                 // [rows*(k+1)]
    uint32_t *thr;            // [rows*(k+1)] top-p threshold key
    unsigned long long *S;    // [rows*(k+1)]
    unsigned long long *Pd;   // [rows*(k+1)]
};
// grammar masks: logits of token i outside its allowed set (bits [M][ceil(V/32)])
// become -inf where on[i]; an empty set leaves the row unchanged
cudaError_t apply_token_masks(float *logits, int M, int V, const uint32_t *bits, const uint8_t *on,
                              cudaStream_t st);
cudaError_t accept_sampled(const RowState &rs, const SpecParams &sp, const int32_t *vtok,
                           const int32_t *count, const float *logits, int V, SampleScratch sc,
                           StepOut out, cudaStream_t st);

// first token after prefill: greedy or sampled at generation index 0
cudaError_t sample_first(const RowState &rs, int row, const float *logits, int V,
                         const int32_t *amax, SampleScratch sc, int32_t *out_token,
                         cudaStream_t st);

// table model (the reference's fake LanguageModel): logits +20 at next[tok]
cudaError_t table_logits(const int32_t *next, const int32_t *tok, int M, int V, float *logits,
                         cudaStream_t st);

}  // namespace mlxcat
