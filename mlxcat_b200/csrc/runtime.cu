// runtime.cu -- context, weights, cache and the speculative step behind the
// C ABI (include/mlxcat_cuda.h).
//
// The host side mirrors ContinuousBatchGenerator.speculativeNext
// (BatchGenerator.swift:875-955) with every row of the batch speculating at
// once: draft (device) -> verify forward over rows x (k+1) tokens (device) ->
// acceptance + in-place rollback (device) -> one device-to-host copy of the
// emitted tokens.  The whole step is captured once per configuration into a
// CUDA graph and replayed.
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <string>
#include <vector>

#include "../../include/mlxcat_cuda.h"
#include "common.cuh"
#include "kernels.h"

using namespace mlxcat;

namespace {

constexpr int PREFILL_CHUNK = 128;   // prompt tokens per prefill forward (q4 kernels)
constexpr int PREFILL_QG = 8;        // prompt tokens per attention group
constexpr int DENSE_CHUNK = 4096;    // prompt tokens per dense prefill forward (fp16 GEMMs)
constexpr int DENSE_MIN = 256;       // prompts at least this long take the dense prefill
constexpr int KEY_CHUNK = 384;       // keys per attention split of the operator entry points
constexpr int KEY_CHUNK_MAX = 1024;  // longest split a cache's verify attention uses

// Keys per split of a cache's verify attention: about 2.5 waves of split CTAs
// (four per SM) over the cache's (row, kv head) pairs at its full length, at
// least KEY_CHUNK.  Long contexts over many rows take longer splits (fewer
// partials to merge, less per-split overhead): at 32 rows x 8 kv heads x 4.4k
// keys, 768 keys per split ran 135 us per layer against 152 at 384; a few rows
// keep 384 (8 x 8 x 2.8k: 29.6 us at 384, 43.6 at 768).
int cache_key_chunk(int rows, int n_kv, int max_len, int sm_count) {
    const double pairs = (double)rows * n_kv, slots = 4.0 * sm_count;
    int kc = (int)(max_len * pairs / (2.5 * slots));
    kc = (kc + 31) / 32 * 32;
    return std::min(KEY_CHUNK_MAX, std::max(KEY_CHUNK, kc));
}

thread_local std::string g_op_err;

struct DevLin {
    uint32_t *wq = nullptr;
    __half *s = nullptr, *b = nullptr;
    uint32_t *sbp = nullptr;   // (scale, bias) pairs in the tensor-core kernel's order
    int N = 0, K = 0;
    Q4WeightTC tcw;       // TMA map over the packed words (built once the buffer exists)
    const Q4WeightTC &tc() const { return tcw; }
    Q4Weight view() const {
        Q4Weight w;
        w.wq = wq; w.scales = s; w.biases = b; w.N = N; w.K = K;
        return w;
    }
    bool build_map() {
        tcw.wq = wq; tcw.scales = s; tcw.biases = b; tcw.sbp = sbp; tcw.N = N; tcw.K = K;
        return make_weight_map(tcw);
    }
    size_t bytes() const { return (size_t)N * K / 2 + (size_t)N * (K / 64) * 4; }
};

// Row placement of a logical tensor inside a fused matrix: logical row n goes
// to (n / group) * stride + n % group + offset.  q|k|v are stacked; gate and up
// are interleaved in blocks of 64 rows so one 128-row tile of the fused
// gate/up linear holds 64 gate rows and the 64 matching up rows.
struct RowMap {
    int offset = 0, group = 0, stride = 0, rows = 0;
    int row(int n) const { return group ? (n / group) * stride + n % group + offset : n + offset; }
};

}  // namespace

struct mlxcat_ctx {
    // cfg: this rank's view (per-rank head / MLP widths when tensor-parallel);
    // gcfg: the model as configured by the caller
    mlxcat_model_config cfg{}, gcfg{};
    int tp = 1, tp_rank = 0;
    int ep = 1, ep_rank = 0, epr = 0;   // expert parallel: ranks, this rank, experts per rank
    void *nccl = nullptr;   // ncclComm_t of the tensor- or expert-parallel group
    int device = 0, sm_count = 148;
    cudaStream_t stream = nullptr;
    std::string err;
    std::vector<void *> allocs;
    DevLin embed, lm_head;
    std::vector<DevLin> qkv, o, gu, down;
    // sparse MoE MLP per layer: bf16 router [E][H]; gate, up [E][I][H/8] and down
    // [E][H][I/8] q4 in the MLX SwitchGLU layout (scales/biases [E][N][K/64])
    struct MoEBank {
        __nv_bfloat16 *router = nullptr;
        uint32_t *wq[3] = {};
        __half *s[3] = {}, *b[3] = {};
    };
    std::vector<MoEBank> moe;
    float *norms = nullptr;     // attn[L][H], mlp[L][H], final[H], qn[L][D], kn[L][D]
    float *inv_freq = nullptr;
    int32_t *table = nullptr;
    bool have_weights = false;
    int64_t launches = 0;
    std::vector<mlxcat_cache *> caches;   // live caches; destroyed with the context

    const float *attn_norm(int l) const { return norms + (size_t)l * cfg.hidden; }
    const float *mlp_norm(int l) const { return norms + (size_t)(cfg.n_layers + l) * cfg.hidden; }
    const float *final_norm() const { return norms + (size_t)2 * cfg.n_layers * cfg.hidden; }
    const float *q_norm(int l) const {
        return cfg.qk_norm ? norms + (size_t)(2 * cfg.n_layers + 1) * cfg.hidden + (size_t)l * cfg.head_dim
                           : nullptr;
    }
    const float *k_norm(int l) const {
        return cfg.qk_norm ? norms + (size_t)(2 * cfg.n_layers + 1) * cfg.hidden +
                                 (size_t)(cfg.n_layers + l) * cfg.head_dim
                           : nullptr;
    }
};

struct mlxcat_cache {
    mlxcat_ctx *ctx = nullptr;
    int rows = 0, max_len = 0, hist_cap = 0;
    std::vector<void *> allocs;
    __half *k = nullptr, *v = nullptr;
    // device row state
    int32_t *hist = nullptr, *hist_len = nullptr, *kv_len = nullptr, *n_gen = nullptr,
            *max_new = nullptr, *active = nullptr, *has_seed = nullptr, *eos = nullptr,
            *n_eos = nullptr, *trigger = nullptr;
    float *temperature = nullptr, *top_p = nullptr;
    uint64_t *seed = nullptr;
    std::vector<float> host_temp;
    // step buffers
    int m_cap = 0;
    int last_m = 0;                    // tokens of the last forward
    int32_t *vtok = nullptr, *count = nullptr, *trow = nullptr, *tpos = nullptr, *amax = nullptr,
            *out_tok = nullptr, *out_n = nullptr, *out_fin = nullptr, *first_tok = nullptr,
            *ptok = nullptr;
    unsigned long long *stats = nullptr;
    float *h = nullptr, *part = nullptr, *logits = nullptr;
    float2 *rope = nullptr;           // (cos, sin) of every position x RoPE frequency
    __half *xn = nullptr, *xa = nullptr, *qbuf = nullptr;
    __half *xg = nullptr;             // MLP input operand (blocked), written by the O projection
    // folded RMSNorm: per-block sums of squares of h [H/128][rows], and the rstd of
    // the attention-norm and MLP-norm inputs of each token row (pre-scales)
    float *norm_part = nullptr, *r_attn = nullptr, *r_mlp = nullptr;
    float *tp_part = nullptr;          // tensor parallel: this rank's O / down partial sums [rows][H]
    // expert / tensor parallel over peer memory (ep.cu, tpx.cu): this cache's
    // exported region (receive slabs or scatter/gather buffers, flags), every
    // rank's mapping of its peers' regions, and for experts the owner side's
    // per-expert lists, SwiGLU activations and scaled outputs over the N * cap
    // received rows
    char *peer_region = nullptr;
    size_t peer_bytes = 0;
    int peer_kind = 0;                 // 1 = expert parallel, 2 = tensor parallel
    int peer_cap = 0;                  // rows per (source, owner) / token rows of the buffers
    EpLayout ep_lay;
    TpxLayout tpx_lay;
    bool peer_connected = false;
    std::vector<char *> peer_opened;   // IPC mappings of the peers' regions
    char **peer_tab = nullptr;         // device [N]
    unsigned *peer_epoch = nullptr, *peer_done = nullptr, *peer_sig = nullptr;
    int *ep_lcount = nullptr;          // [N]
    __half *ep_act = nullptr;
    int *ep_exp_count = nullptr;       // [layer][local experts]
    int32_t *ep_exp_list = nullptr;
    float *ep_scale = nullptr, *ep_w = nullptr, *ep_ys = nullptr;
    // sparse MoE: routing, per-expert assignment lists (counts per layer, zeroed
    // once per forward), SwiGLU activations per assignment, scaled expert outputs
    int32_t *moe_id = nullptr, *moe_list = nullptr;
    int *moe_count = nullptr;
    float *moe_w = nullptr, *moe_scale = nullptr, *moe_y = nullptr, *moe_logits = nullptr;
    __half *moe_act = nullptr;
    size_t part_floats = 0;
    unsigned *counters = nullptr;     // split-K tickets of the q4 linear (self-resetting)
    unsigned long long *amax_part = nullptr;   // split argmax partial keys
    unsigned *amax_ctr = nullptr;              // split argmax tickets (self-resetting)
    int *err = nullptr;               // device-side wait timeouts
    int32_t *h_err = nullptr;
    AttnScratch attn;
    int attn_splits = 1, key_chunk = KEY_CHUNK;
    SampleScratch samp{};
    // dense prefill: fp16 weights of one linear, row-major activations of one
    // chunk of DENSE_CHUNK prompt tokens, attention scratch (one key split)
    struct Prefill {
        bool ready = false;
        int qg = 0, key_chunk = 0;
        __half *wdq = nullptr, *x = nullptr, *act = nullptr, *q = nullptr;
        float *h = nullptr, *y = nullptr;
        int32_t *tok = nullptr, *trow = nullptr, *tpos = nullptr;
        AttnScratch attn;
    } pf;
    // grammar masks for the next acceptance: allowed-token bitsets per verify
    // token [rows*(k+1)][ceil(vocab/32)] and their enable flags (allocated on
    // first use); mask_k = the k they were set for, -1 = none pending
    uint32_t *mask_bits = nullptr;
    uint8_t *mask_on = nullptr;
    int mask_k = -1;
    // pinned host mirrors
    int32_t *h_tok = nullptr, *h_n = nullptr, *h_fin = nullptr;
    unsigned long long *h_stats = nullptr;
    // graph of the speculative step
    cudaGraphExec_t graph = nullptr;
    mlxcat_spec_config gkey{};
    bool gsampled = false;
    int64_t graph_launches = 0;
    cudaEvent_t ev0 = nullptr, ev1 = nullptr;     // verify forward
    cudaEvent_t es0 = nullptr, es1 = nullptr;     // whole step
    int last_k = -1;
    // per-kernel profiling: event pairs around q4 linears / attention
    bool profiling = false;
    std::vector<cudaEvent_t> prof_ev;
    std::vector<int> prof_class;       // 0 = q4 linear, 1 = attention (per pair)
    size_t prof_used = 0;
    bool prof_recording = false;

    RowState rs() const {
        RowState r;
        r.hist = hist; r.hist_len = hist_len; r.kv_len = kv_len; r.n_gen = n_gen;
        r.max_new = max_new; r.active = active; r.temperature = temperature; r.top_p = top_p;
        r.seed = seed; r.has_seed = has_seed; r.eos = eos; r.n_eos = n_eos; r.trigger = trigger;
        r.hist_cap = hist_cap; r.rows = rows;
        return r;
    }
    KVLayer layer(int l) const {
        const mlxcat_model_config &c = ctx->cfg;
        KVLayer kv;
        const size_t per = (size_t)rows * c.n_kv_heads * max_len * c.head_dim;
        kv.k = k + (size_t)l * per;
        kv.v = v + (size_t)l * per;
        kv.max_len = max_len;
        return kv;
    }
};

namespace {

int set_err(mlxcat_ctx *ctx, int code, const char *fmt, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof buf, fmt, ap);
    va_end(ap);
    if (ctx) ctx->err = buf;
    return code;
}

int op_err(int code, const char *fmt, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof buf, fmt, ap);
    va_end(ap);
    g_op_err = buf;
    return code;
}

#define CK(ctx_, expr)                                                                      \
    do {                                                                                    \
        cudaError_t e_ = (expr);                                                            \
        if (e_ != cudaSuccess)                                                              \
            return set_err((ctx_), e_ == cudaErrorMemoryAllocation ? MLXCAT_E_OOM : MLXCAT_E_CUDA, \
                           "%s: %s (%s:%d)", #expr, cudaGetErrorString(e_), __FILE__, __LINE__); \
    } while (0)

#define LK(ctx_, expr)                                                                      \
    do {                                                                                    \
        (ctx_)->launches++;                                                                 \
        CK(ctx_, expr);                                                                     \
    } while (0)

template <typename T>
cudaError_t dalloc(std::vector<void *> &list, T **p, size_t n) {
    void *q = nullptr;
    cudaError_t e = cudaMalloc(&q, std::max<size_t>(n, 1) * sizeof(T));
    if (e != cudaSuccess) return e;
    list.push_back(q);
    *p = static_cast<T *>(q);
    return cudaSuccess;
}

bool valid_config(const mlxcat_model_config *c, std::string &why) {
    if (c->kind == MLXCAT_MODEL_TABLE) {
        if (c->vocab <= 0) { why = "vocab must be positive"; return false; }
        return true;
    }
    if (c->kind != MLXCAT_MODEL_TRANSFORMER) { why = "unknown model kind"; return false; }
    if (c->group_size != 64 || c->bits != 4) { why = "only MLX affine q4 group 64 is supported"; return false; }
    if (c->n_layers <= 0 || c->hidden <= 0 || c->n_heads <= 0 || c->n_kv_heads <= 0 ||
        c->head_dim <= 0 || c->intermediate <= 0 || c->vocab <= 0) {
        why = "dimensions must be positive";
        return false;
    }
    if (c->n_heads % c->n_kv_heads) { why = "n_heads must be a multiple of n_kv_heads"; return false; }
    if (c->head_dim != 64 && c->head_dim != 128) { why = "head_dim must be 64 or 128"; return false; }
    // the exchange's flag waits run one thread per peer in a single warp
    if (c->tp_size > 32 || c->ep_size > 32) { why = "tp_size and ep_size are at most 32"; return false; }
    if (c->tp_size > 1) {
        const int T = c->tp_size;
        if (c->tp_rank < 0 || c->tp_rank >= T) { why = "tp_rank must be in [0, tp_size)"; return false; }
        if (c->n_kv_heads % T) { why = "n_kv_heads must be a multiple of tp_size"; return false; }
        if (c->intermediate % T || (c->intermediate / T) % 128) {
            why = "intermediate / tp_size must be a multiple of 128";
            return false;
        }
        if (c->n_experts > 0) { why = "tensor parallelism is for dense models"; return false; }
    }
    if (c->ep_size > 1) {
        if (c->n_experts <= 0 || c->n_experts % c->ep_size) { why = "ep_size must divide n_experts (MoE models)"; return false; }
        if (c->ep_rank < 0 || c->ep_rank >= c->ep_size) { why = "ep_rank must be in [0, ep_size)"; return false; }
        if (c->tp_size > 1) { why = "tensor and expert parallelism are not combined"; return false; }
    }
    if (c->n_experts < 0) { why = "n_experts must be >= 0"; return false; }
    if (c->n_experts > 0) {
        if (c->n_experts % 32 || c->n_experts > 256) { why = "n_experts must be a multiple of 32, at most 256"; return false; }
        if (c->top_k < 1 || c->top_k > 8 || c->top_k > c->n_experts) { why = "top_k must be in 1..min(8, n_experts)"; return false; }
        if (c->hidden % 256) { why = "MoE models need hidden a multiple of 256"; return false; }
    }
    const int qkv = (c->n_heads + 2 * c->n_kv_heads) * c->head_dim;
    const int dims[] = {c->hidden, c->intermediate, c->n_heads * c->head_dim, qkv, 2 * c->intermediate, c->vocab};
    for (int d : dims)
        if (d % 128) { why = "hidden, intermediate, q/kv widths and vocab must be multiples of 128"; return false; }
    return true;
}

// bracket one launch with a pair of events when the step is being profiled
struct ProfScope {
    mlxcat_cache *c;
    cudaEvent_t e1 = nullptr;
    ProfScope(mlxcat_cache *cc, int cls) : c(cc) {
        if (!c->prof_recording) return;
        if (c->prof_used + 2 > c->prof_ev.size()) {
            for (int i = 0; i < 64; ++i) {
                cudaEvent_t e;
                if (cudaEventCreate(&e) != cudaSuccess) return;
                c->prof_ev.push_back(e);
            }
        }
        cudaEvent_t e0 = c->prof_ev[c->prof_used];
        e1 = c->prof_ev[c->prof_used + 1];
        c->prof_used += 2;
        c->prof_class.push_back(cls);
        cudaEventRecordWithFlags(e0, c->ctx->stream, cudaEventRecordExternal);
    }
    ~ProfScope() {
        if (e1) cudaEventRecordWithFlags(e1, c->ctx->stream, cudaEventRecordExternal);
    }
};

// Expert-parallel MoE MLP of layer l (after the route): every assignment's
// operand row is stored into the owning rank's receive slab over NVLink, the
// owner runs the grouped expert kernels over all rows it received, stores the
// scaled fp32 outputs back into each source's return buffer, and the source's
// combine reads them in assignment order (ep.cu).
int ep_moe(mlxcat_cache *c, int l, int M) {
    mlxcat_ctx *ctx = c->ctx;
    const mlxcat_model_config &cf = ctx->cfg;
    const int H = cf.hidden, I = cf.intermediate, TK = cf.top_k, N = ctx->ep, epr = ctx->epr, R = c->m_cap;
    const int rows = N * c->peer_cap;
    cudaStream_t st = ctx->stream;
    EpArgs a;
    a.peers = c->peer_tab; a.layout = c->ep_lay; a.N = N; a.me = ctx->ep_rank; a.cap = c->peer_cap; a.H = H;
    a.TK = TK; a.epr = epr; a.set = l & 1; a.layer = l;
    a.epoch = c->peer_epoch; a.lcount = c->ep_lcount; a.done = c->peer_done; a.err = c->err;
    const size_t asg = (size_t)c->m_cap * TK;
    LK(ctx, ep_dispatch(a, c->moe_id + l * asg, c->moe_w + l * asg, c->moe_scale, c->xg, R, M * TK, st));
    LK(ctx, ep_wait_dispatch(a, st));
    int *ecnt = c->ep_exp_count + (size_t)l * epr;
    LK(ctx, ep_lists(a, ecnt, c->ep_exp_list, c->ep_scale, c->ep_w, st));
    const auto &mb = ctx->moe[l];
    MoEExpertArgs xa;
    xa.wq = mb.wq[0]; xa.scales = mb.s[0]; xa.biases = mb.b[0];
    xa.wq2 = mb.wq[1]; xa.scales2 = mb.s[1]; xa.biases2 = mb.b[1];
    xa.N = I; xa.K = H; xa.E = epr; xa.x = ep_received(a, c->peer_region); xa.ldx_rows = rows; xa.x_div = 1;
    xa.exp_count = ecnt; xa.exp_list = c->ep_exp_list; xa.list_cap = rows;
    xa.tok_scale = c->ep_scale; xa.act = c->ep_act; xa.act_rows = rows;
    { ProfScope ps(c, 0); LK(ctx, moe_expert(xa, 0, st)); }
    MoEExpertArgs da;
    da.wq = mb.wq[2]; da.scales = mb.s[2]; da.biases = mb.b[2];
    da.N = H; da.K = I; da.E = epr; da.x = c->ep_act; da.ldx_rows = rows; da.x_div = 1;
    da.exp_count = ecnt; da.exp_list = c->ep_exp_list; da.list_cap = rows;
    da.topk_w = c->ep_w; da.y = c->ep_ys;
    { ProfScope ps(c, 0); LK(ctx, moe_expert(da, 1, st)); }
    LK(ctx, ep_return(a, c->ep_ys, st));
    LK(ctx, ep_wait_return(a, st));
    MoECombineArgs ca;
    ca.h = c->h; ca.y = ep_returned(a, c->peer_region); ca.M = M; ca.H = H; ca.TK = TK;
    ca.norm_w = l + 1 < cf.n_layers ? ctx->attn_norm(l + 1) : ctx->final_norm(); ca.norm_scale = c->r_mlp;
    ca.xout = c->xn; ca.ldx_rows = R; ca.norm_part = c->norm_part; ca.norm_rows = R;
    LK(ctx, moe_combine(ca, st));
    return MLXCAT_OK;
}

// Tensor-parallel residual step: this rank's slice of a row-split projection
// (O or down) as fp32 partial sums, summed over the group, then h += y with the
// next linear's folded-norm operand fp16(h * norm_w * s) and per-block sums of
// squares -- what the RESID epilogue does on one GPU.  With the cache's peer
// regions connected the sum is the fused scatter / reduce / gather of tpx.cu
// (call = 2 * layer + {0: O, 1: down}); otherwise one NCCL allreduce.
int tp_residual(mlxcat_cache *c, const DevLin &w, const __half *x, int M, const float *norm_w,
                const float *norm_scale, __half *xout, int call) {
    mlxcat_ctx *ctx = c->ctx;
    const int H = ctx->cfg.hidden, R = c->m_cap;
    cudaStream_t st = ctx->stream;
    Q4Epilogue e;
    e.part = c->part; e.counters = c->counters; e.err = c->err; e.pdl = 1;
    e.op = Q4Epilogue::STORE; e.out = c->tp_part; e.ldo = H;
    const float *y = c->tp_part;
    if (c->peer_connected) {
        TpxArgs a;
        a.peers = c->peer_tab; a.layout = c->tpx_lay; a.N = ctx->tp; a.me = ctx->tp_rank; a.mcap = c->peer_cap;
        a.H = H; a.set = call & 1; a.call = call;
        a.epoch = c->peer_epoch; a.done = c->peer_done; a.sig = c->peer_sig; a.err = c->err;
        tpx_scatter_epilogue(a, e);
        { ProfScope ps(c, 0); LK(ctx, q4_tc(w.tc(), x, R, 0, M, ctx->sm_count, e, st)); }
        ctx->launches += 2;
        LK(ctx, tpx_reduce(a, M, ctx->sm_count, st));
        LK(ctx, tpx_wait(a, st));
        y = tpx_gathered(a, c->peer_region);
    } else {
        { ProfScope ps(c, 0); LK(ctx, q4_tc(w.tc(), x, R, 0, M, ctx->sm_count, e, st)); }
        if (const char *er = tp_allreduce_sum(ctx->nccl, c->tp_part, (size_t)M * H, st))
            return set_err(ctx, MLXCAT_E_CUDA, "allreduce: %s", er);
    }
    MoECombineArgs ca;
    ca.h = c->h; ca.y = y; ca.M = M; ca.H = H; ca.TK = 1;
    ca.norm_w = norm_w; ca.norm_scale = norm_scale; ca.xout = xout; ca.ldx_rows = R;
    ca.norm_part = c->norm_part; ca.norm_rows = R;
    LK(ctx, moe_combine(ca, st));
    return MLXCAT_OK;
}

// ---------------------------------------------------------------------------
// forward over M tokens (tok/trow/tpos on device); logits for tokens
// [lg_from, M) into c->logits (rows in that order); lg_from = M: no logits
// ---------------------------------------------------------------------------
int forward(mlxcat_cache *c, int M, int qg, const int32_t *tok, const int32_t *trow,
            const int32_t *tpos, int lg_from) {
    mlxcat_ctx *ctx = c->ctx;
    const mlxcat_model_config &cf = ctx->cfg;
    cudaStream_t st = ctx->stream;
    if (cf.kind == MLXCAT_MODEL_TABLE) {
        if (lg_from < M) LK(ctx, table_logits(ctx->table, tok + lg_from, M - lg_from, cf.vocab, c->logits, st));
        return MLXCAT_OK;
    }
    const int H = cf.hidden, D = cf.head_dim, Hq = cf.n_heads, Hkv = cf.n_kv_heads,
              I = cf.intermediate, L = cf.n_layers;
    const float eps = cf.rms_eps;
    const int R = c->m_cap;   // token rows of the blocked activation buffers
    c->last_m = M;
    // The RMSNorms between the linears are folded into them: a residual linear
    // writes fp16(h * w * s) with s an earlier rstd of the row and the per-block
    // sums of squares of h; the next linear scales its accumulators by rstd / s.
    // Layer 0's input is normalised exactly here.
    LK(ctx, embed_norm(ctx->embed.view(), tok, M, ctx->attn_norm(0), eps, c->h, c->xn, R, st, c->r_attn));
    if (cf.n_experts) CK(ctx, cudaMemsetAsync(c->moe_count, 0, sizeof(int) * (size_t)L * cf.n_experts, st));
    if (cf.n_experts && ctx->ep > 1) {
        if (!c->peer_connected)
            return set_err(ctx, MLXCAT_E_STATE, "expert-parallel cache not connected (mlxcat_cache_peer_connect)");
        CK(ctx, cudaMemsetAsync(c->ep_exp_count, 0, sizeof(int) * (size_t)L * ctx->epr, st));
    }
    if (c->peer_connected) {
        ctx->launches++;
        LK(ctx, ep_begin(c->peer_epoch, st));   // the forward's epoch, part of every exchange flag
    }
    Q4Epilogue ep;
    ep.part = c->part;
    ep.counters = c->counters;
    ep.err = c->err;
    ep.pdl = 1;   // each linear streams its weights while its predecessor finishes
    for (int l = 0; l < L; ++l) {
        const KVLayer kv = c->layer(l);
        {   // q|k|v projection + q/k norm + RoPE + KV append
            Q4Epilogue e = ep;
            e.op = Q4Epilogue::QKV;
            e.qbuf = c->qbuf; e.kc = kv.k; e.vc = kv.v; e.max_len = kv.max_len;
            e.n_heads = Hq; e.n_kv = Hkv; e.head_dim = D;
            e.q_norm = ctx->q_norm(l); e.k_norm = ctx->k_norm(l); e.eps = eps;
            e.inv_freq = ctx->inv_freq; e.rope = c->rope; e.trow = trow; e.tpos = tpos;
            if (l > 0) {   // operand = down projection's fp16(h * attn_norm * r_mlp)
                e.col_part = c->norm_part; e.col_prev = c->r_mlp; e.col_rstd = c->r_attn;
                e.col_eps = eps; e.norm_rows = R;
            }
            ProfScope ps(c, 0);
            LK(ctx, q4_tc(ctx->qkv[l].tc(), c->xn, R, 0, M, ctx->sm_count, e, st));
        }
        ctx->launches++;  // attention is two kernels
        { ProfScope ps(c, 1);
          LK(ctx, attention(c->qbuf, kv, trow, tpos, M, qg, Hq, Hkv, D, c->key_chunk, c->attn_splits,
                            c->attn, c->xn, true, R, st, true)); }
        if (ctx->tp > 1) {   // row-split output projection: partial sums, allreduce, residual
            int rc = tp_residual(c, ctx->o[l], c->xn, M, ctx->mlp_norm(l), c->r_attn, c->xg, 2 * l);
            if (rc) return rc;
        } else {   // output projection into the residual stream
            Q4Epilogue e = ep;
            e.op = Q4Epilogue::RESID; e.out = c->h; e.ldo = H;
            // + the MLP input fp16(h * mlp_norm * r_attn) (not into xn: other CTAs
            // may still be reading this projection's own operand there)
            e.norm_w = ctx->mlp_norm(l); e.norm_scale = c->r_attn; e.xout = c->xg; e.ldx_rows = R;
            e.norm_part = c->norm_part; e.norm_rows = R;
            ProfScope ps(c, 0);
            LK(ctx, q4_tc(ctx->o[l].tc(), c->xn, R, 0, M, ctx->sm_count, e, st));
        }
        if (cf.n_experts) {   // sparse MoE MLP: route, experts, combine into the residual
            const int E = cf.n_experts, TK = cf.top_k;
            int *cnt = c->moe_count + (size_t)l * E;
            MoERouteArgs ra;
            ra.x = c->xg; ra.ldx_rows = R; ra.M = M; ra.H = H; ra.E = E; ra.TK = TK; ra.norm_topk = cf.norm_topk;
            ra.wr = ctx->moe[l].router;
            ra.col_part = c->norm_part; ra.col_prev = c->r_attn; ra.col_rstd = c->r_mlp; ra.norm_rows = R;
            const size_t asg = (size_t)c->m_cap * TK;   // routing kept per layer (inspection)
            ra.eps = eps; ra.tok_scale = c->moe_scale; ra.topk_id = c->moe_id + l * asg; ra.topk_w = c->moe_w + l * asg;
            ra.exp_count = cnt; ra.exp_list = c->moe_list; ra.list_cap = c->m_cap; ra.logits = c->moe_logits;
            ctx->launches++;   // logits + top-k
            LK(ctx, moe_route(ra, st));
            const auto &mb = ctx->moe[l];
            if (ctx->ep > 1) {
                int rc = ep_moe(c, l, M);
                if (rc) return rc;
                continue;
            }
            MoEExpertArgs xa;
            xa.wq = mb.wq[0]; xa.scales = mb.s[0]; xa.biases = mb.b[0];
            xa.wq2 = mb.wq[1]; xa.scales2 = mb.s[1]; xa.biases2 = mb.b[1];
            xa.N = I; xa.K = H; xa.E = E; xa.x = c->xg; xa.ldx_rows = R; xa.x_div = TK;
            xa.exp_count = cnt; xa.exp_list = c->moe_list; xa.list_cap = c->m_cap;
            xa.tok_scale = c->moe_scale; xa.act = c->moe_act; xa.act_rows = c->m_cap * TK;
            { ProfScope ps(c, 0); LK(ctx, moe_expert(xa, 0, st)); }
            MoEExpertArgs da;
            da.wq = mb.wq[2]; da.scales = mb.s[2]; da.biases = mb.b[2];
            da.N = H; da.K = I; da.E = E; da.x = c->moe_act; da.ldx_rows = c->m_cap * TK; da.x_div = 1;
            da.exp_count = cnt; da.exp_list = c->moe_list; da.list_cap = c->m_cap;
            da.topk_w = c->moe_w + l * asg; da.y = c->moe_y;
            { ProfScope ps(c, 0); LK(ctx, moe_expert(da, 1, st)); }
            MoECombineArgs ca;
            ca.h = c->h; ca.y = c->moe_y; ca.M = M; ca.H = H; ca.TK = TK;
            ca.norm_w = l + 1 < L ? ctx->attn_norm(l + 1) : ctx->final_norm(); ca.norm_scale = c->r_mlp;
            ca.xout = c->xn; ca.ldx_rows = R; ca.norm_part = c->norm_part; ca.norm_rows = R;
            LK(ctx, moe_combine(ca, st));
            continue;
        }
        {   // gate/up + SwiGLU
            Q4Epilogue e = ep;
            e.op = Q4Epilogue::SWIGLU; e.xout = c->xa; e.ldx_rows = R;
            e.col_part = c->norm_part; e.col_prev = c->r_attn; e.col_rstd = c->r_mlp;
            e.col_eps = eps; e.norm_rows = R;
            ProfScope ps(c, 0);
            LK(ctx, q4_tc(ctx->gu[l].tc(), c->xg, R, 0, M, ctx->sm_count, e, st));
        }
        if (ctx->tp > 1) {   // row-split down projection
            int rc = tp_residual(c, ctx->down[l], c->xa, M, l + 1 < L ? ctx->attn_norm(l + 1) : ctx->final_norm(),
                                 c->r_mlp, c->xn, 2 * l + 1);
            if (rc) return rc;
            continue;
        }
        {   // down projection into the residual stream
            Q4Epilogue e = ep;
            e.op = Q4Epilogue::RESID; e.out = c->h; e.ldo = H;
            // + the next layer's (or the head's) input fp16(h * norm * r_mlp)
            e.norm_w = l + 1 < L ? ctx->attn_norm(l + 1) : ctx->final_norm(); e.norm_scale = c->r_mlp;
            e.xout = c->xn; e.ldx_rows = R;
            e.norm_part = c->norm_part; e.norm_rows = R;
            ProfScope ps(c, 0);
            LK(ctx, q4_tc(ctx->down[l].tc(), c->xa, R, 0, M, ctx->sm_count, e, st));
        }
    }
    if (lg_from < M) {
        const DevLin &head = cf.tie_embeddings ? ctx->embed : ctx->lm_head;
        Q4Epilogue e = ep;
        e.op = Q4Epilogue::STORE; e.out = c->logits; e.ldo = cf.vocab;
        e.col_part = c->norm_part; e.col_prev = c->r_mlp; e.col_eps = eps; e.norm_rows = R;
        ProfScope ps(c, 0);
        LK(ctx, q4_tc(head.tc(), c->xn, R, lg_from, M - lg_from, ctx->sm_count, e, st));
    }
    return MLXCAT_OK;
}

int check_weights(mlxcat_cache *c) {
    mlxcat_ctx *ctx = c->ctx;
    if (!ctx->have_weights) return set_err(ctx, MLXCAT_E_STATE, "weights not loaded");
    if (ctx->tp > 1 && !ctx->nccl && !c->peer_connected)
        return set_err(ctx, MLXCAT_E_STATE,
                       "tensor-parallel cache not connected (mlxcat_cache_peer_connect or mlxcat_ctx_tp_connect)");
    if (ctx->ep > 1 && ctx->cfg.n_experts && !c->peer_connected)
        return set_err(ctx, MLXCAT_E_STATE, "expert-parallel cache not connected (mlxcat_cache_peer_connect)");
    return MLXCAT_OK;
}

int validate_spec(mlxcat_ctx *ctx, const mlxcat_spec_config *s) {
    if (!s) return set_err(ctx, MLXCAT_E_INVALID, "spec config is NULL");
    if (s->max_proposal < 0 || s->max_proposal > MLXCAT_MAX_PROPOSAL)
        return set_err(ctx, MLXCAT_E_INVALID, "max_proposal must be in [0, %d]", MLXCAT_MAX_PROPOSAL);
    if (s->max_suffix < 1 || s->min_context < 2 || (s->mode != 0 && s->mode != 1))
        return set_err(ctx, MLXCAT_E_INVALID, "bad spec config");
    return MLXCAT_OK;
}

SpecParams params_of(const mlxcat_spec_config *s) {
    SpecParams p;
    p.mode = s->mode;
    p.enabled = s->enabled;
    p.k = s->enabled ? s->max_proposal : 0;
    p.n = s->max_suffix;
    p.min_ctx = s->min_context;
    return p;
}

StepOut step_out(mlxcat_cache *c) {
    StepOut o;
    o.tokens = c->out_tok; o.n = c->out_n; o.finished = c->out_fin; o.stats = c->stats;
    return o;
}

bool any_sampled(const mlxcat_cache *c) {
    for (float t : c->host_temp)
        if (t != 0.0f) return true;
    return false;
}

// draft -> verify -> accept, enqueued on the context stream
int enqueue_step(mlxcat_cache *c, const SpecParams &sp, bool sampled, bool timed) {
    mlxcat_ctx *ctx = c->ctx;
    cudaStream_t st = ctx->stream;
    const int K1 = sp.k + 1, M = c->rows * K1;
    if (timed) CK(ctx, cudaEventRecordWithFlags(c->es0, st, cudaEventRecordExternal));
    LK(ctx, draft(c->rs(), sp, c->vtok, c->count, c->trow, c->tpos, st));
    if (timed) CK(ctx, cudaEventRecordWithFlags(c->ev0, st, cudaEventRecordExternal));
    c->prof_used = 0;
    c->prof_class.clear();
    c->prof_recording = timed && c->profiling;
    int rc = forward(c, M, K1, c->vtok, c->trow, c->tpos, 0);
    c->prof_recording = false;
    if (rc) return rc;
    if (timed) CK(ctx, cudaEventRecordWithFlags(c->ev1, st, cudaEventRecordExternal));
    LK(ctx, argmax_rows(c->logits, M, ctx->cfg.vocab, c->amax, st, c->amax_part, c->amax_ctr));
    LK(ctx, accept_greedy(c->rs(), sp, c->vtok, c->count, c->amax, step_out(c), st));
    if (sampled) {
        ctx->launches++;
        LK(ctx, accept_sampled(c->rs(), sp, c->vtok, c->count, c->logits, ctx->cfg.vocab, c->samp,
                               step_out(c), st));
    }
    CK(ctx, cudaMemcpyAsync(c->h_tok, c->out_tok, sizeof(int32_t) * M, cudaMemcpyDeviceToHost, st));
    CK(ctx, cudaMemcpyAsync(c->h_n, c->out_n, sizeof(int32_t) * c->rows, cudaMemcpyDeviceToHost, st));
    CK(ctx, cudaMemcpyAsync(c->h_fin, c->out_fin, sizeof(int32_t) * c->rows, cudaMemcpyDeviceToHost, st));
    CK(ctx, cudaMemcpyAsync(c->h_stats, c->stats, sizeof(unsigned long long) * 4, cudaMemcpyDeviceToHost, st));
    if (c->err) CK(ctx, cudaMemcpyAsync(c->h_err, c->err, sizeof(int), cudaMemcpyDeviceToHost, st));
    if (timed) CK(ctx, cudaEventRecordWithFlags(c->es1, st, cudaEventRecordExternal));
    return MLXCAT_OK;
}

void copy_out(mlxcat_cache *c, int K1, int32_t *out_tokens, int32_t *out_counts, int32_t *out_fin,
              mlxcat_stats *stats) {
    if (out_tokens) memcpy(out_tokens, c->h_tok, sizeof(int32_t) * c->rows * K1);
    if (out_counts) memcpy(out_counts, c->h_n, sizeof(int32_t) * c->rows);
    if (out_fin) memcpy(out_fin, c->h_fin, sizeof(int32_t) * c->rows);
    if (stats) {
        stats->proposed = (int64_t)c->h_stats[0];
        stats->accepted = (int64_t)c->h_stats[1];
        stats->proposal_batches = (int64_t)c->h_stats[2];
        stats->rejected_batches = (int64_t)c->h_stats[3];
    }
    for (int r = 0; r < c->rows; ++r)
        if (c->h_fin[r]) c->host_temp[r] = 0.0f;
}

// a device wait that timed out (bounded mbarrier polls) poisons the cache's
// results: report it and clear the flag
int device_err(mlxcat_cache *c, bool from_pinned) {
    int e = 0;
    if (!c->err) return MLXCAT_OK;
    if (from_pinned) {
        e = *c->h_err;
    } else if (cudaMemcpy(&e, c->err, sizeof(int), cudaMemcpyDeviceToHost) != cudaSuccess) {
        return set_err(c->ctx, MLXCAT_E_CUDA, "reading the device error flag failed");
    }
    if (e == 0) return MLXCAT_OK;
    cudaMemset(c->err, 0, sizeof(int));
    *c->h_err = 0;
    return set_err(c->ctx, MLXCAT_E_CUDA, "a device pipeline wait timed out (code %d)", e);
}

void drop_graph(mlxcat_cache *c) {
    if (c->graph) cudaGraphExecDestroy(c->graph);
    c->graph = nullptr;
}

}  // namespace

namespace {
// The dense prefill path needs a dense (non-MoE) model on one GPU.
bool dense_prefill_ok(const mlxcat_ctx *ctx) {
    const mlxcat_model_config &cf = ctx->cfg;
    return cf.kind == MLXCAT_MODEL_TRANSFORMER && !cf.n_experts && ctx->tp == 1 && ctx->ep == 1 &&
           cf.hidden % 128 == 0 && cf.intermediate % 128 == 0 && (cf.n_heads * cf.head_dim) % 128 == 0;
}

int ensure_prefill(mlxcat_cache *c) {
    auto &pf = c->pf;
    if (pf.ready) return MLXCAT_OK;
    mlxcat_ctx *ctx = c->ctx;
    const mlxcat_model_config &cf = ctx->cfg;
    const int H = cf.hidden, I = cf.intermediate, D = cf.head_dim, Hq = cf.n_heads, Hkv = cf.n_kv_heads;
    const size_t P = DENSE_CHUNK, Nqkv = (size_t)(Hq + 2 * Hkv) * D;
    const size_t xw = std::max<size_t>(std::max(H, I), (size_t)Hq * D);
    const size_t wmax = std::max(std::max(Nqkv * H, (size_t)H * Hq * D), (size_t)2 * I * H);
    auto &A = c->allocs;
    CK(ctx, dalloc(A, &pf.wdq, wmax));
    CK(ctx, dalloc(A, &pf.x, P * xw));
    CK(ctx, dalloc(A, &pf.act, P * I));
    CK(ctx, dalloc(A, &pf.q, P * Hq * D));
    CK(ctx, dalloc(A, &pf.h, P * H));
    CK(ctx, dalloc(A, &pf.y, P * std::max(Nqkv, (size_t)H)));   // q|k|v, or the O / down output
    CK(ctx, dalloc(A, &pf.tok, P));
    CK(ctx, dalloc(A, &pf.trow, P));
    CK(ctx, dalloc(A, &pf.tpos, P));
    // attention: the longest query group whose heads fit one CTA's 64 query rows;
    // every key of a group in one split (prefill has many groups to spread)
    pf.qg = std::max(1, std::min(16, 64 / (Hq / Hkv)));
    pf.key_chunk = (c->max_len + 31) / 32 * 32;
    const int groups = (int)((P + pf.qg - 1) / pf.qg);
    const int qrows = attention_qrows(pf.qg, Hq, Hkv);
    pf.attn.items = attention_scratch_items(groups, Hkv, 1);
    CK(ctx, dalloc(A, &pf.attn.o, pf.attn.items * qrows * D));
    CK(ctx, dalloc(A, &pf.attn.ml, pf.attn.items * qrows * 2));
    pf.ready = true;
    return MLXCAT_OK;
}

// Prompt positions [s0, s0 + n) of `row` (tokens tok, on the device) through
// every layer with fp16 GEMMs on tcgen05 (gemm_tc.cu): each q4 weight is
// dequantised once per chunk, activations are row-major, the norms are exact
// (x = fp16(h * rstd * w)).  K/V of the positions land in the row's cache; with
// `logits` the last position's logits go to row 0 of c->logits.
int prefill_dense(mlxcat_cache *c, int row, const int32_t *tok, int s0, int n, bool logits) {
    mlxcat_ctx *ctx = c->ctx;
    const mlxcat_model_config &cf = ctx->cfg;
    auto &pf = c->pf;
    cudaStream_t st = ctx->stream;
    const int H = cf.hidden, I = cf.intermediate, D = cf.head_dim, Hq = cf.n_heads, Hkv = cf.n_kv_heads,
              L = cf.n_layers, sm = ctx->sm_count;
    const int Nqkv = (Hq + 2 * Hkv) * D;
    const float eps = cf.rms_eps;
    LK(ctx, prefill_rows(pf.trow, pf.tpos, row, s0, n, st));
    LK(ctx, prefill_embed(ctx->embed.view(), tok, n, pf.h, st));
    LK(ctx, prefill_rmsnorm(pf.h, n, H, ctx->attn_norm(0), eps, pf.x, st));
    for (int l = 0; l < L; ++l) {
        const KVLayer kv = c->layer(l);
        LK(ctx, dequant_q4(ctx->qkv[l].view(), pf.wdq, st));
        LK(ctx, gemm_tc(pf.wdq, Nqkv, H, pf.x, n, GEMM_STORE, pf.y, Nqkv, sm, c->err, st));
        LK(ctx, prefill_qkv(pf.y, n, Hq, Hkv, D, ctx->q_norm(l), ctx->k_norm(l), eps, c->rope, row, pf.tpos, pf.q,
                            kv, st));
        if (fa_prefill_supported(D)) {   // tensor-core flash attention; output reuses x (row-major [n][Hq*D])
            LK(ctx, fa_prefill(pf.q, DENSE_CHUNK, kv, c->rows, row, s0, n, Hq, Hkv, D, pf.x, c->err, st));
        } else {
            ctx->launches++;   // split-K attention is two kernels
            LK(ctx, attention(pf.q, kv, pf.trow, pf.tpos, n, pf.qg, Hq, Hkv, D, pf.key_chunk, 1, pf.attn, pf.x,
                              false, n, st, false));
        }
        LK(ctx, dequant_q4(ctx->o[l].view(), pf.wdq, st));
        LK(ctx, gemm_tc(pf.wdq, H, Hq * D, pf.x, n, GEMM_STORE, pf.y, H, sm, c->err, st));
        LK(ctx, prefill_add_rmsnorm(pf.h, pf.y, n, H, ctx->mlp_norm(l), eps, pf.x, st));
        LK(ctx, dequant_q4(ctx->gu[l].view(), pf.wdq, st));
        LK(ctx, gemm_tc(pf.wdq, 2 * I, H, pf.x, n, GEMM_SWIGLU, pf.act, I, sm, c->err, st));
        LK(ctx, dequant_q4(ctx->down[l].view(), pf.wdq, st));
        LK(ctx, gemm_tc(pf.wdq, H, I, pf.act, n, GEMM_STORE, pf.y, H, sm, c->err, st));
        LK(ctx, prefill_add_rmsnorm(pf.h, pf.y, n, H, l + 1 < L ? ctx->attn_norm(l + 1) : ctx->final_norm(), eps,
                                    pf.x, st));
    }
    if (logits) {   // the last position through the q4 head (one token: the GEMV-shaped kernel)
        LK(ctx, prefill_to_blocked(pf.x + (size_t)(n - 1) * H, H, c->xn, c->m_cap, st));
        const DevLin &head = cf.tie_embeddings ? ctx->embed : ctx->lm_head;
        Q4Epilogue e;
        e.part = c->part; e.counters = c->counters; e.err = c->err;
        e.op = Q4Epilogue::STORE; e.out = c->logits; e.ldo = cf.vocab;
        LK(ctx, q4_tc(head.tc(), c->xn, c->m_cap, 0, 1, sm, e, st));
    }
    return MLXCAT_OK;
}
}  // namespace

namespace {
// Admission of `row`: row state, then prefill of prompt positions [start, len)
// (positions below `start` are already in the cache: a prefix-cache import)
// and the first token from the last position's logits.
int admit_row(mlxcat_cache *c, int32_t row, const int32_t *prompt, int32_t len, int32_t start,
              int32_t max_new_tokens, const mlxcat_sampling *sp, int32_t *first_token) {
    mlxcat_ctx *ctx = c->ctx;
    if (row < 0 || row >= c->rows || !prompt || len < 1 || max_new_tokens < 1 || !sp)
        return set_err(ctx, MLXCAT_E_INVALID, "bad insert arguments");
    if ((int64_t)len + max_new_tokens + MLXCAT_MAX_PROPOSAL + 1 > c->max_len)
        return set_err(ctx, MLXCAT_E_INVALID, "prompt %d + max_new %d exceeds cache length %d", len,
                       max_new_tokens, c->max_len);
    if (sp->n_eos < 0 || sp->n_eos > MLXCAT_MAX_EOS) return set_err(ctx, MLXCAT_E_INVALID, "too many EOS ids");
    if (sp->temperature < 0.0f) return set_err(ctx, MLXCAT_E_INVALID, "negative temperature");
    for (int i = 0; i < len; ++i)
        if (prompt[i] < 0 || prompt[i] >= ctx->cfg.vocab) return set_err(ctx, MLXCAT_E_INVALID, "prompt token out of range");
    int rc = check_weights(c);
    if (rc) return rc;
    CK(ctx, cudaSetDevice(ctx->device));
    cudaStream_t st = ctx->stream;
    CK(ctx, cudaStreamSynchronize(st));
    // row state (host -> device)
    const int32_t zero = 0, one = 1;
    const int32_t eos_pad[MLXCAT_MAX_EOS] = {sp->eos[0], sp->eos[1], sp->eos[2], sp->eos[3],
                                             sp->eos[4], sp->eos[5], sp->eos[6], sp->eos[7]};
    CK(ctx, cudaMemcpy(c->hist + (size_t)row * c->hist_cap, prompt, sizeof(int32_t) * len, cudaMemcpyHostToDevice));
    CK(ctx, cudaMemcpy(c->hist_len + row, &len, 4, cudaMemcpyHostToDevice));
    CK(ctx, cudaMemcpy(c->kv_len + row, &len, 4, cudaMemcpyHostToDevice));
    CK(ctx, cudaMemcpy(c->n_gen + row, &zero, 4, cudaMemcpyHostToDevice));
    CK(ctx, cudaMemcpy(c->max_new + row, &max_new_tokens, 4, cudaMemcpyHostToDevice));
    CK(ctx, cudaMemcpy(c->active + row, &one, 4, cudaMemcpyHostToDevice));
    CK(ctx, cudaMemcpy(c->temperature + row, &sp->temperature, 4, cudaMemcpyHostToDevice));
    CK(ctx, cudaMemcpy(c->top_p + row, &sp->top_p, 4, cudaMemcpyHostToDevice));
    CK(ctx, cudaMemcpy(c->seed + row, &sp->seed, 8, cudaMemcpyHostToDevice));
    CK(ctx, cudaMemcpy(c->has_seed + row, &sp->has_seed, 4, cudaMemcpyHostToDevice));
    CK(ctx, cudaMemcpy(c->eos + (size_t)row * MLXCAT_MAX_EOS, eos_pad, sizeof eos_pad, cudaMemcpyHostToDevice));
    CK(ctx, cudaMemcpy(c->n_eos + row, &sp->n_eos, 4, cudaMemcpyHostToDevice));
    CK(ctx, cudaMemcpy(c->trigger + row, &sp->trigger, 4, cudaMemcpyHostToDevice));
    c->host_temp[row] = sp->temperature;
    // prefill in chunks; logits only for the last prompt token
    const bool dense = len - start >= DENSE_MIN && dense_prefill_ok(ctx);
    if (dense) {
        if ((rc = ensure_prefill(c))) return rc;
        for (int s0 = start; s0 < len; s0 += DENSE_CHUNK) {
            const int n = std::min(DENSE_CHUNK, len - s0);
            // stream-ordered after the previous chunk's kernels, which read the same buffer
            CK(ctx, cudaMemcpyAsync(c->pf.tok, prompt + s0, 4 * n, cudaMemcpyHostToDevice, st));
            if ((rc = prefill_dense(c, row, c->pf.tok, s0, n, s0 + n == len))) return rc;
        }
    }
    std::vector<int32_t> rr(PREFILL_CHUNK, row), pp(PREFILL_CHUNK);
    for (int s0 = dense ? len : start; s0 < len; s0 += PREFILL_CHUNK) {
        const int n = std::min(PREFILL_CHUNK, len - s0);
        for (int i = 0; i < n; ++i) pp[i] = s0 + i;
        CK(ctx, cudaMemcpyAsync(c->ptok, prompt + s0, 4 * n, cudaMemcpyHostToDevice, st));
        CK(ctx, cudaMemcpyAsync(c->trow, rr.data(), 4 * n, cudaMemcpyHostToDevice, st));
        CK(ctx, cudaMemcpyAsync(c->tpos, pp.data(), 4 * n, cudaMemcpyHostToDevice, st));
        const bool last = s0 + n == len;
        rc = forward(c, n, PREFILL_QG, c->ptok, c->trow, c->tpos, last ? n - 1 : n);
        if (rc) return rc;
        CK(ctx, cudaStreamSynchronize(st));   // host staging vectors are reused
    }
    LK(ctx, argmax_rows(c->logits, 1, ctx->cfg.vocab, c->amax, st, c->amax_part, c->amax_ctr));
    LK(ctx, sample_first(c->rs(), row, c->logits, ctx->cfg.vocab, c->amax, c->samp, c->first_tok, st));
    int32_t t0 = 0;
    CK(ctx, cudaMemcpyAsync(&t0, c->first_tok, 4, cudaMemcpyDeviceToHost, st));
    CK(ctx, cudaStreamSynchronize(st));
    if ((rc = device_err(c, false))) return rc;
    if (first_token) *first_token = t0;
    return MLXCAT_OK;
}
}  // namespace

// ===========================================================================
// C ABI
// ===========================================================================
extern "C" {

const char *mlxcat_last_error(const mlxcat_ctx *ctx) { return ctx ? ctx->err.c_str() : "null context"; }
const char *mlxcat_op_last_error(void) { return g_op_err.c_str(); }

int mlxcat_ctx_create(const mlxcat_model_config *cfg, int32_t device, mlxcat_ctx **out) {
    if (!cfg || !out) return op_err(MLXCAT_E_INVALID, "null argument");
    *out = nullptr;
    std::string why;
    if (!valid_config(cfg, why)) return op_err(MLXCAT_E_INVALID, "%s", why.c_str());
    int ndev = 0;
    cudaError_t e = cudaGetDeviceCount(&ndev);
    if (e != cudaSuccess || ndev == 0)
        return op_err(MLXCAT_E_CUDA, "no CUDA device: %s", cudaGetErrorString(e));
    if (device < 0 || device >= ndev) return op_err(MLXCAT_E_INVALID, "device %d out of range", device);
    mlxcat_ctx *ctx = new mlxcat_ctx();
    ctx->cfg = *cfg;
    ctx->gcfg = *cfg;
    ctx->device = device;
    if (cfg->kind == MLXCAT_MODEL_TRANSFORMER && cfg->n_experts > 0) {
        ctx->ep = cfg->ep_size > 1 ? cfg->ep_size : 1;
        ctx->ep_rank = ctx->ep > 1 ? cfg->ep_rank : 0;
        ctx->epr = cfg->n_experts / ctx->ep;
    }
    if (cfg->kind == MLXCAT_MODEL_TRANSFORMER && cfg->tp_size > 1) {
        // this rank's slice: whole KV heads with their query-head groups, a
        // contiguous block of MLP rows
        ctx->tp = cfg->tp_size;
        ctx->tp_rank = cfg->tp_rank;
        ctx->cfg.n_heads = cfg->n_heads / ctx->tp;
        ctx->cfg.n_kv_heads = cfg->n_kv_heads / ctx->tp;
        ctx->cfg.intermediate = cfg->intermediate / ctx->tp;
        ctx->cfg.tp_size = 1;
        ctx->cfg.tp_rank = 0;
        std::string lwhy;
        if (!valid_config(&ctx->cfg, lwhy)) {
            delete ctx;
            return op_err(MLXCAT_E_INVALID, "per-rank slice: %s", lwhy.c_str());
        }
    }
    auto fail = [&](int code) {
        g_op_err = ctx->err;
        mlxcat_ctx_destroy(ctx);
        return code;
    };
    if (cudaSetDevice(device) != cudaSuccess) { set_err(ctx, MLXCAT_E_CUDA, "cudaSetDevice failed"); return fail(MLXCAT_E_CUDA); }
    cudaDeviceGetAttribute(&ctx->sm_count, cudaDevAttrMultiProcessorCount, device);
    if (cudaStreamCreateWithFlags(&ctx->stream, cudaStreamNonBlocking) != cudaSuccess) {
        set_err(ctx, MLXCAT_E_CUDA, "stream creation failed");
        return fail(MLXCAT_E_CUDA);
    }
    const mlxcat_model_config &c = ctx->cfg;   // this rank's view (the slice when tensor-parallel)
    int rc = MLXCAT_OK;
    auto alloc_lin = [&](DevLin &w, int N, int K) {
        w.N = N; w.K = K;
        if (dalloc(ctx->allocs, &w.wq, (size_t)N * K / 8) != cudaSuccess ||
            dalloc(ctx->allocs, &w.s, (size_t)N * K / 64) != cudaSuccess ||
            dalloc(ctx->allocs, &w.b, (size_t)N * K / 64) != cudaSuccess ||
            dalloc(ctx->allocs, &w.sbp, q4_sbp_words(N, K)) != cudaSuccess)
            rc = set_err(ctx, MLXCAT_E_OOM, "weight allocation failed (%d x %d)", N, K);
        else if (!w.build_map())
            rc = set_err(ctx, MLXCAT_E_CUDA, "TMA descriptor for a %d x %d weight failed", N, K);
    };
    if (c.kind == MLXCAT_MODEL_TABLE) {
        if (dalloc(ctx->allocs, &ctx->table, (size_t)c.vocab) != cudaSuccess)
            rc = set_err(ctx, MLXCAT_E_OOM, "table allocation failed");
    } else {
        const int H = c.hidden, D = c.head_dim, L = c.n_layers;
        alloc_lin(ctx->embed, c.vocab, H);
        if (!c.tie_embeddings) alloc_lin(ctx->lm_head, c.vocab, H);
        ctx->qkv.resize(L); ctx->o.resize(L);
        if (c.n_experts) ctx->moe.resize(L);
        else { ctx->gu.resize(L); ctx->down.resize(L); }
        for (int l = 0; l < L && rc == MLXCAT_OK; ++l) {
            alloc_lin(ctx->qkv[l], (c.n_heads + 2 * c.n_kv_heads) * D, H);
            alloc_lin(ctx->o[l], H, c.n_heads * D);
            if (c.n_experts) {
                auto &mb = ctx->moe[l];
                const size_t n = (size_t)ctx->epr * c.intermediate * H;   // this rank's experts, per projection
                bool ok = dalloc(ctx->allocs, &mb.router, (size_t)c.n_experts * H) == cudaSuccess;
                for (int p = 0; p < 3 && ok; ++p)
                    ok = dalloc(ctx->allocs, &mb.wq[p], n / 8) == cudaSuccess &&
                         dalloc(ctx->allocs, &mb.s[p], n / 64) == cudaSuccess &&
                         dalloc(ctx->allocs, &mb.b[p], n / 64) == cudaSuccess;
                if (!ok) rc = set_err(ctx, MLXCAT_E_OOM, "expert weight allocation failed (layer %d)", l);
            } else {
                alloc_lin(ctx->gu[l], 2 * c.intermediate, H);
                alloc_lin(ctx->down[l], H, c.intermediate);
            }
        }
        const size_t nn = (size_t)(2 * L + 1) * H + (size_t)2 * L * D;
        if (rc == MLXCAT_OK && dalloc(ctx->allocs, &ctx->norms, nn) != cudaSuccess)
            rc = set_err(ctx, MLXCAT_E_OOM, "norm allocation failed");
        if (rc == MLXCAT_OK && dalloc(ctx->allocs, &ctx->inv_freq, (size_t)D / 2) != cudaSuccess)
            rc = set_err(ctx, MLXCAT_E_OOM, "rope table allocation failed");
        if (rc == MLXCAT_OK) {
            // RMSNorm weights: ones (random-init checkpoints carry unit norms)
            std::vector<float> ones(nn, 1.0f);
            std::vector<float> inv(D / 2);
            for (int i = 0; i < D / 2; ++i)
                inv[i] = (float)(1.0 / pow((double)c.rope_theta, (2.0 * i) / (double)D));
            if (cudaMemcpy(ctx->norms, ones.data(), nn * 4, cudaMemcpyHostToDevice) != cudaSuccess ||
                cudaMemcpy(ctx->inv_freq, inv.data(), inv.size() * 4, cudaMemcpyHostToDevice) != cudaSuccess)
                rc = set_err(ctx, MLXCAT_E_CUDA, "norm / rope upload failed");
        }
    }
    if (rc != MLXCAT_OK) return fail(rc);
    *out = ctx;
    return MLXCAT_OK;
}

int mlxcat_tp_unique_id(uint8_t id[128]) {
    if (!id) return op_err(MLXCAT_E_INVALID, "null id buffer");
    if (const char *e = tp_unique_id(id)) return op_err(MLXCAT_E_STATE, "tensor parallel id: %s", e);
    return MLXCAT_OK;
}

int mlxcat_ctx_tp_connect(mlxcat_ctx *ctx, const uint8_t id[128]) {
    if (!ctx || !id) return MLXCAT_E_INVALID;
    if (ctx->ep > 1)
        return set_err(ctx, MLXCAT_E_STATE, "expert-parallel contexts connect their caches (mlxcat_cache_ep_connect)");
    if (ctx->tp <= 1) return set_err(ctx, MLXCAT_E_STATE, "context is not tensor-parallel");
    if (ctx->nccl) return set_err(ctx, MLXCAT_E_STATE, "context already connected");
    CK(ctx, cudaSetDevice(ctx->device));
    if (const char *e = tp_connect(&ctx->nccl, id, ctx->tp, ctx->tp_rank))
        return set_err(ctx, MLXCAT_E_STATE, "tensor parallel connect: %s", e);
    return MLXCAT_OK;
}

int mlxcat_ctx_destroy(mlxcat_ctx *ctx) {
    if (!ctx) return MLXCAT_OK;
    // caches hold the context's stream and buffers: they go first
    while (!ctx->caches.empty()) mlxcat_cache_destroy(ctx->caches.back());
    cudaSetDevice(ctx->device);
    if (ctx->stream) cudaStreamSynchronize(ctx->stream);
    tp_destroy(ctx->nccl);
    for (void *p : ctx->allocs) cudaFree(p);
    if (ctx->stream) cudaStreamDestroy(ctx->stream);
    delete ctx;
    return MLXCAT_OK;
}

int mlxcat_ctx_stream(mlxcat_ctx *ctx, void **stream) {
    if (!ctx || !stream) return MLXCAT_E_INVALID;
    *stream = (void *)ctx->stream;
    return MLXCAT_OK;
}

int mlxcat_ctx_synchronize(mlxcat_ctx *ctx) {
    if (!ctx) return MLXCAT_E_INVALID;
    CK(ctx, cudaStreamSynchronize(ctx->stream));
    return MLXCAT_OK;
}

int64_t mlxcat_ctx_launch_count(const mlxcat_ctx *ctx) { return ctx ? ctx->launches : -1; }

// A MoE expert tensor (MLXCAT_TENSOR_EXPERT ids) as a non-owning view into its
// layer's expert bank.
static bool expert_view(mlxcat_ctx *ctx, uint32_t id, DevLin *v, RowMap *rm) {
    const mlxcat_model_config &c = ctx->cfg;
    if (c.kind != MLXCAT_MODEL_TRANSFORMER || !c.n_experts || (id & 0xC0000000u) != 0x40000000u) return false;
    const int l = (int)((id >> 12) & 0x3FFFFu), eg = (int)((id >> 2) & 0x3FFu), kind = (int)(id & 3u);
    if (l >= c.n_layers || eg >= c.n_experts || kind > 2) return false;
    const int e = eg - ctx->ep_rank * ctx->epr;   // this rank's bank holds experts [ep_rank*epr, +epr)
    if (e < 0 || e >= ctx->epr) return false;
    const auto &mb = ctx->moe[l];
    const size_t per = (size_t)c.intermediate * c.hidden;   // weights of one expert projection
    *rm = RowMap();
    *v = DevLin();
    v->wq = mb.wq[kind] + (size_t)e * per / 8;
    v->s = mb.s[kind] + (size_t)e * per / 64;
    v->b = mb.b[kind] + (size_t)e * per / 64;
    v->N = kind < 2 ? c.intermediate : c.hidden;
    v->K = kind < 2 ? c.hidden : c.intermediate;
    rm->rows = v->N;
    return true;
}

static DevLin *lin_for(mlxcat_ctx *ctx, uint32_t id, RowMap *rm) {
    const mlxcat_model_config &c = ctx->cfg;
    if (c.kind != MLXCAT_MODEL_TRANSFORMER) return nullptr;
    if ((id & 0xC0000000u) == 0x40000000u) return nullptr;
    *rm = RowMap();
    if (id == 0xFFFF0000u) { rm->rows = c.vocab; return &ctx->embed; }
    if (id == 0xFFFF0001u) {
        if (c.tie_embeddings) return nullptr;
        rm->rows = c.vocab; return &ctx->lm_head;
    }
    const int l = (int)(id / 16u), kind = (int)(id % 16u);
    if (l >= c.n_layers) return nullptr;
    const int D = c.head_dim, qd = c.n_heads * D, kvd = c.n_kv_heads * D;
    switch (kind) {
    case 0: rm->rows = qd; return &ctx->qkv[l];
    case 1: rm->offset = qd; rm->rows = kvd; return &ctx->qkv[l];
    case 2: rm->offset = qd + kvd; rm->rows = kvd; return &ctx->qkv[l];
    case 3: rm->rows = c.hidden; return &ctx->o[l];
    }
    if (c.n_experts) return nullptr;   // MoE layers have no dense MLP
    switch (kind) {
    case 4: rm->group = 64; rm->stride = 128; rm->rows = c.intermediate; return &ctx->gu[l];
    case 5: rm->group = 64; rm->stride = 128; rm->offset = 64; rm->rows = c.intermediate; return &ctx->gu[l];
    case 6: rm->rows = c.hidden; return &ctx->down[l];
    default: return nullptr;
    }
}

// copy `rows` logical rows between a host tensor and their placement in a fused matrix
static cudaError_t copy_rows(const DevLin *w, const RowMap &rm, void *host_wq, void *host_s, void *host_b,
                             bool to_device) {
    const size_t wb = (size_t)w->K / 2, sb = (size_t)w->K / 64 * 2;
    const int run = rm.group ? rm.group : rm.rows;
    for (int n0 = 0; n0 < rm.rows; n0 += run) {
        const int cnt = std::min(run, rm.rows - n0);
        const size_t dr = (size_t)rm.row(n0);
        char *dw = reinterpret_cast<char *>(w->wq) + dr * wb, *hw = static_cast<char *>(host_wq) + n0 * wb;
        char *ds = reinterpret_cast<char *>(w->s) + dr * sb, *hs = static_cast<char *>(host_s) + n0 * sb;
        char *db = reinterpret_cast<char *>(w->b) + dr * sb, *hb = static_cast<char *>(host_b) + n0 * sb;
        cudaError_t e;
        if (to_device) {
            if ((e = cudaMemcpy(dw, hw, cnt * wb, cudaMemcpyHostToDevice)) != cudaSuccess) return e;
            if ((e = cudaMemcpy(ds, hs, cnt * sb, cudaMemcpyHostToDevice)) != cudaSuccess) return e;
            if ((e = cudaMemcpy(db, hb, cnt * sb, cudaMemcpyHostToDevice)) != cudaSuccess) return e;
        } else {
            if (host_wq && (e = cudaMemcpy(hw, dw, cnt * wb, cudaMemcpyDeviceToHost)) != cudaSuccess) return e;
            if (host_s && (e = cudaMemcpy(hs, ds, cnt * sb, cudaMemcpyDeviceToHost)) != cudaSuccess) return e;
            if (host_b && (e = cudaMemcpy(hb, db, cnt * sb, cudaMemcpyDeviceToHost)) != cudaSuccess) return e;
        }
    }
    return cudaSuccess;
}

int mlxcat_weights_synth(mlxcat_ctx *ctx, uint64_t seed, float stddev) {
    if (!ctx) return MLXCAT_E_INVALID;
    const mlxcat_model_config &c = ctx->cfg;
    if (c.kind != MLXCAT_MODEL_TRANSFORMER) return set_err(ctx, MLXCAT_E_INVALID, "synth needs a transformer model");
    CK(ctx, cudaSetDevice(ctx->device));
    std::vector<uint32_t> ids = {0xFFFF0000u};
    if (!c.tie_embeddings) ids.push_back(0xFFFF0001u);
    for (int l = 0; l < c.n_layers; ++l)
        for (int k = 0; k < (c.n_experts ? 4 : 7); ++k) ids.push_back((uint32_t)l * 16u + (uint32_t)k);
    for (int l = 0; l < c.n_layers && c.n_experts; ++l) {
        LK(ctx, router_synth(seed, (uint32_t)l * 16u + 7u, stddev, c.n_experts, c.hidden, ctx->moe[l].router,
                             ctx->stream));
        for (int e = ctx->ep_rank * ctx->epr; e < (ctx->ep_rank + 1) * ctx->epr; ++e)
            for (int kind = 0; kind < 3; ++kind) {
                const uint32_t id = MLXCAT_TENSOR_EXPERT(l, e, kind);
                DevLin v;
                RowMap rm;
                expert_view(ctx, id, &v, &rm);
                LK(ctx, synth_q4(seed, id, stddev, rm.rows, v.K, v.wq, v.s, v.b, rm.offset, ctx->stream,
                                 rm.group, rm.stride));
            }
    }
    for (uint32_t id : ids) {
        RowMap rm;
        DevLin *w = lin_for(ctx, id, &rm);
        // tensor parallel: this rank's rows (q, k, v, gate, up) or columns (o, down)
        // of the full tensor, drawn from the full tensor's weight stream
        int row_base = 0, col_base = 0, k_total = 0;
        if (ctx->tp > 1 && id < 0xFFFF0000u) {
            const int kind = (int)(id % 16u), r = ctx->tp_rank, D = c.head_dim;
            switch (kind) {
            case 0: row_base = r * c.n_heads * D; break;
            case 1: case 2: row_base = r * c.n_kv_heads * D; break;
            case 3: col_base = r * c.n_heads * D; k_total = ctx->gcfg.n_heads * D; break;
            case 4: case 5: row_base = r * c.intermediate; break;
            case 6: col_base = r * c.intermediate; k_total = ctx->gcfg.intermediate; break;
            default: break;
            }
        }
        LK(ctx, synth_q4(seed, id, stddev, rm.rows, w->K, w->wq, w->s, w->b, rm.offset, ctx->stream,
                         rm.group, rm.stride, row_base, col_base, k_total));
    }
    for (uint32_t id : ids) {   // fused matrices are packed once per distinct buffer (repeats are harmless)
        RowMap rm;
        DevLin *w = lin_for(ctx, id, &rm);
        LK(ctx, pack_q4_sb(w->s, w->b, w->N, w->K, w->sbp, ctx->stream));
    }
    CK(ctx, cudaStreamSynchronize(ctx->stream));
    ctx->have_weights = true;
    return MLXCAT_OK;
}

int mlxcat_weights_set_q4(mlxcat_ctx *ctx, uint32_t id, const uint32_t *wq, const uint16_t *scales,
                          const uint16_t *biases) {
    if (!ctx || !wq || !scales || !biases) return MLXCAT_E_INVALID;
    RowMap rm;
    DevLin ev;
    if (expert_view(ctx, id, &ev, &rm)) {
        CK(ctx, cudaSetDevice(ctx->device));
        CK(ctx, copy_rows(&ev, rm, const_cast<uint32_t *>(wq), const_cast<uint16_t *>(scales),
                          const_cast<uint16_t *>(biases), true));
        ctx->have_weights = true;
        return MLXCAT_OK;
    }
    DevLin *w = lin_for(ctx, id, &rm);
    if (!w) return set_err(ctx, MLXCAT_E_INVALID, "unknown tensor id 0x%x", id);
    CK(ctx, cudaSetDevice(ctx->device));
    CK(ctx, copy_rows(w, rm, const_cast<uint32_t *>(wq), const_cast<uint16_t *>(scales),
                      const_cast<uint16_t *>(biases), true));
    CK(ctx, pack_q4_sb(w->s, w->b, w->N, w->K, w->sbp, ctx->stream));
    CK(ctx, cudaStreamSynchronize(ctx->stream));
    ctx->have_weights = true;
    return MLXCAT_OK;
}

int mlxcat_weights_get_q4(mlxcat_ctx *ctx, uint32_t id, uint32_t *wq, uint16_t *scales, uint16_t *biases) {
    if (!ctx) return MLXCAT_E_INVALID;
    RowMap rm;
    DevLin ev;
    DevLin *w = expert_view(ctx, id, &ev, &rm) ? &ev : lin_for(ctx, id, &rm);
    if (!w) return set_err(ctx, MLXCAT_E_INVALID, "unknown tensor id 0x%x", id);
    CK(ctx, cudaSetDevice(ctx->device));
    CK(ctx, cudaStreamSynchronize(ctx->stream));
    CK(ctx, copy_rows(w, rm, wq, scales, biases, false));
    return MLXCAT_OK;
}

static __nv_bfloat16 *bf16_for(mlxcat_ctx *ctx, uint32_t id, size_t *n) {
    const mlxcat_model_config &c = ctx->cfg;
    if (c.kind != MLXCAT_MODEL_TRANSFORMER || !c.n_experts || id % 16u != 7u || (int)(id / 16u) >= c.n_layers)
        return nullptr;
    *n = (size_t)c.n_experts * c.hidden;
    return ctx->moe[id / 16u].router;
}

int mlxcat_weights_set_bf16(mlxcat_ctx *ctx, uint32_t id, const uint16_t *w) {
    if (!ctx || !w) return MLXCAT_E_INVALID;
    size_t n = 0;
    __nv_bfloat16 *d = bf16_for(ctx, id, &n);
    if (!d) return set_err(ctx, MLXCAT_E_INVALID, "unknown bf16 tensor id 0x%x", id);
    CK(ctx, cudaSetDevice(ctx->device));
    CK(ctx, cudaMemcpy(d, w, n * 2, cudaMemcpyHostToDevice));
    return MLXCAT_OK;
}

int mlxcat_weights_get_bf16(mlxcat_ctx *ctx, uint32_t id, uint16_t *w) {
    if (!ctx || !w) return MLXCAT_E_INVALID;
    size_t n = 0;
    __nv_bfloat16 *d = bf16_for(ctx, id, &n);
    if (!d) return set_err(ctx, MLXCAT_E_INVALID, "unknown bf16 tensor id 0x%x", id);
    CK(ctx, cudaSetDevice(ctx->device));
    CK(ctx, cudaStreamSynchronize(ctx->stream));
    CK(ctx, cudaMemcpy(w, d, n * 2, cudaMemcpyDeviceToHost));
    return MLXCAT_OK;
}

int mlxcat_weights_set_norm(mlxcat_ctx *ctx, uint32_t id, const float *w) {
    if (!ctx || !w) return MLXCAT_E_INVALID;
    const mlxcat_model_config &c = ctx->cfg;
    if (c.kind != MLXCAT_MODEL_TRANSFORMER || !ctx->norms) return set_err(ctx, MLXCAT_E_STATE, "model has no norms");
    const float *dst = nullptr;
    int n = c.hidden;
    const int l = (int)(id / 16u), kind = (int)(id % 16u);
    if (id == MLXCAT_NORM_FINAL) dst = ctx->final_norm();
    else if (id < 0x40000000u && l < c.n_layers && kind == 8) dst = ctx->attn_norm(l);
    else if (id < 0x40000000u && l < c.n_layers && kind == 9) dst = ctx->mlp_norm(l);
    else if (id < 0x40000000u && l < c.n_layers && kind == 10 && c.qk_norm) { dst = ctx->q_norm(l); n = c.head_dim; }
    else if (id < 0x40000000u && l < c.n_layers && kind == 11 && c.qk_norm) { dst = ctx->k_norm(l); n = c.head_dim; }
    if (!dst) return set_err(ctx, MLXCAT_E_INVALID, "unknown norm id 0x%x", id);
    CK(ctx, cudaSetDevice(ctx->device));
    CK(ctx, cudaStreamSynchronize(ctx->stream));
    CK(ctx, cudaMemcpy(const_cast<float *>(dst), w, sizeof(float) * n, cudaMemcpyHostToDevice));
    for (mlxcat_cache *cc : ctx->caches) drop_graph(cc);
    return MLXCAT_OK;
}

int mlxcat_weights_set_table(mlxcat_ctx *ctx, const int32_t *next, int32_t vocab) {
    if (!ctx || !next) return MLXCAT_E_INVALID;
    if (ctx->cfg.kind != MLXCAT_MODEL_TABLE || vocab != ctx->cfg.vocab)
        return set_err(ctx, MLXCAT_E_INVALID, "table model of vocab %d expected", ctx->cfg.vocab);
    for (int i = 0; i < vocab; ++i)
        if (next[i] < 0 || next[i] >= vocab) return set_err(ctx, MLXCAT_E_INVALID, "table entry out of range");
    CK(ctx, cudaSetDevice(ctx->device));
    CK(ctx, cudaMemcpy(ctx->table, next, sizeof(int32_t) * vocab, cudaMemcpyHostToDevice));
    ctx->have_weights = true;
    return MLXCAT_OK;
}

int64_t mlxcat_weights_bytes(const mlxcat_ctx *ctx) {
    if (!ctx || ctx->cfg.kind != MLXCAT_MODEL_TRANSFORMER) return 0;
    size_t b = ctx->cfg.tie_embeddings ? ctx->embed.bytes() : ctx->lm_head.bytes();
    const mlxcat_model_config &c = ctx->cfg;
    for (int l = 0; l < c.n_layers; ++l) {
        b += ctx->qkv[l].bytes() + ctx->o[l].bytes();
        if (c.n_experts)   // every (local) expert is touched by a verify step's assignments; router replicated
            b += (size_t)ctx->epr * 3 * ((size_t)c.intermediate * c.hidden / 2 +
                                         (size_t)c.intermediate * c.hidden / 64 * 4) +
                 (size_t)c.n_experts * c.hidden * 2;
        else
            b += ctx->gu[l].bytes() + ctx->down[l].bytes();
    }
    return (int64_t)b;
}

int mlxcat_cache_create(mlxcat_ctx *ctx, int32_t max_rows, int32_t max_len, mlxcat_cache **out) {
    if (!ctx || !out || max_rows <= 0 || max_len <= MLXCAT_MAX_PROPOSAL + 2)
        return set_err(ctx, MLXCAT_E_INVALID, "bad cache shape");
    *out = nullptr;
    CK(ctx, cudaSetDevice(ctx->device));
    const mlxcat_model_config &cf = ctx->cfg;
    mlxcat_cache *c = new mlxcat_cache();
    c->ctx = ctx;
    c->rows = max_rows;
    c->max_len = max_len;
    c->hist_cap = max_len + 1;
    c->host_temp.assign(max_rows, 0.0f);
    auto &A = c->allocs;
    int rc = MLXCAT_OK;
    auto chk = [&](cudaError_t e) {
        if (e != cudaSuccess && rc == MLXCAT_OK)
            rc = set_err(ctx, e == cudaErrorMemoryAllocation ? MLXCAT_E_OOM : MLXCAT_E_CUDA,
                         "cache allocation: %s", cudaGetErrorString(e));
    };
    const bool tr = cf.kind == MLXCAT_MODEL_TRANSFORMER;
    const int R = max_rows;
    c->m_cap = std::max(R * (MLXCAT_MAX_PROPOSAL + 1), PREFILL_CHUNK);
    const int Mc = c->m_cap;
    if (tr) {
        const size_t kvn = (size_t)cf.n_layers * R * cf.n_kv_heads * max_len * cf.head_dim;
        chk(dalloc(A, &c->k, kvn));
        chk(dalloc(A, &c->v, kvn));
    }
    chk(dalloc(A, &c->hist, (size_t)R * c->hist_cap));
    chk(dalloc(A, &c->hist_len, R)); chk(dalloc(A, &c->kv_len, R)); chk(dalloc(A, &c->n_gen, R));
    chk(dalloc(A, &c->max_new, R)); chk(dalloc(A, &c->active, R)); chk(dalloc(A, &c->has_seed, R));
    chk(dalloc(A, &c->eos, (size_t)R * MLXCAT_MAX_EOS)); chk(dalloc(A, &c->n_eos, R));
    chk(dalloc(A, &c->trigger, R)); chk(dalloc(A, &c->temperature, R)); chk(dalloc(A, &c->top_p, R));
    chk(dalloc(A, &c->seed, R));
    chk(dalloc(A, &c->vtok, Mc)); chk(dalloc(A, &c->count, R)); chk(dalloc(A, &c->trow, Mc));
    chk(dalloc(A, &c->tpos, Mc)); chk(dalloc(A, &c->amax, Mc)); chk(dalloc(A, &c->out_tok, Mc));
    chk(dalloc(A, &c->out_n, R)); chk(dalloc(A, &c->out_fin, R)); chk(dalloc(A, &c->first_tok, 1));
    chk(dalloc(A, &c->ptok, Mc)); chk(dalloc(A, &c->stats, 4));
    chk(dalloc(A, &c->amax_part, argmax_scratch_words(Mc))); chk(dalloc(A, &c->amax_ctr, Mc));
    if (rc == MLXCAT_OK) chk(cudaMemset(c->amax_ctr, 0, sizeof(unsigned) * Mc));
    chk(dalloc(A, &c->logits, (size_t)Mc * cf.vocab));
    const int KS = Mc;   // sampling scratch slots (rows*(k+1))
    chk(dalloc(A, &c->samp.m, KS)); chk(dalloc(A, &c->samp.thr, KS));
    chk(dalloc(A, &c->samp.S, KS)); chk(dalloc(A, &c->samp.Pd, KS));
    if (tr) {
        const int H = cf.hidden, I = cf.intermediate, D = cf.head_dim;
        const int Hq = cf.n_heads, Hkv = cf.n_kv_heads;
        const int xw = std::max(std::max(H, I), Hq * D);
        chk(dalloc(A, &c->h, (size_t)Mc * H));
        chk(dalloc(A, &c->xn, (size_t)Mc * xw));
        chk(dalloc(A, &c->xa, (size_t)Mc * I));
        chk(dalloc(A, &c->xg, (size_t)Mc * H));
        chk(dalloc(A, &c->norm_part, (size_t)Mc * ((H + 127) / 128)));
        chk(dalloc(A, &c->r_attn, (size_t)Mc));
        chk(dalloc(A, &c->r_mlp, (size_t)Mc));
        chk(dalloc(A, &c->qbuf, (size_t)Mc * Hq * D));
        if (ctx->tp > 1) {
            chk(dalloc(A, &c->tp_part, (size_t)Mc * H));
            c->peer_kind = 2;
            c->peer_cap = Mc;
            c->tpx_lay = tpx_layout(ctx->tp, Mc, H);
            c->peer_bytes = c->tpx_lay.total;
        }
        if (cf.n_experts) {
            const size_t asg = (size_t)Mc * cf.top_k;
            chk(dalloc(A, &c->moe_id, asg * cf.n_layers));
            chk(dalloc(A, &c->moe_w, asg * cf.n_layers));
            chk(dalloc(A, &c->moe_scale, (size_t)Mc));
            chk(dalloc(A, &c->moe_list, (size_t)cf.n_experts * Mc));
            chk(dalloc(A, &c->moe_count, (size_t)cf.n_layers * cf.n_experts));
            chk(dalloc(A, &c->moe_act, asg * I));
            chk(dalloc(A, &c->moe_y, asg * H));
            chk(dalloc(A, &c->moe_logits, (size_t)Mc * cf.n_experts));
            if (ctx->ep > 1) {
                // per (source, owner) capacity: all of a rank's assignments of one forward
                const int N = ctx->ep;
                c->peer_kind = 1;
                c->peer_cap = (int)asg;
                c->ep_lay = ep_layout(N, c->peer_cap, H);
                c->peer_bytes = c->ep_lay.total;
                const size_t rows = (size_t)N * c->peer_cap;
                chk(dalloc(A, &c->ep_lcount, (size_t)N));
                if (rc == MLXCAT_OK) chk(cudaMemset(c->ep_lcount, 0, sizeof(int) * N));
                chk(dalloc(A, &c->ep_act, rows * I));
                chk(dalloc(A, &c->ep_exp_count, (size_t)cf.n_layers * ctx->epr));
                chk(dalloc(A, &c->ep_exp_list, (size_t)ctx->epr * rows));
                chk(dalloc(A, &c->ep_scale, rows));
                chk(dalloc(A, &c->ep_w, rows));
                chk(dalloc(A, &c->ep_ys, rows * H));
            }
        }
        if (c->peer_kind) {   // the exported region is its own allocation (mapped whole by the peers)
            const int N = c->peer_kind == 1 ? ctx->ep : ctx->tp;
            chk(dalloc(A, &c->peer_region, c->peer_bytes));
            if (rc == MLXCAT_OK) chk(cudaMemset(c->peer_region, 0, c->peer_bytes));
            chk(dalloc(A, &c->peer_tab, (size_t)N));
            chk(dalloc(A, &c->peer_epoch, 1));
            chk(dalloc(A, &c->peer_done, 1));
            chk(dalloc(A, &c->peer_sig, 1));
            if (rc == MLXCAT_OK) chk(cudaMemset(c->peer_epoch, 0, sizeof(unsigned)));
            if (rc == MLXCAT_OK) chk(cudaMemset(c->peer_done, 0, sizeof(unsigned)));
            if (rc == MLXCAT_OK) chk(cudaMemset(c->peer_sig, 0, sizeof(unsigned)));
        }
        chk(dalloc(A, &c->rope, (size_t)max_len * (D / 2)));
        if (rc == MLXCAT_OK) chk(rope_table(ctx->inv_freq, D / 2, max_len, c->rope, ctx->stream));
        if (rc == MLXCAT_OK) chk(cudaStreamSynchronize(ctx->stream));
        // split-K partials and tickets: max over the linears and every token count
        size_t pf = 0, nc = 0;
        const int NK[5][2] = {{(Hq + 2 * Hkv) * D, H}, {H, Hq * D}, {2 * I, H}, {H, I}, {cf.vocab, H}};
        for (int m = 1; m <= Mc; ++m)
            for (auto &nk : NK) {
                pf = std::max(pf, q4_tc_partial_floats(nk[0], nk[1], m, ctx->sm_count));
                nc = std::max(nc, q4_tc_counters(nk[0], m));
            }
        c->part_floats = pf;
        chk(dalloc(A, &c->part, pf));
        chk(dalloc(A, &c->counters, nc));
        if (rc == MLXCAT_OK) chk(cudaMemset(c->counters, 0, nc * sizeof(unsigned)));
        // attention scratch
        c->key_chunk = cache_key_chunk(R, Hkv, max_len, ctx->sm_count);
        c->attn_splits = attention_max_splits(max_len, c->key_chunk);
        int groups = std::max(R, (PREFILL_CHUNK + PREFILL_QG - 1) / PREFILL_QG);
        int qrows = 16;
        for (int k = 0; k <= MLXCAT_MAX_PROPOSAL; ++k) qrows = std::max(qrows, attention_qrows(k + 1, Hq, Hkv));
        qrows = std::max(qrows, attention_qrows(PREFILL_QG, Hq, Hkv));
        groups = std::max(groups, R);
        const size_t items = attention_scratch_items(groups, Hkv, c->attn_splits);
        c->attn.items = items;
        chk(dalloc(A, &c->attn.o, items * qrows * D));
        chk(dalloc(A, &c->attn.ml, items * qrows * 2));
    }
    chk(cudaMallocHost((void **)&c->h_tok, sizeof(int32_t) * Mc));
    chk(cudaMallocHost((void **)&c->h_n, sizeof(int32_t) * R));
    chk(cudaMallocHost((void **)&c->h_fin, sizeof(int32_t) * R));
    chk(cudaMallocHost((void **)&c->h_stats, sizeof(unsigned long long) * 4));
    chk(cudaMallocHost((void **)&c->h_err, sizeof(int32_t)));
    chk(dalloc(A, &c->err, 1));
    if (rc == MLXCAT_OK) chk(cudaMemset(c->err, 0, sizeof(int)));
    chk(cudaEventCreate(&c->ev0));
    chk(cudaEventCreate(&c->ev1));
    chk(cudaEventCreate(&c->es0));
    chk(cudaEventCreate(&c->es1));
    if (rc == MLXCAT_OK) {
        chk(cudaMemset(c->active, 0, sizeof(int32_t) * R));
        chk(cudaMemset(c->hist_len, 0, sizeof(int32_t) * R));
        chk(cudaMemset(c->kv_len, 0, sizeof(int32_t) * R));
        chk(cudaMemset(c->n_gen, 0, sizeof(int32_t) * R));
        chk(cudaMemset(c->max_new, 0, sizeof(int32_t) * R));
        chk(cudaMemset(c->temperature, 0, sizeof(float) * R));
        chk(cudaMemset(c->top_p, 0, sizeof(float) * R));
        chk(cudaMemset(c->has_seed, 0, sizeof(int32_t) * R));
        chk(cudaMemset(c->n_eos, 0, sizeof(int32_t) * R));
        chk(cudaMemset(c->seed, 0, sizeof(uint64_t) * R));
        chk(cudaMemset(c->stats, 0, sizeof(unsigned long long) * 4));
        std::vector<int32_t> neg(R, -1);
        chk(cudaMemcpy(c->trigger, neg.data(), sizeof(int32_t) * R, cudaMemcpyHostToDevice));
    }
    if (rc != MLXCAT_OK) {
        mlxcat_cache_destroy(c);
        return rc;
    }
    ctx->caches.push_back(c);
    *out = c;
    return MLXCAT_OK;
}

int mlxcat_cache_destroy(mlxcat_cache *c) {
    if (!c) return MLXCAT_OK;
    auto &live = c->ctx->caches;
    live.erase(std::remove(live.begin(), live.end(), c), live.end());
    cudaSetDevice(c->ctx->device);
    cudaStreamSynchronize(c->ctx->stream);
    drop_graph(c);
    for (char *p : c->peer_opened) cudaIpcCloseMemHandle(p);
    for (void *p : c->allocs) cudaFree(p);
    if (c->h_tok) cudaFreeHost(c->h_tok);
    if (c->h_n) cudaFreeHost(c->h_n);
    if (c->h_fin) cudaFreeHost(c->h_fin);
    if (c->h_stats) cudaFreeHost(c->h_stats);
    if (c->h_err) cudaFreeHost(c->h_err);
    if (c->ev0) cudaEventDestroy(c->ev0);
    if (c->ev1) cudaEventDestroy(c->ev1);
    if (c->es0) cudaEventDestroy(c->es0);
    if (c->es1) cudaEventDestroy(c->es1);
    for (cudaEvent_t e : c->prof_ev) cudaEventDestroy(e);
    delete c;
    return MLXCAT_OK;
}

int mlxcat_cache_set_token_masks(mlxcat_cache *c, int32_t k, const uint32_t *bits, const uint8_t *enabled) {
    if (!c) return MLXCAT_E_INVALID;
    mlxcat_ctx *ctx = c->ctx;
    if (!enabled) {   // clear
        c->mask_k = -1;
        return MLXCAT_OK;
    }
    if (k < 0 || k > MLXCAT_MAX_PROPOSAL) return set_err(ctx, MLXCAT_E_INVALID, "k must be in [0, %d]", MLXCAT_MAX_PROPOSAL);
    if (!bits) return set_err(ctx, MLXCAT_E_INVALID, "null mask bits");
    CK(ctx, cudaSetDevice(ctx->device));
    const size_t W = ((size_t)ctx->cfg.vocab + 31) / 32, T = (size_t)c->rows * (MLXCAT_MAX_PROPOSAL + 1);
    const size_t n = (size_t)c->rows * (k + 1);
    if (!c->mask_bits) {
        CK(ctx, dalloc(c->allocs, &c->mask_bits, T * W));
        CK(ctx, dalloc(c->allocs, &c->mask_on, T));
    }
    CK(ctx, cudaMemcpyAsync(c->mask_bits, bits, n * W * sizeof(uint32_t), cudaMemcpyHostToDevice, ctx->stream));
    CK(ctx, cudaMemcpyAsync(c->mask_on, enabled, n, cudaMemcpyHostToDevice, ctx->stream));
    CK(ctx, cudaStreamSynchronize(ctx->stream));
    c->mask_k = k;
    return MLXCAT_OK;
}

namespace {
// The bytes one rank hands to the others for expert or tensor parallelism.
struct PeerHandle {
    char magic[4];              // "MXPR"
    int32_t version;            // 1
    int32_t kind;               // 1 = expert parallel, 2 = tensor parallel
    int32_t rank, ranks, cap, hidden;
    int32_t pad;
    uint64_t bytes;             // size of the exported region
    cudaIpcMemHandle_t ipc;     // the region (its own cudaMalloc allocation)
};
static_assert(sizeof(PeerHandle) <= MLXCAT_PEER_HANDLE_BYTES, "peer handle too large");

int group_rank(const mlxcat_ctx *ctx) { return ctx->ep > 1 ? ctx->ep_rank : ctx->tp_rank; }
int group_size(const mlxcat_ctx *ctx) { return ctx->ep > 1 ? ctx->ep : ctx->tp; }
}  // namespace

int mlxcat_cache_peer_handle(mlxcat_cache *c, uint8_t out[MLXCAT_PEER_HANDLE_BYTES]) {
    if (!c || !out) return c ? set_err(c->ctx, MLXCAT_E_INVALID, "null handle buffer") : MLXCAT_E_INVALID;
    mlxcat_ctx *ctx = c->ctx;
    if (!c->peer_region) return set_err(ctx, MLXCAT_E_STATE, "cache is neither expert- nor tensor-parallel");
    CK(ctx, cudaSetDevice(ctx->device));
    PeerHandle h;
    std::memset(&h, 0, sizeof h);
    std::memcpy(h.magic, "MXPR", 4);
    h.version = 1;
    h.kind = c->peer_kind;
    h.rank = group_rank(ctx); h.ranks = group_size(ctx); h.cap = c->peer_cap; h.hidden = ctx->cfg.hidden;
    h.bytes = c->peer_bytes;
    CK(ctx, cudaIpcGetMemHandle(&h.ipc, c->peer_region));
    std::memset(out, 0, MLXCAT_PEER_HANDLE_BYTES);
    std::memcpy(out, &h, sizeof h);
    return MLXCAT_OK;
}

int mlxcat_cache_peer_connect(mlxcat_cache *c, const uint8_t *handles) {
    if (!c || !handles) return c ? set_err(c->ctx, MLXCAT_E_INVALID, "null handles") : MLXCAT_E_INVALID;
    mlxcat_ctx *ctx = c->ctx;
    if (!c->peer_region) return set_err(ctx, MLXCAT_E_STATE, "cache is neither expert- nor tensor-parallel");
    if (c->peer_connected) return set_err(ctx, MLXCAT_E_STATE, "cache already connected");
    CK(ctx, cudaSetDevice(ctx->device));
    const int N = group_size(ctx), me = group_rank(ctx);
    std::vector<PeerHandle> hs(N);
    for (int p = 0; p < N; ++p) {
        std::memcpy(&hs[p], handles + (size_t)p * MLXCAT_PEER_HANDLE_BYTES, sizeof(PeerHandle));
        const PeerHandle &h = hs[p];
        if (std::memcmp(h.magic, "MXPR", 4) || h.version != 1 || h.kind != c->peer_kind)
            return set_err(ctx, MLXCAT_E_INVALID, "handle %d is not a %s cache handle", p,
                           c->peer_kind == 1 ? "expert-parallel" : "tensor-parallel");
        if (h.rank != p || h.ranks != N)
            return set_err(ctx, MLXCAT_E_INVALID, "handle %d is rank %d of %d (want rank %d of %d, in rank order)", p,
                           h.rank, h.ranks, p, N);
        if (h.cap != c->peer_cap || h.hidden != ctx->cfg.hidden || h.bytes != c->peer_bytes)
            return set_err(ctx, MLXCAT_E_INVALID,
                           "rank %d's cache has another shape (capacity %d rows, hidden %d; this rank: %d, %d): "
                           "every rank's cache needs the same max_rows",
                           p, h.cap, h.hidden, c->peer_cap, ctx->cfg.hidden);
    }
    if (c->peer_kind == 2 && ctx->cfg.hidden % (128 * N))
        return set_err(ctx, MLXCAT_E_INVALID, "the fused allreduce needs hidden (%d) to be a multiple of 128 x %d ranks",
                       ctx->cfg.hidden, N);
    std::vector<char *> peers(N, nullptr), opened;
    for (int p = 0; p < N; ++p) {
        if (p == me) { peers[p] = c->peer_region; continue; }
        void *q = nullptr;
        const cudaError_t e = cudaIpcOpenMemHandle(&q, hs[p].ipc, cudaIpcMemLazyEnablePeerAccess);
        if (e != cudaSuccess) {
            for (char *o : opened) cudaIpcCloseMemHandle(o);
            return set_err(ctx, MLXCAT_E_CUDA, "mapping rank %d's region: %s", p, cudaGetErrorString(e));
        }
        peers[p] = static_cast<char *>(q);
        opened.push_back(peers[p]);
    }
    const cudaError_t e = cudaMemcpy(c->peer_tab, peers.data(), sizeof(char *) * N, cudaMemcpyHostToDevice);
    if (e != cudaSuccess) {
        for (char *o : opened) cudaIpcCloseMemHandle(o);
        return set_err(ctx, MLXCAT_E_CUDA, "peer table upload: %s", cudaGetErrorString(e));
    }
    c->peer_opened = opened;
    c->peer_connected = true;
    drop_graph(c);   // a captured step would still use the other allreduce
    return MLXCAT_OK;
}

int mlxcat_cache_insert_row(mlxcat_cache *c, int32_t row, const int32_t *prompt, int32_t len,
                            int32_t max_new_tokens, const mlxcat_sampling *sp, int32_t *first_token) {
    if (!c) return MLXCAT_E_INVALID;
    return admit_row(c, row, prompt, len, 0, max_new_tokens, sp, first_token);
}

int mlxcat_cache_insert_row_prefix(mlxcat_cache *c, int32_t row, const int32_t *prompt, int32_t len,
                                   int32_t prefix_len, const uint16_t *k_prefix, const uint16_t *v_prefix,
                                   int32_t max_new_tokens, const mlxcat_sampling *sp, int32_t *first_token) {
    if (!c) return MLXCAT_E_INVALID;
    mlxcat_ctx *ctx = c->ctx;
    if (ctx->cfg.kind != MLXCAT_MODEL_TRANSFORMER)
        return set_err(ctx, MLXCAT_E_INVALID, "prefix import needs a transformer model");
    if (prefix_len < 0 || prefix_len >= len || (prefix_len > 0 && (!k_prefix || !v_prefix)))
        return set_err(ctx, MLXCAT_E_INVALID, "prefix_len must be in [0, len) with K and V given");
    if (row < 0 || row >= c->rows || (int64_t)len + max_new_tokens + MLXCAT_MAX_PROPOSAL + 1 > c->max_len)
        return set_err(ctx, MLXCAT_E_INVALID, "bad insert arguments");
    if (prefix_len > 0) {
        CK(ctx, cudaSetDevice(ctx->device));
        CK(ctx, cudaStreamSynchronize(ctx->stream));
        const mlxcat_model_config &cf = ctx->cfg;
        const size_t D = cf.head_dim, Hkv = cf.n_kv_heads;
        const size_t host_pitch = (size_t)prefix_len * D * 2, dev_pitch = (size_t)c->max_len * D * 2;
        for (int l = 0; l < cf.n_layers; ++l) {
            const KVLayer kv = c->layer(l);
            const size_t host_off = (size_t)l * Hkv * prefix_len * D;
            const size_t dev_off = (size_t)row * Hkv * c->max_len * D;
            CK(ctx, cudaMemcpy2DAsync(kv.k + dev_off, dev_pitch, k_prefix + host_off, host_pitch, host_pitch, Hkv,
                                      cudaMemcpyHostToDevice, ctx->stream));
            CK(ctx, cudaMemcpy2DAsync(kv.v + dev_off, dev_pitch, v_prefix + host_off, host_pitch, host_pitch, Hkv,
                                      cudaMemcpyHostToDevice, ctx->stream));
        }
    }
    return admit_row(c, row, prompt, len, prefix_len, max_new_tokens, sp, first_token);
}


int mlxcat_cache_remove_row(mlxcat_cache *c, int32_t row) {
    if (!c || row < 0 || row >= c->rows) return MLXCAT_E_INVALID;
    mlxcat_ctx *ctx = c->ctx;
    CK(ctx, cudaSetDevice(ctx->device));
    CK(ctx, cudaStreamSynchronize(ctx->stream));
    const int32_t zero = 0;
    CK(ctx, cudaMemcpy(c->active + row, &zero, 4, cudaMemcpyHostToDevice));
    CK(ctx, cudaMemcpy(c->kv_len + row, &zero, 4, cudaMemcpyHostToDevice));
    CK(ctx, cudaMemcpy(c->hist_len + row, &zero, 4, cudaMemcpyHostToDevice));
    c->host_temp[row] = 0.0f;
    return MLXCAT_OK;
}

int mlxcat_cache_trim(mlxcat_cache *c, int32_t n, int32_t *trimmed) {
    if (!c || n < 0) return MLXCAT_E_INVALID;
    mlxcat_ctx *ctx = c->ctx;
    CK(ctx, cudaSetDevice(ctx->device));
    CK(ctx, cudaStreamSynchronize(ctx->stream));
    std::vector<int32_t> len(c->rows);
    CK(ctx, cudaMemcpy(len.data(), c->kv_len, 4 * c->rows, cudaMemcpyDeviceToHost));
    int idx = 0;
    for (int x : len) idx = std::max(idx, x);
    const int t = std::min(n, idx);
    for (int &x : len) x -= std::min(t, x);
    CK(ctx, cudaMemcpy(c->kv_len, len.data(), 4 * c->rows, cudaMemcpyHostToDevice));
    if (trimmed) *trimmed = t;
    return MLXCAT_OK;
}

int mlxcat_cache_filter(mlxcat_cache *c, const int32_t *keep, int32_t n) {
    if (!c || n < 0 || (n > 0 && !keep)) return MLXCAT_E_INVALID;
    mlxcat_ctx *ctx = c->ctx;
    std::vector<char> kept(c->rows, 0);
    for (int i = 0; i < n; ++i) {
        if (keep[i] < 0 || keep[i] >= c->rows) return set_err(ctx, MLXCAT_E_INVALID, "filter: row %d out of range", keep[i]);
        kept[keep[i]] = 1;
    }
    for (int r = 0; r < c->rows; ++r)
        if (!kept[r]) {
            const int rc = mlxcat_cache_remove_row(c, r);
            if (rc) return rc;
        }
    return MLXCAT_OK;
}

int mlxcat_cache_trim_row(mlxcat_cache *c, int32_t row, int32_t n, int32_t *trimmed) {
    if (!c || row < 0 || row >= c->rows || n < 0) return MLXCAT_E_INVALID;
    mlxcat_ctx *ctx = c->ctx;
    CK(ctx, cudaSetDevice(ctx->device));
    CK(ctx, cudaStreamSynchronize(ctx->stream));
    int32_t len = 0;
    CK(ctx, cudaMemcpy(&len, c->kv_len + row, 4, cudaMemcpyDeviceToHost));
    const int32_t t = std::min(n, len);
    len -= t;
    CK(ctx, cudaMemcpy(c->kv_len + row, &len, 4, cudaMemcpyHostToDevice));
    if (trimmed) *trimmed = t;
    return MLXCAT_OK;
}

int mlxcat_cache_lengths(mlxcat_cache *c, int32_t *out) {
    if (!c || !out) return MLXCAT_E_INVALID;
    mlxcat_ctx *ctx = c->ctx;
    CK(ctx, cudaSetDevice(ctx->device));
    CK(ctx, cudaStreamSynchronize(ctx->stream));
    CK(ctx, cudaMemcpy(out, c->kv_len, 4 * c->rows, cudaMemcpyDeviceToHost));
    return MLXCAT_OK;
}

int mlxcat_cache_moe_routing(mlxcat_cache *c, int32_t layer, int32_t *ids, float *weights, int32_t *m) {
    if (!c) return MLXCAT_E_INVALID;
    mlxcat_ctx *ctx = c->ctx;
    const mlxcat_model_config &cf = ctx->cfg;
    if (!cf.n_experts || layer < 0 || layer >= cf.n_layers)
        return set_err(ctx, MLXCAT_E_INVALID, "no MoE layer %d", layer);
    if (m) *m = c->last_m;
    CK(ctx, cudaSetDevice(ctx->device));
    CK(ctx, cudaStreamSynchronize(ctx->stream));
    const size_t asg = (size_t)c->m_cap * cf.top_k, n = (size_t)c->last_m * cf.top_k;
    if (ids && n) CK(ctx, cudaMemcpy(ids, c->moe_id + layer * asg, n * 4, cudaMemcpyDeviceToHost));
    if (weights && n) CK(ctx, cudaMemcpy(weights, c->moe_w + layer * asg, n * 4, cudaMemcpyDeviceToHost));
    return MLXCAT_OK;
}

int mlxcat_cache_active(mlxcat_cache *c, int32_t *out) {
    if (!c || !out) return MLXCAT_E_INVALID;
    mlxcat_ctx *ctx = c->ctx;
    CK(ctx, cudaSetDevice(ctx->device));
    CK(ctx, cudaStreamSynchronize(ctx->stream));
    CK(ctx, cudaMemcpy(out, c->active, 4 * c->rows, cudaMemcpyDeviceToHost));
    return MLXCAT_OK;
}

int mlxcat_cache_history(mlxcat_cache *c, int32_t row, int32_t *out, int32_t cap, int32_t *len) {
    if (!c || row < 0 || row >= c->rows) return MLXCAT_E_INVALID;
    mlxcat_ctx *ctx = c->ctx;
    CK(ctx, cudaSetDevice(ctx->device));
    CK(ctx, cudaStreamSynchronize(ctx->stream));
    int32_t L = 0;
    CK(ctx, cudaMemcpy(&L, c->hist_len + row, 4, cudaMemcpyDeviceToHost));
    if (len) *len = L;
    if (out && cap > 0)
        CK(ctx, cudaMemcpy(out, c->hist + (size_t)row * c->hist_cap, 4 * (size_t)std::min(L, cap),
                           cudaMemcpyDeviceToHost));
    return MLXCAT_OK;
}

int mlxcat_cache_extract_row(mlxcat_cache *c, int32_t row, int32_t layer, uint16_t *k_out,
                             uint16_t *v_out) {
    if (!c || row < 0 || row >= c->rows) return MLXCAT_E_INVALID;
    mlxcat_ctx *ctx = c->ctx;
    const mlxcat_model_config &cf = ctx->cfg;
    if (cf.kind != MLXCAT_MODEL_TRANSFORMER || layer < 0 || layer >= cf.n_layers)
        return set_err(ctx, MLXCAT_E_INVALID, "no such layer");
    CK(ctx, cudaSetDevice(ctx->device));
    CK(ctx, cudaStreamSynchronize(ctx->stream));
    int32_t L = 0;
    CK(ctx, cudaMemcpy(&L, c->kv_len + row, 4, cudaMemcpyDeviceToHost));
    const KVLayer kv = c->layer(layer);
    const size_t D = cf.head_dim;
    for (int h = 0; h < cf.n_kv_heads; ++h) {
        const size_t src = (((size_t)row * cf.n_kv_heads + h) * c->max_len) * D;
        if (k_out) CK(ctx, cudaMemcpy(k_out + (size_t)h * L * D, kv.k + src, 2 * L * D, cudaMemcpyDeviceToHost));
        if (v_out) CK(ctx, cudaMemcpy(v_out + (size_t)h * L * D, kv.v + src, 2 * L * D, cudaMemcpyDeviceToHost));
    }
    return MLXCAT_OK;
}

int mlxcat_draft(mlxcat_cache *c, const mlxcat_spec_config *spec, int32_t *drafts, int32_t *counts) {
    if (!c) return MLXCAT_E_INVALID;
    mlxcat_ctx *ctx = c->ctx;
    int rc = validate_spec(ctx, spec);
    if (rc) return rc;
    CK(ctx, cudaSetDevice(ctx->device));
    const SpecParams sp = params_of(spec);
    const int K1 = sp.k + 1;
    cudaStream_t st = ctx->stream;
    LK(ctx, draft(c->rs(), sp, c->vtok, c->count, c->trow, c->tpos, st));
    c->last_k = sp.k;
    std::vector<int32_t> vt((size_t)c->rows * K1);
    CK(ctx, cudaMemcpyAsync(vt.data(), c->vtok, 4 * vt.size(), cudaMemcpyDeviceToHost, st));
    if (counts) CK(ctx, cudaMemcpyAsync(counts, c->count, 4 * c->rows, cudaMemcpyDeviceToHost, st));
    CK(ctx, cudaStreamSynchronize(st));
    if (drafts)
        for (int r = 0; r < c->rows; ++r)
            for (int i = 0; i < sp.k; ++i) drafts[r * sp.k + i] = vt[(size_t)r * K1 + 1 + i];
    return MLXCAT_OK;
}

int mlxcat_verify_forward(mlxcat_cache *c, const mlxcat_spec_config *spec, float *logits) {
    if (!c) return MLXCAT_E_INVALID;
    mlxcat_ctx *ctx = c->ctx;
    int rc = validate_spec(ctx, spec);
    if (rc) return rc;
    if ((rc = check_weights(c))) return rc;
    const SpecParams sp = params_of(spec);
    if (c->last_k != sp.k) return set_err(ctx, MLXCAT_E_STATE, "mlxcat_draft with the same config must come first");
    CK(ctx, cudaSetDevice(ctx->device));
    const int K1 = sp.k + 1, M = c->rows * K1;
    rc = forward(c, M, K1, c->vtok, c->trow, c->tpos, 0);
    if (rc) return rc;
    if (logits)
        CK(ctx, cudaMemcpyAsync(logits, c->logits, sizeof(float) * (size_t)M * ctx->cfg.vocab,
                                cudaMemcpyDeviceToHost, ctx->stream));
    CK(ctx, cudaStreamSynchronize(ctx->stream));
    if ((rc = device_err(c, false))) return rc;
    return MLXCAT_OK;
}

int mlxcat_accept(mlxcat_cache *c, const mlxcat_spec_config *spec, int32_t *out_tokens,
                  int32_t *out_counts, int32_t *out_fin, mlxcat_stats *stats) {
    if (!c) return MLXCAT_E_INVALID;
    mlxcat_ctx *ctx = c->ctx;
    int rc = validate_spec(ctx, spec);
    if (rc) return rc;
    const SpecParams sp = params_of(spec);
    if (c->last_k != sp.k) return set_err(ctx, MLXCAT_E_STATE, "mlxcat_verify_forward with the same config must come first");
    CK(ctx, cudaSetDevice(ctx->device));
    cudaStream_t st = ctx->stream;
    const int K1 = sp.k + 1, M = c->rows * K1;
    if (c->mask_k >= 0) {
        if (c->mask_k != sp.k)
            return set_err(ctx, MLXCAT_E_STATE, "token masks were set for k = %d, this step has k = %d", c->mask_k, sp.k);
        ctx->launches++;
        LK(ctx, apply_token_masks(c->logits, M, ctx->cfg.vocab, c->mask_bits, c->mask_on, st));
        c->mask_k = -1;   // consumed by this acceptance
    }
    LK(ctx, argmax_rows(c->logits, M, ctx->cfg.vocab, c->amax, st, c->amax_part, c->amax_ctr));
    LK(ctx, accept_greedy(c->rs(), sp, c->vtok, c->count, c->amax, step_out(c), st));
    if (any_sampled(c)) {
        ctx->launches++;
        LK(ctx, accept_sampled(c->rs(), sp, c->vtok, c->count, c->logits, ctx->cfg.vocab, c->samp, step_out(c), st));
    }
    CK(ctx, cudaMemcpyAsync(c->h_tok, c->out_tok, sizeof(int32_t) * M, cudaMemcpyDeviceToHost, st));
    CK(ctx, cudaMemcpyAsync(c->h_n, c->out_n, sizeof(int32_t) * c->rows, cudaMemcpyDeviceToHost, st));
    CK(ctx, cudaMemcpyAsync(c->h_fin, c->out_fin, sizeof(int32_t) * c->rows, cudaMemcpyDeviceToHost, st));
    CK(ctx, cudaMemcpyAsync(c->h_stats, c->stats, 32, cudaMemcpyDeviceToHost, st));
    CK(ctx, cudaStreamSynchronize(st));
    copy_out(c, K1, out_tokens, out_counts, out_fin, stats);
    c->last_k = -1;
    return MLXCAT_OK;
}

int mlxcat_spec_step(mlxcat_cache *c, const mlxcat_spec_config *spec, int32_t *out_tokens,
                     int32_t *out_counts, int32_t *out_fin, mlxcat_stats *stats) {
    if (!c) return MLXCAT_E_INVALID;
    mlxcat_ctx *ctx = c->ctx;
    int rc = validate_spec(ctx, spec);
    if (rc) return rc;
    if ((rc = check_weights(c))) return rc;
    if (c->mask_k >= 0)
        return set_err(ctx, MLXCAT_E_STATE,
                       "token masks are pending: they depend on the drafts, so they apply to the split step "
                       "(mlxcat_draft, mlxcat_verify_forward, mlxcat_accept)");
    CK(ctx, cudaSetDevice(ctx->device));
    const SpecParams sp = params_of(spec);
    const bool sampled = any_sampled(c);
    const bool same = c->graph && memcmp(&c->gkey, spec, sizeof *spec) == 0 && c->gsampled == sampled;
    cudaStream_t st = ctx->stream;
    if (!same) {
        drop_graph(c);
        CK(ctx, cudaStreamSynchronize(st));
        const int64_t before = ctx->launches;
        cudaGraph_t g = nullptr;
        CK(ctx, cudaStreamBeginCapture(st, cudaStreamCaptureModeThreadLocal));
        rc = enqueue_step(c, sp, sampled, true);
        cudaError_t ec = cudaStreamEndCapture(st, &g);
        if (rc) { if (g) cudaGraphDestroy(g); return rc; }
        CK(ctx, ec);
        cudaError_t ei = cudaGraphInstantiate(&c->graph, g, 0);
        cudaGraphDestroy(g);
        CK(ctx, ei);
        c->graph_launches = ctx->launches - before;
        ctx->launches = before;
        c->gkey = *spec;
        c->gsampled = sampled;
    }
    CK(ctx, cudaGraphLaunch(c->graph, st));
    ctx->launches += c->graph_launches;
    CK(ctx, cudaStreamSynchronize(st));
    if ((rc = device_err(c, true))) return rc;
    copy_out(c, sp.k + 1, out_tokens, out_counts, out_fin, stats);
    c->last_k = -1;
    return MLXCAT_OK;
}

int mlxcat_last_verify_ms(mlxcat_cache *c, float *ms) {
    if (!c || !ms) return MLXCAT_E_INVALID;
    CK(c->ctx, cudaEventElapsedTime(ms, c->ev0, c->ev1));
    return MLXCAT_OK;
}

int mlxcat_last_step_ms(mlxcat_cache *c, float *ms) {
    if (!c || !ms) return MLXCAT_E_INVALID;
    CK(c->ctx, cudaEventElapsedTime(ms, c->es0, c->es1));
    return MLXCAT_OK;
}

int mlxcat_cache_set_profiling(mlxcat_cache *c, int32_t enabled) {
    if (!c) return MLXCAT_E_INVALID;
    if (c->profiling != (enabled != 0)) drop_graph(c);
    c->profiling = enabled != 0;
    return MLXCAT_OK;
}

int mlxcat_cache_profile(mlxcat_cache *c, float *q4_ms, float *attn_ms, int32_t *q4_n, int32_t *attn_n) {
    if (!c) return MLXCAT_E_INVALID;
    float sum[2] = {0.f, 0.f};
    int cnt[2] = {0, 0};
    for (size_t i = 0; i < c->prof_class.size(); ++i) {
        float ms = 0.f;
        CK(c->ctx, cudaEventElapsedTime(&ms, c->prof_ev[2 * i], c->prof_ev[2 * i + 1]));
        sum[c->prof_class[i]] += ms;
        cnt[c->prof_class[i]] += 1;
    }
    if (q4_ms) *q4_ms = sum[0];
    if (attn_ms) *attn_ms = sum[1];
    if (q4_n) *q4_n = cnt[0];
    if (attn_n) *attn_n = cnt[1];
    return MLXCAT_OK;
}

// ---------------------------------------------------------------------------
// device-pointer operators
// ---------------------------------------------------------------------------
static int op_sm_count() {
    int dev = 0, sm = 148;
    if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sm, cudaDevAttrMultiProcessorCount, dev);
    return sm;
}

// workspace: [x in perm8 order | packed (scale, bias) | split-K partials |
//             split-K tickets | error flag]
static void q4_ws_layout(int32_t N, int32_t K, int32_t M, size_t *off_sbp, size_t *off_part, size_t *off_ctr,
                         size_t *off_err, size_t *total) {
    const int sm = op_sm_count();
    auto up = [](size_t v) { return (v + 255) & ~(size_t)255; };
    *off_sbp = up((size_t)M * K * 2);
    *off_part = *off_sbp + up(q4_sbp_words(N, K) * 4);
    *off_ctr = *off_part + up(q4_tc_partial_floats(N, K, M, sm) * 4);
    *off_err = *off_ctr + up(q4_tc_counters(N, M) * 4);
    *total = *off_err + 256;
}

size_t mlxcat_op_q4_linear_workspace(int32_t N, int32_t K, int32_t M) {
    if (N <= 0 || K <= 0 || M <= 0) return 0;
    size_t a, b, c, d, t;
    q4_ws_layout(N, K, M, &a, &b, &c, &d, &t);
    return t;
}

int mlxcat_op_q4_linear(const uint32_t *wq, const uint16_t *scales, const uint16_t *biases, int32_t N,
                        int32_t K, const uint16_t *x, int32_t M, float *y, void *ws, size_t ws_bytes,
                        void *stream) {
    if (!wq || !scales || !biases || !x || !y || N <= 0 || K <= 0 || M <= 0)
        return op_err(MLXCAT_E_INVALID, "bad q4_linear arguments");
    if (N % 128 || K % 128) return op_err(MLXCAT_E_INVALID, "N and K must be multiples of 128");
    size_t off_sbp, off_part, off_ctr, off_err, need;
    q4_ws_layout(N, K, M, &off_sbp, &off_part, &off_ctr, &off_err, &need);
    if (!ws || ws_bytes < need) return op_err(MLXCAT_E_INVALID, "workspace of %zu bytes required", need);
    cudaStream_t st = (cudaStream_t)stream;
    char *w8 = static_cast<char *>(ws);
    Q4WeightTC w;
    w.wq = wq; w.scales = reinterpret_cast<const __half *>(scales);
    w.biases = reinterpret_cast<const __half *>(biases); w.N = N; w.K = K;
    w.sbp = reinterpret_cast<const uint32_t *>(w8 + off_sbp);
    if (!make_weight_map(w)) return op_err(MLXCAT_E_CUDA, "TMA descriptor for the weights failed");
    Q4Epilogue ep;
    ep.op = Q4Epilogue::STORE; ep.out = y; ep.ldo = N;
    ep.part = reinterpret_cast<float *>(w8 + off_part);
    ep.counters = reinterpret_cast<unsigned *>(w8 + off_ctr);
    ep.err = reinterpret_cast<int *>(w8 + off_err);
    __half *xp = reinterpret_cast<__half *>(w8);
    cudaError_t e = cudaMemsetAsync(w8 + off_ctr, 0, need - off_ctr, st);
    if (e == cudaSuccess) e = permute_activations(reinterpret_cast<const __half *>(x), xp, M, K, st);
    if (e == cudaSuccess)
        e = pack_q4_sb(w.scales, w.biases, N, K, reinterpret_cast<uint32_t *>(w8 + off_sbp), st);
    if (e == cudaSuccess) e = q4_tc(w, xp, M, 0, M, op_sm_count(), ep, st);
    if (e != cudaSuccess) return op_err(MLXCAT_E_CUDA, "q4_linear: %s", cudaGetErrorString(e));
    return MLXCAT_OK;
}

// ---- sparse MoE MLP operator ------------------------------------------------
static void moe_ws_layout(int32_t M, int32_t H, int32_t I, int32_t E, int32_t TK, size_t off[9]) {
    const size_t sz[9] = {(size_t)M * H * 2, (size_t)M * 4, (size_t)M * TK * 4, (size_t)M * TK * 4,
                          (size_t)E * 4, (size_t)E * M * 4, (size_t)M * TK * I * 2, (size_t)M * E * 4,
                          (size_t)M * TK * H * 4};
    size_t o = 0;
    for (int i = 0; i < 9; ++i) {
        off[i] = o;
        o += (sz[i] + 255) & ~(size_t)255;
    }
}

size_t mlxcat_op_moe_workspace(int32_t M, int32_t hidden, int32_t intermediate, int32_t n_experts, int32_t top_k) {
    if (M <= 0 || hidden <= 0 || intermediate <= 0 || n_experts <= 0 || top_k <= 0) return 0;
    size_t off[9];
    moe_ws_layout(M, hidden, intermediate, n_experts, top_k, off);
    return off[8] + (size_t)M * top_k * hidden * 4;
}

int mlxcat_op_moe(const uint16_t *x, int32_t M, int32_t hidden, int32_t intermediate, int32_t n_experts,
                  int32_t top_k, int32_t norm_topk, const uint16_t *router, const uint32_t *const wq[3],
                  const uint16_t *const scales[3], const uint16_t *const biases[3], float *y, int32_t *ids,
                  float *weights, void *ws, size_t ws_bytes, void *stream) {
    if (!x || !router || !wq || !scales || !biases || !y || M <= 0)
        return op_err(MLXCAT_E_INVALID, "bad moe arguments");
    for (int p = 0; p < 3; ++p)
        if (!wq[p] || !scales[p] || !biases[p]) return op_err(MLXCAT_E_INVALID, "bad moe weight pointers");
    const int H = hidden, I = intermediate, E = n_experts, TK = top_k;
    if (H % 256 || I % 128 || E % 32 || E > 256 || TK < 1 || TK > 8 || TK > E)
        return op_err(MLXCAT_E_INVALID, "moe shape: hidden %% 256, intermediate %% 128, n_experts %% 32 (<= 256), "
                                        "1 <= top_k <= min(8, n_experts)");
    const size_t need = mlxcat_op_moe_workspace(M, H, I, E, TK);
    if (!ws || ws_bytes < need) return op_err(MLXCAT_E_INVALID, "workspace of %zu bytes required", need);
    size_t off[9];
    moe_ws_layout(M, H, I, E, TK, off);
    char *w8 = static_cast<char *>(ws);
    cudaStream_t st = (cudaStream_t)stream;
    __half *xb = reinterpret_cast<__half *>(w8 + off[0]);
    float *tsc = reinterpret_cast<float *>(w8 + off[1]);
    int32_t *tid = ids ? ids : reinterpret_cast<int32_t *>(w8 + off[2]);
    float *tw = weights ? weights : reinterpret_cast<float *>(w8 + off[3]);
    int *cnt = reinterpret_cast<int *>(w8 + off[4]);
    int32_t *list = reinterpret_cast<int32_t *>(w8 + off[5]);
    __half *act = reinterpret_cast<__half *>(w8 + off[6]);
    float *lg = reinterpret_cast<float *>(w8 + off[7]);
    float *yt = reinterpret_cast<float *>(w8 + off[8]);
    cudaError_t e = permute_activations(reinterpret_cast<const __half *>(x), xb, M, H, st);
    if (e == cudaSuccess) e = cudaMemsetAsync(cnt, 0, sizeof(int) * E, st);
    if (e == cudaSuccess) e = cudaMemsetAsync(y, 0, sizeof(float) * (size_t)M * H, st);
    MoERouteArgs ra;
    ra.x = xb; ra.ldx_rows = M; ra.M = M; ra.H = H; ra.E = E; ra.TK = TK; ra.norm_topk = norm_topk;
    ra.wr = reinterpret_cast<const __nv_bfloat16 *>(router);
    ra.tok_scale = tsc; ra.topk_id = tid; ra.topk_w = tw; ra.exp_count = cnt; ra.exp_list = list; ra.list_cap = M;
    ra.logits = lg;
    if (e == cudaSuccess) e = moe_route(ra, st);
    MoEExpertArgs ga;
    ga.wq = wq[0]; ga.scales = reinterpret_cast<const __half *>(scales[0]); ga.biases = reinterpret_cast<const __half *>(biases[0]);
    ga.wq2 = wq[1]; ga.scales2 = reinterpret_cast<const __half *>(scales[1]); ga.biases2 = reinterpret_cast<const __half *>(biases[1]);
    ga.N = I; ga.K = H; ga.E = E; ga.x = xb; ga.ldx_rows = M; ga.x_div = TK;
    ga.exp_count = cnt; ga.exp_list = list; ga.list_cap = M; ga.tok_scale = tsc; ga.act = act; ga.act_rows = M * TK;
    if (e == cudaSuccess) e = moe_expert(ga, 0, st);
    MoEExpertArgs da;
    da.wq = wq[2]; da.scales = reinterpret_cast<const __half *>(scales[2]); da.biases = reinterpret_cast<const __half *>(biases[2]);
    da.N = H; da.K = I; da.E = E; da.x = act; da.ldx_rows = M * TK; da.x_div = 1;
    da.exp_count = cnt; da.exp_list = list; da.list_cap = M; da.topk_w = tw; da.y = yt;
    if (e == cudaSuccess) e = moe_expert(da, 1, st);
    MoECombineArgs ca;
    ca.h = y; ca.y = yt; ca.M = M; ca.H = H; ca.TK = TK;
    if (e == cudaSuccess) e = moe_combine(ca, st);
    if (e != cudaSuccess) return op_err(MLXCAT_E_CUDA, "moe: %s", cudaGetErrorString(e));
    return MLXCAT_OK;
}

size_t mlxcat_op_attention_workspace(int32_t M, int32_t qg, int32_t n_heads, int32_t n_kv, int32_t D,
                                     int32_t max_len) {
    if (M <= 0 || qg <= 0 || n_kv <= 0) return 0;
    const int groups = (M + qg - 1) / qg;
    const int splits = attention_max_splits(max_len, KEY_CHUNK);
    const size_t items = attention_scratch_items(groups, n_kv, splits);
    const int qrows = attention_qrows(qg, n_heads, n_kv);
    return items * qrows * (size_t)D * 4 + 256 + items * qrows * 2 * 4;
}

int mlxcat_op_attention(const uint16_t *q, const uint16_t *k_cache, const uint16_t *v_cache,
                        int32_t max_len, const int32_t *trow, const int32_t *tpos, int32_t M, int32_t qg,
                        int32_t n_heads, int32_t n_kv, int32_t D, uint16_t *out, void *ws,
                        size_t ws_bytes, void *stream) {
    if (!q || !k_cache || !v_cache || !trow || !tpos || !out || M <= 0 || qg <= 0 || n_kv <= 0 ||
        n_heads % n_kv || (D != 64 && D != 128) || qg * (n_heads / n_kv) > 64)
        return op_err(MLXCAT_E_INVALID, "bad attention arguments");
    const size_t need = mlxcat_op_attention_workspace(M, qg, n_heads, n_kv, D, max_len);
    if (!ws || ws_bytes < need) return op_err(MLXCAT_E_INVALID, "workspace of %zu bytes required", need);
    const int groups = (M + qg - 1) / qg;
    const int splits = attention_max_splits(max_len, KEY_CHUNK);
    const size_t items = attention_scratch_items(groups, n_kv, splits);
    const int qrows = attention_qrows(qg, n_heads, n_kv);
    AttnScratch sc;
    sc.o = static_cast<float *>(ws);
    sc.ml = reinterpret_cast<float *>(static_cast<char *>(ws) + ((items * qrows * (size_t)D * 4 + 255) & ~(size_t)255));
    sc.items = items;
    KVLayer kv;
    kv.k = const_cast<__half *>(reinterpret_cast<const __half *>(k_cache));
    kv.v = const_cast<__half *>(reinterpret_cast<const __half *>(v_cache));
    kv.max_len = max_len;
    cudaError_t e = attention(reinterpret_cast<const __half *>(q), kv, trow, tpos, M, qg, n_heads, n_kv, D,
                              KEY_CHUNK, splits, sc, reinterpret_cast<__half *>(out), false, M,
                              (cudaStream_t)stream);
    if (e != cudaSuccess) return op_err(MLXCAT_E_CUDA, "attention: %s", cudaGetErrorString(e));
    return MLXCAT_OK;
}

int mlxcat_op_prefill_attention(const uint16_t *q, const uint16_t *k_cache, const uint16_t *v_cache, int32_t rows,
                                int32_t max_len, int32_t row, int32_t s0, int32_t n, int32_t n_heads, int32_t n_kv,
                                int32_t D, uint16_t *out, int32_t *err, void *stream) {
    if (!q || !k_cache || !v_cache || !out || !err || n <= 0 || n_kv <= 0 || n_heads % n_kv || rows <= 0 ||
        row < 0 || row >= rows || s0 < 0 || s0 + n > max_len || !fa_prefill_supported(D))
        return op_err(MLXCAT_E_INVALID, "bad prefill attention arguments (head_dim must be 128)");
    KVLayer kv;
    kv.k = const_cast<__half *>(reinterpret_cast<const __half *>(k_cache));
    kv.v = const_cast<__half *>(reinterpret_cast<const __half *>(v_cache));
    kv.max_len = max_len;
    const cudaError_t e = fa_prefill(reinterpret_cast<const __half *>(q), n, kv, rows, row, s0, n, n_heads, n_kv, D,
                                     reinterpret_cast<__half *>(out), err, (cudaStream_t)stream);
    if (e != cudaSuccess) return op_err(MLXCAT_E_CUDA, "prefill attention: %s", cudaGetErrorString(e));
    return MLXCAT_OK;
}

// ---------------------------------------------------------------------------
// attention for callers that cannot allocate device memory
// ---------------------------------------------------------------------------
// Some callers of the attention operator have no way to allocate device
// memory where they call it: a host runtime whose device buffers all come
// from a foreign arena it does not own (a Swift / MLX-style buffer pool, a
// ctypes or JNI binding without a CUDA allocator), or an inference loop that
// must not allocate between steps.  For them the split-K scratch (partial
// outputs and running max / sum per key split) lives in one fixed device array
// of MLXCAT_NOALLOC_ATTN_SCRATCH_BYTES, declared below at file scope.  Every
// GPU that loads this library holds that array until the process exits.
//
// In host code `g_attn_noalloc_scratch` is only a stand-in for the device
// symbol; its device address comes from cudaGetSymbolAddress on the current
// device.  It is fetched again on every call made outside a stream capture (a
// device reset reloads the module, after which an old address would be
// stale); inside a capture, where that query is not allowed, the address
// cached by the device's last uncaptured call is used.
static __device__ __align__(256) unsigned char g_attn_noalloc_scratch[MLXCAT_NOALLOC_ATTN_SCRATCH_BYTES];

namespace {
std::mutex g_noalloc_mu;
void *g_noalloc_base[64] = {};   // device address of the array, per device ordinal
}  // namespace

int mlxcat_op_attention_noalloc(const uint16_t *q, const uint16_t *k_cache, const uint16_t *v_cache,
                                int32_t max_len, const int32_t *trow, const int32_t *tpos, int32_t M,
                                int32_t qg, int32_t n_heads, int32_t n_kv, int32_t D, uint16_t *out,
                                void *stream) {
    if (!q || !k_cache || !v_cache || !trow || !tpos || !out || M <= 0 || qg <= 0 || n_kv <= 0 ||
        n_heads % n_kv || (D != 64 && D != 128) || qg * (n_heads / n_kv) > 64)
        return op_err(MLXCAT_E_INVALID, "bad attention arguments");
    const size_t need = mlxcat_op_attention_workspace(M, qg, n_heads, n_kv, D, max_len);
    if (need > (size_t)MLXCAT_NOALLOC_ATTN_SCRATCH_BYTES)
        return op_err(MLXCAT_E_INVALID,
                      "attention_noalloc: this shape needs %zu bytes of scratch but the fixed array holds %zu; "
                      "use mlxcat_op_attention with a workspace",
                      need, (size_t)MLXCAT_NOALLOC_ATTN_SCRATCH_BYTES);
    int dev = -1;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return op_err(MLXCAT_E_CUDA, "attention_noalloc: %s", cudaGetErrorString(e));
    if (dev < 0 || dev >= 64) return op_err(MLXCAT_E_INVALID, "attention_noalloc: device ordinal %d >= 64", dev);
    char *base = nullptr;
    {
        cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
        e = cudaStreamIsCapturing((cudaStream_t)stream, &cap);
        if (e != cudaSuccess) return op_err(MLXCAT_E_CUDA, "attention_noalloc: %s", cudaGetErrorString(e));
        std::lock_guard<std::mutex> lock(g_noalloc_mu);
        if (cap == cudaStreamCaptureStatusNone) {
            // resolve the array's address on the current device
            void *p = nullptr;
            e = cudaGetSymbolAddress(&p, g_attn_noalloc_scratch);
            if (e != cudaSuccess)
                return op_err(MLXCAT_E_CUDA, "attention_noalloc: cudaGetSymbolAddress: %s", cudaGetErrorString(e));
            g_noalloc_base[dev] = p;
        } else if (!g_noalloc_base[dev]) {
            return op_err(MLXCAT_E_STATE,
                          "attention_noalloc: first call on device %d inside a stream capture; call it once "
                          "outside a capture first",
                          dev);
        }
        base = static_cast<char *>(g_noalloc_base[dev]);
    }
    // Nothing in the array needs clearing: every partial and every (max, sum)
    // pair the combine pass reads is written by the split pass of the same call.
    const int groups = (M + qg - 1) / qg;
    const int splits = attention_max_splits(max_len, KEY_CHUNK);
    const size_t items = attention_scratch_items(groups, n_kv, splits);
    const int qrows = attention_qrows(qg, n_heads, n_kv);
    AttnScratch sc;
    sc.o = reinterpret_cast<float *>(base);
    sc.ml = reinterpret_cast<float *>(base + ((items * qrows * (size_t)D * 4 + 255) & ~(size_t)255));
    sc.items = items;
    KVLayer kv;
    kv.k = const_cast<__half *>(reinterpret_cast<const __half *>(k_cache));
    kv.v = const_cast<__half *>(reinterpret_cast<const __half *>(v_cache));
    kv.max_len = max_len;
    e = attention(reinterpret_cast<const __half *>(q), kv, trow, tpos, M, qg, n_heads, n_kv, D, KEY_CHUNK,
                  splits, sc, reinterpret_cast<__half *>(out), false, M, (cudaStream_t)stream);
    if (e != cudaSuccess) return op_err(MLXCAT_E_CUDA, "attention_noalloc: %s", cudaGetErrorString(e));
    return MLXCAT_OK;
}

int mlxcat_op_dequant_q4(const uint32_t *wq, const uint16_t *scales, const uint16_t *biases, int32_t N, int32_t K,
                         uint16_t *w_out, void *stream) {
    if (!wq || !scales || !biases || !w_out || N <= 0 || K <= 0 || K % 64)
        return op_err(MLXCAT_E_INVALID, "dequant_q4: bad arguments");
    Q4Weight w;
    w.wq = wq; w.scales = reinterpret_cast<const __half *>(scales); w.biases = reinterpret_cast<const __half *>(biases);
    w.N = N; w.K = K;
    cudaError_t e = dequant_q4(w, reinterpret_cast<__half *>(w_out), (cudaStream_t)stream);
    if (e != cudaSuccess) return op_err(MLXCAT_E_CUDA, "dequant_q4: %s", cudaGetErrorString(e));
    return MLXCAT_OK;
}

int mlxcat_op_gemm_f16(const uint16_t *w, int32_t N, int32_t K, const uint16_t *x, int32_t M, int32_t epilogue,
                       void *out, int32_t ldo, int32_t *err_flag, void *stream) {
    if (!w || !x || !out || N <= 0 || K <= 0 || M <= 0 || N % 128 || K % 64 || epilogue < 0 || epilogue > 2)
        return op_err(MLXCAT_E_INVALID, "gemm_f16: bad arguments (N %% 128, K %% 64)");
    if (ldo < (epilogue == MLXCAT_GEMM_SWIGLU ? N / 2 : N)) return op_err(MLXCAT_E_INVALID, "gemm_f16: ldo too small");
    cudaError_t e = gemm_tc(reinterpret_cast<const __half *>(w), N, K, reinterpret_cast<const __half *>(x), M,
                            epilogue, out, ldo, op_sm_count(), err_flag, (cudaStream_t)stream);
    if (e != cudaSuccess) return op_err(MLXCAT_E_CUDA, "gemm_f16: %s", cudaGetErrorString(e));
    return MLXCAT_OK;
}

int mlxcat_op_synth_q4(uint64_t seed, uint32_t tensor_id, float stddev, int32_t N, int32_t K, uint32_t *wq,
                       uint16_t *scales, uint16_t *biases, void *stream) {
    if (!wq || !scales || !biases || N <= 0 || K <= 0 || K % 64)
        return op_err(MLXCAT_E_INVALID, "bad synth arguments");
    cudaError_t e = synth_q4(seed, tensor_id, stddev, N, K, wq, reinterpret_cast<__half *>(scales),
                             reinterpret_cast<__half *>(biases), 0, (cudaStream_t)stream);
    if (e != cudaSuccess) return op_err(MLXCAT_E_CUDA, "synth: %s", cudaGetErrorString(e));
    return MLXCAT_OK;
}

static RowState rows_of(const mlxcat_rows *r) {
    RowState s;
    s.hist = r->hist; s.hist_cap = r->hist_cap; s.rows = r->rows; s.hist_len = r->hist_len;
    s.kv_len = r->kv_len; s.n_gen = r->n_gen; s.max_new = r->max_new; s.active = r->active;
    s.temperature = r->temperature; s.top_p = r->top_p; s.seed = r->seed; s.has_seed = r->has_seed;
    s.eos = r->eos; s.n_eos = r->n_eos; s.trigger = r->trigger;
    return s;
}

int mlxcat_op_draft(const mlxcat_rows *rows, const mlxcat_spec_config *spec, int32_t *vtok, int32_t *count,
                    int32_t *trow, int32_t *tpos, void *stream) {
    if (!rows || !spec || !vtok || !count || !trow || !tpos || rows->rows <= 0)
        return op_err(MLXCAT_E_INVALID, "bad draft arguments");
    if (spec->max_proposal < 0 || spec->max_proposal > 16 || spec->max_suffix < 1)
        return op_err(MLXCAT_E_INVALID, "bad spec config");
    cudaError_t e = draft(rows_of(rows), params_of(spec), vtok, count, trow, tpos, (cudaStream_t)stream);
    if (e != cudaSuccess) return op_err(MLXCAT_E_CUDA, "draft: %s", cudaGetErrorString(e));
    return MLXCAT_OK;
}

size_t mlxcat_op_accept_workspace(int32_t rows, int32_t k) {
    const size_t n = (size_t)rows * (k + 1);
    return n * 4 + n * 4 + n * 8 + n * 8 + n * 4 + argmax_scratch_words((int)n) * 8 + n * 4 + 2560;
}

int mlxcat_op_accept(const mlxcat_rows *rows, const mlxcat_spec_config *spec, const int32_t *vtok,
                     const int32_t *count, const float *logits, int32_t vocab, int32_t *tokens, int32_t *n,
                     int32_t *finished, uint64_t *stats, void *ws, size_t ws_bytes, void *stream) {
    if (!rows || !spec || !vtok || !count || !logits || !tokens || !n || !finished || !stats || vocab <= 0)
        return op_err(MLXCAT_E_INVALID, "bad accept arguments");
    if (spec->max_proposal < 0 || spec->max_proposal > 16) return op_err(MLXCAT_E_INVALID, "bad k");
    const SpecParams sp = params_of(spec);
    const size_t need = mlxcat_op_accept_workspace(rows->rows, sp.k);
    if (!ws || ws_bytes < need) return op_err(MLXCAT_E_INVALID, "workspace of %zu bytes required", need);
    const size_t cnt = (size_t)rows->rows * (sp.k + 1);
    char *p = static_cast<char *>(ws);
    auto take = [&](size_t bytes) { void *q = p; p += (bytes + 255) & ~(size_t)255; return q; };
    SampleScratch sc;
    sc.S = static_cast<unsigned long long *>(take(cnt * 8));
    sc.Pd = static_cast<unsigned long long *>(take(cnt * 8));
    sc.m = static_cast<float *>(take(cnt * 4));
    sc.thr = static_cast<uint32_t *>(take(cnt * 4));
    int32_t *amax = static_cast<int32_t *>(take(cnt * 4));
    unsigned long long *amax_part = static_cast<unsigned long long *>(take(argmax_scratch_words((int)cnt) * 8));
    unsigned *amax_ctr = static_cast<unsigned *>(take(cnt * 4));
    (void)p;
    cudaStream_t st = (cudaStream_t)stream;
    StepOut out;
    out.tokens = tokens; out.n = n; out.finished = finished;
    out.stats = reinterpret_cast<unsigned long long *>(stats);
    cudaError_t e = cudaMemsetAsync(amax_ctr, 0, cnt * 4, st);
    if (e == cudaSuccess) e = argmax_rows(logits, (int)cnt, vocab, amax, st, amax_part, amax_ctr);
    if (e == cudaSuccess) e = accept_greedy(rows_of(rows), sp, vtok, count, amax, out, st);
    if (e == cudaSuccess) e = accept_sampled(rows_of(rows), sp, vtok, count, logits, vocab, sc, out, st);
    if (e != cudaSuccess) return op_err(MLXCAT_E_CUDA, "accept: %s", cudaGetErrorString(e));
    return MLXCAT_OK;
}

}  // extern "C"
