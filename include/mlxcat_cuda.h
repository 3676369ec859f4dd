/*
 * mlxcat_cuda.h -- C ABI of the B200 (sm_100a) n-gram speculative-decode path.
 *
 * A Swift shim (SwiftPM system-library target) keeps the Swift surface of
 * mlxcat's ContinuousBatchGenerator / BatchKVCache / Scheduler / TokenSampler
 * and calls these entry points in place of the MLX graph.  Plain pointers and
 * sizes only; every call returns 0 on success or a negative MLXCAT_E* code
 * (message: mlxcat_last_error / mlxcat_op_last_error).  Calls on one context
 * must be serialised by the caller (the reference runs them on the Scheduler
 * actor, Sources/MLXCat/TrackB/Scheduler.swift:13).  No CPU fallback exists:
 * without a CUDA device every compute call fails with MLXCAT_E_CUDA.
 *
 * Reference paths below are inside the mlxcat project.
 */
#ifndef MLXCAT_CUDA_H
#define MLXCAT_CUDA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#if defined(__GNUC__)
#define MLXCAT_API __attribute__((visibility("default")))
#else
#define MLXCAT_API
#endif

#define MLXCAT_OK 0
#define MLXCAT_E_INVALID (-1)   /* bad argument / shape                    */
#define MLXCAT_E_CUDA (-2)      /* CUDA runtime error or no device         */
#define MLXCAT_E_OOM (-3)       /* device allocation failed                */
#define MLXCAT_E_STATE (-4)     /* call out of order (e.g. no weights)     */

#define MLXCAT_MODEL_TRANSFORMER 0   /* Llama / Qwen3 dense, MLX affine q4 g64   */
#define MLXCAT_MODEL_TABLE 1         /* next-token table (the reference's fake
                                        LanguageModel test doubles)            */

#define MLXCAT_ACCEPT_COMPAT 0  /* BatchGenerator.swift:906-940 semantics   */
#define MLXCAT_ACCEPT_PREFIX 1  /* batched prefix match / rejection sampling */

#define MLXCAT_MAX_PROPOSAL 8   /* k upper bound                           */
#define MLXCAT_MAX_EOS 8

/* Model description.  Replaces the model half of mlx-swift-lm's
 * LanguageModel as injected through LanguageModelBox (Scheduler.swift:5-11,
 * 68-89). */
typedef struct {
    int32_t kind;                 /* MLXCAT_MODEL_*                         */
    int32_t n_layers, hidden, n_heads, n_kv_heads, head_dim, intermediate, vocab;
    int32_t tie_embeddings;       /* lm_head = embedding table              */
    int32_t qk_norm;              /* Qwen3 per-head q/k RMSNorm             */
    float rms_eps, rope_theta;
    int32_t group_size, bits;     /* must be 64 and 4 (MLX affine q4 g64)   */
    /* Sparse MoE MLP in every layer (Qwen3-MoE, mlx-swift-lm's SwitchGLU
     * block) when n_experts > 0: bf16 router [n_experts][hidden], top_k
     * experts per token, each a q4 SwiGLU of width `intermediate`;
     * norm_topk renormalises the k routing weights.  0 = dense MLP. */
    int32_t n_experts, top_k, norm_topk;
    /* Tensor parallelism over tp_size GPUs (0 or 1: off), this context being
     * rank tp_rank: q/k/v heads and gate/up rows split by rank (column-split),
     * o/down inputs split (row-split), one allreduce after the attention and
     * one after the MLP block of every layer (NCCL, see mlxcat_ctx_tp_connect).
     * Embedding, lm_head and norms are replicated; every rank runs the same
     * rows.  Weight and KV-cache calls on such a context address the rank's
     * slice (n_heads/tp_size heads, intermediate/tp_size MLP rows). */
    int32_t tp_size, tp_rank;
    /* Expert parallelism for MoE models over ep_size GPUs (0 or 1: off): rank
     * ep_rank holds experts [ep_rank*E/ep_size, (ep_rank+1)*E/ep_size) and runs
     * its own rows; every MoE layer stores each routed operand row straight
     * into its expert owner's memory and the owner stores the result back
     * (NVLink peer memory, see mlxcat_cache_peer_connect).  The other weights
     * are replicated.  Every rank must run the same NUMBER of forwards in the
     * same order (each inserted prompt chunk and each verify is one); their
     * token counts may differ.  A rank that stops participating makes the
     * others' next forward fail with MLXCAT_E_CUDA ("exchange timed out")
     * after about 10 s.  Not combinable with tp_size > 1. */
    int32_t ep_size, ep_rank;
} mlxcat_model_config;

/* SamplingParameters subset on the path (Sampling.swift:139-217). */
typedef struct {
    float temperature;            /* 0 = greedy                             */
    float top_p;                  /* (0,1) enables the nucleus filter       */
    uint64_t seed;                /* per-request RNG seed                   */
    int32_t has_seed;             /* request carried its own seed           */
    int32_t eos[MLXCAT_MAX_EOS];
    int32_t n_eos;
    int32_t trigger;              /* tool-call start token, -1 if none      */
} mlxcat_sampling;

/* SpeculativeDecodingConfiguration (BatchGenerator.swift:10-29) plus mode. */
typedef struct {
    int32_t mode;                 /* MLXCAT_ACCEPT_*                        */
    int32_t enabled;
    int32_t max_proposal;         /* k, 0..MLXCAT_MAX_PROPOSAL              */
    int32_t max_suffix;           /* n, >= 1                                */
    int32_t min_context;          /* >= 2                                   */
} mlxcat_spec_config;

/* SpeculativeDecodingStats (BatchGenerator.swift:31-38). */
typedef struct {
    int64_t proposed, accepted, proposal_batches, rejected_batches;
} mlxcat_stats;

typedef struct mlxcat_ctx mlxcat_ctx;
typedef struct mlxcat_cache mlxcat_cache;

/* ---- context -------------------------------------------------------------
 * replaces: model construction + MLX device stream (NativeModelEngine.swift:44-54) */
MLXCAT_API int mlxcat_ctx_create(const mlxcat_model_config *cfg, int32_t device, mlxcat_ctx **out);
/* also destroys every cache still open on the context (their handles become invalid) */
MLXCAT_API int mlxcat_ctx_destroy(mlxcat_ctx *ctx);
/* Tensor parallelism: one rank creates an id (ncclGetUniqueId), the host
 * hands the 128 bytes to every rank, each rank connects its context
 * (ncclCommInitRank; collective: all ranks call it).  NCCL is loaded at run
 * time (libnccl.so.2); without it these return MLXCAT_E_STATE.  Must precede
 * the first forward on a context with tp_size > 1.  (Expert-parallel
 * contexts use no NCCL: their caches connect, mlxcat_cache_peer_connect, which also
 * gives tensor-parallel caches the fused allreduce over peer memory.) */
MLXCAT_API int mlxcat_tp_unique_id(uint8_t id[128]);
MLXCAT_API int mlxcat_ctx_tp_connect(mlxcat_ctx *ctx, const uint8_t id[128]);
MLXCAT_API const char *mlxcat_last_error(const mlxcat_ctx *ctx);
/* the context's CUDA stream (cudaStream_t), for callers that time or order work */
MLXCAT_API int mlxcat_ctx_stream(mlxcat_ctx *ctx, void **stream);
MLXCAT_API int mlxcat_ctx_synchronize(mlxcat_ctx *ctx);
/* number of kernel launches issued by the context (graph replays count their nodes) */
MLXCAT_API int64_t mlxcat_ctx_launch_count(const mlxcat_ctx *ctx);

/* ---- weights ---------------------------------------------------------------
 * replaces: MLX QuantizedLinear / QuantizedEmbedding parameter loading.
 * tensor ids: layer*16 + {0 q,1 k,2 v,3 o,4 gate,5 up,6 down},
 * 0xFFFF0000 embedding, 0xFFFF0001 lm_head (untied only).
 * MoE models: layer*16 + 7 is the bf16 router [n_experts][hidden]
 * (mlxcat_weights_set_bf16); expert tensors are
 * MLXCAT_TENSOR_EXPERT(layer, expert, {0 gate, 1 up, 2 down}) (q4). */
#define MLXCAT_TENSOR_EXPERT(layer, expert, kind) \
    (0x40000000u | ((uint32_t)(layer) << 12) | ((uint32_t)(expert) << 2) | (uint32_t)(kind))
MLXCAT_API int mlxcat_weights_synth(mlxcat_ctx *ctx, uint64_t seed, float stddev);
MLXCAT_API int mlxcat_weights_set_q4(mlxcat_ctx *ctx, uint32_t tensor_id, const uint32_t *wq,
                          const uint16_t *scales, const uint16_t *biases);
MLXCAT_API int mlxcat_weights_get_q4(mlxcat_ctx *ctx, uint32_t tensor_id, uint32_t *wq, uint16_t *scales,
                          uint16_t *biases);
MLXCAT_API int mlxcat_weights_set_table(mlxcat_ctx *ctx, const int32_t *next_token, int32_t vocab);
/* bf16 tensors (the MoE router, id layer*16 + 7): [n_experts][hidden] */
MLXCAT_API int mlxcat_weights_set_bf16(mlxcat_ctx *ctx, uint32_t tensor_id, const uint16_t *w);
MLXCAT_API int mlxcat_weights_get_bf16(mlxcat_ctx *ctx, uint32_t tensor_id, uint16_t *w);
/* RMSNorm weights (fp32; all ones until set): id layer*16 + {8 input_layernorm,
 * 9 post_attention_layernorm, 10 q_norm, 11 k_norm} ([hidden], q/k: [head_dim],
 * Qwen3 only), MLXCAT_NORM_FINAL ([hidden]).  Replaces the RMSNorm parameter
 * loading of the mlx-swift-lm model (un-vendored). */
#define MLXCAT_NORM_FINAL 0xFFFF0002u
#define MLXCAT_NORM(layer, kind) ((uint32_t)(layer) * 16u + 8u + (uint32_t)(kind))
MLXCAT_API int mlxcat_weights_set_norm(mlxcat_ctx *ctx, uint32_t norm_id, const float *w);
/* bytes of q4 weights one forward streams (packed words + scales + biases) */
MLXCAT_API int64_t mlxcat_weights_bytes(const mlxcat_ctx *ctx);

/* ---- cache: BatchKVCache + per-row generator state --------------------------
 * replaces: BatchKVCache (BatchCache.swift:37-89) and the per-row arrays of
 * ContinuousBatchGenerator (BatchGenerator.swift:144-215) on the device.
 * Layout: K and V fp16 [layer][row][kv_head][max_len][head_dim], right-ragged
 * with one length per row. */
MLXCAT_API int mlxcat_cache_create(mlxcat_ctx *ctx, int32_t max_rows, int32_t max_len, mlxcat_cache **out);
MLXCAT_API int mlxcat_cache_destroy(mlxcat_cache *cache);
/* Expert parallelism (ep_size > 1) and the fused tensor-parallel allreduce
 * (tp_size > 1): each rank's cache owns one device region (expert parallel:
 * receive slabs, return rows, flags; tensor parallel: scatter and gather
 * buffers of the row-split projections, flags) that every other rank maps
 * and writes over NVLink.  Each rank writes its cache's handle (a CUDA IPC
 * handle plus the region's shape), the host gathers the group's handles in
 * rank order and hands all of them to every rank's mlxcat_cache_peer_connect.
 * Caches of different shape (max_rows) are rejected with MLXCAT_E_INVALID.
 * Connect before the first insert_row.  Expert parallelism needs it; tensor
 * parallelism uses NCCL (mlxcat_ctx_tp_connect) instead while the cache is
 * not peer-connected.  No counterpart in the reference (the MLX path runs on
 * one device). */
#define MLXCAT_PEER_HANDLE_BYTES 128
MLXCAT_API int mlxcat_cache_peer_handle(mlxcat_cache *cache, uint8_t handle[MLXCAT_PEER_HANDLE_BYTES]);
MLXCAT_API int mlxcat_cache_peer_connect(mlxcat_cache *cache, const uint8_t *handles /* [group][128] */);
/* admission: prefill prompt into `row`, sample the first token (generation
 * index 0).  Scheduler.completeAdmission + generator.insert
 * (Scheduler.swift:599-668, BatchGenerator.swift:380-460).  Requires
 * len + max_new_tokens + MLXCAT_MAX_PROPOSAL + 1 <= max_len. */
MLXCAT_API int mlxcat_cache_insert_row(mlxcat_cache *cache, int32_t row, const int32_t *prompt, int32_t len,
                            int32_t max_new_tokens, const mlxcat_sampling *sampling,
                            int32_t *first_token);
/* Admission on a prefix-cache hit: the reference installs the KV its prefix
 * cache reconstructed for the first `prefix_len` prompt tokens and prefills
 * only positions [prefix_len, len) (Scheduler.swift:931-985 prepareHitRow,
 * TrackA/BlockAwarePrefixCache.swift:57-87 reconstructCache).  k_prefix and
 * v_prefix: host fp16 [n_layers][n_kv_heads][prefix_len][head_dim] (the
 * rank's heads when tensor-parallel), copied into the row's cache slots; then
 * the rest of the prompt is prefilled and the first token sampled as in
 * mlxcat_cache_insert_row.  0 <= prefix_len < len (a full match is shortened
 * by the caller, as the reference does, so one position produces logits). */
MLXCAT_API int mlxcat_cache_insert_row_prefix(mlxcat_cache *cache, int32_t row, const int32_t *prompt,
                                              int32_t len, int32_t prefix_len, const uint16_t *k_prefix,
                                              const uint16_t *v_prefix, int32_t max_new_tokens,
                                              const mlxcat_sampling *sampling, int32_t *first_token);
/* generator.remove(uid:) */
MLXCAT_API int mlxcat_cache_remove_row(mlxcat_cache *cache, int32_t row);
/* BatchKVCache.trim(n) (BatchCache.swift:403-424): every row loses
 * min(n, its length); *trimmed = min(n, longest row) */
MLXCAT_API int mlxcat_cache_trim(mlxcat_cache *cache, int32_t n, int32_t *trimmed);
/* BatchKVCache.filter(keeping:) (BatchCache.swift:217-245): every row not
 * listed in keep[0..n) is removed as by mlxcat_cache_remove_row; listed rows
 * stay active in their slot (the device batch is addressed by slot, so no KV
 * moves and the caller's row-to-slot map is unchanged).  n = 0 removes all. */
MLXCAT_API int mlxcat_cache_filter(mlxcat_cache *cache, const int32_t *keep, int32_t n);
/* trim(n) for one row: the right-ragged form of BatchCache.swift:403-424 --
 * the row's KV loses min(n, its length) positions; *trimmed (may be NULL)
 * receives that count.  Like mlxcat_cache_trim it changes KV lengths only. */
MLXCAT_API int mlxcat_cache_trim_row(mlxcat_cache *cache, int32_t row, int32_t n, int32_t *trimmed);
/* per-row KV lengths (BatchKVCache.offset / ropeOffset) */
MLXCAT_API int mlxcat_cache_lengths(mlxcat_cache *cache, int32_t *out_rows);
/* speculativeTokenHistory[row] (BatchGenerator.swift:452-456, 1012-1014) */
MLXCAT_API int mlxcat_cache_history(mlxcat_cache *cache, int32_t row, int32_t *out, int32_t cap,
                         int32_t *len);
/* BatchKVCache.extract(row) state: fp16 [n_kv][len][head_dim] for one layer */
MLXCAT_API int mlxcat_cache_extract_row(mlxcat_cache *cache, int32_t row, int32_t layer, uint16_t *k_out,
                             uint16_t *v_out);
MLXCAT_API int mlxcat_cache_active(mlxcat_cache *cache, int32_t *out_rows);
/* Expert routing of the last forward on a MoE model (the SwitchGLU gate's
 * top-k choice, un-vendored mlx-swift-lm Qwen3-MoE): ids and renormalised
 * weights [M][top_k] of `layer`, M = the last forward's token count (rows x
 * (k+1) after a verify forward), returned in *m.  Inspection for tests and
 * hosts that log routing; either output may be NULL. */
MLXCAT_API int mlxcat_cache_moe_routing(mlxcat_cache *cache, int32_t layer, int32_t *ids, float *weights,
                                        int32_t *m);


/* ---- hot path ----------------------------------------------------------------
 * mlxcat_draft: proposeSuffixTokens for every row (BatchGenerator.swift:982-1010)
 *   with the gate and limit of :877-892, :957-975.
 *   drafts: [max_rows][k] (unused slots repeat the current token), counts: [max_rows].
 * mlxcat_verify_forward: the (k+1)-token verify forward of :897-904 for every
 *   row on the tokens [current, drafts...]; KV appended at each row's length;
 *   logits [max_rows][k+1][vocab] fp32 (NULL to skip the copy).  Lengths are
 *   NOT advanced (mlxcat_accept does that).
 * mlxcat_accept: the acceptance loop + rollback of :906-954 on the logits of
 *   the last verify forward; tokens [max_rows][k+1], counts [max_rows].
 * mlxcat_spec_step: draft -> verify -> accept fused on the device, one host
 *   synchronisation per step (replays a CUDA graph per configuration).
 *   With spec->enabled == 0 it is one ordinary decode step. */
MLXCAT_API int mlxcat_draft(mlxcat_cache *cache, const mlxcat_spec_config *spec, int32_t *drafts,
                 int32_t *counts);
MLXCAT_API int mlxcat_verify_forward(mlxcat_cache *cache, const mlxcat_spec_config *spec, float *logits);
MLXCAT_API int mlxcat_accept(mlxcat_cache *cache, const mlxcat_spec_config *spec, int32_t *out_tokens,
                  int32_t *out_counts, int32_t *out_finished, mlxcat_stats *stats);
/* Grammar-constrained speculation (the device side of the allow masks of
 * Sampling.swift:557-590, which today keep a grammar row out of speculation,
 * BatchGenerator.swift:957-975).  A grammar's allowed set at verify position p
 * depends on drafts 0..p-1, so the host runs mlxcat_draft, advances its matcher
 * along each row's drafts, and sets one allowed-token bitset per row and
 * position: bits [max_rows][k+1][ceil(vocab/32)] (bit v of word v/32 = token v
 * allowed), enabled [max_rows][k+1] (0 = that position is unconstrained).  The
 * next mlxcat_accept sets every disallowed logit to -inf before it samples or
 * takes the argmax; a position whose set holds no valid token id is left
 * unchanged (as applyAllowedTokenMask does).  The masks are consumed by that
 * acceptance; enabled == NULL clears pending masks.  While masks are pending,
 * mlxcat_spec_step returns MLXCAT_E_STATE (its drafts are not known on the
 * host before it runs). */
MLXCAT_API int mlxcat_cache_set_token_masks(mlxcat_cache *cache, int32_t k, const uint32_t *bits,
                                            const uint8_t *enabled);
MLXCAT_API int mlxcat_spec_step(mlxcat_cache *cache, const mlxcat_spec_config *spec, int32_t *out_tokens,
                     int32_t *out_counts, int32_t *out_finished, mlxcat_stats *stats);
/* device time (ms) of the verify forward inside the last mlxcat_spec_step */
MLXCAT_API int mlxcat_last_verify_ms(mlxcat_cache *cache, float *ms);
/* device time (ms) of the whole last mlxcat_spec_step (draft through the
 * device-to-host copy of its outputs) */
MLXCAT_API int mlxcat_last_step_ms(mlxcat_cache *cache, float *ms);
/* Per-kernel CUDA-event timing inside the captured step (off by default):
 * when enabled, every q4 linear and attention launch of the verify forward is
 * bracketed by events; mlxcat_cache_profile returns the summed device time of
 * each class in the last step and the number of launches timed. */
MLXCAT_API int mlxcat_cache_set_profiling(mlxcat_cache *cache, int32_t enabled);
MLXCAT_API int mlxcat_cache_profile(mlxcat_cache *cache, float *q4_linear_ms, float *attention_ms,
                                    int32_t *q4_linear_launches, int32_t *attention_launches);

/* ---- device-pointer operators ------------------------------------------------
 * Stream-ordered kernels on caller-owned device memory (fp16 passed as
 * uint16_t).  `stream` is a cudaStream_t (NULL = legacy default stream).
 * Operators that need scratch take a caller-owned device workspace whose size
 * the matching *_workspace query returns. */
MLXCAT_API const char *mlxcat_op_last_error(void);

/* quantizedMatmul (mlx-swift, called by QuantizedLinear): y[M][N] fp32 =
 * x[M][K] fp16 . dequant(W)^T, W MLX affine q4 g64 (tcgen05 tensor cores).
 * The workspace holds the re-ordered activations, the scales and biases
 * re-packed per 512-wide k unit, split-K partials and tickets, and a device
 * error flag (non-zero after a pipeline wait timed out). */
MLXCAT_API size_t mlxcat_op_q4_linear_workspace(int32_t N, int32_t K, int32_t M);
MLXCAT_API int mlxcat_op_q4_linear(const uint32_t *wq, const uint16_t *scales, const uint16_t *biases,
                        int32_t N, int32_t K, const uint16_t *x, int32_t M, float *y,
                        void *workspace, size_t workspace_bytes, void *stream);

/* MLXFast.scaledDotProductAttention with the causal mask of CausalMask.swift:4-28
 * on a right-ragged cache.  q [M][n_heads][head_dim] fp16; token m belongs
 * to row trow[m] at position tpos[m] and sees keys 0..tpos[m]; tokens come in
 * groups of `qg` consecutive positions of one row.  out [M][n_heads*head_dim]. */
MLXCAT_API size_t mlxcat_op_attention_workspace(int32_t M, int32_t qg, int32_t n_heads, int32_t n_kv_heads,
                                     int32_t head_dim, int32_t max_len);
MLXCAT_API int mlxcat_op_attention(const uint16_t *q, const uint16_t *k_cache, const uint16_t *v_cache,
                        int32_t max_len, const int32_t *trow, const int32_t *tpos, int32_t M,
                        int32_t qg, int32_t n_heads, int32_t n_kv_heads, int32_t head_dim,
                        uint16_t *out, void *workspace, size_t workspace_bytes, void *stream);

/* The same attention for a prompt chunk (the admission prefill,
 * Scheduler.swift:599-668), on the tensor cores: n tokens of cache row `row`
 * at positions s0..s0+n-1, each seeing keys 0..its position.  q [n][n_heads *
 * head_dim], out [n][n_heads * head_dim] fp16; caches as above with `rows`
 * rows; head_dim 128.  err: a device int the kernel sets when a pipeline wait
 * timed out (0 otherwise).  No workspace. */
MLXCAT_API int mlxcat_op_prefill_attention(const uint16_t *q, const uint16_t *k_cache, const uint16_t *v_cache,
                                           int32_t rows, int32_t max_len, int32_t row, int32_t s0, int32_t n,
                                           int32_t n_heads, int32_t n_kv_heads, int32_t head_dim, uint16_t *out,
                                           int32_t *err, void *stream);

/* Sparse MoE MLP: the SwitchGLU block of mlx-swift-lm's Qwen3-MoE model
 * (un-vendored) that the verify forward (BatchGenerator.swift:900) runs in
 * every layer of a MoE model, on an already normalised input x [M][hidden]
 * fp16.  router: bf16 [n_experts][hidden]; wq/scales/biases[0..2]: gate and up
 * [n_experts][intermediate][hidden/8] and down [n_experts][hidden][intermediate/8]
 * (the MLX SwitchLinear layout; scales/biases [n_experts][N][K/64]).
 * Routing: bf16 logits, fp32 softmax, top_k largest (ties to the lower
 * index), weights renormalised over the k when norm_topk.
 * y [M][hidden] fp32 = sum_j w_j down_e(silu(gate_e x) * up_e x); ids and
 * weights [M][top_k] (each may be NULL) receive the routing. */
MLXCAT_API size_t mlxcat_op_moe_workspace(int32_t M, int32_t hidden, int32_t intermediate, int32_t n_experts,
                                          int32_t top_k);
MLXCAT_API int mlxcat_op_moe(const uint16_t *x, int32_t M, int32_t hidden, int32_t intermediate,
                             int32_t n_experts, int32_t top_k, int32_t norm_topk, const uint16_t *router,
                             const uint32_t *const wq[3], const uint16_t *const scales[3],
                             const uint16_t *const biases[3], float *y, int32_t *ids, float *weights,
                             void *workspace, size_t workspace_bytes, void *stream);

/* No counterpart in the reference: the attention operator above for callers
 * that cannot allocate device memory.  Same arguments and result as
 * mlxcat_op_attention, but its scratch lives in a fixed device array of
 * MLXCAT_NOALLOC_ATTN_SCRATCH_BYTES inside the library (held on every GPU that
 * loads it until exit); a shape whose mlxcat_op_attention_workspace exceeds
 * that size is rejected with MLXCAT_E_INVALID.  It allocates nothing.  Each
 * call made outside a stream capture resolves the array's address on the
 * current device with cudaGetSymbolAddress (the first such call can load the
 * library's device code on that device; after a device reset it picks up the
 * new address); a call inside a capture uses the address found by the
 * device's last uncaptured call, so make one call on each device before any
 * stream capture (a first call inside a capture returns MLXCAT_E_STATE).  All
 * calls share the one array, so calls whose kernels overlap on the GPU
 * (different streams without ordering) race on it. */
#define MLXCAT_NOALLOC_ATTN_SCRATCH_BYTES (16u << 20)
MLXCAT_API int mlxcat_op_attention_noalloc(const uint16_t *q, const uint16_t *k_cache, const uint16_t *v_cache,
                        int32_t max_len, const int32_t *trow, const int32_t *tpos, int32_t M,
                        int32_t qg, int32_t n_heads, int32_t n_kv_heads, int32_t head_dim,
                        uint16_t *out, void *stream);

/* The prefill path's linears (Scheduler.swift:670-1016 admission prefill, which
 * runs mlx-swift's quantizedMatmul at M = prompt length): at hundreds to
 * thousands of tokens the contraction is dense, so the q4 weight is
 * dequantised once into fp16 and multiplied on the tensor cores.
 * mlxcat_op_dequant_q4: w_out fp16 [N][K] = scale * q + bias (fp16 FMA, as
 * the q4 linear dequantises).  mlxcat_op_gemm_f16: y[m][n] = sum_k x[m][k]
 * w[n][k], w fp16 [N][K] (N % 128 == 0), x fp16 [M][K] row-major (K % 64 ==
 * 0), fp32 accumulation; MLXCAT_GEMM_STORE: out fp32 [M][ldo] = y;
 * MLXCAT_GEMM_ADD: out fp32 [M][ldo] += y (residual stream);
 * MLXCAT_GEMM_SWIGLU: w is a fused gate/up matrix (per 128-row block 64 gate
 * rows then the matching 64 up rows), out fp16 [M][ldo] = silu(g) * u for
 * the N/2 outputs.  err_flag (device int, may be NULL) becomes non-zero if a
 * pipeline wait timed out. */
#define MLXCAT_GEMM_STORE 0
#define MLXCAT_GEMM_ADD 1
#define MLXCAT_GEMM_SWIGLU 2
MLXCAT_API int mlxcat_op_dequant_q4(const uint32_t *wq, const uint16_t *scales, const uint16_t *biases, int32_t N,
                                    int32_t K, uint16_t *w_out, void *stream);
MLXCAT_API int mlxcat_op_gemm_f16(const uint16_t *w, int32_t N, int32_t K, const uint16_t *x, int32_t M,
                                  int32_t epilogue, void *out, int32_t ldo, int32_t *err_flag, void *stream);

/* Seeded N(0, stddev) weights quantised to MLX affine q4 g64 (bit-identical
 * with the CPU restatement). */
MLXCAT_API int mlxcat_op_synth_q4(uint64_t seed, uint32_t tensor_id, float stddev, int32_t N, int32_t K,
                       uint32_t *wq, uint16_t *scales, uint16_t *biases, void *stream);

/* Per-row generator state on the device, for the drafter / acceptance
 * operators.  All arrays have `rows` entries (eos: rows x MLXCAT_MAX_EOS). */
typedef struct {
    int32_t *hist;                /* [rows][hist_cap]                        */
    int32_t hist_cap;
    int32_t rows;
    int32_t *hist_len, *kv_len, *n_gen, *max_new, *active;
    float *temperature, *top_p;
    uint64_t *seed;
    int32_t *has_seed, *eos, *n_eos, *trigger;
} mlxcat_rows;

/* proposeSuffixTokens + gate for every row: vtok [rows][k+1] = current token
 * then drafts (padding repeats the current token), count [rows], and the
 * verify tokens' row / position descriptors trow, tpos [rows*(k+1)]. */
MLXCAT_API int mlxcat_op_draft(const mlxcat_rows *rows, const mlxcat_spec_config *spec, int32_t *vtok,
                    int32_t *count, int32_t *trow, int32_t *tpos, void *stream);

/* Acceptance + rollback on given logits [rows][k+1][vocab] fp32 (greedy rows
 * by argmax, temperature rows by rejection sampling).  Updates the row state
 * in place; tokens [rows][k+1], n [rows], finished [rows]; stats[4] device
 * uint64 counters (proposed, accepted, proposal_batches, rejected_batches)
 * are incremented. */
MLXCAT_API size_t mlxcat_op_accept_workspace(int32_t rows, int32_t k);
MLXCAT_API int mlxcat_op_accept(const mlxcat_rows *rows, const mlxcat_spec_config *spec, const int32_t *vtok,
                     const int32_t *count, const float *logits, int32_t vocab, int32_t *tokens,
                     int32_t *n, int32_t *finished, uint64_t *stats, void *workspace,
                     size_t workspace_bytes, void *stream);

#ifdef __cplusplus
}
#endif
#endif
