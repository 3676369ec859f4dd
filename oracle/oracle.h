/*
 * oracle.h -- CPU restatement of mlxcat's n-gram speculative-decode path.
 *
 * TEST INFRASTRUCTURE ONLY.  This library is the checker for the CUDA
 * implementation in mlxcat_b200/csrc.  Only tests/, __graft_entry__.smoke()
 * and bench.py's cpu_baseline / --impl reference legs may load it.  The
 * product never links, loads or calls anything here.
 *
 * Parity pinning:
 *   - drafter, gate, acceptance, stats, history: restated from
 *     Sources/MLXCat/TrackB/BatchGenerator.swift:875-1035 and pinned by the
 *     known-answer tests of Tests/MLXCatTests/SchedulerSpeculativeDecodingTests.swift
 *     (restated in tests/test_oracle_kat.py with the same fake models);
 *   - top-p keep rule: Sources/MLXCat/TrackB/Sampling.swift:847-858, pinned by
 *     Tests/MLXCatTests/TopPSamplingTests.swift:10-54;
 *   - KV trim: Sources/MLXCat/TrackB/BatchCache.swift:403-424, pinned by
 *     Tests/MLXCatTests/BatchCacheShapeTests.swift:170-193.
 *   - q4 linear / attention / RoPE / RMSNorm arithmetic lives in the
 *     un-vendored mlx-swift (ea227ae6) and mlx-swift-lm (dcfa3aa1); the
 *     reference ships no test vectors for it that run without real
 *     checkpoints, so that part is "parity unpinned" against mlxcat and is
 *     restated from the published MLX affine format (w = scale*q + bias,
 *     8 nibbles per uint32, lowest nibble first, group 64).
 *   - single-draft rejection sampling, fixed-point distributions and the
 *     Philox uniform streams are extensions with no reference counterpart;
 *     they are defined here and the CUDA kernels must match them bit-exactly.
 */
#ifndef MLXCAT_ORACLE_H
#define MLXCAT_ORACLE_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- deterministic arithmetic (bit-identical with the device versions) --- */
/* OpenMP threads of the parallel loops below (n < 1: every host core);
 * returns the count in effect.  Hosts launched by torchrun inherit
 * OMP_NUM_THREADS=1, which would serialise the CPU baseline. */
int orc_set_threads(int n);
void orc_philox4x32_10(const uint32_t ctr[4], const uint32_t key[2], uint32_t out[4]);
float orc_exp_neg(float x);          /* e^x for x <= 0 (0 below -87)          */
float orc_log(float x);              /* natural log, x > 0 normal             */
uint16_t orc_f32_to_f16(float x);    /* IEEE round-to-nearest-even            */
float orc_f16_to_f32(uint16_t h);
float orc_normal(uint64_t seed, uint32_t tensor_id, uint64_t index);
uint32_t orc_uniform_u32(uint64_t seed, uint64_t gen_index, uint32_t purpose);

/* ---- MLX affine 4-bit, group 64 ------------------------------------------ */
void orc_q4_quantize_row(const float *w, int K, uint32_t *wq, uint16_t *scales,
                         uint16_t *biases);
void orc_q4_synth(uint64_t seed, uint32_t tensor_id, float stddev, int N, int K,
                  uint32_t *wq, uint16_t *scales, uint16_t *biases);
void orc_q4_dequant(const uint32_t *wq, const uint16_t *scales, const uint16_t *biases,
                    int N, int K, float *w);
/* y[M,N] = x[M,K] . dequant(W)^T, fp32 */
void orc_q4_linear(const uint32_t *wq, const uint16_t *scales, const uint16_t *biases,
                   int N, int K, const float *x, int M, float *y);

/* ---- drafter (BatchGenerator.swift:982-1010) ------------------------------ */
int orc_propose_suffix(const int32_t *ctx, int n_ctx, int max_suffix, int min_ctx,
                       int limit, int32_t *out);

/* ---- sampling ------------------------------------------------------------- */
int orc_argmax(const float *logits, int V);
/* top-p keep mask (Sampling.swift:847-858), fixed-point restatement */
void orc_top_p_keep(const float *logits, int V, float top_p, uint8_t *keep);
/* fixed-point tempered distribution: P[i] (2^24 scale); returns sum */
uint64_t orc_fixed_dist(const float *logits, int V, float temperature, float top_p,
                        uint32_t *P);
/* inverse-CDF pick of T=floor(u*S/2^32) in token order, skipping `skip` */
int orc_pick(const uint32_t *P, int V, uint64_t S, uint32_t u, int skip);

/* ---- per-row acceptance (one verify step) --------------------------------- */
enum { ORC_MODE_COMPAT = 0, ORC_MODE_PREFIX = 1 };
typedef struct {
    float temperature;
    float top_p;
    uint64_t seed;
    int32_t has_seed;           /* request carried its own seed           */
    int32_t eos[8];
    int32_t n_eos;
    int32_t trigger;            /* tool-call start token, -1 if none */
} orc_sampling;

/* logits: (count+1) x V.  drafts: count tokens.  gen_index: tokens this request
 * has generated so far (uniform stream position).  Writes emitted tokens (<=
 * count+1) to out; returns the number emitted; *rejected = 1 when the proposal
 * was not taken whole. */
int orc_accept_row(int mode, const float *logits, int V, const int32_t *drafts, int count,
                   const orc_sampling *sp, uint64_t gen_index, int32_t *out, int *rejected);

/* ---- model ---------------------------------------------------------------- */
typedef struct {
    int n_layers, hidden, n_heads, n_kv_heads, head_dim, intermediate, vocab;
    int tie_embeddings, qk_norm;
    float rms_eps, rope_theta;
    /* sparse MoE MLP in every layer when n_experts > 0 (Qwen3-MoE): a bf16
     * router [n_experts][hidden], top_k experts per token, each expert a q4
     * SwiGLU of width `intermediate`; norm_topk renormalises the k weights */
    int n_experts, top_k, norm_topk;
} orc_config;

typedef struct orc_model orc_model;
typedef struct orc_kv orc_kv;

enum { ORC_T_Q = 0, ORC_T_K, ORC_T_V, ORC_T_O, ORC_T_GATE, ORC_T_UP, ORC_T_DOWN, ORC_T_ROUTER };
#define ORC_TENSOR_EMBED 0xFFFF0000u
#define ORC_TENSOR_LM_HEAD 0xFFFF0001u
uint32_t orc_tensor_id(int layer, int kind);
/* expert tensors: kind 0 gate, 1 up, 2 down */
#define ORC_TENSOR_EXPERT(layer, expert, kind) \
    (0x40000000u | ((uint32_t)(layer) << 12) | ((uint32_t)(expert) << 2) | (uint32_t)(kind))

/* bf16 round-to-nearest-even (NaN not produced by the callers) */
uint16_t orc_f32_to_bf16(float x);
float orc_bf16_to_f32(uint16_t h);
/* router weights: bf16(N(0, stddev)) from the weight stream of tensor
 * orc_tensor_id(layer, ORC_T_ROUTER), element index e*hidden + k */
void orc_router_synth(uint64_t seed, uint32_t tensor_id, float stddev, int E, int H,
                      uint16_t *w);
int orc_model_set_router(orc_model *m, int layer, const uint16_t *w);
/* RMSNorm weights: id = layer*16 + {8 input, 9 post-attention, 10 q, 11 k},
 * 0xFFFF0002 final (hidden or head_dim floats); -1 for an unknown id */
int orc_model_set_norm(orc_model *m, uint32_t id, const float *w);
/* MoE routing of one token (x: normalised MLP input, fp32): bf16 router
 * logits, fp32 softmax, top-k (ties to the lower expert index), optional
 * renormalisation.  Writes ids[k], weights[k]; returns the gap between the
 * k-th and (k+1)-th largest logit (the margin of the selection). */
float orc_moe_route(const orc_model *m, int layer, const float *x, int32_t *ids, float *weights);
/* smallest routing margin over all tokens routed since the last reset: a
 * parity test on a MoE model skips inputs whose expert choice is a near tie */
float orc_moe_min_margin(int reset);
/* the MoE MLP of `layer` alone on given normalised inputs x[M][hidden]:
 * y[M][hidden] += sum_j w_j expert_j(x); ids/weights [M][top_k] and routing
 * margins [M] (each may be NULL) */
/* test hook: force the expert choices of the next forwards, ids
 * [n_layers][M][top_k] (token i of a forward of M tokens), and with weights
 * (may be NULL) their routing weights too; ids NULL clears */
void orc_moe_force(int n_layers, int M, int top_k, const int32_t *ids, const float *weights);
/* largest distance, in bf16 steps, between a forced choice and the oracle's own */
float orc_moe_force_deviation(int reset);
/* largest relative difference between a forced routing weight and the oracle's own */
float orc_moe_force_weight_deviation(int reset);
void orc_moe_mlp(const orc_model *m, int layer, const float *x, int M, float *y, int32_t *ids,
                 float *weights, float *margins);

orc_model *orc_model_synth(const orc_config *cfg, uint64_t seed, float stddev);
/* table model: logits +20 at next[token], -20 elsewhere (the reference test doubles) */
orc_model *orc_model_table(const int32_t *next, int vocab);
/* model over caller-provided q4 tensors (pointers are copied) */
orc_model *orc_model_empty(const orc_config *cfg);
int orc_model_set_q4(orc_model *m, uint32_t tensor_id, const uint32_t *wq,
                     const uint16_t *scales, const uint16_t *biases);
void orc_model_get_q4(const orc_model *m, uint32_t tensor_id, const uint32_t **wq,
                      const uint16_t **scales, const uint16_t **biases, int *N, int *K);
void orc_model_free(orc_model *m);
const orc_config *orc_model_config(const orc_model *m);

orc_kv *orc_kv_create(const orc_model *m, int max_rows, int max_len);
void orc_kv_free(orc_kv *kv);
int orc_kv_len(const orc_kv *kv, int row);
void orc_kv_set_len(orc_kv *kv, int row, int len);
/* uniform trim (BatchCache.swift:403-424 semantics on a right-ragged cache):
 * every row loses min(n, len[row]) positions; returns min(n, max len) */
int orc_kv_trim(orc_kv *kv, int n);
/* raw access for state transfer: layer-major [layer][kvh][pos][d] fp32 */
float *orc_kv_k(orc_kv *kv, int row, int layer);
float *orc_kv_v(orc_kv *kv, int row, int layer);

/* forward M tokens; token m belongs to rows[m] at position pos[m]; writes its K/V
 * to the cache at pos[m] and attends causally to positions 0..pos[m] of its
 * row.  logits: M x vocab fp32 (may be NULL). */
void orc_forward(const orc_model *m, orc_kv *kv, int M, const int32_t *tokens,
                 const int32_t *rows, const int32_t *pos, float *logits);

/* ---- batched speculative step (mirrors the device step) ------------------- */
typedef struct {
    int mode;                  /* ORC_MODE_*                           */
    int enabled;
    int max_proposal;          /* k                                    */
    int max_suffix;            /* n                                    */
    int min_context;
} orc_spec_config;

typedef struct {
    int64_t proposed, accepted, proposal_batches, rejected_batches;
} orc_stats;

typedef struct {
    int32_t *hist;             /* row history: prompt + generated      */
    int hist_len, hist_cap;
    int n_gen;                 /* tokens generated so far              */
    int max_new;
    int active;
    orc_sampling sp;
} orc_row;

/* One decode step over all active rows (speculative when cfg->enabled).
 * out: rows x (k+1) emitted tokens; n_out: per-row emitted counts.
 * Histories, n_gen and kv lengths are advanced in place. */
void orc_spec_step(const orc_model *m, orc_kv *kv, orc_row *rows, int n_rows,
                   const orc_spec_config *cfg, int32_t *out, int32_t *n_out,
                   orc_stats *stats);

/* admission: prefill prompt[0..len) into row `row`, sample the first token
 * (generation index 0); returns it. */
int orc_admit(const orc_model *m, orc_kv *kv, orc_row *r, int row, const int32_t *prompt,
              int len, int chunk);

#ifdef __cplusplus
}
#endif
#endif
