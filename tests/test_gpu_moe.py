"""Sparse MoE MLP (Qwen3-MoE shape) on the GPU against the CPU oracle.

* weights: expert q4 tensors and the bf16 router synthesised bit-identically;
* mlxcat_op_moe on the same fp16 input as the oracle: the router's fp32
  accumulation order is pinned on both sides, so the bf16 logits, and with
  them the expert ids of every token, are identical; renormalised weights
  within 1e-5, outputs within 2e-2 of the output scale -- at a small shape
  and at the Qwen3-30B-A3B shape (128 experts, top-8, hidden 2048, M = 320);
* the verify forward of a MoE model against the oracle's forward on every
  row and verify position: the router's logits are bf16 by spec and the
  device's router input is fp16, so a logit can round to the neighbouring
  bf16 value -- which moves its routing weight by up to a bf16 step of the
  logit and can resolve a near tie the other way.  The oracle therefore takes
  the device's expert choices and weights, and the test bounds both against
  the oracle's own: every forced choice within NEAR_TIE_STEPS bf16 steps,
  every forced weight within WEIGHT_RTOL; the logits then agree within 2e-2;
* batch invariance (the reference's own MoE gate,
  Tests/MLXCatTests/MoEBatchIntegrationTests.swift:37: batched greedy tokens
  equal single-row tokens)."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")
if not torch.cuda.is_available():
    pytest.skip("needs a CUDA device", allow_module_level=True)

import mlxcat_b200 as M  # noqa: E402
from mlxcat_b200 import _abi as A  # noqa: E402
from oracle import oracle as O  # noqa: E402
from tests.gpu_util import dev, ptr  # noqa: E402

L = A.lib()
TOL = 2e-2
NEAR_TIE_STEPS = 2.0   # a forced choice may differ from the oracle's only within this many bf16 steps
WEIGHT_RTOL = 2e-2     # two bf16 steps of a logit of magnitude <= 2.5 move exp(logit) by at most ~2 %

MOE_SMALL = M.ModelConfig(2, 512, 8, 2, 64, 256, 4096, False, True, 1e-6, 1e6, name="moe-small",
                          n_experts=32, top_k=4, norm_topk=True)
# Qwen3-30B-A3B layer shape (hidden 2048, 32/4 heads of 128, 128 experts of
# width 768, top-8, full vocabulary) at two layers
MOE_30B = M.ModelConfig(2, 2048, 32, 4, 128, 768, 151936, False, True, 1e-6, 1e6, name="qwen3-30b-a3b-2l",
                        n_experts=128, top_k=8, norm_topk=True)


def oracle_model(cfg, seed):
    ocfg = O.make_config(cfg.n_layers, cfg.hidden, cfg.n_heads, cfg.n_kv_heads, cfg.head_dim,
                         cfg.intermediate, cfg.vocab, cfg.tie_embeddings, cfg.qk_norm, cfg.rms_eps,
                         cfg.rope_theta, cfg.n_experts, cfg.top_k, cfg.norm_topk)
    return O.Model.synth(ocfg, seed, 0.02)


def segment_prompt(vocab, n_seg, seg_len, length, seed):
    rng = np.random.default_rng(seed)
    pool = rng.integers(0, vocab, size=(n_seg, seg_len))
    out = []
    while len(out) < length:
        out += pool[rng.integers(0, n_seg)].tolist()
    return out[:length]


def test_moe_weights_synth_bit_identical():
    cfg = MOE_SMALL
    ctx = M.Context(cfg)
    ctx.synth_weights(42)
    om = oracle_model(cfg, 42)
    I, H, E = cfg.intermediate, cfg.hidden, cfg.n_experts
    for layer, e in ((0, 0), (1, 17), (1, E - 1)):
        for kind, (N, K) in enumerate(((I, H), (I, H), (H, I))):
            tid = O.tensor_expert(layer, e, kind)
            got = ctx.get_q4(tid, N, K)
            for g, w in zip(got, om.get_q4(tid)):
                np.testing.assert_array_equal(g, w)
    for layer in range(cfg.n_layers):
        rid = layer * 16 + 7
        np.testing.assert_array_equal(ctx.get_bf16(rid, (E, H)), O.router_synth(42, rid, 0.02, E, H))


def stacked(om, layer, cfg):
    """gate, up, down of every expert of a layer in the SwitchLinear layout"""
    out = []
    for kind in range(3):
        parts = [om.get_q4(O.tensor_expert(layer, e, kind)) for e in range(cfg.n_experts)]
        out.append(tuple(np.ascontiguousarray(np.stack([p[i] for p in parts])) for i in range(3)))
    return out


@pytest.mark.parametrize("cfg,M_tok", [(MOE_SMALL, 48), (MOE_SMALL, 300), (MOE_30B, 320)],
                         ids=["small-48", "small-300", "30b-a3b-320"])
def test_op_moe_matches_oracle(cfg, M_tok):
    om = oracle_model(cfg, 5)
    H, I, E, TK = cfg.hidden, cfg.intermediate, cfg.n_experts, cfg.top_k
    rng = np.random.default_rng(M_tok)
    x = rng.standard_normal((M_tok, H)).astype(np.float16)
    y_ref, ids_ref, w_ref, margin = om.moe_mlp(1, x.astype(np.float32))
    W = stacked(om, 1, cfg)
    dW = [[dev(t) for t in w] for w in W]
    router = dev(O.router_synth(5, 1 * 16 + 7, 0.02, E, H).view(np.int16))
    xd = dev(x.view(np.int16))
    y = torch.zeros((M_tok, H), dtype=torch.float32, device="cuda")
    ids = torch.zeros((M_tok, TK), dtype=torch.int32, device="cuda")
    wts = torch.zeros((M_tok, TK), dtype=torch.float32, device="cuda")
    ws_bytes = L.mlxcat_op_moe_workspace(M_tok, H, I, E, TK)
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device="cuda")
    wq = A._vp3(*[dW[k][0].data_ptr() for k in range(3)])
    sc = A._vp3(*[dW[k][1].data_ptr() for k in range(3)])
    bi = A._vp3(*[dW[k][2].data_ptr() for k in range(3)])
    for _ in range(2):   # a second call on the same workspace gives the same result
        A.check(L.mlxcat_op_moe(ptr(xd), M_tok, H, I, E, TK, 1, ptr(router), wq, sc, bi, ptr(y), ptr(ids),
                                ptr(wts), ptr(ws), ws_bytes, None))
        torch.cuda.synchronize()
        yg, ig, wg = y.cpu().numpy(), ids.cpu().numpy(), wts.cpu().numpy()
        # same operand, same pinned accumulation order: identical routing on every token
        np.testing.assert_array_equal(ig, ids_ref)
        np.testing.assert_allclose(wg, w_ref, rtol=1e-5, atol=1e-7)
        scale = float(np.abs(y_ref).max())
        np.testing.assert_allclose(yg, y_ref, rtol=TOL, atol=TOL * scale)
        np.testing.assert_allclose(wg.sum(1), 1.0, rtol=1e-5)


def moe_verify_against_oracle(cfg, rows, ctx_len, k, seed):
    """Device verify forward of every row vs the oracle's forward over the same
    padded verify tokens, with the oracle's expert choices and weights forced
    to the device's (admission and verify forwards); returns the largest
    distance, in bf16 steps, between a forced choice and the oracle's own, and
    the largest relative difference between a forced weight and the oracle's
    own.  Prompt KV comes from a prefix-cache import of random fp16
    keys/values, so each admission computes one position (the last prompt
    token) on both sides."""
    ctx = M.Context(cfg)
    ctx.synth_weights(seed)
    om = oracle_model(cfg, seed)
    K1, L = k + 1, cfg.n_layers
    max_len = ctx_len + 64
    prompts = [segment_prompt(cfg.vocab, 6, 12, ctx_len - (r % 3), 300 + r) for r in range(rows)]
    spec = M.SpeculativeDecodingConfiguration(True, k, 3, 8, A.ACCEPT_PREFIX)
    cache = M.BatchKVCache(ctx, rows, max_len)
    kv = O.KV(om, rows, max_len)
    rng = np.random.default_rng(seed)
    O.moe_force_deviation(reset=True)
    O.moe_force_weight_deviation(reset=True)
    for r, p in enumerate(prompts):
        shape = (L, cfg.n_kv_heads, len(p) - 1, cfg.head_dim)
        kp = rng.standard_normal(shape).astype(np.float16)
        vp = rng.standard_normal(shape).astype(np.float16)
        first = cache.insert_row_prefix(r, p, kp, vp, 32, M.SamplingParameters())
        for l in range(L):
            kv.k(r, l, cfg.n_kv_heads, cfg.head_dim)[:, :len(p) - 1] = kp[l].astype(np.float32)
            kv.v(r, l, cfg.n_kv_heads, cfg.head_dim)[:, :len(p) - 1] = vp[l].astype(np.float32)
        rt = [cache.moe_routing(l) for l in range(L)]
        O.moe_force(np.stack([x[0] for x in rt]), np.stack([x[1] for x in rt]))
        ol = O.forward(om, kv, [p[-1]], [r], [len(p) - 1])[0]
        top2 = np.sort(ol)[-2:]
        assert first == int(np.argmax(ol)) or top2[1] - top2[0] < 1e-2, (r, first)
    hist = [cache.history(r) for r in range(rows)]
    drafts = cache.draft(spec)
    logits = cache.verify_forward(spec)
    rt = [cache.moe_routing(l) for l in range(L)]
    routing, weights = np.stack([x[0] for x in rt]), np.stack([x[1] for x in rt])
    assert routing.shape[1] == rows * K1
    toks, trow, tpos = [], [], []
    for r in range(rows):
        d = drafts[r]
        toks += [hist[r][-1]] + d + [hist[r][-1]] * (k - len(d))   # the device's padded verify tokens
        trow += [r] * K1
        tpos += list(range(len(prompts[r]), len(prompts[r]) + K1))
    O.moe_force(routing, weights)
    ol = O.forward(om, kv, toks, trow, tpos)
    dist = O.moe_force_deviation(reset=True)
    wdev = O.moe_force_weight_deviation(reset=True)
    O.moe_force(None)
    for r in range(rows):   # every verify position, the padding too
        np.testing.assert_allclose(logits[r], ol[r * K1:(r + 1) * K1], rtol=TOL, atol=TOL)
    tok, n, fin, stats = cache.accept(spec)
    lens = cache.lengths()
    for r in range(rows):
        assert lens[r] == len(prompts[r]) + int(n[r])
    return dist, wdev


def test_moe_verify_logits_match_oracle():
    dist, wdev = moe_verify_against_oracle(MOE_SMALL, 2, 72, 4, 7)
    assert dist <= NEAR_TIE_STEPS, f"a device expert choice is {dist} bf16 steps from the oracle's"
    assert wdev <= WEIGHT_RTOL, f"a device routing weight is {wdev:.3g} (relative) from the oracle's"


def test_moe_30b_shape_verify_matches_oracle():
    """Qwen3-30B-A3B shapes (128 experts, top-8, hidden 2048, vocab 151936) at
    64 rows x (k+1 = 5) = 320 verify tokens over 1024-token contexts."""
    dist, wdev = moe_verify_against_oracle(MOE_30B, 64, 1024, 4, 31)
    assert dist <= NEAR_TIE_STEPS, f"a device expert choice is {dist} bf16 steps from the oracle's"
    assert wdev <= WEIGHT_RTOL, f"a device routing weight is {wdev:.3g} (relative) from the oracle's"


def test_moe_batched_rows_match_single_row_runs():
    """MoEBatchIntegrationTests.swift:37-95 on the device: a row's greedy tokens
    do not depend on its neighbours (expert columns are computed independently)."""
    cfg = MOE_SMALL
    ctx = M.Context(cfg)
    ctx.synth_weights(9)
    prompts = [segment_prompt(cfg.vocab, 4, 20, L, 50 + i) for i, L in enumerate([96, 64, 120])]
    spec = M.SpeculativeDecodingConfiguration(True, 4, 3, 8, A.ACCEPT_PREFIX)

    def run(ps):
        sched = M.Scheduler(ctx, len(ps), 256, spec)
        for i, p in enumerate(ps):
            sched.submit(M.Request(f"r{i}", p, 24, M.SamplingParameters()))
        out = {f"r{i}": [] for i in range(len(ps))}
        while not sched.is_idle:
            for r in sched.step():
                out[r.uid].append(r.token)
        return out

    together = run(prompts)
    for i, p in enumerate(prompts):
        alone = run([p])["r0"]
        assert together[f"r{i}"] == alone
