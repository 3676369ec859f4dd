"""The CPU restatement of the sparse MoE MLP (Qwen3-MoE routing + expert
SwiGLU), checked on its own before it serves as the checker of the CUDA MoE
kernels.

The block's arithmetic lives in un-vendored mlx-swift-lm (dcfa3aa1); the
reference's own MoE gate (Tests/MLXCatTests/MoEBatchIntegrationTests.swift:37)
needs a real checkpoint.  These tests pin the restatement structurally:
a one-expert MoE equals the dense MLP bit for bit, and the routing agrees with
an independent numpy statement of bf16 logits -> softmax -> top-k -> renorm."""
import numpy as np

from oracle import oracle as O


def bf16_round(x):
    u = np.asarray(x, np.float32).view(np.uint32).astype(np.uint64)
    u = (u + 0x7FFF + ((u >> 16) & 1)) >> 16
    return (u.astype(np.uint32) << 16).view(np.float32)


def test_bf16_rounding_matches_numpy():
    xs = np.array([1.0, -2.5, 3.14159, 1e-3, 65504.0, 1.00390625, 1.01171875], np.float32)
    for x in xs:
        got = np.array([O.lib().orc_f32_to_bf16(float(x))], np.uint16).astype(np.uint32) << 16
        np.testing.assert_array_equal(got.view(np.float32), bf16_round(x))


def test_single_expert_moe_equals_dense_mlp():
    dense = O.make_config(2, 256, 4, 2, 64, 384, 512, True, False, 1e-5, 10000.0)
    moe = O.make_config(2, 256, 4, 2, 64, 384, 512, True, False, 1e-5, 10000.0,
                        n_experts=1, top_k=1, norm_topk=True)
    md = O.Model.synth(dense, 11, 0.02)
    mm = O.Model.synth(moe, 11, 0.02)
    for layer in range(2):
        for kind, tk in ((0, O.T_GATE), (1, O.T_UP), (2, O.T_DOWN)):
            wq, s, b = mm.get_q4(O.tensor_expert(layer, 0, kind))
            md.set_q4(O.lib().orc_tensor_id(layer, tk), wq, s, b)
    toks = [5, 17, 301, 42, 7]
    pos = list(range(len(toks)))
    kd = O.KV(md, 1, 16)
    km = O.KV(mm, 1, 16)
    ld = O.forward(md, kd, toks, [0] * len(toks), pos)
    lm = O.forward(mm, km, toks, [0] * len(toks), pos)
    np.testing.assert_array_equal(ld, lm)


def test_routing_matches_numpy_statement():
    cfg = O.make_config(1, 512, 4, 2, 64, 128, 256, True, False, 1e-5, 10000.0,
                        n_experts=32, top_k=4, norm_topk=True)
    m = O.Model.synth(cfg, 5, 0.02)
    W = O.router_synth(5, O.lib().orc_tensor_id(0, O.T_ROUTER), 0.02, 32, 512)
    Wf = (W.astype(np.uint32) << 16).view(np.float32).astype(np.float64)
    rng = np.random.default_rng(3)
    checked = 0
    for _ in range(50):
        x = rng.standard_normal(512).astype(np.float32)
        ids, w, margin = m.route(0, x)
        lg = bf16_round((Wf @ x.astype(np.float64)).astype(np.float32)).astype(np.float64)
        order = np.lexsort((np.arange(32), -lg))
        assert abs(w.sum() - 1.0) < 1e-5
        if margin < 1e-2:
            continue
        np.testing.assert_array_equal(ids, order[:4])
        p = np.exp(lg - lg.max())
        p /= p.sum()
        np.testing.assert_allclose(w, p[order[:4]] / p[order[:4]].sum(), rtol=1e-4, atol=1e-6)
        checked += 1
    assert checked >= 30


def test_router_weights_are_bf16_normals():
    W = O.router_synth(9, 7, 0.02, 8, 256)
    f = (W.astype(np.uint32) << 16).view(np.float32)
    assert abs(float(f.std()) - 0.02) < 0.003
    # every value is the bf16 rounding of the weight stream's normal
    for i in (0, 1, 100, 2047):
        e, k = divmod(i, 256)
        ref = bf16_round(np.float32(O.normal(9, 7, e * 256 + k)) * np.float32(0.02))
        assert f[e, k] == ref
