"""The dense prefill path on the GPU (admission of prompts of 256 tokens or
more: Scheduler.completeAdmission, Scheduler.swift:599-668).

* mlxcat_op_dequant_q4 against the oracle's dequantisation (fp16 rounding of
  scale * q + bias);
* mlxcat_op_gemm_f16 (tcgen05, both operands TMA-staged) against a torch fp32
  matmul of the same fp16 operands, in its three epilogues, at shapes with
  partial token tiles;
* whole-prompt admissions against the CPU oracle: the KV of every prompt
  position within rtol/atol 2e-2, the first token equal except at top-2 gaps
  under 1e-2, and the next verify step's logits within 2e-2 -- at prompt
  lengths that take one and two 4096-token chunks, with and without the
  Qwen3 q/k norm, and at the Llama-3-8B layer widths.
"""
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
TIE = 1e-2


def test_dequant_q4_matches_oracle():
    N, K = 384, 1408
    wq, s, b = O.q4_synth(3, 9, 0.02, N, K)
    ref = O.q4_dequant(wq, s, b)
    dw, ds, db = dev(wq.view(np.int32)), dev(s.view(np.int16)), dev(b.view(np.int16))
    out = torch.zeros((N, K), dtype=torch.float16, device="cuda")
    A.check(L.mlxcat_op_dequant_q4(ptr(dw), ptr(ds), ptr(db), N, K, ptr(out), None))
    torch.cuda.synchronize()
    got = out.float().cpu().numpy()
    # one fp16 rounding of scale * q + bias
    np.testing.assert_allclose(got, ref, rtol=1e-3, atol=1e-6)


def gemm(w, x, epi, out, ldo, err):
    A.check(L.mlxcat_op_gemm_f16(ptr(w), w.shape[0], w.shape[1], ptr(x), x.shape[0], epi, ptr(out), ldo, ptr(err),
                                 None))
    torch.cuda.synchronize()
    assert int(err.item()) == 0, "a pipeline wait timed out"


@pytest.mark.parametrize("M_,N,K", [(1, 128, 64), (300, 256, 512), (2048, 1536, 2560), (700, 4096, 14336),
                                    (257, 6144, 4096)])
def test_gemm_f16_store_and_add_match_torch(M_, N, K):
    g = torch.Generator(device="cuda").manual_seed(M_ + N + K)
    w = (torch.randn((N, K), device="cuda", generator=g) * 0.02).half()
    x = torch.randn((M_, K), device="cuda", generator=g).half()
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    ref = x.float() @ w.float().t()
    out = torch.full((M_, N + 8), 7.0, device="cuda")   # ldo > N: the padding columns stay untouched
    gemm(w, x, A.GEMM_STORE, out, N + 8, err)
    scale = float(ref.abs().max())
    torch.testing.assert_close(out[:, :N], ref, rtol=1e-3, atol=1e-3 * scale)
    assert bool((out[:, N:] == 7.0).all())
    base = torch.randn((M_, N), device="cuda", generator=g)
    acc = base.clone()
    gemm(w, x, A.GEMM_ADD, acc, N, err)
    torch.testing.assert_close(acc, base + ref, rtol=1e-3, atol=1e-3 * scale)


@pytest.mark.parametrize("M_,I,K", [(100, 128, 256), (1100, 1408, 512), (2048, 14336, 4096)])
def test_gemm_f16_swiglu_matches_torch(M_, I, K):
    g = torch.Generator(device="cuda").manual_seed(M_ + I)
    gate = (torch.randn((I, K), device="cuda", generator=g) * 0.05).half()
    up = (torch.randn((I, K), device="cuda", generator=g) * 0.05).half()
    # fused layout: per 128-row block, 64 gate rows then the matching 64 up rows
    fused = torch.stack([gate.view(I // 64, 64, K), up.view(I // 64, 64, K)], 1).reshape(2 * I, K).contiguous()
    x = torch.randn((M_, K), device="cuda", generator=g).half()
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    out = torch.zeros((M_, I), dtype=torch.float16, device="cuda")
    gemm(fused, x, A.GEMM_SWIGLU, out, I, err)
    gg, uu = x.float() @ gate.float().t(), x.float() @ up.float().t()
    ref = gg * torch.sigmoid(gg) * uu
    torch.testing.assert_close(out.float(), ref, rtol=2e-3, atol=2e-3 * float(ref.abs().max()))


# --------------------------------------------------------------------------- #
# whole-prompt admissions against the oracle
# --------------------------------------------------------------------------- #
TINY2 = M.ModelConfig(2, 512, 8, 2, 64, 1408, 32000, True, False, 1e-5, 500000.0, name="tiny2")
QWEN_SMALL = M.ModelConfig(2, 1024, 16, 4, 128, 2816, 4096, True, True, 1e-6, 1e6, name="qwen-small")
LLAMA8B_LAYER = M.ModelConfig(1, 4096, 32, 8, 128, 14336, 8192, False, False, 1e-5, 500000.0,
                              name="llama8b-layer")


def segment_prompt(vocab, n_seg, seg_len, length, seed):
    rng = np.random.default_rng(seed)
    pool = rng.integers(0, vocab, size=(n_seg, seg_len))
    picks = rng.integers(0, n_seg, size=(length + seg_len - 1) // seg_len)
    return pool[picks].reshape(-1)[:length].tolist()


@pytest.mark.parametrize("cfg,lens", [(TINY2, [4500, 256]), (QWEN_SMALL, [700, 300]), (LLAMA8B_LAYER, [600])],
                         ids=lambda v: getattr(v, "name", str(v)))
def test_dense_prefill_matches_oracle(cfg, lens):
    seed, k = 19, 4
    ctx = M.Context(cfg)
    ctx.synth_weights(seed)
    ocfg = O.make_config(cfg.n_layers, cfg.hidden, cfg.n_heads, cfg.n_kv_heads, cfg.head_dim, cfg.intermediate,
                         cfg.vocab, cfg.tie_embeddings, cfg.qk_norm, cfg.rms_eps, cfg.rope_theta)
    om = O.Model.synth(ocfg, seed, 0.02)
    rows, max_len = len(lens), max(lens) + 64
    prompts = [segment_prompt(cfg.vocab, 16, 32, n, 400 + r) for r, n in enumerate(lens)]
    cache = M.BatchKVCache(ctx, rows, max_len)
    gen = O.Generator(om, rows, max_len, O.SpecConfig(A.ACCEPT_PREFIX, 1, k, 3, 8))
    for r, p in enumerate(prompts):
        first = cache.insert_row(r, p, 32, M.SamplingParameters())
        ofirst = gen.admit(r, p, 32, O.sampling())
        if first != ofirst:   # only at a near tie of the last prompt position's logits
            kv2 = O.KV(om, 1, max_len)
            lg = O.forward(om, kv2, p, [0] * len(p), list(range(len(p))))[-1]
            top2 = np.sort(lg)[-2:]
            assert top2[1] - top2[0] < TIE, (r, first, ofirst)
        for layer in sorted({0, cfg.n_layers - 1}):
            kk, vv = cache.extract_row(r, layer)
            ok = gen.kv.k(r, layer, cfg.n_kv_heads, cfg.head_dim)[:, :len(p)]
            ov = gen.kv.v(r, layer, cfg.n_kv_heads, cfg.head_dim)[:, :len(p)]
            np.testing.assert_allclose(kk.astype(np.float32), ok, rtol=TOL, atol=TOL)
            np.testing.assert_allclose(vv.astype(np.float32), ov, rtol=TOL, atol=TOL)
    # the next verify step reads the prefilled KV
    spec = M.SpeculativeDecodingConfiguration(True, k, 3, 8, A.ACCEPT_PREFIX)
    drafts = cache.draft(spec)
    logits = cache.verify_forward(spec)
    for r in range(rows):
        h = cache.history(r)
        toks = [h[-1]] + drafts[r]
        kvlen = len(prompts[r])
        ol = O.forward(om, gen.kv, toks, [r] * len(toks), list(range(kvlen, kvlen + len(toks))))
        np.testing.assert_allclose(logits[r, :len(toks)], ol, rtol=TOL, atol=TOL)


@pytest.mark.parametrize("s0,n", [(0, 1), (0, 77), (0, 128), (300, 700), (5, 300), (1000, 129)])
def test_prefill_attention_matches_torch(s0, n):
    """mlxcat_op_prefill_attention (tcgen05 flash attention, head_dim 128)
    against a torch fp32 causal softmax(q K^T / sqrt(d)) V of the same fp16
    inputs; GQA 32 query / 8 kv heads, row 1 of a 2-row cache."""
    rows, Hkv, Hq, D, max_len, row = 2, 8, 32, 128, 1200, 1
    g = torch.Generator(device="cuda").manual_seed(s0 * 7 + n)
    kc = torch.randn((rows, Hkv, max_len, D), device="cuda", generator=g).half()
    vc = torch.randn((rows, Hkv, max_len, D), device="cuda", generator=g).half()
    q = torch.randn((n, Hq * D), device="cuda", generator=g).half()
    out = torch.zeros((n, Hq * D), dtype=torch.float16, device="cuda")
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    A.check(L.mlxcat_op_prefill_attention(ptr(q), ptr(kc), ptr(vc), rows, max_len, row, s0, n, Hq, Hkv, D,
                                          ptr(out), ptr(err), None))
    torch.cuda.synchronize()
    assert int(err.item()) == 0, "a pipeline wait timed out"
    T = s0 + n
    k = kc[row, :, :T].float().repeat_interleave(Hq // Hkv, dim=0)      # [Hq][T][D]
    v = vc[row, :, :T].float().repeat_interleave(Hq // Hkv, dim=0)
    qq = q.float().view(n, Hq, D).transpose(0, 1)                        # [Hq][n][D]
    s = qq @ k.transpose(1, 2) / D ** 0.5                                # [Hq][n][T]
    pos = torch.arange(s0, s0 + n, device="cuda")[:, None]
    s = s.masked_fill(torch.arange(T, device="cuda")[None, :] > pos, float("-inf"))
    ref = (torch.softmax(s, dim=-1) @ v).transpose(0, 1).reshape(n, Hq * D)
    got = out.float()
    scale = ref.abs().max().item()
    assert torch.isfinite(got).all()
    assert (got - ref).abs().max().item() <= 5e-3 * max(scale, 1.0), (got - ref).abs().max().item()
