"""RMSNorm weights and MLX checkpoints on the GPU.

* norm weights (mlxcat_weights_set_norm) other than one: the verify logits
  match the oracle with the same weights within the verify tolerance (the
  folded RMSNorm carries the weight into every linear's operand);
* a context written as an MLX checkpoint (safetensors + config.json, mlx-lm
  tensor names) and loaded back (mlxcat_b200.checkpoint) gives bit-identical
  first tokens and verify logits, dense and MoE."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")
if not torch.cuda.is_available():
    pytest.skip("needs a CUDA device", allow_module_level=True)

import mlxcat_b200 as M  # noqa: E402
from mlxcat_b200 import _abi as A  # noqa: E402
from mlxcat_b200 import checkpoint as CK  # noqa: E402
from oracle import oracle as O  # noqa: E402

TOL = 2e-2
QWEN_SMALL = M.ModelConfig(2, 1024, 16, 4, 128, 2816, 4096, True, True, 1e-6, 1e6, name="qwen-small")
LLAMA_SMALL = M.ModelConfig(2, 512, 8, 2, 64, 1408, 4096, False, False, 1e-5, 500000.0, name="llama-small")
MOE_SMALL = M.ModelConfig(2, 512, 8, 2, 64, 256, 4096, False, True, 1e-6, 1e6, name="moe-small",
                          n_experts=32, top_k=4, norm_topk=True)
K = 4


def random_norms(cfg, seed):
    rng = np.random.default_rng(seed)
    return {nid: (1.0 + 0.25 * rng.standard_normal(n)).astype(np.float32) for _, nid, n in CK.norm_tensors(cfg)}


def prompts(vocab):
    return [[int(t) for t in np.random.default_rng(70 + r).integers(0, vocab, n)] for r, n in enumerate((75, 40))]


def run(ctx):
    spec = M.SpeculativeDecodingConfiguration(True, K, 3, 8, A.ACCEPT_PREFIX)
    ps = prompts(ctx.cfg.vocab)
    cache = M.BatchKVCache(ctx, len(ps), 256)
    firsts = [cache.insert_row(r, p, 16, M.SamplingParameters()) for r, p in enumerate(ps)]
    drafts = cache.draft(spec)
    logits = cache.verify_forward(spec)
    cache.accept(spec)
    cache.close()
    return firsts, drafts, logits


@pytest.mark.parametrize("cfg", [QWEN_SMALL, LLAMA_SMALL], ids=lambda c: c.name)
def test_norm_weights_match_oracle(cfg):
    seed = 23
    norms = random_norms(cfg, 5)
    ctx = M.Context(cfg)
    ctx.synth_weights(seed)
    for nid, w in norms.items():
        ctx.set_norm(nid, w)
    om = O.Model.synth(O.make_config(cfg.n_layers, cfg.hidden, cfg.n_heads, cfg.n_kv_heads, cfg.head_dim,
                                     cfg.intermediate, cfg.vocab, cfg.tie_embeddings, cfg.qk_norm, cfg.rms_eps,
                                     cfg.rope_theta), seed, 0.02)
    for nid, w in norms.items():
        om.set_norm(nid, w)
    firsts, drafts, logits = run(ctx)
    ctx.close()
    ps = prompts(cfg.vocab)
    gen = O.Generator(om, len(ps), 256, O.SpecConfig(A.ACCEPT_PREFIX, 1, K, 3, 8))
    for r, p in enumerate(ps):
        gen.admit(r, p, 16, O.sampling())
    for r, p in enumerate(ps):
        toks = [firsts[r]] + drafts[r]
        ol = O.forward(om, gen.kv, toks, [r] * len(toks), list(range(len(p), len(p) + len(toks))))
        np.testing.assert_allclose(logits[r, :len(toks)], ol, rtol=TOL, atol=TOL)


@pytest.mark.parametrize("cfg", [QWEN_SMALL, LLAMA_SMALL, MOE_SMALL], ids=lambda c: c.name)
def test_checkpoint_round_trip_is_bit_identical(cfg, tmp_path):
    norms = random_norms(cfg, 9)
    a = M.Context(cfg)
    a.synth_weights(41)
    for nid, w in norms.items():
        a.set_norm(nid, w)
    CK.save_mlx_checkpoint(a, str(tmp_path), norms)
    want = run(a)
    a.close()
    b = CK.load_mlx_checkpoint(str(tmp_path))
    assert b.cfg.n_layers == cfg.n_layers and b.cfg.qk_norm == cfg.qk_norm and b.cfg.n_experts == cfg.n_experts
    got = run(b)
    b.close()
    assert got[0] == want[0] and got[1] == want[1]
    np.testing.assert_array_equal(got[2], want[2])
