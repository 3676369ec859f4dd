"""Tensor-parallel weight slices on one GPU: contexts for rank 0 and rank 1 of
a two-way split hold exactly their part of every full tensor of the oracle
(q/k/v and gate/up rows, o and down input columns), and replicated tensors
whole.  Weight synthesis needs no communicator, so both ranks' contexts live in
one process here; the forward with its allreduce is tests/test_gpu_tp.py."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")
if not torch.cuda.is_available():
    pytest.skip("needs a CUDA device", allow_module_level=True)

import mlxcat_b200 as M  # noqa: E402
from oracle import oracle as O  # noqa: E402

CFG = dict(n_layers=2, hidden=512, n_heads=8, n_kv_heads=4, head_dim=64, intermediate=512,
           vocab=4096, tie_embeddings=False, qk_norm=False, rms_eps=1e-5, rope_theta=500000.0)


def test_tensor_parallel_slices_equal_the_full_tensors():
    T, seed = 2, 23
    om = O.Model.synth(O.make_config(**CFG), seed, 0.02)
    H, D, Hq, Hkv, I = CFG["hidden"], CFG["head_dim"], CFG["n_heads"], CFG["n_kv_heads"], CFG["intermediate"]
    qd, kvd, il = Hq * D // T, Hkv * D // T, I // T
    for r in range(T):
        ctx = M.Context(M.ModelConfig(**CFG, name="tp-slices", tp_size=T, tp_rank=r))
        ctx.synth_weights(seed)
        for layer in range(CFG["n_layers"]):
            for kind, (N, K), rows, cols in (
                    (0, (qd, H), slice(r * qd, (r + 1) * qd), None),
                    (1, (kvd, H), slice(r * kvd, (r + 1) * kvd), None),
                    (2, (kvd, H), slice(r * kvd, (r + 1) * kvd), None),
                    (3, (H, qd), None, slice(r * qd, (r + 1) * qd)),
                    (4, (il, H), slice(r * il, (r + 1) * il), None),
                    (5, (il, H), slice(r * il, (r + 1) * il), None),
                    (6, (H, il), None, slice(r * il, (r + 1) * il))):
                tid = layer * 16 + kind
                got = ctx.get_q4(tid, N, K)
                full = om.get_q4(tid)
                for g, f, per_k in zip(got, full, (8, 64, 64)):
                    want = f[rows] if rows is not None else f[:, cols.start // per_k: cols.stop // per_k]
                    np.testing.assert_array_equal(g, want)
        for tid in (O.TENSOR_EMBED, O.TENSOR_LM_HEAD):   # replicated
            for g, f in zip(ctx.get_q4(tid, CFG["vocab"], H), om.get_q4(tid)):
                np.testing.assert_array_equal(g, f)
        ctx.close()


def test_tensor_parallel_context_refuses_to_run_unconnected():
    ctx = M.Context(M.ModelConfig(**CFG, name="tp-slices", tp_size=2, tp_rank=0))
    ctx.synth_weights(1)
    cache = M.BatchKVCache(ctx, 1, 128)
    with pytest.raises(Exception, match="not connected"):
        cache.insert_row(0, list(range(1, 20)), 4, M.SamplingParameters())
