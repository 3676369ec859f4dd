"""Argument checking of the multi-GPU connect path on one GPU (no peer is
mapped and no exchange runs): a parallel cache refuses to run forwards before
it is connected, and mlxcat_cache_peer_connect rejects handle sets that do
not describe a group of equal caches in rank order -- the rule that keeps
every rank's exchange buffers the same shape."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")
if not torch.cuda.is_available():
    pytest.skip("needs a CUDA device", allow_module_level=True)

import mlxcat_b200 as M  # noqa: E402
from mlxcat_b200 import _abi as A  # noqa: E402

MOE = dict(n_layers=1, hidden=512, n_heads=8, n_kv_heads=2, head_dim=64, intermediate=256, vocab=1024,
           tie_embeddings=False, qk_norm=True, rms_eps=1e-6, rope_theta=1e6, n_experts=32, top_k=4,
           norm_topk=True)
DENSE = dict(n_layers=1, hidden=512, n_heads=8, n_kv_heads=4, head_dim=64, intermediate=512, vocab=1024,
             tie_embeddings=False, qk_norm=False, rms_eps=1e-5, rope_theta=500000.0)


def forged(handle, rank=None, ranks=None, cap=None, magic=None):
    """a copy of a handle with header fields replaced (layout: magic[4],
    version, kind, rank, ranks, cap, hidden as int32)"""
    b = bytearray(handle)
    if magic is not None:
        b[0:4] = magic
    for off, v in ((12, rank), (16, ranks), (20, cap)):
        if v is not None:
            b[off:off + 4] = int(v).to_bytes(4, "little", signed=True)
    return bytes(b)


@pytest.mark.parametrize("kind", ["ep", "tp"])
def test_parallel_cache_refuses_forwards_before_connect(kind):
    cfg = (M.ModelConfig(**MOE, name="ep", ep_size=2, ep_rank=0) if kind == "ep"
           else M.ModelConfig(**DENSE, name="tp", tp_size=2, tp_rank=0))
    ctx = M.Context(cfg, 0)
    ctx.synth_weights(3)
    cache = M.BatchKVCache(ctx, 2, 64)
    with pytest.raises(A.MlxcatError, match="not connected"):
        cache.insert_row(0, list(range(20)), 8, M.SamplingParameters())
    cache.close()
    ctx.close()


def test_peer_connect_rejects_bad_handle_sets():
    ctx = M.Context(M.ModelConfig(**MOE, name="ep", ep_size=2, ep_rank=0), 0)
    cache = M.BatchKVCache(ctx, 2, 64)
    h = cache.peer_handle()
    assert len(h) == M.BatchKVCache.PEER_HANDLE_BYTES and h[:4] == b"MXPR"
    other = forged(h, rank=1)
    bad = [
        ([forged(h, magic=b"XXXX"), other], "not a"),
        ([other, h], "rank order"),                       # ranks swapped
        ([h, forged(h, rank=1, ranks=4)], "rank 1 of 4"),   # a member of another group
        ([h, forged(h, rank=1, cap=7)], "another shape"),   # a cache of another max_rows
    ]
    for handles, msg in bad:
        with pytest.raises(A.MlxcatError, match=msg):
            cache.peer_connect(handles)
    # a dense one-GPU cache has no region to export
    ctx1 = M.Context(M.ModelConfig(**DENSE, name="one"), 0)
    c1 = M.BatchKVCache(ctx1, 1, 64)
    with pytest.raises(A.MlxcatError, match="neither"):
        c1.peer_handle()
    c1.close()
    ctx1.close()
    cache.close()
    ctx.close()
