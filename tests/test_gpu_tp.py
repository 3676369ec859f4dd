"""Tensor-parallel verify forward (the partitioning of the Llama-3-70B
configuration) on two GPUs, one process per GPU, against the CPU oracle of the
whole model.

Each rank holds its slice of every linear (q/k/v heads and gate/up rows
column-split, o/down inputs row-split), synthesised from the full tensor's
weight stream, so the slices together are the oracle's weights; one
allreduce follows the attention block and one the MLP block -- either NCCL
(mlxcat_ctx_tp_connect) or the fused scatter / reduce / gather over the
caches' peer regions (mlxcat_cache_peer_connect: the row-split projection
writes its partial sums straight into the owning rank's memory).  Both ranks
must produce the same logits and tokens, and the logits must match the oracle
within the verify tolerance.  Needs two GPUs (skipped otherwise)."""
import multiprocessing as mp
import os
import queue

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")
if not torch.cuda.is_available() or torch.cuda.device_count() < 2:
    pytest.skip("needs two CUDA devices", allow_module_level=True)

import mlxcat_b200 as M  # noqa: E402
from mlxcat_b200 import _abi as A  # noqa: E402
from oracle import oracle as O  # noqa: E402

TOL = 2e-2
TP_SMALL = dict(n_layers=2, hidden=512, n_heads=8, n_kv_heads=4, head_dim=64, intermediate=512,
                vocab=4096, tie_embeddings=False, qk_norm=False, rms_eps=1e-5, rope_theta=500000.0)
SEED = 31
K = 4


def prompts():
    return [[int(t) for t in np.random.default_rng(40 + r).integers(0, 4096, n)] for r, n in enumerate((90, 57))]


def rank_main(rank, world, mode, boxes, results):
    try:
        os.environ["NCCL_NVLS_ENABLE"] = "0"
        cfg = M.ModelConfig(**TP_SMALL, name="tp-small", tp_size=world, tp_rank=rank)
        ctx = M.Context(cfg, rank)
        if mode == "nccl":
            if rank == 0:
                uid = M.Context.tp_unique_id()
                for r in range(1, world):
                    boxes[r].put((0, uid))
            else:
                uid = boxes[rank].get(timeout=60)[1]
            ctx.tp_connect(uid)
        ctx.synth_weights(SEED)
        spec = M.SpeculativeDecodingConfiguration(True, K, 3, 8, A.ACCEPT_PREFIX)
        ps = prompts()
        cache = M.BatchKVCache(ctx, len(ps), 256)
        if mode == "peer":
            mine = cache.peer_handle()
            for r in range(world):
                if r != rank:
                    boxes[r].put((rank, mine))
            handles = {rank: mine}
            while len(handles) < world:
                r, h = boxes[rank].get(timeout=60)
                handles[r] = h
            cache.peer_connect([handles[r] for r in range(world)])
        firsts = [cache.insert_row(r, p, 16, M.SamplingParameters()) for r, p in enumerate(ps)]
        drafts = cache.draft(spec)
        logits = cache.verify_forward(spec)
        cache.accept(spec)
        hist = [cache.history(r) for r in range(len(ps))]
        cache.close()
        ctx.close()
        results.put((rank, firsts, drafts, logits, hist))
    except Exception as e:  # reported to the parent
        results.put((rank, "error", repr(e), None, None))


@pytest.mark.parametrize("mode", ["nccl", "peer"])
def test_tensor_parallel_verify_matches_oracle(mode):
    world = 2
    ctx_mp = mp.get_context("spawn")
    boxes, results = [ctx_mp.Queue() for _ in range(world)], ctx_mp.Queue()
    procs = [ctx_mp.Process(target=rank_main, args=(r, world, mode, boxes, results)) for r in range(world)]
    for p in procs:
        p.start()
    out = {}
    try:
        for _ in range(world):
            r = results.get(timeout=240)
            out[r[0]] = r
            if r[1] == "error":   # the other ranks would wait in a collective
                break
    except queue.Empty:
        pass
    for p in procs:
        p.join(timeout=5 if any(v[1] == "error" for v in out.values()) else 30)
        if p.is_alive():
            p.kill()
    for r in out.values():
        assert r[1] != "error", f"rank {r[0]}: {r[2]}"
    assert len(out) == world, f"ranks reported: {sorted(out)}"
    for r in range(1, world):   # replicated results on every rank
        assert out[r][1] == out[0][1] and out[r][2] == out[0][2] and out[r][4] == out[0][4]
        np.testing.assert_array_equal(out[r][3], out[0][3])
    _, firsts, drafts, logits, hist = out[0]
    ps = prompts()
    om = O.Model.synth(O.make_config(**TP_SMALL), SEED, 0.02)
    gen = O.Generator(om, len(ps), 256, O.SpecConfig(A.ACCEPT_PREFIX, 1, K, 3, 8))
    for r, p in enumerate(ps):
        gen.admit(r, p, 16, O.sampling())
    for r, p in enumerate(ps):
        assert hist[r][:len(p)] == p
        toks = [firsts[r]] + drafts[r]
        ol = O.forward(om, gen.kv, toks, [r] * len(toks), list(range(len(p), len(p) + len(toks))))
        np.testing.assert_allclose(logits[r, :len(toks)], ol, rtol=TOL, atol=TOL)
