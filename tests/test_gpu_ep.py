"""Expert-parallel MoE verify forward (the partitioning of the Qwen3-30B-A3B
configuration) on two GPUs, one process per GPU, against the one-GPU forward.

Each rank holds half of every layer's experts and runs its own rows; every MoE
layer stores each routed operand row into the owning rank's memory over
NVLink and the owner stores the scaled expert output back (mlxcat_cache_peer_*).
The expert kernels compute every assignment's output independently of which
other tokens share its tile, and the results travel in fp32, so each rank's
first tokens, drafts, per-layer routing and verify logits must equal a
one-GPU run of the same rows bit for bit.  The one-GPU MoE forward itself is
checked against the oracle in tests/test_gpu_moe.py.  The model is the
Qwen3-30B-A3B layer shape (hidden 2048, 32/4 heads of 128, 128 experts of
width 768, top-8) at two layers and a 4096-token vocabulary.

Ranks start with NVLS off (NCCL_NVLS_ENABLE=0), exchange their 128-byte
handles through the parent, and report errors instead of hanging: every
device wait of the exchange is bounded (10 s).  Needs two GPUs (skipped
otherwise)."""
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

MOE = dict(n_layers=2, hidden=2048, n_heads=32, n_kv_heads=4, head_dim=128, intermediate=768, vocab=4096,
           tie_embeddings=False, qk_norm=True, rms_eps=1e-6, rope_theta=1e6, n_experts=128, top_k=8,
           norm_topk=True)
SEED = 17
K = 4
WORLD = 2
MAX_LEN = 160


def prompts(rank):
    # equal lengths on every rank: each rank runs the same number of forwards
    return [[int(t) for t in np.random.default_rng(100 * rank + r).integers(0, 4096, n)]
            for r, n in enumerate((48, 33, 57))]


def run_rows(cache, ps, spec):
    firsts = [cache.insert_row(r, p, 16, M.SamplingParameters()) for r, p in enumerate(ps)]
    routing = [cache.moe_routing(l) for l in range(MOE["n_layers"])]   # the last forward: row 2's prefill
    drafts = cache.draft(spec)
    logits = cache.verify_forward(spec)
    vrouting = [cache.moe_routing(l) for l in range(MOE["n_layers"])]
    cache.accept(spec)
    return firsts, drafts, logits, routing, vrouting


def rank_main(rank, world, inbox, outboxes, results):
    try:
        os.environ["NCCL_NVLS_ENABLE"] = "0"
        ctx = M.Context(M.ModelConfig(**MOE, name="ep-30b-shape", ep_size=world, ep_rank=rank), rank)
        ctx.synth_weights(SEED)
        spec = M.SpeculativeDecodingConfiguration(True, K, 3, 8, A.ACCEPT_PREFIX)
        ps = prompts(rank)
        cache = M.BatchKVCache(ctx, len(ps), MAX_LEN)
        mine = cache.peer_handle()
        for r in range(world):
            if r != rank:
                outboxes[r].put((rank, mine))
        handles = {rank: mine}
        while len(handles) < world:
            r, h = inbox.get(timeout=60)
            handles[r] = h
        cache.peer_connect([handles[r] for r in range(world)])
        out = run_rows(cache, ps, spec)
        cache.close()
        ctx.close()
        results.put((rank, "ok", out))
    except Exception as e:  # reported to the parent
        results.put((rank, "error", repr(e)))


def test_expert_parallel_equals_one_gpu_forward():
    ctx_mp = mp.get_context("spawn")
    boxes = [ctx_mp.Queue() for _ in range(WORLD)]
    results = ctx_mp.Queue()
    procs = [ctx_mp.Process(target=rank_main, args=(r, WORLD, boxes[r], boxes, results)) for r in range(WORLD)]
    for p in procs:
        p.start()
    out = {}
    try:
        for _ in range(WORLD):
            r = results.get(timeout=300)
            out[r[0]] = r
            if r[1] == "error":
                break
    except queue.Empty:
        pass
    for p in procs:
        p.join(timeout=30)
        if p.is_alive():
            p.kill()
    for r in out.values():
        assert r[1] != "error", f"rank {r[0]}: {r[2]}"
    assert len(out) == WORLD, f"ranks reported: {sorted(out)}"

    # the same rows through the one-GPU forward (all experts on one device)
    ctx = M.Context(M.ModelConfig(**MOE, name="ep-30b-shape"), 0)
    ctx.synth_weights(SEED)
    spec = M.SpeculativeDecodingConfiguration(True, K, 3, 8, A.ACCEPT_PREFIX)
    try:
        for rank in range(WORLD):
            cache = M.BatchKVCache(ctx, len(prompts(rank)), MAX_LEN)
            ref = run_rows(cache, prompts(rank), spec)
            cache.close()
            firsts, drafts, logits, routing, vrouting = out[rank][2]
            assert firsts == ref[0], f"rank {rank}: first tokens differ"
            assert drafts == ref[1], f"rank {rank}: drafts differ"
            for l in range(MOE["n_layers"]):
                for got, want, what in ((routing, ref[3], "prefill"), (vrouting, ref[4], "verify")):
                    assert np.array_equal(got[l][0], want[l][0]), f"rank {rank} layer {l}: {what} experts differ"
                    assert np.array_equal(got[l][1], want[l][1]), f"rank {rank} layer {l}: {what} weights differ"
            assert logits.shape == ref[2].shape
            diff = np.abs(logits - ref[2])
            assert np.array_equal(logits, ref[2]), f"rank {rank}: verify logits differ (max {diff.max():.3g})"
    finally:
        ctx.close()
