"""The whole-job aggregation of bench.py over ranks (max of times, sum of
tokens), run as two gloo processes on the CPU."""
import os
import socket

import pytest

torch = pytest.importorskip("torch")
import torch.multiprocessing as mp  # noqa: E402


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, out):
    import datetime
    import sys
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path.insert(0, root)
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.distributed.init_process_group("gloo", rank=rank, world_size=world,
                                         timeout=datetime.timedelta(seconds=60))
    import bench
    dev_ms = [12.5, 14.0][rank]
    wall = [0.020, 0.018][rank]
    tokens = [48, 40][rank]
    out[rank] = bench.reduce_over_ranks(dev_ms, wall, tokens, world, "cpu")
    torch.distributed.barrier()
    torch.distributed.destroy_process_group()


def test_reduce_over_two_gloo_ranks():
    world = 2
    mgr = mp.Manager()
    out = mgr.dict()
    mp.spawn(_worker, args=(world, _free_port(), out), nprocs=world, join=True)
    for r in range(world):
        dev_ms, wall, tokens = out[r]
        assert dev_ms == 14.0 and wall == 0.020 and tokens == 88.0


def _tp_worker(rank, world, port, out):
    import datetime
    import sys
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path.insert(0, root)
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.distributed.init_process_group("gloo", rank=rank, world_size=world,
                                         timeout=datetime.timedelta(seconds=60))
    import bench
    uid = bytes((7 * i + 3) % 256 for i in range(128)) if rank == 0 else None
    got = bench.share_tp_id(uid, rank, "cpu")
    # tensor parallel: every rank emits the same 48 tokens; the job emitted 48
    red = bench.reduce_over_ranks([9.0, 11.0][rank], 0.01, bench.job_tokens(48, rank, True), world, "cpu")
    out[rank] = (got, red)
    torch.distributed.barrier()
    torch.distributed.destroy_process_group()


def test_tensor_parallel_host_plumbing_on_two_gloo_ranks():
    """The NCCL id created on rank 0 reaches every rank unchanged, and the
    tensor-parallel job counts its tokens once."""
    world = 2
    mgr = mp.Manager()
    out = mgr.dict()
    mp.spawn(_tp_worker, args=(world, _free_port(), out), nprocs=world, join=True)
    want = bytes((7 * i + 3) % 256 for i in range(128))
    for r in range(world):
        got, (dev_ms, wall, tokens) = out[r]
        assert got == want
        assert dev_ms == 11.0 and tokens == 48.0


def test_reduce_single_rank_is_identity():
    import sys
    sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    import bench
    assert bench.reduce_over_ranks(3.0, 0.5, 7, 1, "cpu") == (3.0, 0.5, 7.0)
