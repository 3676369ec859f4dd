"""The attention entry point for callers that cannot allocate device memory
(mlxcat_op_attention_noalloc) against the workspace entry point
(mlxcat_op_attention) on the same inputs, through the C ABI.

It runs last (file name) because its scratch is a device array shared by every
call: calls in a row with different shapes, the first filling the array to its
limit, check that leftover contents from a previous call do not leak into the
next result."""
import os
import re

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")
if not torch.cuda.is_available():
    pytest.skip("needs a CUDA device", allow_module_level=True)

from mlxcat_b200 import _abi as A  # noqa: E402
from tests.gpu_util import dev, ptr  # noqa: E402

L = A.lib()
RTOL = ATOL = 2e-2   # the attention tolerance of the kernel parity tests


def scratch_limit():
    header = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "include",
                          "mlxcat_cuda.h")
    m = re.search(r"#define MLXCAT_NOALLOC_ATTN_SCRATCH_BYTES \((\d+)u << (\d+)\)", open(header).read())
    return int(m.group(1)) << int(m.group(2))


def make_case(seed, rows, Hq, Hkv, D, qg, max_len, lens):
    rng = np.random.default_rng(seed)
    kc = rng.normal(size=(rows, Hkv, max_len, D)).astype(np.float16)
    vc = rng.normal(size=(rows, Hkv, max_len, D)).astype(np.float16)
    trow = [r for r in range(rows) for _ in range(qg)]
    tpos = [lens[r] + j for r in range(rows) for j in range(qg)]
    q = rng.normal(size=(len(trow), Hq, D)).astype(np.float16)
    return dict(q=dev(q.view(np.int16)), k=dev(kc.view(np.int16)), v=dev(vc.view(np.int16)),
                trow=dev(np.array(trow, np.int32)), tpos=dev(np.array(tpos, np.int32)),
                M=len(trow), qg=qg, Hq=Hq, Hkv=Hkv, D=D, max_len=max_len,
                host=(q.astype(np.float32), kc.astype(np.float32), vc.astype(np.float32), trow, tpos))


def attention_fp32(c):
    """Causal GQA attention in fp32 on the host: token m (row r, position p)
    sees keys 0..p of its row; output [M][Hq*D]."""
    q, kc, vc, trow, tpos = c["host"]
    G, D = c["Hq"] // c["Hkv"], c["D"]
    out = np.zeros((c["M"], c["Hq"] * D), np.float32)
    for m in range(c["M"]):
        r, p = trow[m], tpos[m]
        for h in range(c["Hq"]):
            k, v = kc[r, h // G, :p + 1], vc[r, h // G, :p + 1]
            s = k @ q[m, h] / np.sqrt(D)
            w = np.exp(s - s.max())
            out[m, h * D:(h + 1) * D] = (w / w.sum()) @ v
    return out


def run_workspace(c):
    ws_bytes = L.mlxcat_op_attention_workspace(c["M"], c["qg"], c["Hq"], c["Hkv"], c["D"], c["max_len"])
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device="cuda")
    out = torch.zeros((c["M"], c["Hq"] * c["D"]), dtype=torch.int16, device="cuda")
    A.check(L.mlxcat_op_attention(ptr(c["q"]), ptr(c["k"]), ptr(c["v"]), c["max_len"], ptr(c["trow"]),
                                  ptr(c["tpos"]), c["M"], c["qg"], c["Hq"], c["Hkv"], c["D"], ptr(out),
                                  ptr(ws), ws_bytes, None))
    torch.cuda.synchronize()
    return out.cpu().numpy().view(np.float16).astype(np.float32)


def run_noalloc(c):
    out = torch.zeros((c["M"], c["Hq"] * c["D"]), dtype=torch.int16, device="cuda")
    A.check(L.mlxcat_op_attention_noalloc(ptr(c["q"]), ptr(c["k"]), ptr(c["v"]), c["max_len"],
                                          ptr(c["trow"]), ptr(c["tpos"]), c["M"], c["qg"], c["Hq"],
                                          c["Hkv"], c["D"], ptr(out), None))
    torch.cuda.synchronize()
    return out.cpu().numpy().view(np.float16).astype(np.float32)


def test_noalloc_attention_matches_workspace_entry_point_twice():
    # first call: long contexts, many key splits; second call: a smaller shape
    # whose scratch reuses the start of the array
    first = make_case(11, rows=4, Hq=32, Hkv=8, D=128, qg=6, max_len=2900, lens=[2800, 1500, 40, 2047])
    second = make_case(12, rows=3, Hq=8, Hkv=2, D=64, qg=5, max_len=700, lens=[37, 300, 650])
    for c in (first, second):
        need = L.mlxcat_op_attention_workspace(c["M"], c["qg"], c["Hq"], c["Hkv"], c["D"], c["max_len"])
        assert need <= scratch_limit()
    want1, want2 = run_workspace(first), run_workspace(second)
    got1 = run_noalloc(first)
    got2 = run_noalloc(second)
    np.testing.assert_allclose(got1, want1, rtol=RTOL, atol=ATOL)
    np.testing.assert_allclose(got2, want2, rtol=RTOL, atol=ATOL)


def test_noalloc_attention_near_the_limit_then_smaller_shapes():
    """A shape whose scratch fills the array to within a few KB, then two
    smaller shapes that run on its leftovers; the smallest is also checked
    against an fp32 attention computed on the host."""
    full = make_case(13, rows=14, Hq=32, Hkv=8, D=128, qg=8, max_len=3456,
                     lens=[3440 - 37 * r for r in range(14)])
    need = L.mlxcat_op_attention_workspace(full["M"], full["qg"], full["Hq"], full["Hkv"], full["D"],
                                           full["max_len"])
    assert 0.99 * scratch_limit() < need <= scratch_limit()
    mid = make_case(14, rows=2, Hq=32, Hkv=8, D=128, qg=5, max_len=2000, lens=[1990, 700])
    small = make_case(15, rows=3, Hq=8, Hkv=2, D=64, qg=5, max_len=400, lens=[17, 200, 390])
    want = [run_workspace(c) for c in (full, mid, small)]
    got = [run_noalloc(c) for c in (full, mid, small)]
    for g, w in zip(got, want):
        np.testing.assert_allclose(g, w, rtol=RTOL, atol=ATOL)
    np.testing.assert_allclose(got[2], attention_fp32(small), rtol=RTOL, atol=ATOL)


def test_noalloc_attention_rejects_shapes_beyond_the_array():
    # a shape whose scratch exceeds the fixed array: refused before any launch
    M, qg, Hq, Hkv, D, max_len = 64, 1, 64, 64, 128, 4096
    assert L.mlxcat_op_attention_workspace(M, qg, Hq, Hkv, D, max_len) > scratch_limit()
    dummy = torch.zeros(16, dtype=torch.int32, device="cuda")
    rc = L.mlxcat_op_attention_noalloc(ptr(dummy), ptr(dummy), ptr(dummy), max_len, ptr(dummy), ptr(dummy),
                                       M, qg, Hq, Hkv, D, ptr(dummy), None)
    assert rc == A.E_INVALID
    assert b"fixed array" in L.mlxcat_op_last_error()
