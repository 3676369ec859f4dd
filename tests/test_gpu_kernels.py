"""Kernel parity on the GPU: each operator of the C ABI against the CPU oracle
on the same seeded inputs.  Integer work (synthesis, drafter, acceptance) is
compared bit-exactly; floating-point work within rtol 2e-2 / atol 2e-2."""
import ctypes as C
import random

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")
if not torch.cuda.is_available():
    pytest.skip("needs a CUDA device", allow_module_level=True)

from mlxcat_b200 import _abi as A  # noqa: E402
from oracle import oracle as O  # noqa: E402
from tests.gpu_util import DeviceRows, dev, ptr  # noqa: E402

L = A.lib()
RTOL = ATOL = 2e-2


# --------------------------------------------------------------------------- #
# weight synthesis: bit-exact
# --------------------------------------------------------------------------- #
@pytest.mark.parametrize("N,K,tid", [(128, 512, 0), (64, 1408, 37), (256, 2560, 0xFFFF0000)])
def test_synth_q4_bit_exact(N, K, tid):
    wq = torch.zeros((N, K // 8), dtype=torch.int32, device="cuda")
    s = torch.zeros((N, K // 64), dtype=torch.int16, device="cuda")
    b = torch.zeros((N, K // 64), dtype=torch.int16, device="cuda")
    A.check(L.mlxcat_op_synth_q4(77, tid, 0.02, N, K, ptr(wq), ptr(s), ptr(b), None))
    torch.cuda.synchronize()
    owq, os_, ob = O.q4_synth(77, tid, 0.02, N, K)
    np.testing.assert_array_equal(wq.cpu().numpy().view(np.uint32), owq)
    np.testing.assert_array_equal(s.cpu().numpy().view(np.uint16), os_)
    np.testing.assert_array_equal(b.cpu().numpy().view(np.uint16), ob)


# --------------------------------------------------------------------------- #
# q4 linear
# --------------------------------------------------------------------------- #
@pytest.mark.parametrize("M", [1, 5, 16, 17, 48, 64, 100, 144, 150, 160, 200, 300])   # 129..160: one wide tile
@pytest.mark.parametrize("N,K", [(256, 512), (384, 1408), (1024, 2560), (128, 9728), (128, 128)])
def test_q4_linear_matches_oracle(M, N, K):
    rng = np.random.default_rng(M * 7 + N)
    wq, s, b = O.q4_synth(5, N, 0.02, N, K)
    x = rng.normal(size=(M, K)).astype(np.float16)
    ref = O.q4_linear(wq, s, b, x.astype(np.float32))
    ws_bytes = L.mlxcat_op_q4_linear_workspace(N, K, M)
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device="cuda")
    y = torch.zeros((M, N), dtype=torch.float32, device="cuda")
    dw, ds, db, dx = dev(wq.view(np.int32)), dev(s.view(np.int16)), dev(b.view(np.int16)), dev(x.view(np.int16))
    A.check(L.mlxcat_op_q4_linear(ptr(dw), ptr(ds), ptr(db), N, K, ptr(dx), M, ptr(y), ptr(ws),
                                  ws_bytes, None))
    torch.cuda.synchronize()
    np.testing.assert_allclose(y.cpu().numpy(), ref, rtol=RTOL, atol=ATOL)
    # much tighter in practice: fp16 dequant rounding only
    assert np.abs(y.cpu().numpy() - ref).max() < 5e-3 * max(1.0, np.abs(ref).max())


def test_q4_linear_deterministic():
    N, K, M = 2560, 9728, 48
    wq, s, b = O.q4_synth(9, 1, 0.02, N, K)
    x = np.random.default_rng(1).normal(size=(M, K)).astype(np.float16)
    ws_bytes = L.mlxcat_op_q4_linear_workspace(N, K, M)
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device="cuda")
    dw, ds, db, dx = dev(wq.view(np.int32)), dev(s.view(np.int16)), dev(b.view(np.int16)), dev(x.view(np.int16))
    outs = []
    for _ in range(3):
        y = torch.zeros((M, N), dtype=torch.float32, device="cuda")
        A.check(L.mlxcat_op_q4_linear(ptr(dw), ptr(ds), ptr(db), N, K, ptr(dx), M, ptr(y), ptr(ws),
                                      ws_bytes, None))
        outs.append(y.cpu().numpy())
    assert all(np.array_equal(outs[0], o) for o in outs[1:])


def test_q4_linear_token_columns_independent():
    """Batch invariance (BatchInvarianceTests.swift:72-86 property): a token's
    output does not depend on which other tokens share the launch."""
    N, K = 1024, 2560
    wq, s, b = O.q4_synth(3, 2, 0.02, N, K)
    x = np.random.default_rng(2).normal(size=(48, K)).astype(np.float16)
    dw, ds, db = dev(wq.view(np.int32)), dev(s.view(np.int16)), dev(b.view(np.int16))

    def run(xm):
        M = xm.shape[0]
        ws_bytes = L.mlxcat_op_q4_linear_workspace(N, K, M)
        ws = torch.empty(ws_bytes, dtype=torch.uint8, device="cuda")
        y = torch.zeros((M, N), dtype=torch.float32, device="cuda")
        dx = dev(xm.view(np.int16))
        A.check(L.mlxcat_op_q4_linear(ptr(dw), ptr(ds), ptr(db), N, K, ptr(dx), M, ptr(y), ptr(ws),
                                      ws_bytes, None))
        return y.cpu().numpy()

    full = run(x)
    np.testing.assert_allclose(run(x[:5]), full[:5], rtol=1e-6, atol=1e-6)


# --------------------------------------------------------------------------- #
# attention
# --------------------------------------------------------------------------- #
def attention_ref(q, kc, vc, trow, tpos, Hq, Hkv, D):
    M = q.shape[0]
    G = Hq // Hkv
    out = np.zeros((M, Hq * D), np.float32)
    for m in range(M):
        for hq in range(Hq):
            h = hq // G
            T = tpos[m] + 1
            K = kc[trow[m], h, :T].astype(np.float32)
            V = vc[trow[m], h, :T].astype(np.float32)
            s = K @ q[m, hq].astype(np.float32) / np.sqrt(D)
            p = np.exp(s - s.max())
            out[m, hq * D:(hq + 1) * D] = (p / p.sum()) @ V
    return out


@pytest.mark.parametrize("Hq,Hkv,D", [(8, 2, 64), (32, 8, 128), (16, 2, 128)])
@pytest.mark.parametrize("qg", [1, 5, 8])
@pytest.mark.parametrize("max_len", [700, 340])   # several key splits + combine / one split, direct output
def test_attention_matches_reference(Hq, Hkv, D, qg, max_len):
    rng = np.random.default_rng(Hq + qg)
    rows = 3
    if qg * Hq // Hkv > 64:
        pytest.skip("query tile limit")
    lens = [37, 300, 650] if max_len == 700 else [5, 170, 330]
    kc = rng.normal(size=(rows, Hkv, max_len, D)).astype(np.float16)
    vc = rng.normal(size=(rows, Hkv, max_len, D)).astype(np.float16)
    trow, tpos = [], []
    for r in range(rows):
        for j in range(qg):
            trow.append(r)
            tpos.append(lens[r] + j)
    M = len(trow)
    q = rng.normal(size=(M, Hq, D)).astype(np.float16)
    ref = attention_ref(q, kc, vc, trow, tpos, Hq, Hkv, D)
    ws_bytes = L.mlxcat_op_attention_workspace(M, qg, Hq, Hkv, D, max_len)
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device="cuda")
    out = torch.zeros((M, Hq * D), dtype=torch.int16, device="cuda")
    dq, dk, dv = dev(q.view(np.int16)), dev(kc.view(np.int16)), dev(vc.view(np.int16))
    dr, dp = dev(np.array(trow, np.int32)), dev(np.array(tpos, np.int32))
    A.check(L.mlxcat_op_attention(ptr(dq), ptr(dk), ptr(dv), max_len, ptr(dr), ptr(dp), M, qg, Hq, Hkv,
                                  D, ptr(out), ptr(ws), ws_bytes, None))
    torch.cuda.synchronize()
    got = out.cpu().numpy().view(np.float16).astype(np.float32)
    np.testing.assert_allclose(got, ref, rtol=RTOL, atol=ATOL)
    # fp16 P and output rounding only: much tighter relative to the output scale
    assert np.abs(got - ref).max() < 5e-3 * np.abs(ref).max()


# --------------------------------------------------------------------------- #
# drafter: bit-exact with proposeSuffixTokens
# --------------------------------------------------------------------------- #
def run_draft(rows: DeviceRows, mode, enabled, k, n, min_ctx):
    R = rows.R
    vtok = torch.zeros((R, k + 1), dtype=torch.int32, device="cuda")
    cnt = torch.zeros(R, dtype=torch.int32, device="cuda")
    trow = torch.zeros(R * (k + 1), dtype=torch.int32, device="cuda")
    tpos = torch.zeros(R * (k + 1), dtype=torch.int32, device="cuda")
    st = rows.struct()
    sc = A.SpecConfigC(mode, enabled, k, n, min_ctx)
    A.check(L.mlxcat_op_draft(C.byref(st), C.byref(sc), ptr(vtok), ptr(cnt), ptr(trow), ptr(tpos), None))
    torch.cuda.synchronize()
    return vtok.cpu().numpy(), cnt.cpu().numpy(), trow.cpu().numpy(), tpos.cpu().numpy()


@pytest.mark.parametrize("trial", range(6))
def test_drafter_bit_exact(trial):
    rnd = random.Random(trial)
    R = 24
    hists, max_new, n_gen = [], [], []
    for r in range(R):
        vocab = rnd.choice([2, 4, 16, 32000])
        seg = [[rnd.randrange(vocab) for _ in range(rnd.randint(1, 40))] for _ in range(6)]
        h = []
        target = rnd.choice([1, 5, 9, 60, 700, 4000])
        while len(h) < target:
            h += seg[rnd.randrange(6)]
        hists.append(h[:target])
        max_new.append(rnd.choice([1, 2, 3, 50, 500]))
        n_gen.append(rnd.choice([0, 1, 1, 2]))
    k, n, min_ctx = rnd.choice([(4, 3, 8), (5, 3, 8), (4, 16, 8), (8, 7, 2), (1, 1, 2)])
    rows = DeviceRows(hists, max_new, n_gen=n_gen)
    vtok, cnt, trow, tpos = run_draft(rows, A.ACCEPT_PREFIX, 1, k, n, min_ctx)
    for r in range(R):
        remaining = max_new[r] - n_gen[r]
        want = None
        if remaining > 1:
            want = O.propose_suffix(hists[r], n, min_ctx, min(k, remaining - 1))
        want = want or []
        assert cnt[r] == len(want), (r, want, vtok[r])
        assert vtok[r, 0] == hists[r][-1]
        assert vtok[r, 1:1 + cnt[r]].tolist() == want
        assert all(x == hists[r][-1] for x in vtok[r, 1 + cnt[r]:])
        assert trow[r * (k + 1):(r + 1) * (k + 1)].tolist() == [r] * (k + 1)
        assert tpos[r * (k + 1):(r + 1) * (k + 1)].tolist() == list(range(len(hists[r]) - 1,
                                                                           len(hists[r]) + k))


@pytest.mark.parametrize("n", [64, 65, 100, 300])
def test_drafter_long_suffix_bit_exact(n):
    """Suffix lengths past the 64 tail tokens staged in shared memory: an older
    occurrence of the row's last 100 tokens (match length 100) must beat a more
    recent one that matches only 70, exactly as proposeSuffixTokens scans
    L = min(n, |ctx| - 1) down to 1 (BatchGenerator.swift:987-1008)."""
    rnd = random.Random(n)
    T = [rnd.randrange(1000, 30000) for _ in range(100)]
    d1, d2 = [11, 12, 13, 14], [21, 22, 23, 24]
    hist = [5] * 20 + T + d1 + [7] * 9 + [3] + T[30:] + d2 + [8] * 13 + T
    rows = DeviceRows([hist, hist[:-1]], [500, 500])
    vtok, cnt, _, _ = run_draft(rows, A.ACCEPT_PREFIX, 1, 4, n, 8)
    for r, h in enumerate([hist, hist[:-1]]):
        want = O.propose_suffix(h, n, 8, 4) or []
        assert vtok[r, 1:1 + cnt[r]].tolist() == want, (n, r, want)
    assert O.propose_suffix(hist, n, 8, 4) == (d1 if n >= 71 else d2)


def test_drafter_compat_gate_width_one():
    """COMPAT speculates only at width 1, greedy, unseeded (BatchGenerator.swift:957-975)."""
    h = [1, 2, 3, 1, 2, 3, 1, 2, 3]
    one = DeviceRows([h], [10])
    _, cnt, _, _ = run_draft(one, A.ACCEPT_COMPAT, 1, 4, 16, 8)
    assert cnt.tolist() == [3]
    two = DeviceRows([h, h], [10, 10])
    _, cnt, _, _ = run_draft(two, A.ACCEPT_COMPAT, 1, 4, 16, 8)
    assert cnt.tolist() == [0, 0]
    seeded = DeviceRows([h], [10], has_seed=[1])
    assert run_draft(seeded, A.ACCEPT_COMPAT, 1, 4, 16, 8)[1].tolist() == [0]
    hot = DeviceRows([h], [10], temperature=[0.7])
    assert run_draft(hot, A.ACCEPT_COMPAT, 1, 4, 16, 8)[1].tolist() == [0]
    assert run_draft(two, A.ACCEPT_PREFIX, 1, 4, 16, 8)[1].tolist() == [3, 3]
    assert run_draft(two, A.ACCEPT_PREFIX, 0, 4, 16, 8)[1].tolist() == [0, 0]


# --------------------------------------------------------------------------- #
# acceptance: bit-exact given identical logits and uniforms
# --------------------------------------------------------------------------- #
@pytest.mark.parametrize("mode", [A.ACCEPT_COMPAT, A.ACCEPT_PREFIX])
@pytest.mark.parametrize("sampled", [False, True])
def test_accept_bit_exact(mode, sampled):
    if sampled and mode == A.ACCEPT_COMPAT:
        pytest.skip("COMPAT never speculates on temperature rows")
    rng = np.random.default_rng(11 + mode + 2 * sampled)
    R, k, V = 16 if mode == A.ACCEPT_PREFIX else 1, 5, 4096
    hists = [rng.integers(0, V, size=rng.integers(10, 200)).tolist() for _ in range(R)]
    counts = rng.integers(0, k + 1, size=R)
    drafts = rng.integers(0, V, size=(R, k))
    logits = rng.normal(size=(R, k + 1, V)).astype(np.float32) * (3.0 if sampled else 1.0)
    # make proposals survive often: put each draft on (or near) the top
    for r in range(R):
        for p in range(k):
            if rng.random() < 0.75:
                logits[r, p, drafts[r, p]] = logits[r, p].max() + (2.0 if not sampled else rng.random() * 4)
    temps = [0.7 if sampled else 0.0] * R
    top_ps = [0.9 if (sampled and r % 2 == 0) else 0.0 for r in range(R)]
    seeds = [1000 + r for r in range(R)]
    eos = [[int(drafts[r, 2])] if r % 5 == 3 else [] for r in range(R)]
    trig = [int(drafts[r, 1]) if r % 7 == 6 else -1 for r in range(R)]
    n_gen = rng.integers(1, 50, size=R).tolist()
    max_new = [n_gen[r] + int(rng.integers(1, 20)) for r in range(R)]
    rows = DeviceRows(hists, max_new, n_gen=n_gen, temperature=temps, top_p=top_ps, seed=seeds,
                      has_seed=[1] * R, eos=eos, trigger=trig)
    vt = np.zeros((R, k + 1), np.int32)
    for r in range(R):
        vt[r, 0] = hists[r][-1]
        vt[r, 1:] = drafts[r]
    dvt, dcnt, dlog = dev(vt), dev(counts.astype(np.int32)), dev(logits)
    tokens = torch.zeros((R, k + 1), dtype=torch.int32, device="cuda")
    n = torch.zeros(R, dtype=torch.int32, device="cuda")
    fin = torch.zeros(R, dtype=torch.int32, device="cuda")
    stats = torch.zeros(4, dtype=torch.int64, device="cuda")
    ws_bytes = L.mlxcat_op_accept_workspace(R, k)
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device="cuda")
    st = rows.struct()
    sc = A.SpecConfigC(mode, 1, k, 3, 8)
    A.check(L.mlxcat_op_accept(C.byref(st), C.byref(sc), ptr(dvt), ptr(dcnt), ptr(dlog), V, ptr(tokens),
                               ptr(n), ptr(fin), ptr(stats), ptr(ws), ws_bytes, None))
    torch.cuda.synchronize()
    tokens, n, fin = tokens.cpu().numpy(), n.cpu().numpy(), fin.cpu().numpy()
    want_stats = np.zeros(4, np.int64)
    for r in range(R):
        sp = O.sampling(temperature=temps[r], top_p=top_ps[r], seed=seeds[r], eos=eos[r], trigger=trig[r])
        c = int(counts[r])
        out, rej = O.accept_row(mode, logits[r, :c + 1], drafts[r, :c].tolist(), sp, n_gen[r])
        assert n[r] == len(out), (r, out, tokens[r])
        assert tokens[r, :n[r]].tolist() == out
        assert rows.history(r) == hists[r] + out
        assert int(rows.kv_len[r]) == len(hists[r]) - 1 + len(out)
        assert int(rows.n_gen[r]) == n_gen[r] + len(out)
        done = (out[-1] in eos[r]) or n_gen[r] + len(out) >= max_new[r]
        assert bool(fin[r]) == done and int(rows.active[r]) == (0 if done else 1)
        if c > 0:
            want_stats += [c, len(out) - 1, 1, int(rej)]
    np.testing.assert_array_equal(stats.cpu().numpy(), want_stats)


def test_top_p_threshold_matches_oracle_on_hard_cases():
    """Ties, -inf, tiny and ordinary top-p on one row: sampled tokens agree."""
    V = 3000
    rng = np.random.default_rng(4)
    base = np.round(rng.normal(size=V) * 2, 1).astype(np.float32)   # many ties
    base[::97] = -np.inf
    for top_p in (1e-8, 1e-3, 0.3, 0.7, 0.9, 0.999):
        rows = DeviceRows([[1, 2, 3]], [100], n_gen=[3], temperature=[0.8], top_p=[top_p],
                          seed=[5], has_seed=[1])
        logits = np.stack([base] * 1)[None]
        vt = np.array([[3]], np.int32)
        tokens = torch.zeros((1, 1), dtype=torch.int32, device="cuda")
        n = torch.zeros(1, dtype=torch.int32, device="cuda")
        fin = torch.zeros(1, dtype=torch.int32, device="cuda")
        stats = torch.zeros(4, dtype=torch.int64, device="cuda")
        ws_bytes = L.mlxcat_op_accept_workspace(1, 0)
        ws = torch.empty(ws_bytes, dtype=torch.uint8, device="cuda")
        st = rows.struct()
        sc = A.SpecConfigC(A.ACCEPT_PREFIX, 1, 0, 3, 8)
        dl = dev(logits.astype(np.float32))
        dvt, dcnt = dev(vt), dev(np.zeros(1, np.int32))   # alive across the call
        A.check(L.mlxcat_op_accept(C.byref(st), C.byref(sc), ptr(dvt), ptr(dcnt),
                                   ptr(dl), V, ptr(tokens), ptr(n), ptr(fin), ptr(stats), ptr(ws),
                                   ws_bytes, None))
        torch.cuda.synchronize()
        sp = O.sampling(temperature=0.8, top_p=top_p, seed=5)
        out, _ = O.accept_row(A.ACCEPT_PREFIX, logits[0], [], sp, 3)
        assert tokens.cpu().numpy()[0, :int(n[0])].tolist() == out, top_p
