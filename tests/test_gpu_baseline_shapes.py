"""Parity at the benchmarked shapes, on the GPU through the C ABI.

* The verify forward of the Qwen3-4B and Llama-3-8B architectures at their
  full widths and vocabularies (two layers each, so the CPU oracle stays
  bounded) over the batch and context lengths the bench times: 8 rows x 6
  verify tokens over 2048-token contexts (M = 48, greedy), and 32 rows x 5
  verify tokens over 4096-token contexts (M = 160, temperature 0.7, top-p 0.9,
  single-draft rejection sampling with per-request seeds).  Prompt KV comes
  from a prefix-cache import of random fp16 keys/values (the reference's
  prepareHitRow path, Scheduler.swift:957-985), so each admission computes only
  the last prompt position.  Checked: drafts bit-exact, verify logits within
  rtol/atol 2e-2 of the oracle, acceptance bit-exact on the device's logits,
  greedy tokens equal to the oracle's except at top-2 gaps under 1e-2, the
  appended KV within 2e-2.
* A ragged token count: 29 rows x 5 verify tokens = 145, which the gate/up
  projection runs as one 160-column tile with 15 padding columns and the
  other projections as two 80-token tiles (reduced widths, greedy).
* The q4 linear operator at every (N, K, M) the benchmarks launch, against the
  oracle's fp32 restatement on three 128-row blocks of each output (the first,
  a middle and the last block), so the stream-K split, token tiles and the
  last partial block are those of the real launches.
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

QWEN3_4B_2L = M.ModelConfig(2, 2560, 32, 8, 128, 9728, 151936, True, True, 1e-6, 1e6, name="qwen3-4b-2l")
LLAMA3_8B_2L = M.ModelConfig(2, 4096, 32, 8, 128, 14336, 128256, False, False, 1e-5, 500000.0,
                             name="llama3-8b-2l")
RAGGED_SMALL = M.ModelConfig(2, 1024, 16, 4, 128, 2816, 8192, False, False, 1e-5, 500000.0,
                             name="llama-small-ragged")


def segment_prompt(vocab, n_seg, seg_len, length, seed):
    rng = np.random.default_rng(seed)
    pool = rng.integers(0, vocab, size=(n_seg, seg_len))
    picks = rng.integers(0, n_seg, size=(length + seg_len - 1) // seg_len)
    return pool[picks].reshape(-1)[:length].tolist()


def oracle_model(cfg, seed):
    ocfg = O.make_config(cfg.n_layers, cfg.hidden, cfg.n_heads, cfg.n_kv_heads, cfg.head_dim,
                         cfg.intermediate, cfg.vocab, cfg.tie_embeddings, cfg.qk_norm, cfg.rms_eps,
                         cfg.rope_theta)
    return O.Model.synth(ocfg, seed, 0.02)


def verify_at_shape(cfg, rows, ctx_len, k, n, temperature, top_p, seed):
    ctx = M.Context(cfg)
    ctx.synth_weights(seed)
    om = oracle_model(cfg, seed)
    K1, Ly = k + 1, cfg.n_layers
    max_len = ctx_len + 128   # prompt + 64 new tokens + the verify window
    # segment-pool prompts (64 segments of 48 tokens) so the drafter proposes tokens
    prompts = [segment_prompt(cfg.vocab, 64, 48, ctx_len - (r % 5), 1000 + r) for r in range(rows)]
    sps = [M.SamplingParameters(temperature=temperature, top_p=top_p, seed=7000 + r) for r in range(rows)]
    osps = [O.sampling(temperature=temperature, top_p=top_p, seed=7000 + r) for r in range(rows)]
    spec = M.SpeculativeDecodingConfiguration(True, k, n, 8, A.ACCEPT_PREFIX)
    cache = M.BatchKVCache(ctx, rows, max_len)
    kv = O.KV(om, rows, max_len)
    rng = np.random.default_rng(seed)
    for r, p in enumerate(prompts):
        shape = (Ly, cfg.n_kv_heads, len(p) - 1, cfg.head_dim)
        kp = rng.standard_normal(shape).astype(np.float16)
        vp = rng.standard_normal(shape).astype(np.float16)
        first = cache.insert_row_prefix(r, p, kp, vp, 64, sps[r])
        for l in range(Ly):
            kv.k(r, l, cfg.n_kv_heads, cfg.head_dim)[:, :len(p) - 1] = kp[l].astype(np.float32)
            kv.v(r, l, cfg.n_kv_heads, cfg.head_dim)[:, :len(p) - 1] = vp[l].astype(np.float32)
        ol = O.forward(om, kv, [p[-1]], [r], [len(p) - 1])[0]
        if temperature == 0.0:
            top2 = np.sort(ol)[-2:]
            assert first == int(np.argmax(ol)) or top2[1] - top2[0] < TIE, (r, first)
    hist = [cache.history(r) for r in range(rows)]
    drafts = cache.draft(spec)
    logits = cache.verify_forward(spec)
    if temperature == 0.0:   # (a sampled first token rarely occurs in the prompt: rows may not draft)
        assert sum(len(d) for d in drafts) > 0, "the segment-pool prompts should yield drafts"
    toks, trow, tpos = [], [], []
    for r in range(rows):
        assert drafts[r] == (O.propose_suffix(hist[r], n, 8, k) or [])
        d = drafts[r]
        toks += [hist[r][-1]] + d + [hist[r][-1]] * (k - len(d))   # the device's padded verify tokens
        trow += [r] * K1
        tpos += list(range(len(prompts[r]), len(prompts[r]) + K1))
    ol = O.forward(om, kv, toks, trow, tpos)
    # every verify position, the padding too (the oracle ran the same padded tokens)
    for r in range(rows):
        np.testing.assert_allclose(logits[r], ol[r * K1:(r + 1) * K1], rtol=TOL, atol=TOL)
    tok, cnt, fin, stats = cache.accept(spec)
    for r in range(rows):
        m = len(drafts[r]) + 1
        n_gen = len(hist[r]) - len(prompts[r])
        # acceptance is integer work given the logits: bit-exact on the device's logits
        want, _ = O.accept_row(A.ACCEPT_PREFIX, logits[r, :m], drafts[r], osps[r], n_gen)
        assert tok[r, :cnt[r]].tolist() == want, r
        if temperature == 0.0:   # and on the oracle's logits, except at near ties
            ref, _ = O.accept_row(A.ACCEPT_PREFIX, ol[r * K1:r * K1 + m], drafts[r], osps[r], n_gen)
            for i, (a, b) in enumerate(zip(want, ref)):
                if a != b:
                    top2 = np.sort(ol[r * K1 + i])[-2:]
                    assert top2[1] - top2[0] < TIE, (r, i, a, b)
                    break
    # the KV appended for the accepted positions (last layer) and the rolled-back lengths
    lens = cache.lengths()
    for r in range(0, rows, max(1, rows // 4)):
        assert lens[r] == len(prompts[r]) + int(cnt[r])
        kk, vv = cache.extract_row(r, Ly - 1)
        lo = len(prompts[r])
        ok = kv.k(r, Ly - 1, cfg.n_kv_heads, cfg.head_dim)[:, lo:lens[r]]
        ovv = kv.v(r, Ly - 1, cfg.n_kv_heads, cfg.head_dim)[:, lo:lens[r]]
        np.testing.assert_allclose(kk[:, lo:].astype(np.float32), ok, rtol=TOL, atol=TOL)
        np.testing.assert_allclose(vv[:, lo:].astype(np.float32), ovv, rtol=TOL, atol=TOL)
    return drafts


def test_ragged_token_count_verify_matches_oracle():
    """145 verify tokens (29 rows x 5): the one-tile gate/up launch with padding columns."""
    verify_at_shape(RAGGED_SMALL, 29, 600, 4, 3, 0.0, 0.0, 43)


def test_qwen3_4b_shape_verify_matches_oracle():
    """Qwen3-4B widths, vocab 151936, 8 rows x (k+1 = 6) over 2048-token contexts, greedy."""
    verify_at_shape(QWEN3_4B_2L, 8, 2048, 5, 3, 0.0, 0.0, 41)


def test_llama3_8b_shape_sampled_verify_matches_oracle():
    """Llama-3-8B widths, vocab 128256, 32 rows x (k+1 = 5) over 4096-token
    contexts, temperature 0.7 / top-p 0.9 rejection sampling."""
    verify_at_shape(LLAMA3_8B_2L, 32, 4096, 4, 4, 0.7, 0.9, 43)


# --------------------------------------------------------------------------- #
# q4 linear at the launched shapes
# --------------------------------------------------------------------------- #
def launched_shapes():
    out = []
    for (H, Hq, Hkv, D, I, V, M_) in [(2560, 32, 8, 128, 9728, 151936, 48),      # Qwen3-4B verify
                                      (4096, 32, 8, 128, 14336, 128256, 160)]:   # Llama-3-8B verify
        out += [((Hq + 2 * Hkv) * D, H, M_), (H, Hq * D, M_), (2 * I, H, M_), (H, I, M_), (V, H, M_)]
    # Qwen3-30B-A3B attention projections and head at 64 x 5 tokens
    out += [((32 + 8) * 128, 2048, 320), (2048, 32 * 128, 320), (151936, 2048, 320)]
    # Llama-3-70B tensor-parallel slices at 64 x 7 tokens (2 and 8 ranks) and its head
    for T in (2, 8):
        out += [((64 // T + 2 * 8 // T) * 128, 8192, 448), (8192, 64 // T * 128, 448),
                (2 * 28672 // T, 8192, 448), (8192, 28672 // T, 448)]
    out.append((128256, 8192, 448))
    return out


@pytest.mark.parametrize("N,K,M_", launched_shapes(), ids=lambda v: str(v))
def test_q4_linear_at_launched_shape(N, K, M_):
    rng = np.random.default_rng(N * 31 + K * 7 + M_)
    wq = rng.integers(0, 2**32, size=(N, K // 8), dtype=np.uint32)
    s = (rng.random((N, K // 64), dtype=np.float32) * 4e-3 + 1e-3).astype(np.float16)
    b = (-rng.random((N, K // 64), dtype=np.float32) * 3e-2).astype(np.float16)
    x = rng.standard_normal((M_, K)).astype(np.float16)
    blocks = sorted({0, (N // 256) * 128, N - 128})
    rows = np.concatenate([np.arange(r, r + 128) for r in blocks])
    ref = O.q4_linear(wq[rows], s[rows].view(np.uint16), b[rows].view(np.uint16), x.astype(np.float32))
    ws_bytes = L.mlxcat_op_q4_linear_workspace(N, K, M_)
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device="cuda")
    y = torch.zeros((M_, N), dtype=torch.float32, device="cuda")
    dw, ds, db, dx = dev(wq.view(np.int32)), dev(s.view(np.int16)), dev(b.view(np.int16)), dev(x.view(np.int16))
    A.check(L.mlxcat_op_q4_linear(ptr(dw), ptr(ds), ptr(db), N, K, ptr(dx), M_, ptr(y), ptr(ws), ws_bytes, None))
    torch.cuda.synchronize()
    got = y[:, torch.as_tensor(rows, device="cuda")].cpu().numpy()
    scale = float(np.abs(ref).max())
    np.testing.assert_allclose(got, ref, rtol=TOL, atol=TOL * max(1.0, scale))
    # fp16 dequantisation rounding only: much tighter in practice
    assert np.abs(got - ref).max() < 5e-3 * max(1.0, scale)
