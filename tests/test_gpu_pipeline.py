"""End-to-end parity on the GPU through the C ABI.

* the reference's speculation tests (SchedulerSpeculativeDecodingTests.swift)
  with the same fake models, run through the device step;
* the tiny Llama-style model against the CPU oracle: verify logits within
  rtol/atol 2e-2, token streams equal except at near-ties, KV rollback exact;
* speculative == plain greedy decode on the device (COMPAT and PREFIX);
* per-request seeded sampling independent of batch composition;
* BatchKVCache.trim known answer.
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

TOL = 2e-2


# --------------------------------------------------------------------------- #
# SchedulerSpeculativeDecodingTests.swift:9-106 on the device
# --------------------------------------------------------------------------- #
def repeating_table(vocab=8, mismatch=False):
    nxt = [1] * vocab
    nxt[1], nxt[2] = 2, 3
    if mismatch:
        nxt[3] = 4
    return nxt


def run_scheduler(table, prompt, spec, max_tokens=10, trigger=None):
    ctx = M.Context(M.ModelConfig.table(len(table)))
    ctx.set_table(table)
    sched = M.Scheduler(ctx, 1, 64, spec)
    sched.submit(M.Request("repeat", prompt, max_tokens,
                           M.SamplingParameters(temperature=0.0, tool_call_start_token_id=trigger)))
    tokens = []
    while not sched.is_idle:
        tokens += [r.token for r in sched.step() if r.uid == "repeat" and r.token >= 0]
    return tokens, sched.speculative_decoding_stats, sched.generator.decode_calls


def spec_cfg(min_ctx=8, mode=A.ACCEPT_COMPAT, k=4):
    return M.SpeculativeDecodingConfiguration(True, k, 16, min_ctx, mode)


def test_ngram_speculation_identical_tokens_with_fewer_decode_calls():
    prompt = [1, 2, 3, 1, 2, 3, 1, 2]
    base, _, base_calls = run_scheduler(repeating_table(), prompt, M.SpeculativeDecodingConfiguration.disabled)
    spec, stats, spec_calls = run_scheduler(repeating_table(), prompt, spec_cfg())
    assert spec == base == [3, 1, 2, 3, 1, 2, 3, 1, 2, 3]
    assert len(spec) == 10
    assert stats.accepted_token_count > 0 and stats.proposal_batch_count > 0
    assert spec_calls < base_calls


def test_rejected_ngram_proposal_falls_back_without_changing_output():
    prompt = [1, 2, 3, 1, 2, 3, 1, 2]
    base, _, _ = run_scheduler(repeating_table(mismatch=True), prompt, M.SpeculativeDecodingConfiguration.disabled)
    spec, stats, _ = run_scheduler(repeating_table(mismatch=True), prompt, spec_cfg())
    assert spec == base
    assert stats.rejected_batch_count > 0


def test_tool_trigger_keeps_speculation_enabled_before_trigger():
    _, stats, _ = run_scheduler(repeating_table(), [1, 2, 3, 1, 2, 3, 1, 2], spec_cfg(), trigger=7)
    assert stats.proposal_batch_count > 0 and stats.accepted_token_count > 0


def test_speculation_replays_trigger_through_ordinary_path():
    prompt = [1, 2, 3, 1, 2, 3]
    base, _, _ = run_scheduler(repeating_table(), prompt, M.SpeculativeDecodingConfiguration.disabled,
                               max_tokens=5, trigger=2)
    spec, stats, _ = run_scheduler(repeating_table(), prompt, spec_cfg(min_ctx=6), max_tokens=5, trigger=2)
    assert base[:2] == [1, 2]
    assert spec == base
    assert stats.rejected_batch_count > 0


def test_stats_match_oracle_on_table_models():
    for mismatch in (False, True):
        for mode in (A.ACCEPT_COMPAT, A.ACCEPT_PREFIX):
            prompt = [1, 2, 3, 1, 2, 3, 1, 2]
            got, stats, calls = run_scheduler(repeating_table(mismatch=mismatch), prompt,
                                              spec_cfg(mode=mode), max_tokens=30)
            om = O.Model.table(repeating_table(mismatch=mismatch))
            gen = O.Generator(om, 1, 64, O.SpecConfig(mode, 1, 4, 16, 8))
            want = [gen.admit(0, prompt, 30, O.sampling())]
            ocalls = 0
            while gen.active(0):
                want += gen.step()[0]
                ocalls += 1
            assert got == want
            assert calls == ocalls
            s = gen.stats
            assert (stats.proposed_token_count, stats.accepted_token_count, stats.proposal_batch_count,
                    stats.rejected_batch_count) == (s.proposed, s.accepted, s.proposal_batches,
                                                    s.rejected_batches)


def test_trim_keeps_mixed_length_rows_consistent():
    """BatchCacheShapeTests.swift:170-193: lengths 2 and 5, trim(4) -> 0 and 1."""
    ctx = M.Context(M.ModelConfig.table(8))
    ctx.set_table(repeating_table())
    cache = M.BatchKVCache(ctx, 2, 64)
    cache.insert_row(0, [1, 2], 4, M.SamplingParameters())
    cache.insert_row(1, [1, 2, 3, 1, 2], 4, M.SamplingParameters())
    assert cache.lengths() == [2, 5]
    assert cache.trim(4) == 4
    assert cache.lengths() == [0, 1]


# --------------------------------------------------------------------------- #
# tiny Llama-style model vs the CPU oracle
# --------------------------------------------------------------------------- #
TINY2 = M.ModelConfig(2, 512, 8, 2, 64, 1408, 32000, True, False, 1e-5, 500000.0, name="tiny2")
QWEN_SMALL = M.ModelConfig(2, 1024, 16, 4, 128, 2816, 4096, True, True, 1e-6, 1e6, name="qwen-small")


def segment_prompt(vocab, n_seg, seg_len, length, seed):
    rng = np.random.default_rng(seed)
    pool = rng.integers(0, vocab, size=(n_seg, seg_len))
    out = []
    while len(out) < length:
        out += pool[rng.integers(0, n_seg)].tolist()
    return out[:length]


def oracle_model(cfg, seed):
    ocfg = O.make_config(cfg.n_layers, cfg.hidden, cfg.n_heads, cfg.n_kv_heads, cfg.head_dim,
                         cfg.intermediate, cfg.vocab, cfg.tie_embeddings, cfg.qk_norm, cfg.rms_eps,
                         cfg.rope_theta)
    return O.Model.synth(ocfg, seed, 0.02)


@pytest.mark.parametrize("cfg", [TINY2, QWEN_SMALL], ids=lambda c: c.name)
def test_synth_weights_bit_identical_to_oracle(cfg):
    ctx = M.Context(cfg)
    ctx.synth_weights(42)
    om = oracle_model(cfg, 42)
    for tid, (N, K) in [(0, (cfg.n_heads * cfg.head_dim, cfg.hidden)),
                        (1 * 16 + 6, (cfg.hidden, cfg.intermediate)),
                        (A.TENSOR_EMBED, (cfg.vocab, cfg.hidden))]:
        got = ctx.get_q4(tid, N, K)
        want = om.get_q4(tid)
        for g, w in zip(got, want):
            np.testing.assert_array_equal(g, w)


@pytest.mark.parametrize("cfg", [TINY2, QWEN_SMALL], ids=lambda c: c.name)
def test_verify_logits_and_kv_match_oracle(cfg):
    seed, k = 7, 4
    ctx = M.Context(cfg)
    ctx.synth_weights(seed)
    om = oracle_model(cfg, seed)
    rows = 3
    prompts = [segment_prompt(cfg.vocab, 8, 16, L, 100 + r) for r, L in enumerate([150, 40, 333])]
    spec = M.SpeculativeDecodingConfiguration(True, k, 3, 8, A.ACCEPT_PREFIX)
    cache = M.BatchKVCache(ctx, rows, 512)
    gen = O.Generator(om, rows, 512, O.SpecConfig(A.ACCEPT_PREFIX, 1, k, 3, 8))
    firsts = [cache.insert_row(r, p, 64, M.SamplingParameters()) for r, p in enumerate(prompts)]
    ofirst = [gen.admit(r, p, 64, O.sampling()) for r, p in enumerate(prompts)]
    # KV after prefill: fp16 cache vs fp32 oracle
    for r in range(rows):
        kk, vv = cache.extract_row(r, cfg.n_layers - 1)
        ok = gen.kv.k(r, cfg.n_layers - 1, cfg.n_kv_heads, cfg.head_dim)[:, :len(prompts[r])]
        np.testing.assert_allclose(kk.astype(np.float32), ok, rtol=TOL, atol=TOL)
    drafts = cache.draft(spec)
    logits = cache.verify_forward(spec)
    for r in range(rows):
        h = cache.history(r)
        assert h[:-1] == prompts[r] and h[-1] == firsts[r]
        assert gen.history(r)[:-1] == prompts[r]
        assert drafts[r] == (O.propose_suffix(h, 3, 8, k) or [])
        toks = [h[-1]] + drafts[r]
        kvlen = len(prompts[r])
        ol = O.forward(om, gen.kv, toks, [r] * len(toks), list(range(kvlen, kvlen + len(toks))))
        np.testing.assert_allclose(logits[r, :len(toks)], ol, rtol=TOL, atol=TOL)
    tok, n, fin, stats = cache.accept(spec)
    lens = cache.lengths()
    for r in range(rows):
        assert lens[r] == len(prompts[r]) + int(n[r])
        assert cache.history(r) == prompts[r] + [firsts[r]] + tok[r, :n[r]].tolist()


def streams_agree(a, b, logit_gap_ok):
    for i, (x, y) in enumerate(zip(a, b)):
        if x != y:
            return logit_gap_ok(i)
    return len(a) == len(b)


@pytest.mark.parametrize("mode", [A.ACCEPT_COMPAT, A.ACCEPT_PREFIX])
def test_speculative_stream_equals_plain_greedy_on_device(mode):
    cfg = TINY2
    ctx = M.Context(cfg)
    ctx.synth_weights(3)
    prompt = segment_prompt(cfg.vocab, 4, 24, 200, 5)

    def run(spec):
        sched = M.Scheduler(ctx, 1, 512, spec)
        sched.submit(M.Request("a", prompt, 96, M.SamplingParameters()))
        out = []
        while not sched.is_idle:
            out += [r.token for r in sched.step()]
        return out, sched.speculative_decoding_stats, sched.generator.decode_calls

    base, _, base_calls = run(M.SpeculativeDecodingConfiguration.disabled)
    spec, stats, calls = run(M.SpeculativeDecodingConfiguration(True, 4, 3, 8, mode))
    assert spec == base
    assert len(base) == 96
    if stats.accepted_token_count > 0:
        assert calls < base_calls


def test_batched_rows_match_single_row_runs():
    """Batch invariance: a row's greedy tokens do not depend on its neighbours."""
    cfg = TINY2
    ctx = M.Context(cfg)
    ctx.synth_weights(9)
    prompts = [segment_prompt(cfg.vocab, 4, 20, L, 50 + i) for i, L in enumerate([120, 64, 200, 90])]
    spec = M.SpeculativeDecodingConfiguration(True, 4, 3, 8, A.ACCEPT_PREFIX)

    def run(ps):
        sched = M.Scheduler(ctx, len(ps), 512, spec)
        for i, p in enumerate(ps):
            sched.submit(M.Request(f"r{i}", p, 48, M.SamplingParameters()))
        out = {f"r{i}": [] for i in range(len(ps))}
        while not sched.is_idle:
            for r in sched.step():
                out[r.uid].append(r.token)
        return out

    together = run(prompts)
    for i, p in enumerate(prompts):
        alone = run([p])["r0"]
        assert together[f"r{i}"] == alone


def test_greedy_stream_matches_oracle_except_near_ties():
    cfg = TINY2
    seed = 21
    ctx = M.Context(cfg)
    ctx.synth_weights(seed)
    om = oracle_model(cfg, seed)
    prompt = segment_prompt(cfg.vocab, 6, 16, 160, 8)
    spec = M.SpeculativeDecodingConfiguration(True, 4, 3, 8, A.ACCEPT_PREFIX)
    sched = M.Scheduler(ctx, 1, 512, spec)
    sched.submit(M.Request("a", prompt, 40, M.SamplingParameters()))
    got = []
    while not sched.is_idle:
        got += [r.token for r in sched.step()]
    # oracle plain greedy decode, recording the top-2 gap at every position
    kv = O.KV(om, 1, 512)
    logits = O.forward(om, kv, prompt, [0] * len(prompt), list(range(len(prompt))))[-1:]
    want, gaps = [], []
    pos = len(prompt)
    for _ in range(40):
        top2 = np.sort(logits[0])[-2:]
        gaps.append(top2[1] - top2[0])
        t = int(np.argmax(logits[0]))
        want.append(t)
        logits = O.forward(om, kv, [t], [0], [pos])
        pos += 1
    for i, (g, w) in enumerate(zip(got, want)):
        if g != w:
            assert gaps[i] < 1e-2, f"position {i}: {g} != {w} with top-2 gap {gaps[i]}"
            break


def test_seeded_rows_independent_of_batch_composition():
    """PerRequestRNGTests.swift:8-41 on the device: temperature rows with their
    own seed produce the same tokens alone and beside other rows."""
    cfg = TINY2
    ctx = M.Context(cfg)
    ctx.synth_weights(13)
    spec = M.SpeculativeDecodingConfiguration(True, 4, 3, 8, A.ACCEPT_PREFIX)
    pa = segment_prompt(cfg.vocab, 4, 16, 100, 1)
    pb = segment_prompt(cfg.vocab, 4, 16, 80, 2)
    sa = M.SamplingParameters(temperature=1.0, top_p=0.9, seed=11)
    sb = M.SamplingParameters(temperature=0.7, seed=29)

    def run(reqs):
        sched = M.Scheduler(ctx, len(reqs), 512, spec)
        for uid, p, s in reqs:
            sched.submit(M.Request(uid, p, 24, s))
        out = {uid: [] for uid, _, _ in reqs}
        while not sched.is_idle:
            for r in sched.step():
                out[r.uid].append(r.token)
        return out

    mixed = run([("a", pa, sa), ("b", pb, sb), ("g", pb, M.SamplingParameters())])
    assert run([("a", pa, sa)])["a"] == mixed["a"]
    assert run([("b", pb, sb)])["b"] == mixed["b"]
    assert run([("b", pb, sb), ("a", pa, sa)])["a"] == mixed["a"]


def test_sampled_step_matches_oracle_given_device_logits():
    """Rejection sampling on the device equals the oracle's on the logits the
    device verify forward produced (same uniforms: seed + generation index)."""
    cfg = TINY2
    ctx = M.Context(cfg)
    ctx.synth_weights(17)
    spec = M.SpeculativeDecodingConfiguration(True, 4, 3, 8, A.ACCEPT_PREFIX)
    prompts = [segment_prompt(cfg.vocab, 3, 12, 96, 30 + i) for i in range(4)]
    cache = M.BatchKVCache(ctx, 4, 512)
    sps = [M.SamplingParameters(temperature=t, top_p=p, seed=500 + i)
           for i, (t, p) in enumerate([(0.7, 0.9), (1.0, 0.0), (0.3, 0.5), (0.0, 0.0)])]
    for r, p in enumerate(prompts):
        cache.insert_row(r, p, 64, sps[r])
    for _ in range(4):
        hist = [cache.history(r) for r in range(4)]
        drafts = cache.draft(spec)
        logits = cache.verify_forward(spec)
        tok, n, fin, _ = cache.accept(spec)
        for r in range(4):
            s = sps[r]
            osp = O.sampling(temperature=s.temperature, top_p=s.top_p, seed=s.seed)
            n_gen = len(hist[r]) - len(prompts[r])
            out, _ = O.accept_row(A.ACCEPT_PREFIX, logits[r, :len(drafts[r]) + 1], drafts[r], osp, n_gen)
            assert tok[r, :n[r]].tolist() == out


# Llama-3-8B layer shape (hidden 4096, 32/8 heads of 128, SwiGLU 14336, untied
# head, no q/k norm, theta 5e5) at one layer and a reduced vocabulary: the q4
# linears at K = 4096 and 14336 and the sampled acceptance of that config
LLAMA8B_LAYER = M.ModelConfig(1, 4096, 32, 8, 128, 14336, 8192, False, False, 1e-5, 500000.0,
                              name="llama8b-layer")


def test_llama8b_layer_verify_and_sampled_acceptance_match_oracle():
    cfg = LLAMA8B_LAYER
    seed, k = 11, 4
    ctx = M.Context(cfg)
    ctx.synth_weights(seed)
    om = oracle_model(cfg, seed)
    rows = 2
    prompts = [segment_prompt(cfg.vocab, 4, 12, L, 700 + r) for r, L in enumerate([48, 30])]
    sps = [M.SamplingParameters(temperature=0.7, top_p=0.9, seed=9000 + r) for r in range(rows)]
    spec = M.SpeculativeDecodingConfiguration(True, k, 4, 8, A.ACCEPT_PREFIX)
    cache = M.BatchKVCache(ctx, rows, 128)
    gen = O.Generator(om, rows, 128, O.SpecConfig(A.ACCEPT_PREFIX, 1, k, 4, 8))
    for r, p in enumerate(prompts):
        cache.insert_row(r, p, 32, sps[r])
        gen.admit(r, p, 32, O.sampling(temperature=0.7, top_p=0.9, seed=9000 + r))
    hist = [cache.history(r) for r in range(rows)]
    drafts = cache.draft(spec)
    logits = cache.verify_forward(spec)
    tok, n, fin, _ = cache.accept(spec)
    for r in range(rows):
        assert drafts[r] == (O.propose_suffix(hist[r], 4, 8, k) or [])
        toks = [hist[r][-1]] + drafts[r]
        kvlen = len(prompts[r])
        ol = O.forward(om, gen.kv, toks, [r] * len(toks), list(range(kvlen, kvlen + len(toks))))
        np.testing.assert_allclose(logits[r, :len(toks)], ol, rtol=TOL, atol=TOL)
        osp = O.sampling(temperature=0.7, top_p=0.9, seed=9000 + r)
        out, _ = O.accept_row(A.ACCEPT_PREFIX, logits[r, :len(toks)], drafts[r], osp, len(hist[r]) - kvlen)
        assert tok[r, :n[r]].tolist() == out
