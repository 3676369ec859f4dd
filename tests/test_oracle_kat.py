"""Pin the CPU oracle against the reference's own known answers.

Each test restates a test of the mlxcat project (path:line given) with the
same fake models and inputs.  These run without a GPU.
"""
import math
import random

import numpy as np
import pytest


# --------------------------------------------------------------------------- #
# Philox4x32-10 known answers (Random123 kat_vectors, Salmon et al. SC'11)
# --------------------------------------------------------------------------- #
@pytest.mark.parametrize("ctr,key,want", [
    ([0, 0, 0, 0], [0, 0], [0x6627e8d5, 0xe169c58d, 0xbc57ac4c, 0x9b00dbd8]),
    ([0xffffffff] * 4, [0xffffffff] * 2, [0x408f276d, 0x41c83b0e, 0xa20bc7c6, 0x6d5451fd]),
    ([0x243f6a88, 0x85a308d3, 0x13198a2e, 0x03707344], [0xa4093822, 0x299f31d0],
     [0xd16cfe09, 0x94fdcceb, 0x5001e420, 0x24126ea1]),
])
def test_philox_known_answers(orc, ctr, key, want):
    assert orc.philox(ctr, key).tolist() == want


def test_exp_log_accuracy(orc):
    for x in np.linspace(-86.0, 0.0, 4001, dtype=np.float32):
        ref = math.exp(float(x))
        assert abs(orc.exp_neg(float(x)) - ref) <= 2e-7 * ref
    for y in np.exp(np.linspace(-40.0, 0.0, 4001)).astype(np.float32):
        assert abs(orc.log(float(y)) - math.log(float(y))) <= 4e-6


def test_normal_moments(orc):
    z = np.array([orc.normal(7, 0, i) for i in range(40000)])
    assert abs(z.mean()) < 0.02
    assert abs(z.std() - 1.0) < 0.02


# --------------------------------------------------------------------------- #
# MLX affine q4 format
# --------------------------------------------------------------------------- #
def test_q4_roundtrip_and_layout(orc):
    rng = np.random.default_rng(0)
    w = rng.normal(0, 0.02, size=(8, 256)).astype(np.float32)
    wq, s, b = orc.q4_quantize(w)
    deq = orc.q4_dequant(wq, s, b)
    # error bounded by half a quantisation step (+ fp16 rounding of scale/bias)
    step = np.repeat(s.view(np.float16).astype(np.float32), 64, axis=1)
    assert np.all(np.abs(deq - w) <= 0.5 * step + 1e-3 * np.abs(w) + 2e-5)
    # lowest nibble first: nibble i of word j is element 8j+i
    q = ((wq[:, :, None] >> (4 * np.arange(8, dtype=np.uint32))) & 0xF).reshape(8, 256)
    sf = np.repeat(s.view(np.float16).astype(np.float32), 64, axis=1)
    bf = np.repeat(b.view(np.float16).astype(np.float32), 64, axis=1)
    np.testing.assert_array_equal((sf * q.astype(np.float32) + bf).astype(np.float32), deq)


def test_q4_linear_matches_numpy(orc):
    rng = np.random.default_rng(1)
    wq, s, b = orc.q4_synth(3, 5, 0.02, 96, 192)
    w = orc.q4_dequant(wq, s, b)
    x = rng.normal(size=(7, 192)).astype(np.float32)
    np.testing.assert_allclose(orc.q4_linear(wq, s, b, x), x @ w.T, rtol=1e-4, atol=1e-5)


# --------------------------------------------------------------------------- #
# Drafter: BatchGenerator.swift:982-1010
# --------------------------------------------------------------------------- #
def reference_propose(context, max_suffix, min_ctx, limit):
    """Literal transcription of proposeSuffixTokens (small inputs only)."""
    if len(context) < min_ctx or limit <= 0:
        return None
    max_len = min(max_suffix, len(context) - 1)
    if max_len <= 0:
        return None
    for L in range(max_len, 0, -1):
        suffix_start = len(context) - L
        suffix = context[suffix_start:]
        if suffix_start <= 0:
            continue
        for c in range(suffix_start - 1, -1, -1):
            end = c + L
            if end > suffix_start:
                continue
            if context[c:end] == suffix:
                ps, pe = end, min(len(context), end + limit)
                if ps >= pe:
                    continue
                return context[ps:pe]
    return None


def test_drafter_matches_literal_transcription(orc):
    rnd = random.Random(5)
    for _ in range(3000):
        n = rnd.randint(0, 60)
        vocab = rnd.choice([2, 3, 5, 50])
        ctx = [rnd.randrange(vocab) for _ in range(n)]
        ms, mc, lim = rnd.randint(1, 8), rnd.randint(2, 10), rnd.randint(0, 6)
        assert orc.propose_suffix(ctx, ms, mc, lim) == reference_propose(ctx, ms, mc, lim)


def test_drafter_known_cases(orc):
    hist = [1, 2, 3, 1, 2, 3, 1, 2, 3]
    assert orc.propose_suffix(hist, 16, 8, 4) == [1, 2, 3]
    assert orc.propose_suffix(hist, 16, 10, 4) is None          # below minContext
    assert orc.propose_suffix([5, 6, 7, 8, 9, 10, 11, 12], 16, 8, 4) is None


# --------------------------------------------------------------------------- #
# Scheduler speculation tests: SchedulerSpeculativeDecodingTests.swift:9-106
# --------------------------------------------------------------------------- #
def repeating_table(vocab=8, mismatch=False):
    nxt = [1] * vocab
    nxt[1], nxt[2] = 2, 3
    if mismatch:
        nxt[3] = 4
    return nxt


def run_scheduler(orc, table, prompt, spec_enabled, max_tokens=10, k=4, min_ctx=8,
                  trigger=-1, mode=0):
    model = orc.Model.table(table)
    spec = orc.SpecConfig(mode, int(spec_enabled), k, 16, min_ctx)
    gen = orc.Generator(model, 1, 256, spec)
    sp = orc.sampling(temperature=0.0, trigger=trigger)
    tokens = [gen.admit(0, prompt, max_tokens, sp)]
    calls = 0
    while gen.active(0):
        out = gen.step()
        calls += 1
        tokens += out[0]
    return tokens, gen.stats, calls


def test_ngram_speculation_identical_tokens_fewer_calls(orc):
    """:9-38 -- identical tokens, accepted > 0, fewer decode calls."""
    prompt = [1, 2, 3, 1, 2, 3, 1, 2]
    base, _, base_calls = run_scheduler(orc, repeating_table(), prompt, False)
    spec, stats, spec_calls = run_scheduler(orc, repeating_table(), prompt, True)
    assert spec == base
    assert len(spec) == 10
    assert base == [3, 1, 2, 3, 1, 2, 3, 1, 2, 3]
    assert stats.accepted > 0 and stats.proposal_batches > 0
    assert spec_calls < base_calls
    assert (len(spec) - 1) / spec_calls > (len(base) - 1) / base_calls


def test_rejected_proposal_falls_back_without_changing_output(orc):
    """:40-62 -- mismatching model, identical tokens, rejected > 0."""
    prompt = [1, 2, 3, 1, 2, 3, 1, 2]
    base, _, _ = run_scheduler(orc, repeating_table(mismatch=True), prompt, False)
    spec, stats, _ = run_scheduler(orc, repeating_table(mismatch=True), prompt, True)
    assert spec == base
    assert stats.rejected_batches > 0


def test_trigger_token_keeps_speculation_before_trigger(orc):
    """:64-80 -- a trigger that never appears leaves speculation on."""
    prompt = [1, 2, 3, 1, 2, 3, 1, 2]
    _, stats, _ = run_scheduler(orc, repeating_table(), prompt, True, trigger=7)
    assert stats.proposal_batches > 0 and stats.accepted > 0


def test_trigger_token_replays_through_ordinary_path(orc):
    """:82-106 -- a sampled trigger rejects the speculative batch.

    The reference's expected stream [1,2,4,5,6] comes from its tool grammar
    forcing the body tokens after the trigger; grammars are outside this
    path, so the stream here continues with the model's own tokens.  The
    parts that belong to the path are kept: the first two tokens (1, 2), the
    speculative stream equal to the plain one, and rejected batches > 0."""
    prompt = [1, 2, 3, 1, 2, 3]
    base, _, _ = run_scheduler(orc, repeating_table(), prompt, False, max_tokens=5,
                               min_ctx=6, trigger=2)
    spec, stats, _ = run_scheduler(orc, repeating_table(), prompt, True, max_tokens=5,
                                   min_ctx=6, trigger=2)
    assert base[:2] == [1, 2]
    assert spec == base
    assert stats.rejected_batches > 0


@pytest.mark.parametrize("mismatch", [False, True])
def test_prefix_mode_same_stream_as_plain_decode(orc, mismatch):
    prompt = [1, 2, 3, 1, 2, 3, 1, 2]
    base, _, _ = run_scheduler(orc, repeating_table(mismatch=mismatch), prompt, False,
                               max_tokens=40)
    spec, stats, calls = run_scheduler(orc, repeating_table(mismatch=mismatch), prompt, True,
                                       max_tokens=40, mode=orc.MODE_PREFIX)
    assert spec == base
    assert calls < len(base) - 1


# --------------------------------------------------------------------------- #
# Cache trim: BatchCacheShapeTests.swift:170-193
# --------------------------------------------------------------------------- #
def test_trim_keeps_mixed_length_rows_consistent(orc):
    model = orc.Model.table(repeating_table())
    kv = orc.KV(model, 2, 16)
    kv.set_len(0, 2)
    kv.set_len(1, 5)
    assert kv.trim(4) == 4
    assert [kv.len(0), kv.len(1)] == [0, 1]


# --------------------------------------------------------------------------- #
# Top-p: TopPSamplingTests.swift:10-54
# --------------------------------------------------------------------------- #
TINY = [1e-8, 1e-6, 1e-4, 1e-3]


def test_top_p_keeps_only_most_likely_at_tiny_thresholds(orc):
    with np.errstate(divide="ignore"):
        logp = np.log(np.array([0.9, 0, 0, 0.1], np.float32))
    for p in TINY:
        assert orc.top_p_keep(logp, p).tolist() == [True, False, False, False]


def test_top_p_never_masks_every_token(orc):
    rng = np.random.default_rng(0)
    logits = (rng.normal(size=(2, 4096)) * 3).astype(np.float32)
    for row in logits:
        for dt in (np.float32, np.float16):
            typed = row.astype(dt).astype(np.float32)
            for p in TINY:
                keep = orc.top_p_keep(typed, p)
                assert keep.sum() > 0
                assert keep[np.argmax(typed)]


def test_top_p_keeps_nucleus_at_ordinary_threshold(orc):
    logp = np.log(np.array([0.5, 0.3, 0.15, 0.05], np.float32))
    assert orc.top_p_keep(logp, 0.7).tolist() == [True, True, False, False]


# --------------------------------------------------------------------------- #
# Rejection sampling (extension): exactness of the accept rule
# --------------------------------------------------------------------------- #
def test_rejection_sampling_preserves_target_distribution(orc):
    """Accept-then-residual sampling with a point-mass draft reproduces the
    target distribution (checked in expectation over the uniform stream)."""
    logits = np.array([1.0, 0.2, -0.5, 0.7, -2.0], np.float32)
    P, S = orc.fixed_dist(logits, 0.8, 0.0)
    target = P / S
    counts = np.zeros(5)
    n = 20000
    for i in range(n):
        sp = orc.sampling(temperature=0.8, seed=11)
        out, _ = orc.accept_row(orc.MODE_PREFIX, np.stack([logits, logits]), [3], sp, i)
        counts[out[0]] += 1
    assert np.abs(counts / n - target).max() < 0.012


def test_seeded_stream_is_independent_of_batch_composition(orc):
    """PerRequestRNGTests.swift:8-41 property: a seeded row's tokens depend on
    its own seed only, not on the rows beside it."""
    rng = np.random.default_rng(2)
    logits = rng.normal(size=(6, 50)).astype(np.float32)
    sp_a = orc.sampling(temperature=1.0, seed=11)
    alone = [orc.accept_row(orc.MODE_PREFIX, logits[i:i + 1], [], sp_a, i)[0] for i in range(6)]
    again = [orc.accept_row(orc.MODE_PREFIX, logits[i:i + 1], [], sp_a, i)[0] for i in range(6)]
    assert alone == again
    sp_b = orc.sampling(temperature=1.0, seed=29)
    other = [orc.accept_row(orc.MODE_PREFIX, logits[i:i + 1], [], sp_b, i)[0] for i in range(6)]
    assert other != alone
