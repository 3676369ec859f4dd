"""Grammar-constrained speculation on the GPU (mlxcat_cache_set_token_masks).

The tiny two-layer model's verify logits come from the device; the host sets
allowed-token masks per row and verify position; the device acceptance must
equal the oracle's acceptance on the same logits with the same masks applied
by the oracle's restatement of applyAllowedTokenMask (Sampling.swift:557-569),
bit for bit, for greedy and seeded-sampling rows.  Masks that allow only the
draft token force acceptance at that position (a constrained row keeps its
speculation), and every emitted token lies in its position's allowed set.
A choice-constrained row (allowedSequences) decodes exactly one of its
choices while speculating."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")
if not torch.cuda.is_available():
    pytest.skip("needs a CUDA device", allow_module_level=True)

import mlxcat_b200 as M  # noqa: E402
from mlxcat_b200 import _abi as A  # noqa: E402
from oracle import oracle as O  # noqa: E402

TINY2 = M.ModelConfig(2, 512, 8, 2, 64, 1408, 32000, True, False, 1e-5, 500000.0, name="tiny2")
K = 4


def segment_prompt(vocab, n_seg, seg_len, length, seed):
    rng = np.random.default_rng(seed)
    pool = rng.integers(0, vocab, size=(n_seg, seg_len))
    out = []
    while len(out) < length:
        out += pool[rng.integers(0, n_seg)].tolist()
    return out[:length]


def random_masks(rng, drafts, V):
    masks = {}
    for r, d in enumerate(drafts):
        for p in range(len(d) + 1):
            kind = rng.integers(0, 5)
            if kind == 0:
                continue                                   # unconstrained
            if kind == 1 and p < len(d):
                masks[(r, p)] = [d[p]]                     # only the draft: forced acceptance
            elif kind == 2:
                masks[(r, p)] = [V + 5, V + 100]           # no valid id: unchanged
            else:
                ids = rng.choice(V, size=40, replace=False).tolist()
                if p < len(d) and rng.random() < 0.5:
                    ids.append(d[p])
                masks[(r, p)] = ids
    return masks


def test_masked_acceptance_matches_oracle():
    cfg = TINY2
    V = cfg.vocab
    rng = np.random.default_rng(5)
    ctx = M.Context(cfg)
    ctx.synth_weights(17)
    spec = M.SpeculativeDecodingConfiguration(True, K, 3, 8, A.ACCEPT_PREFIX)
    prompts = [segment_prompt(V, 3, 12, 96, 60 + i) for i in range(4)]
    sps = [M.SamplingParameters(temperature=t, top_p=p, seed=900 + i)
           for i, (t, p) in enumerate([(0.0, 0.0), (0.7, 0.9), (0.0, 0.0), (1.0, 0.0)])]
    cache = M.BatchKVCache(ctx, 4, 512)
    for r, p in enumerate(prompts):
        cache.insert_row(r, p, 64, sps[r])
    forced = 0
    for step in range(5):
        hist = [cache.history(r) for r in range(4)]
        drafts = cache.draft(spec)
        logits = cache.verify_forward(spec)
        masks = random_masks(rng, drafts, V)
        cache.set_token_masks(K, masks)
        tok, n, fin, _ = cache.accept(spec)
        for r in range(4):
            s = sps[r]
            osp = O.sampling(temperature=s.temperature, top_p=s.top_p, seed=s.seed)
            c = len(drafts[r])
            ml = np.stack([O.apply_allowed_mask(logits[r, p], masks.get((r, p), [])) for p in range(c + 1)])
            out, _ = O.accept_row(A.ACCEPT_PREFIX, ml, drafts[r], osp, len(hist[r]) - len(prompts[r]))
            assert tok[r, :n[r]].tolist() == out, (step, r)
            for p, t in enumerate(out):
                ids = [i for i in masks.get((r, p), []) if 0 <= i < V]
                if ids:
                    assert t in ids, (step, r, p)
            # a position whose mask allows only its draft accepts it
            for p in range(c):
                if masks.get((r, p)) != [drafts[r][p]]:
                    break
                assert p < len(out) and out[p] == drafts[r][p]
                forced += 1
    assert forced > 0


def test_pending_masks_block_the_fused_step():
    ctx = M.Context(TINY2)
    ctx.synth_weights(3)
    spec = M.SpeculativeDecodingConfiguration(True, K, 3, 8, A.ACCEPT_PREFIX)
    cache = M.BatchKVCache(ctx, 1, 256)
    cache.insert_row(0, segment_prompt(TINY2.vocab, 3, 12, 64, 1), 32, M.SamplingParameters())
    cache.set_token_masks(K, {(0, 0): [1, 2, 3]})
    with pytest.raises(RuntimeError, match="masks are pending"):
        cache.spec_step(spec)
    cache.clear_token_masks()
    cache.spec_step(spec)


def test_choice_row_speculates_and_decodes_a_choice():
    """A choice-constrained greedy row (allowedSequences) through the split
    step: the host computes each position's allowed set along the drafts; the
    output is one of the choices, and drafts along it are accepted."""
    cfg = TINY2
    ctx = M.Context(cfg)
    ctx.synth_weights(29)
    spec = M.SpeculativeDecodingConfiguration(True, K, 3, 8, A.ACCEPT_PREFIX)
    eos = 7
    choices = [[101, 102, 103, 104, 105, 106, eos], [101, 102, 203, 204, 205, eos]]
    # the prompt repeats the first choice so the drafter proposes along it
    prompt = segment_prompt(cfg.vocab, 3, 12, 60, 2) + choices[0][:-1] + [300] + choices[0][:-1] + [300]
    cache = M.BatchKVCache(ctx, 1, 256)
    first = cache.insert_row(0, prompt, 16, M.SamplingParameters(eos_token_ids=[eos]))
    # admission sampled the first token unconstrained; the constraint starts after it
    gen = []
    seqs = [[first] + c for c in choices]
    accepted_drafts = 0
    for _ in range(8):
        d = cache.draft(spec)[0]
        cache.verify_forward(spec, want_logits=False)
        cache.set_token_masks(K, M.speculative_token_masks(0, seqs, [first] + gen, d))
        tok, n, fin, st = cache.accept(spec)
        emitted = tok[0, :n[0]].tolist()
        accepted_drafts += sum(1 for a, b in zip(emitted, d) if a == b)
        gen += emitted
        if fin[0]:
            break
    assert gen in [c for c in choices], gen
    assert accepted_drafts > 0
