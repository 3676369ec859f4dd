"""Host side of grammar-constrained speculation, no GPU: the choice-mode
allowed sets (TokenSampler.allowedNextTokenIDs) against the reference's own
known answers (Tests/MLXCatTests/StructuredOutputTests.swift:327-413), the
per-position sets along a row's drafts, and the oracle's restatement of the
allow mask (Sampling.swift:557-569)."""
import numpy as np

from mlxcat_b200.engine import allowed_next_token_ids, speculative_token_masks
from oracle import oracle as O


def test_allowed_next_token_ids_prefix_cases():
    assert allowed_next_token_ids([[10, 20], [10, 30], [40]], [10]) == [20, 30]


def test_allowed_next_token_ids_excludes_completed_sequences():
    assert allowed_next_token_ids([[10], [10, 20]], [10]) == [20]


def test_allowed_next_token_ids_none_when_only_viable_sequence_is_complete():
    assert allowed_next_token_ids([[10, 20]], [10, 20]) is None


def test_allowed_next_token_ids_forces_eos_after_choice_text():
    eos = 999
    seqs = [[10, 20, eos], [30, 40, eos]]
    assert allowed_next_token_ids(seqs, [10, 20]) == [eos]
    assert allowed_next_token_ids(seqs, [10, 20, eos]) is None


def test_allowed_next_token_ids_none_for_empty_or_unmatched():
    assert allowed_next_token_ids([], []) is None
    assert allowed_next_token_ids([[10, 20]], [99]) is None


def test_choice_mask_constrains_greedy_argmax():
    logits = np.array([0.1, 99.0, 0.2, 0.3, 0.4, 0.5], np.float32)
    allowed = allowed_next_token_ids([[10, 2], [10, 4]], [10])
    masked = O.apply_allowed_mask(logits, allowed)
    assert int(np.argmax(masked)) in (2, 4)
    assert int(np.argmax(masked)) == 4
    assert np.isneginf(masked[[0, 1, 3, 5]]).all() and masked[2] == np.float32(0.2)


def test_mask_with_no_valid_id_leaves_logits_unchanged():
    logits = np.arange(6, dtype=np.float32)
    np.testing.assert_array_equal(O.apply_allowed_mask(logits, [6, 100, -1]), logits)
    np.testing.assert_array_equal(O.apply_allowed_mask(logits, []), logits)


def test_speculative_masks_follow_the_drafts():
    seqs = [[5, 6, 7, 9], [5, 6, 8]]
    # generated [5]; drafts [6, 7]: position 0 after [5], 1 after [5, 6], 2 after [5, 6, 7]
    m = speculative_token_masks(3, seqs, [5], [6, 7])
    assert m == {(3, 0): [6], (3, 1): [7, 8], (3, 2): [9]}
    # a draft that leaves every sequence: later positions unconstrained
    m = speculative_token_masks(0, seqs, [5], [4, 4])
    assert m == {(0, 0): [6]}
