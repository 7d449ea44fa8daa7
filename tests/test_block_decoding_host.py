"""Host logic of block decoding (drafts, children, acceptance) against the oracle's restatement; no GPU."""

from __future__ import annotations

import numpy as np
import pytest

from actfold_b200.speculative.block_decoding import (BlockDecodingConfig, SyntheticDraft, accept_child,
                                                     draft_children)


def test_config_validation():
    with pytest.raises(ValueError):
        BlockDecodingConfig(gen_len=33, block_size=32)
    with pytest.raises(ValueError):
        BlockDecodingConfig(min_edits=3, max_edits=2)
    with pytest.raises(ValueError):
        BlockDecodingConfig(acceptance_threshold=1.5)
    assert BlockDecodingConfig().seq == 2048
    e = BlockDecodingConfig().edits()
    assert e[0] == 2 and e[-1] == 8 and (np.diff(e) >= 0).all()


def test_draft_is_seeded_and_children_take_the_most_confident_positions():
    d = SyntheticDraft(1000, seed=9)
    pos = np.arange(100, 132)
    t1, c1 = d(4, pos)
    t2, c2 = d(4, pos)
    np.testing.assert_array_equal(t1, t2)
    np.testing.assert_array_equal(c1, c2)
    _, many = d(0, np.arange(20000))
    assert 0.16 < (many > 0.9).mean() < 0.22  # Beta(2, 1): P(conf > 0.9) = 0.19
    canvas = np.full(200, 7, np.int64)
    children, n = draft_children(canvas, pos, t1, c1, np.array([1, 3, 40]))
    assert n.tolist() == [1, 3, 32]
    order = np.argsort(-c1, kind="stable")
    for i, k in enumerate(n):
        changed = np.nonzero(children[i] != canvas)[0]
        assert set(changed) <= set(pos[order[:k]])
        np.testing.assert_array_equal(children[i][pos[order[:k]]], t1[order[:k]])


def test_acceptance_rule():
    cfg = BlockDecodingConfig(n_children=4, min_edits=2, max_edits=5, threshold=0.9, acceptance_threshold=0.5)
    n = np.array([2, 3, 4, 5])
    ratio = np.ones(4)
    # three positions above the threshold -> the child with 3 unmasked
    assert accept_child(n, np.array([0.95, 0.99, 0.91, 0.1, 0.2]), ratio, cfg) == 1
    # none above: the most confident one always, raised to min_edits
    assert accept_child(n, np.array([0.1, 0.2]), ratio, cfg) == 0
    # all above, but the largest children fall below the acceptance threshold
    assert accept_child(n, np.full(8, 0.99), np.array([1.0, 0.9, 0.4, 0.3]), cfg) == 1
    # nobody reaches the acceptance threshold: the rule alone decides
    assert accept_child(n, np.full(8, 0.99), np.zeros(4), cfg) == 3
    # equal unmasked counts (fewer masked positions than edits): the first such child
    assert accept_child(np.array([2, 2, 2, 2]), np.full(2, 0.99), ratio, cfg) == 0
