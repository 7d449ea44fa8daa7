"""Host logic of folded generation: the branch tree and the acceptance policies (CPU only).

Mirrors the behaviour of actfold/speculative/branch_tree.py:36-95 and
acceptance_policy.py:12-83 on small hand-made nodes.
"""

from __future__ import annotations

import pytest
import torch

from actfold_b200.speculative import (BranchNode, BranchTree, GreedyAcceptancePolicy, ThresholdAcceptancePolicy,
                                      folded_generate)


def _node(bid, parent, last_logit=None, ratio=None, depth=0):
    n = BranchNode(bid, parent, torch.zeros(1, 3, dtype=torch.long), depth=depth)
    if last_logit is not None:
        lg = torch.zeros(1, 3, 5)
        lg[0, -1, 2] = last_logit
        n.logits = lg
    if ratio is not None:
        n.metadata["stable_ratio"] = ratio
    return n


def test_tree_links_ancestors_prune_and_leaf():
    root = _node("r", None)
    t = BranchTree(root)
    a, b = _node("a", "r", depth=1), _node("b", "r", depth=1)
    c = _node("c", "a", depth=2)
    for n in (a, b, c):
        t.add(n)
    assert root.children == ["a", "b"] and a.children == ["c"]
    assert t.get_ancestors("c") == ["r", "a"] and t.get_ancestors("c", include_self=True) == ["r", "a", "c"]
    assert t.best_accepted_leaf() is c
    t.prune("a")  # the subtree goes, the parent forgets it
    assert t.get("a") is None and t.get("c") is None and root.children == ["b"]
    t.prune("missing")
    b.accepted = False
    root.accepted = False
    assert t.best_accepted_leaf() is root  # none accepted: the root


def test_greedy_policy_takes_the_largest_last_logit_first_on_ties():
    p = GreedyAcceptancePolicy()
    only = _node("x", None)
    assert p.select([only]) is only
    a, b, c = _node("a", None, 1.0), _node("b", None, 3.0), _node("c", None, 3.0)
    assert p.select([a, b, c]) is b
    n = _node("n", None)  # no logits: skipped
    assert p.select([n, a]) is a
    assert p.select([n, _node("m", None)]) is n


def test_threshold_policy_filters_on_stable_ratio():
    with pytest.raises(ValueError):
        ThresholdAcceptancePolicy(1.5)
    p = ThresholdAcceptancePolicy(0.9)
    lo, hi = _node("lo", None, 5.0, ratio=0.5), _node("hi", None, 1.0, ratio=0.95)
    assert p.select([lo, hi]) is hi
    assert p.select([lo, _node("lo2", None, 9.0, ratio=0.1)]).branch_id == "lo2"  # none eligible: greedy over all


def test_folded_generate_without_folding_is_plain_greedy():
    """A model that ignores the branch arguments: the loop is greedy decoding (the reference's fallback test)."""
    class Counter(torch.nn.Module):
        def forward(self, tokens, **kwargs):
            V = 7
            lg = torch.zeros(tokens.shape[0], tokens.shape[1], V)
            lg[:, -1, (tokens[:, -1] + 1) % V] = 1.0
            return lg

    res = folded_generate(Counter(), torch.tensor([[1, 2, 3]]), max_new_tokens=3)
    assert res.tokens.tolist() == [[1, 2, 3, 4, 5, 6]]
    assert res.num_folded_steps == 3 and res.final_branch_id == "root/t0/d0/t1/d0/t2/d0"
    assert res.stable_ratio == 0.0
