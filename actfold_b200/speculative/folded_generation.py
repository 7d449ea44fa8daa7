"""Autoregressive generation in which every new token is verified by folding.

Drop-in for actfold/speculative/folded_generation.py:30-238 (``folded_generate``
and ``FoldedGenerationResult``): at each step candidate children extend the
accepted sequence by one token, each child is verified with the accepted
sequence as its parent (``parent_branch_id``), an AcceptancePolicy keeps one,
and the others are pruned from the branch tree.

Each child is one token longer than its parent: the parent's cached rows
cover the shared prefix and the new position gates against a zero row (the
reference zero-fills positions its parent has no entry for), so on the native
LLaDA / Dream pass every step folds the prefix and recomputes only the
divergent rows, and a verified child is promoted to the next step's parent on
the device. What changes against the reference: when the folded model runs
the native pass, all candidates of a step are verified in ONE batched pass
(branch ids given as a list), instead of one forward per candidate.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Any, Optional

import torch

from actfold_b200.profiler.stability_profiler import GLOBAL_STABILITY_PROFILER
from actfold_b200.speculative.acceptance_policy import AcceptancePolicy, GreedyAcceptancePolicy
from actfold_b200.speculative.branch_tree import BranchNode, BranchTree


@dataclass
class FoldedGenerationResult:
    tokens: torch.Tensor
    stable_ratio: float
    num_folded_steps: int
    final_branch_id: Any


def _next_branch_id(parent_id: Any, token_idx: int, draft_idx: int = 0) -> str:
    """Deterministic child id: ``<parent>/t<token>/d<draft>`` (the reference's naming)."""
    return f"{parent_id}/t{token_idx}/d{draft_idx}"


def _forward(fn, node_tokens: torch.Tensor, branch_id, parent_id, step_idx: int) -> torch.Tensor:
    call = getattr(fn, "forward", fn)
    return call(node_tokens, branch_id=branch_id, parent_branch_id=parent_id, step_idx=step_idx)


def _batched(folded_model) -> bool:
    """True when the folded model verifies a list of children in one pass (the native pass)."""
    return folded_model is not None and bool(getattr(folded_model, "_native", False)) and folded_model.folding_applied


def _evaluate(model, folded_model, nodes: list[BranchNode], step_idx: int) -> None:
    """Run the folded forward of every node (with its parent as parent branch) and store logits / stable ratio."""
    for n in nodes:
        GLOBAL_STABILITY_PROFILER.reset_branch(n.branch_id)
    runner = folded_model if folded_model is not None else model
    parents = {n.parent_id for n in nodes}
    if len(nodes) > 1 and _batched(folded_model) and len(parents) == 1 and len({n.seq_len for n in nodes}) == 1 \
            and all(n.tokens.shape[0] == 1 for n in nodes):
        logits = _forward(runner, torch.cat([n.tokens for n in nodes]), [n.branch_id for n in nodes],
                          nodes[0].parent_id, step_idx)
        for i, n in enumerate(nodes):
            n.logits = logits[i: i + 1]
    else:
        for n in nodes:
            n.logits = _forward(runner, n.tokens, n.branch_id, n.parent_id, step_idx)
    for n in nodes:
        prof = GLOBAL_STABILITY_PROFILER.get_profile(n.branch_id)
        if prof is not None:
            n.metadata["stable_ratio"] = prof.mean_stable_ratio


def _candidates(model, parent: BranchNode, token_idx: int, folded_model, draft_generator, num_branches: int,
                step_idx: int) -> list[BranchNode]:
    if draft_generator is not None and num_branches > 1:
        from actfold_b200.speculative.verification_engine import Branch

        drafts = draft_generator.generate(Branch(parent.branch_id, parent.parent_id, parent.tokens),
                                          num_branches=num_branches, max_new_tokens=1, seed=token_idx)
        return [BranchNode(_next_branch_id(parent.branch_id, token_idx, i), parent.branch_id, d.tokens.clone(),
                           depth=parent.depth + 1) for i, d in enumerate(drafts)]
    if parent.logits is None:
        # The greedy step needs the parent's own logits: one forward of the parent (no folded model).
        _evaluate(model, None, [parent], step_idx)
    if parent.logits is None:
        raise RuntimeError("Failed to obtain logits for greedy candidate generation.")
    nxt = parent.logits[:, -1, :].argmax(dim=-1, keepdim=True).to(parent.tokens.device, parent.tokens.dtype)
    return [BranchNode(_next_branch_id(parent.branch_id, token_idx, 0), parent.branch_id,
                       torch.cat([parent.tokens, nxt], dim=-1), depth=parent.depth + 1)]


def folded_generate(
    model,
    input_ids: torch.Tensor,
    max_new_tokens: int,
    folded_model=None,
    draft_generator=None,
    acceptance_policy: Optional[AcceptancePolicy] = None,
    num_branches_per_step: int = 1,
    record_stability: bool = True,
    step_idx: int = 0,
) -> FoldedGenerationResult:
    """Generate ``max_new_tokens`` tokens after ``input_ids`` [batch, prompt_len], folding every step.

    ``model`` is anything with ``forward(tokens, branch_id=, parent_branch_id=,
    step_idx=)`` -- a FoldedModel, or an adapter that routes to one; the
    candidates run through ``folded_model`` when given. ``draft_generator``
    (``generate(parent, num_branches=, max_new_tokens=1, seed=)``) proposes
    ``num_branches_per_step`` candidates per step; without one the single
    candidate appends the argmax of the accepted sequence's last logits.
    """
    if not record_stability:
        GLOBAL_STABILITY_PROFILER.set_enabled(False)
    policy = acceptance_policy or GreedyAcceptancePolicy()
    root = BranchNode(branch_id="root", parent_id=None, tokens=input_ids.clone(), depth=0)
    tree = BranchTree(root)
    active = root
    for token_idx in range(max_new_tokens):
        cands = _candidates(model, active, token_idx, folded_model, draft_generator, num_branches_per_step, step_idx)
        if not cands:
            break
        for n in cands:
            tree.add(n)
        _evaluate(model, folded_model, cands, step_idx)
        chosen = policy.select(cands)
        chosen.accepted = True
        for n in cands:
            if n.branch_id != chosen.branch_id:
                tree.prune(n.branch_id)
        active = chosen
    if not record_stability:
        GLOBAL_STABILITY_PROFILER.set_enabled(True)
    return FoldedGenerationResult(tokens=active.tokens, stable_ratio=float(active.metadata.get("stable_ratio", 0.0)),
                                  num_folded_steps=active.depth, final_branch_id=active.branch_id)
