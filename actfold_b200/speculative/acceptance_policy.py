"""Which candidate a folded-generation step keeps (actfold/speculative/acceptance_policy.py:12-83).

* GreedyAcceptancePolicy: the candidate whose last position has the largest
  logit (averaged over the batch); a single candidate is returned as is.
* ThresholdAcceptancePolicy: greedy among the candidates whose
  ``metadata["stable_ratio"]`` reaches the threshold (all of them when none does).
"""

from __future__ import annotations

from abc import ABC, abstractmethod

import torch

from actfold_b200.speculative.branch_tree import BranchNode


class AcceptancePolicy(ABC):
    @abstractmethod
    def select(self, candidates: list[BranchNode], logits: torch.Tensor | None = None) -> BranchNode:
        ...


class GreedyAcceptancePolicy(AcceptancePolicy):
    def select(self, candidates: list[BranchNode], logits: torch.Tensor | None = None) -> BranchNode:
        if len(candidates) == 1:
            return candidates[0]
        scored = [n for n in candidates if n.logits is not None]
        if not scored:
            return candidates[0]
        # One device read for all candidates: max over the vocabulary of the last position, batch mean.
        scores = torch.stack([n.logits[:, -1, :].float().amax(dim=-1).mean() for n in scored]).cpu().tolist()
        best = max(range(len(scored)), key=lambda i: (scores[i], -i))  # the first of equal scores wins
        return scored[best]


class ThresholdAcceptancePolicy(AcceptancePolicy):
    def __init__(self, threshold: float = 0.0) -> None:
        if not 0.0 <= threshold <= 1.0:
            raise ValueError(f"threshold must be in [0, 1], got {threshold}")
        self.threshold = threshold
        self.greedy = GreedyAcceptancePolicy()

    def select(self, candidates: list[BranchNode], logits: torch.Tensor | None = None) -> BranchNode:
        eligible = [n for n in candidates
                    if n.logits is not None and n.metadata.get("stable_ratio", 1.0) >= self.threshold]
        return self.greedy.select(eligible or candidates, logits)
