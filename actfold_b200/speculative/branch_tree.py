"""Branch nodes and the branch tree of folded generation.

The node fields and the tree operations (add, get, get_ancestors, prune,
best_accepted_leaf) are those of actfold/speculative/branch_tree.py:11-95,
which callers of ``folded_generate`` and the acceptance policies read.
"""

from __future__ import annotations

from dataclasses import dataclass, field
from typing import Any, Optional

import torch


@dataclass
class BranchNode:
    branch_id: Any
    parent_id: Optional[Any]
    tokens: torch.Tensor                   # [batch, seq_len]
    logits: Optional[torch.Tensor] = None  # [batch, seq_len, vocab]
    accepted: bool = True
    depth: int = 0
    children: list[Any] = field(default_factory=list)
    metadata: dict[str, Any] = field(default_factory=dict)

    @property
    def seq_len(self) -> int:
        return int(self.tokens.shape[1])


class BranchTree:
    """Nodes by id with parent -> children links; pruning drops a whole subtree."""

    def __init__(self, root: BranchNode) -> None:
        self._nodes: dict[Any, BranchNode] = {root.branch_id: root}
        self.root_id = root.branch_id

    def add(self, node: BranchNode) -> None:
        self._nodes[node.branch_id] = node
        parent = self._nodes.get(node.parent_id) if node.parent_id is not None else None
        if parent is not None and node.branch_id not in parent.children:
            parent.children.append(node.branch_id)

    def get(self, branch_id: Any) -> Optional[BranchNode]:
        return self._nodes.get(branch_id)

    def get_ancestors(self, branch_id: Any, include_self: bool = False) -> list[Any]:
        """Ids from the root down to ``branch_id``'s parent (and ``branch_id`` itself if asked)."""
        chain: list[Any] = [branch_id] if include_self else []
        node = self.get(branch_id)
        while node is not None and node.parent_id is not None:
            chain.append(node.parent_id)
            node = self.get(node.parent_id)
        return chain[::-1]

    def prune(self, branch_id: Any) -> None:
        stack = [branch_id]
        first = True
        while stack:
            node = self._nodes.pop(stack.pop(), None)
            if node is None:
                continue
            if first and node.parent_id is not None:
                parent = self._nodes.get(node.parent_id)
                if parent is not None and node.branch_id in parent.children:
                    parent.children.remove(node.branch_id)
            first = False
            stack.extend(node.children)

    def best_accepted_leaf(self) -> BranchNode:
        """The deepest accepted node (the root when none is accepted)."""
        best = None
        for n in self._nodes.values():
            if n.accepted and (best is None or n.depth > best.depth):
                best = n
        return best if best is not None else self._nodes[self.root_id]
