"""Branch context carried from FoldedModel.forward down to each folded layer.

Same contract as actfold/core/folding_context.py:18-55: a ContextVar holds
``{"branch_id", "parent_branch_id", "step_idx"}`` for the duration of a
forward pass, so layers find their branch even when the wrapped model does
not forward extra keyword arguments.
"""

from __future__ import annotations

from contextvars import ContextVar
from typing import Any

FoldingContext = dict[str, Any] | None

FOLDING_CONTEXT: ContextVar[FoldingContext] = ContextVar("actfold_b200_folding_context", default=None)


class folding_scope:
    """Context manager installing the branch context for one forward pass."""

    def __init__(self, branch_id: Any, parent_branch_id: Any | None, step_idx: int) -> None:
        self._ctx = {"branch_id": branch_id, "parent_branch_id": parent_branch_id, "step_idx": step_idx}
        self._token: Any = None

    def __enter__(self) -> None:
        self._token = FOLDING_CONTEXT.set(dict(self._ctx))

    def __exit__(self, *exc: object) -> None:
        if self._token is not None:
            FOLDING_CONTEXT.reset(self._token)
            self._token = None
