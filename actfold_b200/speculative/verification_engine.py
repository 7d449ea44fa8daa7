"""Verification engine: accept or reject child branches against a parent.

Drop-in for actfold/speculative/verification_engine.py:34-294 for models with
a native folded pass (LLaDAModel): ``verify_branch`` has the reference's
signature and result type. Differences, on purpose:

* the parent pass runs once per parent (keyed by branch id and tokens), not on
  every call (verification_engine.py:99, 146-168 re-runs it each time);
* ``verify_branches`` verifies a whole list of children in one batched pass;
* ``stable_ratio`` is the measured mean stable ratio over layers (the
  reference's estimated-ratio fallback is not needed), and ``tflops`` counts
  the FLOPs actually executed by the divergent-row recompute.

``verify_tokens`` is the host-buffer entry point: pinned host token ids in,
per-child scores and per-layer divergent counts back to pinned host memory.
"""

from __future__ import annotations

from dataclasses import dataclass, field
from typing import Any

import numpy as np
import torch

from actfold_b200.core.similarity_gate import SimilarityGate
from actfold_b200.llada import LLaDAModel, ParentCache, round_capacity
from actfold_b200.profiler.stability_profiler import GLOBAL_STABILITY_PROFILER, StabilityProfile


@dataclass
class Branch:
    """A candidate branch: the fields, order and checks of actfold/speculative/branch.py:10-40."""

    branch_id: Any
    parent_id: Any | None
    tokens: torch.Tensor  # [batch, seq_len]
    scores: torch.Tensor | None = None
    accepted: bool = False
    metadata: dict = field(default_factory=dict)

    def __post_init__(self) -> None:
        if self.tokens.dim() != 2:
            raise ValueError(f"tokens must be 2D [batch, seq_len], got {self.tokens.shape}")
        if self.scores is not None and self.scores.shape != self.tokens.shape:
            raise ValueError(f"scores shape {self.scores.shape} must match tokens shape {self.tokens.shape}")


@dataclass(frozen=True)
class VerificationResult:
    accepted: bool
    child_branch: Branch
    parent_branch: Branch
    stable_ratio: float
    tflops: float
    latency_ms: float
    estimated_latency_ms: float = 0.0
    stability_profile: StabilityProfile | None = None


class ActFoldVerificationEngine:
    def __init__(self, model: LLaDAModel, cache=None, gate: SimilarityGate | None = None, scheduler=None,
                 acceptance_threshold: float = 0.0, use_graphs: bool = True) -> None:
        if not 0.0 <= acceptance_threshold <= 1.0:
            raise ValueError(f"acceptance_threshold must be in [0, 1], got {acceptance_threshold}")
        if scheduler is not None:
            raise NotImplementedError("per-layer tau schedules are not supported by the native pass")
        self.model = model
        self.cache = cache
        self.gate = gate or SimilarityGate(0.95)
        self.acceptance_threshold = acceptance_threshold
        self._parents: dict = {}
        self._host: dict = {}
        # verify_tokens replays each plan's pass from a CUDA graph captured over
        # the engine's fixed token / logits / score buffers (use_graphs=False: launch eagerly).
        self.use_graphs = use_graphs
        self._graphs: dict = {}

    # ----------------------------------------------------------------- parent
    def parent_cache(self, parent_branch: Branch) -> ParentCache:
        toks = parent_branch.tokens.reshape(-1)
        key = parent_branch.branch_id
        pc = self._parents.get(key)
        if pc is not None and pc.seq == toks.numel() and pc.tau == self.gate.tau:
            # Same tokens: the cached buffer itself, equal host ids, or (last) a device compare.
            if toks.device == pc.tokens.device and toks.data_ptr() == pc.tokens.data_ptr():
                return pc
            if toks.device.type == "cpu":
                if np.array_equal(toks.numpy(), self._parent_host_tokens(pc)):
                    return pc
            elif torch.equal(pc.tokens, toks.to(pc.tokens.device)):
                return pc
        pc = self.model.parent_pass(toks.to(self.model.device), tau=self.gate.tau)
        self._parents = {key: pc}
        self._graphs = {}
        return pc

    def set_parent_cache(self, parent_branch: Branch, pc: ParentCache) -> None:
        """Install a parent cache computed elsewhere (e.g. broadcast from another rank)."""
        self._parents = {parent_branch.branch_id: pc}

    # ----------------------------------------------------------------- verify
    def _flops(self, n_div: np.ndarray, n_cand: np.ndarray, T: int) -> float:
        d = self.model.dims
        H, q, kv, FF = d.hidden, d.q_dim, d.kv_dim, d.ffn
        f = 0.0
        for l in range(d.n_layers):
            f += 2.0 * n_cand[l] * H * (q + 2 * kv)  # QKV on candidates
            f += 4.0 * n_div[l] * (T + n_cand[l]) * q  # attention of divergent rows
            f += 2.0 * n_div[l] * (q * H + 3 * H * FF)  # O, gate/up, down
        f += 2.0 * n_div[-1] * H * d.vocab
        return f / 1e12

    def verify_tokens(self, parent_branch: Branch, child_tokens_host: torch.Tensor) -> dict:
        """Batched verification from HOST token ids [C, T] (pinned for async copies).

        Returns numpy arrays: ``scores`` [C] (mean logit), ``div_count`` [L, C]
        (divergent rows per layer and child), ``stable_ratio`` [C].
        """
        pc = self.parent_cache(parent_branch)
        dev = self.model.device
        Cn, T = child_tokens_host.shape
        key = (Cn, T)
        bufs = self._host.get(key)
        if bufs is None:
            L = self.model.dims.n_layers
            bufs = {
                "tok": torch.empty((Cn, T), dtype=torch.int64, device=dev),
                "scores": torch.empty((Cn,), dtype=torch.float32, device=dev),
                "logits": torch.empty((Cn, T, self.model.dims.vocab), dtype=torch.bfloat16, device=dev),
                "h_scores": torch.empty((Cn,), dtype=torch.float32, pin_memory=True),
                "h_div": torch.empty((L, Cn), dtype=torch.int32, pin_memory=True),
                "h_status": torch.empty((1,), dtype=torch.int32, pin_memory=True),
            }
            self._host = {key: bufs}
        bufs["tok"].copy_(child_tokens_host, non_blocking=True)
        m_cap, child_cap = self._m_cap(child_tokens_host, pc, Cn, T)
        if self.use_graphs:
            plan = self.model.plan(pc, Cn, m_cap, self.gate.tau, self.gate.metric)
            plan.set_child_cap(child_cap)
            gkey = (id(plan), child_cap, plan.keeps_kv)
            entry = self._graphs.get(gkey)
            if entry is None or entry[1] is not plan or entry[2] is not bufs:
                if len(self._graphs) >= 8:
                    self._graphs = {}
                entry = (plan.capture(bufs["tok"], bufs["logits"], bufs["scores"]), plan, bufs)
                self._graphs[gkey] = entry
            entry[0].replay()
        else:
            plan = self.model.plan(pc, Cn, m_cap, self.gate.tau, self.gate.metric)
            plan.set_child_cap(child_cap)
            _, plan = self.model.verify(bufs["tok"], pc, self.gate.tau, self.gate.metric, logits=bufs["logits"],
                                        scores=bufs["scores"], m_cap=m_cap)
        bufs["h_scores"].copy_(bufs["scores"], non_blocking=True)
        bufs["h_div"].copy_(plan.div_count, non_blocking=True)
        bufs["h_status"].copy_(plan.status, non_blocking=True)
        torch.cuda.current_stream(dev).synchronize()
        if int(bufs["h_status"][0]):
            plan.check_status()
        div = bufs["h_div"].numpy()
        return {
            "scores": bufs["h_scores"].numpy().copy(),
            "div_count": div.copy(),
            "stable_ratio": 1.0 - div.mean(axis=0) / T,
            "logits": bufs["logits"],
            "plan": plan,
        }

    def _m_cap(self, child_tokens_host: torch.Tensor, pc: ParentCache, Cn: int, T: int) -> tuple[int, int]:
        # (capacity, per-child candidate bound) from the host copy of the tokens (no device round trip).
        ptok = self._parent_host_tokens(pc)
        per_child = (child_tokens_host.numpy() != ptok[None]).sum(axis=1)
        su_rows = pc.su_rows_at((self.gate.tau,) * self.model.dims.n_layers)  # one device read per parent
        return round_capacity(int(per_child.sum()) + Cn * su_rows, Cn, T), int(per_child.max()) + su_rows

    def _parent_host_tokens(self, pc: ParentCache) -> np.ndarray:
        cached = getattr(pc, "_host_tokens", None)
        if cached is None:
            cached = pc.tokens.cpu().numpy()
            pc._host_tokens = cached
        return cached

    def verify_branches(self, parent_branch: Branch, child_branches: list[Branch], step_idx: int = 0) -> list[VerificationResult]:
        toks = torch.stack([b.tokens.reshape(-1).cpu() for b in child_branches]).pin_memory()
        start = torch.cuda.Event(enable_timing=True)
        end = torch.cuda.Event(enable_timing=True)
        start.record()
        res = self.verify_tokens(parent_branch, toks)
        end.record()
        end.synchronize()
        ms = start.elapsed_time(end)
        plan = res["plan"]
        masks = plan.stable_masks()
        n_div = plan.n_div.cpu().numpy()
        n_cand = plan.n_cand.cpu().numpy()
        T = toks.shape[1]
        tflops = self._flops(n_div, n_cand, T)
        out = []
        for i, child in enumerate(child_branches):
            GLOBAL_STABILITY_PROFILER.reset_branch(child.branch_id)
            for li in range(masks.shape[0]):
                GLOBAL_STABILITY_PROFILER.record(child.branch_id, parent_branch.branch_id, li, step_idx, masks[li, i][None], self.gate.tau, self.gate.metric)
            ratio = float(res["stable_ratio"][i])
            child.metadata["actfold_score"] = float(res["scores"][i])
            child.metadata["stable_ratio"] = ratio
            accepted = ratio >= self.acceptance_threshold
            child.accepted = accepted
            if not accepted and self.cache is not None:
                self.cache.clear_branch(child.branch_id)
            out.append(
                VerificationResult(accepted, child, parent_branch, ratio, tflops / len(child_branches), ms / len(child_branches),
                                   stability_profile=GLOBAL_STABILITY_PROFILER.get_profile(child.branch_id))
            )
        return out

    def verify_branch(self, parent_branch: Branch, child_branch: Branch, step_idx: int = 0) -> VerificationResult:
        return self.verify_branches(parent_branch, [child_branch], step_idx)[0]
