"""Fast-dLLM-style block decoding whose steps are folded verifications.

Fast-dLLM (the reference's actfold/models/fast_dllm_sampler.py:111-242)
decodes the generation region block by block: every position of the current
block starts as the mask id and, each step, the masked positions whose
predicted probability exceeds a confidence threshold are unmasked, the most
confident one always (:170-195). The reference runs that loop unfolded
(``parent_branch_id=None``, :158-164). Here every step is a speculative
verification on the native folded pass:

* the canvas (prompt + every generation position) is the parent; its
  per-layer activations live in one :class:`ParentCache`, built once by the
  dense pass;
* a draft gives each masked position of the current block a token and a
  confidence (:class:`SyntheticDraft`, seeded, stands in for a trained
  model's predictions);
* child i unmasks the n_i most confident masked positions (n_i rises from
  ``min_edits`` to ``max_edits`` over the children), and all children are
  verified against the parent in one folded pass;
* the accepted child is the one with the most unmasked positions among those
  whose mean stable ratio reaches ``acceptance_threshold`` (the acceptance
  rule of verification_engine.py:121-122) and that unmask no more positions
  than the threshold rule allows; when the rule allows fewer than
  ``min_edits`` positions, ``min_edits`` are committed;
* the accepted child is promoted into the parent cache in place
  (``FoldPlan.promote``): every row it did not change (the prompt, earlier
  blocks, later masked blocks) keeps its cached activations and K/V, which is
  the prefix-cache reuse of block decoding.

A step builds the children on the host, copies them from pinned memory,
replays the pass's CUDA graph, reads back the divergent counts (the one wait
on the device before the acceptance decision), promotes the accepted child and
reads the parent's per-layer self-gate flags (a new plan is made when the
promoted rows changed them).
"""

from __future__ import annotations

from dataclasses import dataclass, field

import numpy as np
import torch

from actfold_b200.llada import LLaDAModel, ParentCache


@dataclass
class BlockDecodingConfig:
    """Sizes and rules of a block-decoding run (defaults: the LLaDA-8B block-decoding workload)."""

    prompt_len: int = 1024
    gen_len: int = 1024
    block_size: int = 32
    n_children: int = 8
    min_edits: int = 2
    max_edits: int = 8
    threshold: float = 0.9
    tau: float = 0.95
    acceptance_threshold: float = 0.0
    seed: int = 42

    def __post_init__(self) -> None:
        if self.block_size < 1 or self.gen_len % self.block_size:
            raise ValueError("gen_len must be a positive multiple of block_size")
        if not 1 <= self.min_edits <= self.max_edits:
            raise ValueError("need 1 <= min_edits <= max_edits")
        if self.n_children < 1:
            raise ValueError("n_children must be >= 1")
        if not 0.0 <= self.acceptance_threshold <= 1.0:
            raise ValueError(f"acceptance_threshold must be in [0, 1], got {self.acceptance_threshold}")

    @property
    def seq(self) -> int:
        return self.prompt_len + self.gen_len

    def edits(self) -> np.ndarray:
        """Unmasked positions per child: min_edits .. max_edits spread over the children."""
        if self.n_children == 1:
            return np.array([self.min_edits])
        return np.rint(np.linspace(self.min_edits, self.max_edits, self.n_children)).astype(np.int64)


class SyntheticDraft:
    """Seeded per-position predictions (token, confidence) for a block's masked positions.

    Stand-in for a trained model's logits: tokens uniform over [0, vocab_limit),
    confidences Beta(a, b) distributed (the defaults put about 19 % of them
    above 0.9). Depends only on (seed, step, positions), so any two runs with
    the same trajectory see the same drafts.
    """

    def __init__(self, vocab_limit: int, seed: int = 42, a: float = 2.0, b: float = 1.0) -> None:
        self.vocab_limit, self.seed, self.a, self.b = int(vocab_limit), int(seed), float(a), float(b)

    def __call__(self, step: int, positions: np.ndarray) -> tuple[np.ndarray, np.ndarray]:
        rng = np.random.default_rng([self.seed, int(step)])
        n = positions.size
        return rng.integers(0, self.vocab_limit, size=n, dtype=np.int64), rng.beta(self.a, self.b, size=n)


def draft_children(canvas: np.ndarray, masked: np.ndarray, tokens: np.ndarray, conf: np.ndarray,
                   edits: np.ndarray) -> tuple[np.ndarray, np.ndarray]:
    """Children [C, T]: child i unmasks the ``edits[i]`` most confident masked positions.

    Returns (children, unmasked count per child); ties in confidence keep position order.
    """
    order = np.argsort(-conf, kind="stable")
    n = np.minimum(edits, masked.size)
    children = np.repeat(canvas[None], edits.size, axis=0)
    for i, k in enumerate(n):
        sel = order[:k]
        children[i, masked[sel]] = tokens[sel]
    return children, n


def accept_child(n: np.ndarray, conf: np.ndarray, stable_ratio: np.ndarray, cfg: BlockDecodingConfig) -> int:
    """Index of the accepted child (see the module docstring)."""
    allowed = max(int((conf > cfg.threshold).sum()), 1, min(cfg.min_edits, int(n.max())))
    ok = (n <= allowed) & (stable_ratio >= cfg.acceptance_threshold)
    if not ok.any():
        ok = n <= allowed
    best = int(n[ok].max())
    return int(np.nonzero(ok & (n == best))[0][0])


@dataclass
class BlockDecodingResult:
    tokens: np.ndarray                  # final canvas [T]
    n_children: int
    seq: int
    steps: int = 0                      # verification passes
    accepted: list = field(default_factory=list)       # accepted child per step
    unmasked: list = field(default_factory=list)       # positions unmasked per step
    stable_ratio: list = field(default_factory=list)   # mean stable ratio of the accepted child per step
    parent: ParentCache | None = None   # parent cache of the final canvas

    @property
    def verified_tokens(self) -> int:
        return self.steps * self.n_children * self.seq


class BlockDecoder:
    """Block decoding of one canvas on an :class:`LLaDAModel` (CUDA), one folded pass per step."""

    def __init__(self, model: LLaDAModel, cfg: BlockDecodingConfig, draft: SyntheticDraft | None = None,
                 use_graph: bool = True) -> None:
        self.model, self.cfg = model, cfg
        self.draft = draft or SyntheticDraft(model.dims.mask_id, cfg.seed)
        self.use_graph = use_graph
        dev = model.device
        C, T = cfg.n_children, cfg.seq
        L = model.dims.n_layers
        self.tok = torch.empty((C, T), dtype=torch.int64, device=dev)
        self.logits = torch.empty((C, T, model.dims.vocab), dtype=torch.bfloat16, device=dev)
        self.scores = torch.empty((C,), dtype=torch.float32, device=dev)
        self.h_tok = torch.empty((C, T), dtype=torch.int64, pin_memory=True)
        self.h_div = torch.empty((L, C), dtype=torch.int32, pin_memory=True)
        self.h_status = torch.empty((1,), dtype=torch.int32, pin_memory=True)
        self.plan = None
        self.graph = None
        self.parent: ParentCache | None = None
        self.canvas: np.ndarray | None = None
        self.step_idx = 0

    # ---------------------------------------------------------------- set-up
    def start(self, prompt: np.ndarray) -> None:
        """Dense pass over prompt + ``gen_len`` mask ids; the canvas becomes the parent."""
        cfg = self.cfg
        prompt = np.asarray(prompt, dtype=np.int64).reshape(-1)
        if prompt.size != cfg.prompt_len:
            raise ValueError(f"prompt must have {cfg.prompt_len} ids, got {prompt.size}")
        self.canvas = np.concatenate([prompt, np.full(cfg.gen_len, self.model.dims.mask_id, dtype=np.int64)])
        self.parent = self.model.parent_pass(torch.from_numpy(self.canvas).to(self.model.device), tau=cfg.tau)
        self.step_idx = 0
        self._make_plan()

    def _make_plan(self) -> None:
        cfg = self.cfg
        su = self.parent.su_layers()
        su_rows = int((self.parent.self_stable == 0).any(dim=0).sum().item()) if su.any() else 0
        C, T = cfg.n_children, cfg.seq
        cap = C * (cfg.max_edits + su_rows)
        m_cap = min(max(16, ((cap + 15) // 16) * 16), ((C * T + 15) // 16) * 16)
        self.plan = self.model.plan(self.parent, C, m_cap, cfg.tau)
        self.plan.set_child_cap(cfg.max_edits + su_rows)
        self.plan.keep_kv(True)
        self._su = su
        self.tok.copy_(torch.from_numpy(self.canvas)[None].expand(C, -1))  # the capture's warm-up run verifies these
        self.graph = self.plan.capture(self.tok, self.logits, self.scores) if self.use_graph else None

    # ---------------------------------------------------------------- steps
    def block_masked(self, block: int) -> np.ndarray:
        lo = self.cfg.prompt_len + block * self.cfg.block_size
        return lo + np.nonzero(self.canvas[lo: lo + self.cfg.block_size] == self.model.dims.mask_id)[0]

    def step(self, block: int) -> dict | None:
        """One verification step on ``block``; None when the block has no masked position left."""
        cfg = self.cfg
        masked = self.block_masked(block)
        if masked.size == 0:
            return None
        tokens, conf = self.draft(self.step_idx, masked)
        children, n = draft_children(self.canvas, masked, tokens, conf, cfg.edits())
        self.h_tok.numpy()[:] = children
        self.tok.copy_(self.h_tok, non_blocking=True)
        if self.graph is not None:
            self.graph.replay()
        else:
            self.plan.run(self.tok, self.logits, self.scores)
        self.h_div.copy_(self.plan.div_count, non_blocking=True)
        self.h_status.copy_(self.plan.status, non_blocking=True)
        torch.cuda.current_stream(self.model.device).synchronize()
        if int(self.h_status[0]):
            self.plan.check_status()
        ratio = 1.0 - self.h_div.numpy().mean(axis=0) / cfg.seq
        i = accept_child(n, conf, ratio, cfg)
        self.plan.promote(i, into=self.parent)
        self.canvas = children[i].copy()
        self.step_idx += 1
        if not np.array_equal(self.parent.su_layers(), self._su):
            self._make_plan()  # the promoted rows changed which layers the parent fails its own gate on
        return {"child": i, "unmasked": int(n[i]), "stable_ratio": float(ratio[i])}

    def run(self, prompt: np.ndarray, max_steps: int | None = None) -> BlockDecodingResult:
        """Decode every block (or stop after ``max_steps`` passes)."""
        self.start(prompt)
        res = BlockDecodingResult(tokens=self.canvas, n_children=self.cfg.n_children, seq=self.cfg.seq)
        for b in range(self.cfg.gen_len // self.cfg.block_size):
            while max_steps is None or res.steps < max_steps:
                out = self.step(b)
                if out is None:
                    break
                res.steps += 1
                res.accepted.append(out["child"])
                res.unmasked.append(out["unmasked"])
                res.stable_ratio.append(out["stable_ratio"])
            if max_steps is not None and res.steps >= max_steps:
                break
        res.tokens = self.canvas
        res.parent = self.parent
        return res
