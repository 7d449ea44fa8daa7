"""LLaDA / Dream-architecture models on the native folded pass.

``LLaDAModel`` is the weight container of a pre-norm Transformer with RMSNorm,
rotate-half RoPE, non-causal multi-head / grouped-query attention and a
SwiGLU FFN (the LLaDA-8B and Dream-7B layouts), stored in bf16 on the GPU in
the layouts the CUDA kernels stream:

* ``w_qkv``   [q_dim + 2 kv_dim, H]: Wq rows, then Wk, then Wv
* ``w_gateup``[2 FF, H]: per 128 rows, 64 gate rows then the 64 matching up rows
* ``w_o`` [H, q_dim], ``w_down`` [H, FF], ``lm_head`` [V, H], norms [H]

``forward(tokens)`` is the dense pass (``af_dense_forward``). Wrapped in
``FoldedModel``, the model verifies whole batches of children with
``native_folded_forward``: the parent pass fills a :class:`ParentCache` that is
registered in the ActivationCache under the parent's branch id, and each child
batch runs ``af_fold_run`` (gate, compaction, divergent-row recompute, merge,
logits) with no host synchronisation until the caller reads a result.
"""

from __future__ import annotations

import ctypes as C
from dataclasses import dataclass, field
from typing import Any, Sequence

import numpy as np
import torch
import torch.nn as nn

from actfold_b200 import _lib
from actfold_b200.kernels import tile_weight
from actfold_b200.workloads import ModelDims

_vp, _i32, _i64, _f32 = C.c_void_p, C.c_int32, C.c_int64, C.c_float


class _Dims(C.Structure):
    _fields_ = [
        ("n_layers", _i32), ("hidden", _i32), ("n_heads", _i32), ("n_kv_heads", _i32),
        ("head_dim", _i32), ("ffn", _i32), ("vocab", _i32), ("rms_eps", _f32),
    ]


class _Layer(C.Structure):
    _fields_ = [("attn_norm", _vp), ("w_qkv", _vp), ("w_o", _vp), ("ffn_norm", _vp), ("w_gateup", _vp), ("w_down", _vp)]


class _Model(C.Structure):
    _fields_ = [
        ("dims", _Dims), ("layers", C.POINTER(_Layer)), ("embed", _vp), ("final_norm", _vp), ("lm_head", _vp),
        ("rope_cos", _vp), ("rope_sin", _vp), ("max_pos", _i64),
    ]


class _Parent(C.Structure):
    _fields_ = [
        ("seq", _i64), ("tokens", _vp), ("layer_in", _vp), ("qkv", _vp), ("logits", _vp),
        ("self_stable", _vp), ("logit_row_sums", _vp), ("kv_headmajor", _vp),
    ]


class _FoldConfig(C.Structure):
    _fields_ = [("n_children", _i64), ("seq", _i64), ("m_cap", _i64), ("tau", _f32), ("metric", _i32), ("su_layers", _vp),
                ("tau_layers", _vp), ("fold_layers", _vp), ("self_stable", _vp), ("partial_always", _i32)]


# int (*)(void* user, int32 kind, int32 layer, void* data, int64 count, void* stream): a cross-rank sum
COLLECTIVE_FN = C.CFUNCTYPE(_i32, _vp, _i32, _i32, _vp, _i64, _vp)


class _FoldOutputs(C.Structure):
    _fields_ = [
        ("n_cand", _vp), ("n_div", _vp), ("div_pos", _vp), ("div_count", _vp), ("status", _vp), ("m_cap", _i64),
        ("n_fresh0", _vp), ("fresh0_pos", _vp),
    ]


_lib.SIGNATURES.update(
    {
        "af_dense_workspace_bytes": (_i32, [C.POINTER(_Dims), _i64, C.POINTER(_i64)]),
        "af_dense_forward": (_i32, [C.POINTER(_Model), _vp, _i64, _f32, _vp, _vp, _vp, _vp, _vp, _vp, _i64, _vp, _vp]),
        "af_dense_forward_static": (_i32, [C.POINTER(_Model), _vp, _i64, _f32, _vp, _vp, _vp, _vp, _vp, _vp, _vp]),
        "af_fold_workspace_bytes": (_i32, [C.POINTER(_Dims), C.POINTER(_FoldConfig), C.POINTER(_i64)]),
        "af_fold_plan_create": (_i32, [C.POINTER(_Model), C.POINTER(_Parent), C.POINTER(_FoldConfig), _vp, _i64, C.POINTER(_vp)]),
        "af_fold_run": (_i32, [_vp, _vp, _vp, _vp, _vp]),
        "af_fold_get_outputs": (_i32, [_vp, C.POINTER(_FoldOutputs)]),
        "af_fold_materialize": (_i32, [_vp, _i64, _vp, _vp]),
        "af_fold_keep_kv": (_i32, [_vp, _vp, _i64]),
        "af_fold_set_child_cap": (_i32, [_vp, _i64]),
        "af_fold_promote": (_i32, [_vp, _i64, _vp, _vp, C.POINTER(_Parent), _vp]),
        "af_fold_plan_destroy": (_i32, [_vp]),
        "af_fold_set_timing": (_i32, [_vp, _i32]),
        "af_fold_get_timing": (_i32, [_vp, C.POINTER(C.c_double), C.POINTER(_i64), _i32, C.POINTER(_i64)]),
        "af_fold_set_tensor_parallel": (_i32, [_vp, _i64, _i64, COLLECTIVE_FN, _vp]),
        "af_parent_kv_headmajor": (_i32, [C.POINTER(_Dims), _i64, _vp, _vp, _vp]),
        "af_fold_peer_bytes": (_i32, [_vp, _i32, C.POINTER(_i64)]),
        "af_fold_set_peer_sum": (_i32, [_vp, _i32, _i32, C.POINTER(_vp)]),
        "af_ipc_export": (_i32, [_vp, _vp, C.POINTER(_i64)]),
        "af_ipc_import": (_i32, [_vp, _i64, C.POINTER(_vp), C.POINTER(_vp)]),
        "af_ipc_close": (_i32, [_vp]),
    }
)

KERNEL_CLASSES = ("setup", "gate", "compact", "gemm_qkv", "attention", "gemm_o", "rmsnorm", "gemm_gateup",
                  "gemm_down", "gemm_lm_head", "logits_fill", "scores", "qkv_finish")


def _bind_late() -> C.CDLL:
    lib = _lib.load()
    for name in ("af_dense_workspace_bytes", "af_dense_forward", "af_fold_workspace_bytes", "af_fold_plan_create",
                 "af_fold_run", "af_fold_get_outputs", "af_fold_materialize", "af_fold_plan_destroy",
                 "af_fold_keep_kv", "af_fold_promote", "af_fold_set_child_cap",
                 "af_fold_set_timing", "af_fold_get_timing", "af_fold_set_tensor_parallel", "af_parent_kv_headmajor",
                 "af_fold_peer_bytes", "af_fold_set_peer_sum", "af_ipc_export", "af_ipc_import", "af_ipc_close"):
        fn = getattr(lib, name)
        fn.restype, fn.argtypes = _lib.SIGNATURES[name]
    return lib


def interleave_gate_up(w_gate: torch.Tensor, w_up: torch.Tensor) -> torch.Tensor:
    """[FF, H] x 2 -> [2 FF, H] with 64 gate rows then 64 up rows per 128-row block."""
    FF, H = w_gate.shape
    if FF % 64:
        raise ValueError("ffn must be a multiple of 64")
    return torch.stack([w_gate.view(FF // 64, 64, H), w_up.view(FF // 64, 64, H)], dim=1).reshape(2 * FF, H).contiguous()


def rope_tables(max_pos: int, head_dim: int, theta: float, device) -> tuple[torch.Tensor, torch.Tensor]:
    """cos/sin [max_pos, head_dim/2]: angle t * theta^(-2i/d) in float64, rounded once to float32."""
    i = torch.arange(0, head_dim, 2, dtype=torch.float64, device=device)
    inv = 1.0 / (float(theta) ** (i / head_dim))
    ang = torch.arange(max_pos, dtype=torch.float64, device=device)[:, None] * inv[None, :]
    return torch.cos(ang).float().contiguous(), torch.sin(ang).float().contiguous()


class LLaDABlock(nn.Module):
    """Weights of one block: bf16 buffers, projections tiled for the GEMM (``kernels.tile_weight``).

    Takes row-major [n, k] projections and stores them tiled; ``shapes`` keeps
    the logical [n, k] of each.
    """

    def __init__(self, attn_norm, w_qkv, w_o, ffn_norm, w_gateup, w_down, tiled: bool = False) -> None:
        super().__init__()
        self.register_buffer("attn_norm", attn_norm.contiguous())
        self.register_buffer("ffn_norm", ffn_norm.contiguous())
        self.shapes = {}
        for k, v in dict(w_qkv=w_qkv, w_o=w_o, w_gateup=w_gateup, w_down=w_down).items():
            if tiled:  # already [n/128, k/64, 128, 64]
                self.shapes[k] = (v.shape[0] * 128, v.shape[1] * 64)
                self.register_buffer(k, v.contiguous())
            else:
                self.shapes[k] = tuple(v.shape)
                self.register_buffer(k, tile_weight(v))

    def forward(self, hidden_states: torch.Tensor, attention_mask: torch.Tensor | None = None) -> torch.Tensor:
        raise RuntimeError("LLaDABlock runs inside the native folded pass; call LLaDAModel or FoldedModel instead")


@dataclass
class ParentCache:
    """Dense parent activations consumed by the folded pass (one per parent branch)."""

    tokens: torch.Tensor        # [T] int64
    layer_in: torch.Tensor      # [L+1, T, H] bf16
    qkv: torch.Tensor           # [L, T, q+2kv] bf16
    logits: torch.Tensor        # [T, V] bf16
    self_stable: torch.Tensor   # [L, T] uint8
    row_sums: torch.Tensor      # [T] fp32
    tau: float
    # Bumped by contents_changed() whenever the arrays are rewritten in place.
    version: int = field(default=0, compare=False)
    # [L, 2, n_kv_heads, T, 128] bf16: the K / V columns of qkv stored
    # head-major, so the attention kernel reads one head's block of parent
    # keys as one contiguous run (kv_headmajor() builds it; promotions keep
    # it current). The buffer lives as long as the cache, so plans may hold it.
    kv_hm: torch.Tensor | None = field(default=None, compare=False, repr=False)
    _kv_hm_at: int = field(default=-1, compare=False, repr=False)

    @property
    def seq(self) -> int:
        return int(self.tokens.shape[0])

    def su_layers(self) -> np.ndarray:
        """Host flags: layers where some parent row fails its own gate (one small copy)."""
        return (self.self_stable == 0).any(dim=1).to(torch.uint8).cpu().numpy()

    def struct(self, model: "LLaDAModel | None" = None) -> _Parent:
        """The C struct; with ``model`` (whose ``kv_headmajor`` is set) the head-major K / V are built or refreshed."""
        hm = self.kv_headmajor(model) if model is not None and model.kv_headmajor else None
        return _Parent(self.seq, self.tokens.data_ptr(), self.layer_in.data_ptr(), self.qkv.data_ptr(),
                       self.logits.data_ptr(), self.self_stable.data_ptr(), self.row_sums.data_ptr(),
                       hm.data_ptr() if hm is not None else None)

    def kv_headmajor(self, model: "LLaDAModel") -> torch.Tensor:
        """The head-major K / V of every layer, rebuilt in place (stream-ordered) when qkv changed since."""
        d = model.dims
        L, T = int(self.qkv.shape[0]), self.seq
        if self.qkv.shape[2] != d.q_dim + 2 * d.kv_dim or L != d.n_layers:
            raise ValueError(f"kv_headmajor: cache qkv {tuple(self.qkv.shape)} does not match the model")
        shape = (L, 2, d.n_kv_heads, T, d.head_dim)
        if self.kv_hm is None or tuple(self.kv_hm.shape) != shape:
            self.kv_hm = torch.empty(shape, dtype=torch.bfloat16, device=self.qkv.device)
            self._kv_hm_at = -1
        if self._kv_hm_at != self.version:
            lib = _bind_late()
            with torch.cuda.device(self.qkv.device):
                _lib.check(lib.af_parent_kv_headmajor(C.byref(model._cdims), T, self.qkv.data_ptr(), self.kv_hm.data_ptr(),
                                                      _lib.stream_ptr(self.qkv.device)), "af_parent_kv_headmajor")
            self._kv_hm_at = self.version
        return self.kv_hm

    def tensors(self) -> list[torch.Tensor]:
        return [self.tokens, self.layer_in, self.qkv, self.logits, self.self_stable, self.row_sums]

    def resized(self, T: int) -> "ParentCache":
        """The cache as seen by children of length ``T`` (a new cache; the last one is kept for reuse).

        The reference gathers the parent's entry of every child position and
        zero-fills the positions the parent has none for
        (actfold/core/fused_ops.py:54-87, 256-324). Rows past this parent's
        length are therefore zero, with token id -1 so that every child counts
        them as edited (they gate as divergent against the zero rows); a
        shorter child sees the first ``T`` rows.
        """
        T = int(T)
        last = getattr(self, "_resized", None)
        if last is not None and last[0] == T:
            return last[1]
        n = min(T, self.seq)

        def fit(a: torch.Tensor, axis: int, fill: float) -> torch.Tensor:
            shape = list(a.shape)
            shape[axis] = T
            b = torch.full(shape, fill, dtype=a.dtype, device=a.device)
            b.narrow(axis, 0, n).copy_(a.narrow(axis, 0, n))
            return b

        out = ParentCache(fit(self.tokens, 0, -1), fit(self.layer_in, 1, 0), fit(self.qkv, 1, 0), fit(self.logits, 0, 0),
                          fit(self.self_stable, 1, 1), fit(self.row_sums, 0, 0), self.tau)
        self._resized = (T, out)
        return out

    def clone(self) -> "ParentCache":
        """Device copy of every array (the destination of a promotion that keeps this cache intact)."""
        return ParentCache(*(t.clone() for t in self.tensors()), self.tau)

    # Values derived from the arrays and kept for reuse: the host copy of the
    # token ids, the self-gate results at other thresholds and the count of
    # rows the parent fails its own gate on, and the last resized view.
    _DERIVED = ("_host_tokens", "_self_stable_at", "_su_rows_at", "_resized")

    def contents_changed(self) -> None:
        """Record an in-place rewrite of the arrays: drop every value derived from them."""
        self.version += 1
        for name in self._DERIVED:
            self.__dict__.pop(name, None)

    def self_stable_at(self, taus: Sequence[float]) -> torch.Tensor:
        """[L, T] uint8: the parent's own gate result of each row, layer l at threshold ``taus[l]``.

        The parent pass stored these at the cache's own ``tau``; layers with
        another threshold are gated again (one SimilarityGate call per
        distinct threshold), and the result is kept until the contents change.
        """
        taus = tuple(float(t) for t in taus)
        if all(t == self.tau for t in taus):
            return self.self_stable
        memo = self.__dict__.setdefault("_self_stable_at", {})
        out = memo.get(taus)
        if out is None:
            from actfold_b200.core.similarity_gate import SimilarityGate

            x = self.layer_in[:-1]
            out = self.self_stable.clone()
            for t in sorted(set(taus) - {self.tau}):
                ls = [i for i, lt in enumerate(taus) if lt == t]
                out[ls] = SimilarityGate(tau=t)(x[ls], x[ls]).to(torch.uint8)
            memo[taus] = out
        return out

    def su_rows_at(self, taus: Sequence[float]) -> int:
        """Rows the parent fails its own gate on at some layer, at thresholds ``taus`` (one device read, kept)."""
        taus = tuple(float(t) for t in taus)
        memo = self.__dict__.setdefault("_su_rows_at", {})
        n = memo.get(taus)
        if n is None:
            n = int((self.self_stable_at(taus) == 0).any(dim=0).sum().item())
            memo[taus] = n
        return n


class FoldPlan:
    """A prepared folded pass for C children of length T with m_cap candidate rows.

    ``layer_taus`` / ``layer_folds`` (optional, one entry per layer) give each
    layer its own gate threshold and say which layers fold at all: the
    per-layer decisions a FoldingScheduler makes inside the reference's folded
    layers (actfold/core/folded_transformer.py:107-119). A layer that does not
    fold recomputes every row of every child, so a plan with one needs
    ``m_cap = C * T``.
    """

    def __init__(self, model: "LLaDAModel", parent: ParentCache, n_children: int, m_cap: int, tau: float,
                 metric: str = "cosine", layer_taus=None, layer_folds=None, partial_always: bool = False) -> None:
        self.lib = _bind_late()
        self.model = model
        self.parent = parent
        L = model.dims.n_layers
        self.C, self.T, self.m_cap, self.tau = n_children, parent.seq, m_cap, tau
        self.layer_taus = tuple(float(t) for t in layer_taus) if layer_taus is not None else (float(tau),) * L
        self.layer_folds = tuple(bool(f) for f in layer_folds) if layer_folds is not None else (True,) * L
        if len(self.layer_taus) != L or len(self.layer_folds) != L:
            raise ValueError(f"layer_taus / layer_folds must have {L} entries")
        if not all(self.layer_folds) and m_cap < n_children * parent.seq:
            raise ValueError("a layer that does not fold recomputes every row: m_cap must be C * T")
        self.self_stable = parent.self_stable_at(self.layer_taus)
        self._parent_version = parent.version
        su = (self.self_stable == 0).any(dim=1).cpu().numpy() | ~np.array(self.layer_folds)
        self._su = np.ascontiguousarray(su.astype(np.uint8))
        self._taus = np.ascontiguousarray(np.array(self.layer_taus, np.float32))
        self._folds = np.ascontiguousarray(np.array(self.layer_folds, np.uint8))
        self._cfg = _FoldConfig(n_children, self.T, m_cap, float(tau), _lib.METRIC[metric], self._su.ctypes.data,
                                self._taus.ctypes.data, self._folds.ctypes.data, self.self_stable.data_ptr(),
                                1 if partial_always else 0)
        nbytes = _i64()
        _lib.check(self.lib.af_fold_workspace_bytes(C.byref(model._cmodel.dims), C.byref(self._cfg), C.byref(nbytes)))
        self.workspace = torch.zeros(int(nbytes.value), dtype=torch.uint8, device=model.device)
        self._pstruct = parent.struct(model)
        plan = _vp()
        _lib.check(self.lib.af_fold_plan_create(C.byref(model._cmodel), C.byref(self._pstruct), C.byref(self._cfg),
                                                self.workspace.data_ptr(), self.workspace.numel(), C.byref(plan)))
        self._plan = plan
        out = _FoldOutputs()
        _lib.check(self.lib.af_fold_get_outputs(plan, C.byref(out)))
        ws = self.workspace
        base = ws.data_ptr()

        def view(ptr, n, dtype):
            off = ptr - base
            itemsize = torch.empty((), dtype=dtype).element_size()
            return ws[off: off + n * itemsize].view(dtype)

        self.n_cand = view(out.n_cand, L + 1, torch.int32)
        self.n_div = view(out.n_div, L, torch.int32)
        self.div_pos = view(out.div_pos, L * m_cap, torch.int32).view(L, m_cap)
        self.div_count = view(out.div_count, L * n_children, torch.int32).view(L, n_children)
        self.status = view(out.status, 1, torch.int32)
        self.n_fresh0 = view(out.n_fresh0, 1, torch.int32)

    def set_tensor_parallel(self, embed_rows: int, vocab_total: int, collective) -> None:
        """Make this plan one rank's shard of a tensor-parallel pass (see actfold_b200.tensor_parallel).

        ``collective(kind, layer, tensor)`` must sum the fp32 ``tensor`` (a view
        of this plan's workspace) over the ranks in place, on the current stream.
        """
        def hook(user, kind, layer, data, count, stream):
            try:
                collective(int(kind), int(layer), self.workspace_view(data, int(count), torch.float32))
                return 0
            except Exception as exc:  # reported through the C status; the message is kept for the caller
                self.collective_error = exc
                return 1

        self._hook = COLLECTIVE_FN(hook)  # kept alive as long as the plan
        _lib.check(self.lib.af_fold_set_tensor_parallel(self._plan, int(embed_rows), int(vocab_total), self._hook, None),
                   "af_fold_set_tensor_parallel")

    collective_error = None

    def peer_bytes(self, world: int) -> int:
        """Bytes of one rank's exchange buffer for peer-memory sums over ``world`` ranks."""
        n = _i64()
        _lib.check(self.lib.af_fold_peer_bytes(self._plan, int(world), C.byref(n)), "af_fold_peer_bytes")
        return int(n.value)

    def set_peer_sum(self, rank: int, world: int, exchange_ptrs) -> None:
        """Route the O / down sums through the ranks' exchange buffers (``exchange_ptrs[q]``: rank q's, as mapped here).

        Every buffer must be zero-filled on every rank before any rank runs
        the plan; after ``set_tensor_parallel``.
        """
        arr = (_vp * int(world))(*[int(x) for x in exchange_ptrs])
        _lib.check(self.lib.af_fold_set_peer_sum(self._plan, int(rank), int(world), arr), "af_fold_set_peer_sum")
        self._exchange_ptrs = arr

    def workspace_view(self, ptr: int, n: int, dtype: torch.dtype) -> torch.Tensor:
        """``n`` elements of ``dtype`` at device address ``ptr`` inside this plan's workspace."""
        off = int(ptr) - self.workspace.data_ptr()
        size = n * torch.empty((), dtype=dtype).element_size()
        if off < 0 or off + size > self.workspace.numel():
            raise ValueError("workspace_view: address outside the plan's workspace")
        return self.workspace[off: off + size].view(dtype)

    def parent_rewritten(self) -> bool:
        """After an in-place rewrite of the parent (a promotion): refresh the plan's self-gate rows.

        Returns True when the plan can no longer run this parent (the layers
        where the parent fails its own gate changed, so the launch sequence
        does); otherwise the plan, and any graph captured from it, stays valid.
        """
        if self._pstruct.kv_headmajor:
            self.parent.kv_headmajor(self.model)  # same buffer, rebuilt from the rewritten qkv
        fresh = self.parent.self_stable_at(self.layer_taus)
        if fresh is not self.self_stable:
            self.self_stable.copy_(fresh)
        su = ((self.self_stable == 0).any(dim=1).cpu().numpy() | ~np.array(self.layer_folds)).astype(np.uint8)
        self._parent_version = self.parent.version
        return not np.array_equal(su, self._su)

    def run(self, child_tokens: torch.Tensor, logits: torch.Tensor, scores: torch.Tensor | None = None) -> None:
        if child_tokens.shape != (self.C, self.T) or child_tokens.dtype != torch.int64 or not child_tokens.is_contiguous():
            raise ValueError(f"child_tokens must be contiguous int64 [{self.C}, {self.T}]")
        st = self.lib.af_fold_run(self._plan, child_tokens.data_ptr(), logits.data_ptr(), _lib.ptr(scores),
                                  _lib.stream_ptr(child_tokens.device))
        if st == _lib.AF_ERR_COMM and self.collective_error is not None:
            err, self.collective_error = self.collective_error, None
            raise err
        _lib.check(st, "af_fold_run")
        self.serial += 1
        self.last_run = (child_tokens, logits)

    serial = 0          # runs so far (a promotion refers to the last one)
    last_run = None     # (child_tokens, logits) of the last run
    _kv_store = None

    def keep_kv(self, enabled: bool = True) -> None:
        """Keep each layer's candidate QKV rows during the next runs, so any child can be promoted.

        Costs one row-copy launch per layer and an [L, m_cap, q+2kv] bf16
        store. Enable it before ``capture``.
        """
        d = self.model.dims
        if enabled and self._kv_store is None:
            self._kv_store = torch.empty((d.n_layers, self.m_cap, d.q_dim + 2 * d.kv_dim), dtype=torch.bfloat16,
                                         device=self.model.device)
        store = self._kv_store if enabled else None
        _lib.check(self.lib.af_fold_keep_kv(self._plan, _lib.ptr(store), 0 if store is None else store.numel() * 2),
                   "af_fold_keep_kv")
        self.keeps_kv = enabled

    keeps_kv = False
    child_cap = 0

    def set_child_cap(self, bound: int) -> None:
        """Bound on any child's candidate rows per layer for the next runs (0: none).

        Lets attention scan only the candidate keys near each tile of packed
        queries (linear instead of quadratic in the child count); a run that
        exceeds it reports a capacity error. Set it before ``capture``.
        """
        bound = int(bound)
        if bound != self.child_cap:
            _lib.check(self.lib.af_fold_set_child_cap(self._plan, bound), "af_fold_set_child_cap")
            self.child_cap = bound

    def promote(self, child: int, into: ParentCache | None = None) -> ParentCache:
        """Parent cache of child ``child`` of the last run (the reference's cached child entries).

        ``into=None`` writes a copy of the plan's parent; ``into=plan.parent``
        promotes in place (the plan then verifies the promoted branch's
        children, as long as ``LLaDAModel.plan`` finds its self-gate flags
        unchanged). Stream-ordered; no host synchronisation.
        """
        if self.last_run is None:
            raise RuntimeError("promote: the plan has not run")
        if not self.keeps_kv:
            raise RuntimeError("promote: enable keep_kv() before the run whose child is promoted")
        if into is None:
            into = self.parent.clone()
        elif into is not self.parent and into.seq != self.T:
            raise ValueError(f"promote: destination length {into.seq} differs from {self.T}")
        toks, logits = self.last_run
        dst = into.struct(self.model)
        _lib.check(self.lib.af_fold_promote(self._plan, int(child), toks.data_ptr(), logits.data_ptr(), C.byref(dst),
                                            _lib.stream_ptr(toks.device)), "af_fold_promote")
        if self.tau != into.tau:
            # Rows the promotion did not touch carry self-gate flags of another tau.
            from actfold_b200.core.similarity_gate import SimilarityGate

            x = into.layer_in[:-1]
            into.self_stable.copy_(SimilarityGate(tau=self.tau)(x, x).to(torch.uint8))
            into.tau = float(self.tau)
        into.contents_changed()  # its token ids and self-gate rows are the child's now
        if dst.kv_headmajor:
            into._kv_hm_at = into.version  # the promotion wrote the head-major rows too
        return into

    def capture(self, child_tokens: torch.Tensor, logits: torch.Tensor, scores: torch.Tensor | None = None
                ) -> torch.cuda.CUDAGraph:
        """Record one pass over these buffers as a CUDA graph; ``graph.replay()`` reruns it.

        The pass has no host synchronisation, so the whole launch sequence
        (with its programmatic-dependency edges) goes into one graph. New
        tokens are passed by copying them into ``child_tokens`` before a replay.
        """
        self.run(child_tokens, logits, scores)  # first run: kernel attributes, flag words
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            self.run(child_tokens, logits, scores)
        return g

    def materialize(self, layer: int) -> torch.Tensor:
        out = torch.empty((self.C, self.T, self.model.dims.hidden), dtype=torch.bfloat16, device=self.model.device)
        _lib.check(self.lib.af_fold_materialize(self._plan, layer, out.data_ptr(), _lib.stream_ptr(out.device)))
        return out

    def stable_masks(self) -> torch.Tensor:
        """[L, C, T] bool stability masks of the last pass, rebuilt on the device from the divergent lists."""
        L = self.model.dims.n_layers
        masks = torch.ones((L, self.C * self.T), dtype=torch.bool, device=self.model.device)
        idx = torch.arange(self.m_cap, device=self.model.device)[None, :]
        valid = idx < self.n_div[:, None].long()
        flat = (torch.arange(L, device=masks.device)[:, None] * (self.C * self.T) + self.div_pos.long())[valid]
        masks.view(-1)[flat] = False
        return masks.view(L, self.C, self.T)

    def set_timing(self, enabled: bool) -> None:
        _lib.check(self.lib.af_fold_set_timing(self._plan, 1 if enabled else 0))

    def get_timing(self) -> tuple[dict, dict, int]:
        """(ms per kernel class, launches per class) accumulated since the last call, launches per run."""
        n = len(KERNEL_CLASSES)
        ms = (C.c_double * n)()
        cnt = (_i64 * n)()
        per_run = _i64()
        _lib.check(self.lib.af_fold_get_timing(self._plan, ms, cnt, n, C.byref(per_run)))
        return ({k: ms[i] for i, k in enumerate(KERNEL_CLASSES)}, {k: int(cnt[i]) for i, k in enumerate(KERNEL_CLASSES)}, int(per_run.value))

    def check_status(self) -> None:
        s = int(self.status.item())
        if s:
            self.status.zero_()
            if s & 1:
                raise TimeoutError(f"folded pass: a device wait timed out (status {s:#x})")
            if s & 2:
                raise ValueError(f"folded pass: candidate rows exceeded m_cap={self.m_cap} or the per-child bound "
                                 f"{self.child_cap} (status {s:#x})")
            raise RuntimeError(f"folded pass: device check failed (status {s:#x})")

    def __del__(self) -> None:
        plan = getattr(self, "_plan", None)
        if plan is not None and plan.value:
            try:
                self.lib.af_fold_plan_destroy(plan)
            except Exception:  # pragma: no cover - interpreter shutdown
                pass
            self._plan = None


class LLaDAModel(nn.Module):
    """LLaDA/Dream-architecture weights + native dense and folded passes (CUDA only)."""

    # Parent caches keep a head-major copy of their keys and values for the
    # folded pass's attention (False: it reads them from the row-major qkv).
    kv_headmajor: bool = True

    def __init__(self, dims: ModelDims, embed, layers: Sequence[LLaDABlock], final_norm, lm_head, max_pos: int = 4096,
                 lm_head_tiled: bool = False) -> None:
        super().__init__()
        self.dims = dims
        self.register_buffer("embed", embed.contiguous())
        self.layers = nn.ModuleList(layers)
        self.register_buffer("final_norm", final_norm.contiguous())
        self.register_buffer("lm_head", lm_head.contiguous() if lm_head_tiled else tile_weight(lm_head))
        cos, sin = rope_tables(max_pos, dims.head_dim, dims.rope_theta, embed.device)
        self.register_buffer("rope_cos", cos)
        self.register_buffer("rope_sin", sin)
        self.max_pos = max_pos
        self._plans: dict = {}
        self._build_struct()

    @property
    def device(self) -> torch.device:
        return self.embed.device

    # ------------------------------------------------------------ construction
    @classmethod
    def from_numpy(cls, dims: ModelDims, w: dict, device="cuda", max_pos: int = 4096) -> "LLaDAModel":
        """From float32 arrays named as in ``workloads.llada_weights_numpy`` (rounded to bf16)."""
        t = lambda a: torch.from_numpy(np.ascontiguousarray(a, np.float32)).to(device=device, dtype=torch.bfloat16)  # noqa: E731
        layers = [
            LLaDABlock(
                t(lw["attn_norm"]),
                torch.cat([t(lw["wq"]), t(lw["wk"]), t(lw["wv"])], dim=0),
                t(lw["wo"]),
                t(lw["ffn_norm"]),
                interleave_gate_up(t(lw["w_gate"]), t(lw["w_up"])),
                t(lw["w_down"]),
            )
            for lw in w["layers"]
        ]
        return cls(dims, t(w["embed"]), layers, t(w["final_norm"]), t(w["lm_head"]), max_pos=max_pos)

    @classmethod
    def random(cls, dims: ModelDims, seed: int = 0, device="cuda", std: float = 0.02, max_pos: int = 4096) -> "LLaDAModel":
        """N(0, std) weights drawn on the device (seeded), unit RMSNorm weights."""
        g = torch.Generator(device=device).manual_seed(seed)
        H = dims.hidden

        def w(*shape):
            out = torch.empty(shape, dtype=torch.bfloat16, device=device)
            # draw in chunks to bound the float32 temporary
            flat = out.view(-1)
            step = 1 << 26
            for i in range(0, flat.numel(), step):
                n = min(step, flat.numel() - i)
                flat[i: i + n] = (torch.randn(n, generator=g, device=device) * std).to(torch.bfloat16)
            return out

        ones = lambda: torch.ones(H, dtype=torch.bfloat16, device=device)  # noqa: E731
        layers = [
            LLaDABlock(ones(), w(dims.q_dim + 2 * dims.kv_dim, H), w(H, dims.q_dim), ones(), w(2 * dims.ffn, H), w(H, dims.ffn))
            for _ in range(dims.n_layers)
        ]
        return cls(dims, w(dims.vocab, H), layers, ones(), w(dims.vocab, H), max_pos=max_pos)

    def _build_struct(self) -> None:
        d = self.dims
        self._cdims = _Dims(d.n_layers, d.hidden, d.n_heads, d.n_kv_heads, d.head_dim, d.ffn, d.vocab, d.rms_eps)
        arr = (_Layer * d.n_layers)()
        for i, b in enumerate(self.layers):
            arr[i] = _Layer(b.attn_norm.data_ptr(), b.w_qkv.data_ptr(), b.w_o.data_ptr(), b.ffn_norm.data_ptr(),
                            b.w_gateup.data_ptr(), b.w_down.data_ptr())
        self._clayers = arr
        self._cmodel = _Model(self._cdims, C.cast(arr, C.POINTER(_Layer)), self.embed.data_ptr(), self.final_norm.data_ptr(),
                              self.lm_head.data_ptr(), self.rope_cos.data_ptr(), self.rope_sin.data_ptr(), self.max_pos)

    # ------------------------------------------------------------ dense pass
    def parent_pass(self, tokens: torch.Tensor, tau: float = 0.95) -> ParentCache:
        """Dense pass over one sequence [T] (or [1, T]); returns the parent cache."""
        _lib.require_cuda(self.embed, what="LLaDAModel")
        tokens = tokens.reshape(-1).to(device=self.device, dtype=torch.int64).contiguous()
        T = tokens.shape[0]
        if T > self.max_pos:
            raise ValueError(f"sequence {T} longer than max_pos {self.max_pos}")
        d = self.dims
        dev = self.device
        lib = _bind_late()
        layer_in = torch.empty((d.n_layers + 1, T, d.hidden), dtype=torch.bfloat16, device=dev)
        qkv = torch.empty((d.n_layers, T, d.q_dim + 2 * d.kv_dim), dtype=torch.bfloat16, device=dev)
        logits = torch.empty((T, d.vocab), dtype=torch.bfloat16, device=dev)
        self_stable = torch.empty((d.n_layers, T), dtype=torch.uint8, device=dev)
        row_sums = torch.empty((T,), dtype=torch.float32, device=dev)
        nb = _i64()
        _lib.check(lib.af_dense_workspace_bytes(C.byref(self._cdims), T, C.byref(nb)))
        ws = torch.zeros(int(nb.value), dtype=torch.uint8, device=dev)
        status = torch.zeros(1, dtype=torch.int32, device=dev)
        with torch.cuda.device(dev):
            st = lib.af_dense_forward(C.byref(self._cmodel), tokens.data_ptr(), T, float(tau), layer_in.data_ptr(), qkv.data_ptr(),
                                      logits.data_ptr(), self_stable.data_ptr(), row_sums.data_ptr(), ws.data_ptr(), ws.numel(),
                                      status.data_ptr(), _lib.stream_ptr(dev))
        _lib.check(st, "af_dense_forward")
        s = int(status.item())
        if s:
            raise TimeoutError(f"dense pass: device status {s:#x}") if s & 1 else RuntimeError(f"dense pass: device status {s:#x}")
        pc = ParentCache(tokens, layer_in, qkv, logits, self_stable, row_sums, float(tau))
        if self.kv_headmajor:
            pc.kv_headmajor(self)
        return pc

    def forward(self, tokens: torch.Tensor, attention_mask: torch.Tensor | None = None) -> torch.Tensor:
        """Plain (unfolded) logits [B, T, V] for tokens [B, T]: one dense pass per row."""
        tokens = tokens.to(self.device)
        if tokens.dim() == 1:
            tokens = tokens[None]
        return torch.stack([self.parent_pass(tokens[b]).logits for b in range(tokens.shape[0])])

    # ------------------------------------------------------------ folded pass
    def schedule(self, tau: float, layer_taus=None, layer_folds=None) -> tuple[tuple, tuple]:
        """(per-layer thresholds, per-layer fold flags), ``tau`` and True everywhere by default."""
        L = self.dims.n_layers
        taus = tuple(float(t) for t in layer_taus) if layer_taus is not None else (float(tau),) * L
        folds = tuple(bool(f) for f in layer_folds) if layer_folds is not None else (True,) * L
        if len(taus) != L or len(folds) != L:
            raise ValueError(f"a schedule needs {L} entries per layer")
        return taus, folds

    def plan(self, parent: ParentCache, n_children: int, m_cap: int, tau: float, metric: str = "cosine",
             layer_taus=None, layer_folds=None) -> FoldPlan:
        taus, folds = self.schedule(tau, layer_taus, layer_folds)
        key = (id(parent), n_children, m_cap, float(tau), metric, taus, folds)
        p = self._plans.get(key)
        if p is not None and p.parent is parent and p._parent_version != parent.version and p.parent_rewritten():
            p = None  # an in-place promotion changed where the parent fails its own gate
        if p is None or p.parent is not parent:
            p = FoldPlan(self, parent, n_children, m_cap, tau, metric, taus, folds)
            self._plans = {k: v for k, v in self._plans.items() if v.parent is parent}
            self._plans[key] = p
        return p

    @staticmethod
    def capacity(child_tokens: torch.Tensor, parent: ParentCache, taus: Sequence[float] | None = None) -> int:
        """Rows a pass can need: edited rows + every child x every row the parent fails its own gate on."""
        return LLaDAModel.capacity_and_bound(child_tokens, parent, taus)[0]

    @staticmethod
    def capacity_and_bound(child_tokens: torch.Tensor, parent: ParentCache, taus: Sequence[float] | None = None,
                           folds: Sequence[bool] | None = None) -> tuple[int, int]:
        """(m_cap, bound on one child's candidate rows per layer), from one small device read.

        With a layer that does not fold every row is a candidate there: m_cap = C * T, bound T.
        """
        C, T = child_tokens.shape
        if folds is not None and not all(folds):
            return round_capacity(C * T, C, T), T
        taus = tuple(taus) if taus is not None else (parent.tau,) * parent.self_stable.shape[0]
        per_child = (child_tokens != parent.tokens[None]).sum(dim=1)
        edited, most = (int(v) for v in torch.stack([per_child.sum(), per_child.max()]).cpu())
        su_rows = parent.su_rows_at(taus)
        return round_capacity(edited + C * su_rows, C, T), most + su_rows

    def verify(self, child_tokens: torch.Tensor, parent: ParentCache, tau: float, metric: str = "cosine",
               logits: torch.Tensor | None = None, scores: torch.Tensor | None = None, m_cap: int | None = None,
               keep_kv: bool = False, layer_taus=None, layer_folds=None) -> tuple[torch.Tensor, FoldPlan]:
        """Folded verification of child_tokens [C, T] against ``parent``; returns (logits [C, T, V], plan).

        ``layer_taus`` / ``layer_folds``: an optional per-layer schedule (see FoldPlan).
        """
        child_tokens = child_tokens.to(device=self.device, dtype=torch.int64).contiguous()
        if child_tokens.dim() != 2 or child_tokens.shape[1] != parent.seq:
            raise ValueError(f"children must be [C, {parent.seq}], got {tuple(child_tokens.shape)}")
        Cn = child_tokens.shape[0]
        taus, folds = self.schedule(tau, layer_taus, layer_folds)
        child_cap = None
        if m_cap is None:
            m_cap, child_cap = self.capacity_and_bound(child_tokens, parent, taus, folds)
        plan = self.plan(parent, Cn, m_cap, tau, metric, taus, folds)
        if child_cap is not None:
            plan.set_child_cap(child_cap)
        if keep_kv and not plan.keeps_kv:
            plan.keep_kv(True)
        if logits is None:
            logits = torch.empty((Cn, parent.seq, self.dims.vocab), dtype=torch.bfloat16, device=self.device)
        plan.run(child_tokens, logits, scores)
        return logits, plan

    def native_folded_forward(self, tokens: torch.Tensor, cache, gate, branch_id: Any, parent_branch_id: Any = None,
                              step_idx: int = 0, scheduler=None, **kwargs: Any) -> torch.Tensor:
        """FoldedModel.forward for this architecture (see actfold_b200.core.model_wrapper).

        With a ``scheduler`` every layer takes the reference's per-layer
        decisions (actfold/core/folded_transformer.py:107-119): a layer where
        ``should_fold(layer, step_idx)`` is False recomputes every row and is
        not recorded by the profiler; a folding layer gates at
        ``get_tau(layer, step_idx, "general")``, which the gate keeps as its
        ``tau`` afterwards (the reference sets it on the shared gate).
        """
        from actfold_b200.profiler.stability_profiler import GLOBAL_STABILITY_PROFILER

        tokens = tokens.to(self.device)
        if tokens.dim() == 1:
            tokens = tokens[None]
        parents = getattr(cache, "native_parents", None)
        if parents is None:
            parents = {}
            cache.native_parents = parents
        if parent_branch_id is None:
            if tokens.shape[0] != 1:
                raise ValueError("a parent pass takes one sequence [1, T]")
            pc = self.parent_pass(tokens[0], tau=gate.tau)
            parents[branch_id] = pc
            register_parent_in_cache(cache, branch_id, pc)
            return pc.logits[None]
        L = self.dims.n_layers
        taus, folds = None, None
        if scheduler is not None:
            folds = [bool(scheduler.should_fold(li, step_idx)) for li in range(L)]
            taus = [float(scheduler.get_tau(layer_idx=li, step_idx=step_idx, task_type="general")) if folds[li]
                    else float(gate.tau) for li in range(L)]
        children = getattr(cache, "native_children", None)
        if children is None:
            children = {}
            cache.native_children = children
        pc = parents.get(parent_branch_id)
        if pc is None:
            pc = _promote_recorded_child(cache, parents, children, parent_branch_id)
        ids = list(branch_id) if isinstance(branch_id, (list, tuple)) else [branch_id] * tokens.shape[0]
        if pc is None:
            # No usable parent activations: every layer recomputes (folded_transformer.py:135-141), and
            # the reference then holds each child's activations under its id, so each row's dense pass
            # becomes a parent cache that later children can fold against.
            rows = []
            for i, bid in enumerate(ids):
                cpc = self.parent_pass(tokens[i], tau=gate.tau)
                if len(set(ids)) == len(ids):
                    children.pop(bid, None)
                    parents[bid] = cpc
                    register_parent_in_cache(cache, bid, cpc)
                rows.append(cpc.logits)
            return torch.stack(rows)
        if pc.seq != tokens.shape[1]:
            pc = pc.resized(tokens.shape[1])  # zero-filled / truncated parent rows, as the reference gathers them
        logits, plan = self.verify(tokens, pc, gate.tau, gate.metric, keep_kv=True, layer_taus=taus, layer_folds=folds)
        plan.check_status()
        if len(set(ids)) == len(ids):
            # Every verified child can be named as a later parent_branch_id (the
            # reference caches each child's activations): it is promoted on
            # first use, while its plan still holds this run.
            for k in [k for k, (pl, _, se) in children.items() if pl.serial != se]:
                del children[k]  # records of runs that are gone
            for c, bid in enumerate(ids):
                parents.pop(bid, None)
                children[bid] = (plan, c, plan.serial)
        folded = [li for li in range(L) if plan.layer_folds[li]]
        if folded:
            masks = plan.stable_masks()[folded]
            layer_tau = [plan.layer_taus[li] for li in folded]
            if len(set(ids)) == len(ids):
                GLOBAL_STABILITY_PROFILER.record_batch(ids, parent_branch_id, step_idx, masks, layer_tau, gate.metric,
                                                       layer_ids=folded)
            else:
                for i, li in enumerate(folded):
                    GLOBAL_STABILITY_PROFILER.record(ids[0], parent_branch_id, li, step_idx, masks[i], layer_tau[i],
                                                     gate.metric)
            if scheduler is not None:
                gate.set_tau(layer_tau[-1])
        return logits


def round_capacity(rows: int, C: int, T: int) -> int:
    """Candidate capacity of a pass: ``rows`` rounded up to 16, at least 16, at most C x T (rounded)."""
    cap = max(16, ((rows + 15) // 16) * 16)
    return min(cap, ((C * T + 15) // 16) * 16)


def _promote_recorded_child(cache, parents: dict, children: dict, branch_id: Any) -> ParentCache | None:
    """Parent cache of a child verified earlier, promoted from its plan's last run; None when that run is gone."""
    rec = children.get(branch_id)
    if rec is None:
        return None
    plan, c, serial = rec
    if plan.serial != serial:
        return None  # the plan has verified another batch since; that child's rows are overwritten
    pc = plan.promote(c)
    parents[branch_id] = pc
    register_parent_in_cache(cache, branch_id, pc)
    return pc


def register_parent_in_cache(cache, branch_id: Any, pc: ParentCache) -> None:
    """Expose the parent's per-layer input / output through the ActivationCache API (views, no copies)."""
    put_views = getattr(cache, "put_views", None)
    if put_views is None:
        return
    L = pc.layer_in.shape[0] - 1
    for li in range(L):
        put_views(branch_id, li, {"ffn_out": pc.layer_in[li + 1][None], "hidden_states": pc.layer_in[li][None]})

