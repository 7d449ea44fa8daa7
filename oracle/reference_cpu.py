"""The reference's per-child verification path on the host cores (TEST / BENCH INFRASTRUCTURE).

Used only by ``bench.py`` (its ``cpu_baseline`` leg and the ``--impl
reference`` arm) to time what the reference does to verify one child branch
on a CPU, with the parent's activations already cached:

* per layer, ``FoldedTransformerLayer.forward`` for a child
  (actfold/core/folded_transformer.py:60-203):

  - ``ActivationCache.get`` of the parent's ``hidden_states`` for every token
    (activation_cache.py:112-153 -> fused_ops.py:256-324: T dict lookups, a
    ``torch.stack`` of T rows, a masked ``torch.where``, an LRU touch per token);
  - ``SimilarityGate``: ``F.cosine_similarity(child, parent, eps=1e-8) > tau``
    (similarity_gate.py:43-83);
  - ``GLOBAL_STABILITY_PROFILER.record``: ``.item()`` of the stable ratio and
    ``nonzero`` of the divergent positions (stability_profiler.py:106-158);
  - the ``.all()`` / ``.any()`` host checks (folded_transformer.py:162, 183);
  - ``_recompute_all``: the wrapped layer on ALL T rows (:224-258);
  - ``ActivationCache.get`` of the parent's ``ffn_out`` under the stable mask,
    ``merge_stable_divergent`` (``torch.where``, fused_ops.py:38-51, 206-253);
  - ``_store_activations``: one ``put`` of T per-token ``.contiguous()`` copies
    of the layer input and output (:260-274, activation_cache.py:50-110);

* the LM head over all T rows (the full ``[T, V]`` logits).

The wrapped layer is a pre-norm LLaDA / Dream block in bf16 (RMSNorm,
rotate-half RoPE, non-causal attention, SwiGLU), the arithmetic of a bf16
checkpoint on ``torch`` CPU kernels (oneDNN, AMX where the host has it). The
reference ships no layer code for these models (they load through Hugging
Face ``trust_remote_code``), so the block is restated here; its FLOPs are the
architecture's.

One timed unit is one child verified completely (every layer and the
full-vocabulary logits). The reference verifies children one after another,
so C such units are one C-child pass. Weights are seeded N(0, std) values:
a pool of normal draws, each matrix a different window of it (weight values
do not change the time of dense bf16 GEMMs, and drawing 8 B fresh normals on
the host would take minutes).
"""

from __future__ import annotations

import os
import time
from collections import OrderedDict

import numpy as np
import torch
import torch.nn.functional as F

BF = torch.bfloat16


class TokenCache:
    """Per-token dict entries with per-layer LRU order (actfold/core/activation_cache.py:50-153)."""

    def __init__(self, max_entries_per_layer: int) -> None:
        self.max_entries = max_entries_per_layer
        self.layers: dict[int, OrderedDict] = {}

    def put(self, branch_id, layer_idx: int, activations: dict, step_idx: int = 0) -> None:
        cache = self.layers.setdefault(layer_idx, OrderedDict())
        T = next(iter(activations.values())).shape[1]
        for t in range(T):
            key = (branch_id, layer_idx, t, step_idx)
            val = {n: a[:, t].contiguous() for n, a in activations.items()}
            if key in cache:
                cache.move_to_end(key)
            cache[key] = val
            if len(cache) > self.max_entries:
                cache.popitem(last=False)

    def get(self, branch_id, layer_idx: int, token_mask: torch.Tensor, step_idx: int = 0) -> dict:
        cache = self.layers.setdefault(layer_idx, OrderedDict())
        B, T = token_mask.shape
        k0 = (branch_id, layer_idx, 0, step_idx)
        if k0 not in cache:
            raise KeyError(f"No cache entry for branch={branch_id}, layer={layer_idx}, step={step_idx}")
        if not all((branch_id, layer_idx, t, step_idx) in cache for t in range(T)):
            raise KeyError("sparse parent entries: the timing sample keeps every parent token cached")
        out = {}
        for name in cache[k0]:
            stacked = torch.stack([cache[(branch_id, layer_idx, t, step_idx)][name] for t in range(T)], dim=1)
            m = token_mask.view(B, T, *([1] * (stacked.ndim - 2)))
            out[name] = torch.where(m, stacked, torch.zeros_like(stacked))
        for t in range(T):
            key = (branch_id, layer_idx, t, step_idx)
            if key in cache and bool(token_mask[:, t].any()):
                cache.move_to_end(key)
        return out

    def clear_branch(self, branch_id) -> None:
        for cache in self.layers.values():
            for key in [k for k in cache if k[0] == branch_id]:
                del cache[key]


def _rms(x: torch.Tensor, w: torch.Tensor, eps: float) -> torch.Tensor:
    xf = x.float()
    return (xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps)).to(BF) * w


def _rope(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
    h = x.shape[-1] // 2
    x1, x2 = x[..., :h], x[..., h:]
    return torch.cat([x1 * cos - x2 * sin, x2 * cos + x1 * sin], dim=-1)


class Block:
    """One bf16 pre-norm block: RMSNorm, QKV, RoPE, non-causal attention, O, RMSNorm, SwiGLU."""

    def __init__(self, w: dict, dims, cos: torch.Tensor, sin: torch.Tensor) -> None:
        self.w, self.d, self.cos, self.sin = w, dims, cos, sin

    def __call__(self, x: torch.Tensor) -> torch.Tensor:
        d, w = self.d, self.w
        B, T, _ = x.shape
        q_dim, kv_dim = d.n_heads * d.head_dim, d.n_kv_heads * d.head_dim
        a = _rms(x, w["attn_norm"], d.rms_eps)
        qkv = F.linear(a, w["w_qkv"])
        q = qkv[..., :q_dim].view(B, T, d.n_heads, d.head_dim).transpose(1, 2)
        k = qkv[..., q_dim:q_dim + kv_dim].view(B, T, d.n_kv_heads, d.head_dim).transpose(1, 2)
        v = qkv[..., q_dim + kv_dim:].view(B, T, d.n_kv_heads, d.head_dim).transpose(1, 2)
        cos, sin = self.cos[:T], self.sin[:T]
        q, k = _rope(q, cos, sin), _rope(k, cos, sin)
        o = F.scaled_dot_product_attention(q, k, v, is_causal=False, enable_gqa=d.n_heads != d.n_kv_heads)
        h = x + F.linear(o.transpose(1, 2).reshape(B, T, q_dim), w["w_o"])
        b = _rms(h, w["ffn_norm"], d.rms_eps)
        f = F.silu(F.linear(b, w["w_gate"])) * F.linear(b, w["w_up"])
        return h + F.linear(f, w["w_down"])


class ReferenceCpuPath:
    """Weights, parent cache and the per-child verification of the reference, on the host cores."""

    def __init__(self, dims, T: int, tau: float = 0.95, seed: int = 0, std: float = 0.02,
                 threads: int | None = None) -> None:
        self.threads = int(threads or os.cpu_count() or 1)
        # torchrun sets OMP_NUM_THREADS=1 for every rank; the sample uses every host thread.
        torch.set_num_threads(self.threads)
        self.d, self.T, self.tau = dims, int(T), float(tau)
        H = dims.hidden
        q_dim, kv_dim = dims.n_heads * dims.head_dim, dims.n_kv_heads * dims.head_dim
        rng = np.random.default_rng(seed)
        pool = torch.from_numpy(rng.standard_normal(1 << 25, dtype=np.float32)).mul_(std).to(BF)

        def mat(n: int, k: int) -> torch.Tensor:
            out = torch.empty(n * k, dtype=BF)
            off, done = int(rng.integers(0, pool.numel())), 0
            while done < out.numel():
                take = min(out.numel() - done, pool.numel() - off)
                out[done:done + take].copy_(pool[off:off + take])
                done += take
                off = 0
            return out.view(n, k)

        ones = torch.ones(H, dtype=BF)
        self.layers = []
        inv = 1.0 / (float(dims.rope_theta) ** (np.arange(0, dims.head_dim, 2, dtype=np.float64) / dims.head_dim))
        ang = np.arange(self.T, dtype=np.float64)[:, None] * inv[None, :]
        cos = torch.from_numpy(np.cos(ang)).to(BF)
        sin = torch.from_numpy(np.sin(ang)).to(BF)
        for _ in range(dims.n_layers):
            w = dict(attn_norm=ones, ffn_norm=ones, w_qkv=mat(q_dim + 2 * kv_dim, H), w_o=mat(H, q_dim),
                     w_gate=mat(dims.ffn, H), w_up=mat(dims.ffn, H), w_down=mat(H, dims.ffn))
            self.layers.append(Block(w, dims, cos, sin))
        self.embed = mat(dims.vocab, H)
        self.final_norm = ones
        self.lm_head = mat(dims.vocab, H)
        # Parent entries for every token of every layer stay cached (capacity for parent + one child).
        self.cache = TokenCache(max_entries_per_layer=2 * self.T)
        self.profile: list = []

    def _gate(self, hc: torch.Tensor, hp: torch.Tensor) -> torch.Tensor:
        return F.cosine_similarity(hc, hp.to(hc.dtype), dim=-1, eps=1e-8) > self.tau

    def _record(self, mask: torch.Tensor) -> None:
        ratio = float(mask.float().mean().item())
        pos = torch.nonzero(~mask, as_tuple=False) if ratio < 1.0 else None
        self.profile.append((ratio, pos))

    def parent_pass(self, tokens: np.ndarray) -> torch.Tensor:
        """Dense pass of the parent with every layer's input / output cached per token."""
        with torch.inference_mode():
            x = self.embed[torch.from_numpy(tokens).long()][None]
            for li, blk in enumerate(self.layers):
                y = blk(x)
                self.cache.put("parent", li, {"ffn_out": y, "hidden_states": x})
                x = y
            return F.linear(_rms(x, self.final_norm, self.d.rms_eps), self.lm_head)

    def verify_child(self, tokens: np.ndarray, branch_id="child") -> torch.Tensor:
        """One child through the reference's folded path; returns its [1, T, V] logits."""
        self.profile = []
        with torch.inference_mode():
            x = self.embed[torch.from_numpy(tokens).long()][None]
            ones = torch.ones(x.shape[:2], dtype=torch.bool)
            for li, blk in enumerate(self.layers):
                hp = self.cache.get("parent", li, ones)["hidden_states"]
                stable = self._gate(x, hp)
                self._record(stable)
                if bool(stable.all()):
                    out = self.cache.get("parent", li, stable)["ffn_out"]
                elif not bool(stable.any()):
                    out = blk(x)
                else:
                    pf = self.cache.get("parent", li, stable)["ffn_out"]
                    out = torch.where(stable[..., None], pf, blk(x))
                self.cache.put(branch_id, li, {"ffn_out": out, "hidden_states": x})
                x = out
            logits = F.linear(_rms(x, self.final_norm, self.d.rms_eps), self.lm_head)
        return logits

    def time_child(self, tokens: np.ndarray) -> float:
        """Seconds to verify one child (its cache entries are dropped afterwards, outside the timing)."""
        t0 = time.perf_counter()
        self.verify_child(tokens, "child")
        dt = time.perf_counter() - t0
        self.cache.clear_branch("child")
        return dt


def host_description(threads: int) -> str:
    """CPU model and bf16 matrix extensions of this host (for the baseline's description)."""
    model, flags = "unknown CPU", set()
    try:
        with open("/proc/cpuinfo") as f:
            for line in f:
                if line.startswith("model name") and model == "unknown CPU":
                    model = line.split(":", 1)[1].strip()
                elif line.startswith("flags"):
                    flags = set(line.split(":", 1)[1].split())
                    break
    except OSError:
        pass
    ext = [x for x in ("amx_bf16", "avx512_bf16") if x in flags]
    return f"{model}, {threads} threads" + (f", {'/'.join(ext)}" if ext else "")


def flops_per_child(dims, T: int) -> float:
    """Dense FLOPs the reference spends per child: every layer on all T rows + the LM head."""
    H = dims.hidden
    q_dim, kv_dim = dims.n_heads * dims.head_dim, dims.n_kv_heads * dims.head_dim
    per_layer = 2 * T * H * (q_dim + 2 * kv_dim) + 2 * T * q_dim * H + 6 * T * H * dims.ffn + 4 * T * T * q_dim
    return dims.n_layers * per_layer + 2.0 * T * H * dims.vocab


__all__ = ["ReferenceCpuPath", "TokenCache", "Block", "host_description", "flops_per_child"]
