"""torch (CPU, bf16) module with the arithmetic of ``oracle.llada`` (TEST INFRASTRUCTURE).

Used by ``tests/golden/make_golden.py`` (the reference's FoldedModel wraps
this module so the golden vectors record the reference's folding decisions
over the restated LLaDA block) and, on the GPU at full LLaDA-8B size, by
``tests/test_full_size_gpu.py`` as the fp32 restatement of one block. Rounding points are those listed in
``oracle.llada``.
"""

from __future__ import annotations

import numpy as np
import torch
import torch.nn as nn

from oracle import llada as L

BF = torch.bfloat16


def _t(a: np.ndarray) -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(a, np.float32)).to(BF)


def _rms(x: torch.Tensor, w: torch.Tensor, eps: float) -> torch.Tensor:
    xf = x.float()
    var = xf.pow(2).mean(-1, keepdim=True)
    xn = (xf * torch.rsqrt(var + eps)).to(BF)
    return (xn.float() * w.float()).to(BF)


def _mm(a: torch.Tensor, w: torch.Tensor) -> torch.Tensor:
    return (a.float() @ w.float().T).to(BF)


class TorchLLaDABlock(nn.Module):
    def __init__(self, lw: dict, dims: L.LLaDADims, cos: np.ndarray, sin: np.ndarray) -> None:
        super().__init__()
        self.dims = dims
        for k, v in lw.items():
            self.register_buffer(k, _t(v))
        self.register_buffer("cos", torch.from_numpy(cos))
        self.register_buffer("sin", torch.from_numpy(sin))

    @classmethod
    def from_tensors(cls, lw: dict, dims: L.LLaDADims, cos: torch.Tensor, sin: torch.Tensor) -> "TorchLLaDABlock":
        """Block over bf16 tensors already on a device (wq, wk, wv, wo, w_gate, w_up, w_down, norms)."""
        blk = cls.__new__(cls)
        nn.Module.__init__(blk)
        blk.dims = dims
        for k, v in lw.items():
            blk.register_buffer(k, v.to(BF))
        blk.register_buffer("cos", cos.float())
        blk.register_buffer("sin", sin.float())
        return blk

    def _rope(self, x: torch.Tensor) -> torch.Tensor:
        T = x.shape[1]
        h = x.shape[-1] // 2
        c = self.cos[:T][None, :, None, :]
        s = self.sin[:T][None, :, None, :]
        xf = x.float()
        x1, x2 = xf[..., :h], xf[..., h:]
        return torch.cat([x1 * c - x2 * s, x2 * c + x1 * s], dim=-1).to(BF)

    def forward(self, hidden_states: torch.Tensor, attention_mask: torch.Tensor | None = None) -> torch.Tensor:
        d = self.dims
        x = hidden_states
        B, T, _ = x.shape
        a = _rms(x, self.attn_norm, d.rms_eps)
        q = self._rope(_mm(a, self.wq).view(B, T, d.n_heads, d.head_dim))
        k = self._rope(_mm(a, self.wk).view(B, T, d.n_kv_heads, d.head_dim))
        v = _mm(a, self.wv).view(B, T, d.n_kv_heads, d.head_dim)
        grp = d.n_heads // d.n_kv_heads
        kf = k.float().repeat_interleave(grp, dim=2)
        vf = v.float().repeat_interleave(grp, dim=2)
        s = torch.einsum("bqhd,bkhd->bhqk", q.float(), kf) / float(np.sqrt(d.head_dim))
        p = torch.softmax(s, dim=-1)
        o = torch.einsum("bhqk,bkhd->bqhd", p, vf).to(BF).reshape(B, T, -1)
        h = (x.float() + _mm(o, self.wo).float()).to(BF)
        b = _rms(h, self.ffn_norm, d.rms_eps)
        g = _mm(b, self.w_gate).float()
        u = _mm(b, self.w_up).float()
        f = (g / (1.0 + torch.exp(-g)) * u).to(BF)
        return (h.float() + _mm(f, self.w_down).float()).to(BF)


class TorchLLaDA(nn.Module):
    def __init__(self, weights: dict, dims: L.LLaDADims, T: int) -> None:
        super().__init__()
        cos, sin = L.rope_tables(T, dims.head_dim, dims.rope_theta)
        self.dims = dims
        self.register_buffer("embed", _t(weights["embed"]))
        self.layers = nn.ModuleList(TorchLLaDABlock(lw, dims, cos, sin) for lw in weights["layers"])
        self.register_buffer("final_norm", _t(weights["final_norm"]))
        self.register_buffer("lm_head", _t(weights["lm_head"]))

    def forward(self, tokens: torch.Tensor) -> torch.Tensor:
        x = self.embed[tokens]
        for layer in self.layers:
            x = layer(x)
        return _mm(_rms(x, self.final_norm, self.dims.rms_eps), self.lm_head)
