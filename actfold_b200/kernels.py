"""Thin torch-facing wrappers of the C-ABI kernels used by the native folded pass.

Each wrapper validates shapes, takes device pointers and the current stream,
and raises on a non-zero af_status. There is no fallback implementation.
"""

from __future__ import annotations

import ctypes as C

import torch

from actfold_b200 import _lib

EPI_STORE, EPI_RESIDUAL, EPI_SWIGLU, EPI_ROPE = 0, 1, 2, 3


def tile_weight(w: torch.Tensor) -> torch.Tensor:
    """[n, k] -> [n/128, k/64, 128, 64]: every 128 x 64 GEMM tile one contiguous 16 KB block.

    A one-time re-layout at model load so the GEMM streams each weight tile from
    HBM as a single contiguous block instead of 128 strided 128-byte pieces.
    """
    n, k = w.shape
    if n % 128 or k % 64:
        raise ValueError(f"tile_weight: shape {tuple(w.shape)} is not a multiple of (128, 64)")
    return w.reshape(n // 128, 128, k // 64, 64).permute(0, 2, 1, 3).contiguous()

class DeviceStatus:
    """Device status word the kernels OR their AF_STATUS bits into (1 timeout, 2 capacity, 4 bounds)."""

    def __init__(self, device: torch.device | str = "cuda") -> None:
        self.status = torch.zeros(1, dtype=torch.int32, device=device)

    def check_status(self) -> None:
        s = int(self.status.item())
        if s:
            self.status.zero_()
            if s & 1:
                raise TimeoutError(f"device wait timed out (status {s:#x})")
            raise RuntimeError(f"device-side check failed (status {s:#x})")


def linear(
    x: torch.Tensor,
    w: torch.Tensor,
    ws: DeviceStatus,
    epilogue: int = EPI_STORE,
    out: torch.Tensor | None = None,
    m_dev: torch.Tensor | None = None,
    out_rows: torch.Tensor | None = None,
    residual: torch.Tensor | None = None,
    res_rows: torch.Tensor | None = None,
    rope: tuple[torch.Tensor, torch.Tensor, torch.Tensor, int] | None = None,
    splits: int = 0,
    w_tiled: bool = False,
    n: int | None = None,
) -> torch.Tensor:
    """``out[m] = epilogue(x[m] . w^T)`` on the tcgen05 GEMM (bf16 in/out, fp32 accumulate).

    x: [m_cap, k] bf16 (row stride may exceed k); w: [n, k] bf16 contiguous, or
    with ``w_tiled`` the output of :func:`tile_weight` (pass ``n``).
    rope = (cos [P, 64] f32, sin [P, 64] f32, positions [m_cap] i32, rope_cols).
    """
    _lib.require_cuda(x, w, what="linear")
    if x.dtype != torch.bfloat16 or w.dtype != torch.bfloat16:
        raise ValueError("linear: bf16 operands required")
    if x.stride(1) != 1 or not w.is_contiguous():
        raise ValueError("linear: operands must have a contiguous inner dimension")
    m_cap, k = x.shape
    if w_tiled:
        if n is None or w.numel() != n * k:
            raise ValueError("linear: a tiled weight needs n with w.numel() == n * k")
    else:
        n = w.shape[0]
        if w.shape[1] != k:
            raise ValueError(f"linear: k mismatch {x.shape} vs {w.shape}")
    out_n = n // 2 if epilogue == EPI_SWIGLU else n
    if out is None:
        out = torch.empty((m_cap, out_n), dtype=torch.bfloat16, device=x.device)
    cos = sin = pos = None
    rope_cols = 0
    if rope is not None:
        cos, sin, pos, rope_cols = rope
    with torch.cuda.device(x.device):
        st = _lib.load().af_linear_bf16(
            x.data_ptr(), x.stride(0), m_cap, _lib.ptr(m_dev), w.data_ptr(), n, k, 1 if w_tiled else 0, epilogue,
            out.data_ptr(), out.stride(0), _lib.ptr(out_rows),
            _lib.ptr(residual), residual.stride(0) if residual is not None else 0, _lib.ptr(res_rows),
            _lib.ptr(cos), _lib.ptr(sin), _lib.ptr(pos), rope_cols,
            splits, ws.status.data_ptr(), _lib.stream_ptr(x.device),
        )
    _lib.check(st, "linear")
    return out


def attention(
    q: torch.Tensor,
    pk: torch.Tensor,
    pv: torch.Tensor,
    n_heads: int,
    n_kv_heads: int,
    out: torch.Tensor | None = None,
    qsrc: torch.Tensor | None = None,
    qchild: torch.Tensor | None = None,
    n_q: torch.Tensor | None = None,
    fresh_bits: torch.Tensor | None = None,
    fk: torch.Tensor | None = None,
    fv: torch.Tensor | None = None,
    fchild: torch.Tensor | None = None,
    n_f: torch.Tensor | None = None,
    n_q_cap: int | None = None,
    status: DeviceStatus | None = None,
) -> torch.Tensor:
    """Non-causal attention of query rows over parent K/V with per-child fresh-key overrides.

    q: rows holding n_heads x 128 query features (row i read at qsrc[i]);
    pk/pv: [T, n_kv_heads * 128]; fk/fv: candidate K/V rows; fresh_bits:
    [children, ceil(T/32)] int32 bitmap of fresh positions per child.
    """
    _lib.require_cuda(q, pk, pv, what="attention")
    T = pk.shape[0]
    cap = n_q_cap if n_q_cap is not None else (qsrc.shape[0] if qsrc is not None else q.shape[0])
    if out is None:
        out = torch.empty((cap, n_heads * 128), dtype=torch.bfloat16, device=q.device)
    n_f_cap = fk.shape[0] if fk is not None else 0
    with torch.cuda.device(q.device):
        st = _lib.load().af_attention_bf16(
            q.data_ptr(), q.stride(0), _lib.ptr(qsrc), _lib.ptr(qchild), _lib.ptr(n_q), cap,
            pk.data_ptr(), pv.data_ptr(), pk.stride(0), T,
            _lib.ptr(fresh_bits), fresh_bits.shape[1] if fresh_bits is not None else 0,
            _lib.ptr(fk), _lib.ptr(fv), fk.stride(0) if fk is not None else 0, _lib.ptr(fchild), _lib.ptr(n_f), n_f_cap,
            out.data_ptr(), out.stride(0), n_heads, n_kv_heads, 128, 128 ** -0.5,
            status.status.data_ptr() if status is not None else None, _lib.stream_ptr(q.device),
        )
    _lib.check(st, "attention")
    return out
