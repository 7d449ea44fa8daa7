"""tcgen05 GEMM numerics against a plain PyTorch fp32 reference of the same op.

Tolerance: bf16 outputs, so max |err| <= 1e-2 * max |ref| (a few bf16 ulps at
the tensor's scale) and mean |err| well below that.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _rel(a: torch.Tensor, b: torch.Tensor) -> float:
    return float((a.float() - b.float()).abs().max() / b.float().abs().max().clamp_min(1e-6))


@pytest.fixture(scope="module")
def ws():
    from actfold_b200.kernels import DeviceStatus

    return DeviceStatus()


@pytest.mark.parametrize("m", [1, 16, 40, 128, 256, 300, 1024])
@pytest.mark.parametrize("splits", [1, 0, 3, 8])
def test_linear_store(ws, m, splits):
    from actfold_b200.kernels import linear

    g = torch.Generator(device="cuda").manual_seed(m)
    x = torch.randn(m, 4096, device="cuda", generator=g).to(torch.bfloat16)
    w = (torch.randn(1024, 4096, device="cuda", generator=g) * 0.02).to(torch.bfloat16)
    out = linear(x, w, ws, splits=splits)
    ref = (x.float() @ w.float().T).to(torch.bfloat16)
    torch.cuda.synchronize()
    ws.check_status()
    assert _rel(out, ref) <= 1e-2


def test_linear_dynamic_m_and_row_maps(ws):
    from actfold_b200.kernels import linear

    m_cap, M = 256, 77
    x = torch.randn(m_cap, 512, device="cuda").to(torch.bfloat16)
    w = (torch.randn(384, 512, device="cuda") * 0.05).to(torch.bfloat16)
    m_dev = torch.tensor([M], dtype=torch.int32, device="cuda")
    rows = torch.randperm(1000, device="cuda")[:m_cap].to(torch.int32)
    out = torch.zeros(1000, 384, dtype=torch.bfloat16, device="cuda")
    linear(x, w, ws, out=out, m_dev=m_dev, out_rows=rows)
    ref = (x[:M].float() @ w.float().T).to(torch.bfloat16)
    assert _rel(out[rows[:M].long()], ref) <= 1e-2
    untouched = torch.ones(1000, dtype=torch.bool, device="cuda")
    untouched[rows[:M].long()] = False
    assert (out[untouched] == 0).all()
    m_dev.zero_()
    out2 = torch.zeros_like(out)
    linear(x, w, ws, out=out2, m_dev=m_dev, out_rows=rows)
    assert (out2 == 0).all()
    torch.cuda.synchronize()
    ws.check_status()


@pytest.mark.parametrize("splits", [1, 0])
def test_linear_residual_and_strided_input(ws, splits):
    from actfold_b200.kernels import EPI_RESIDUAL, linear

    big = torch.randn(64, 8192, device="cuda").to(torch.bfloat16)
    x = big[:, 1024:5120]  # row stride 8192
    w = (torch.randn(4096, 4096, device="cuda") * 0.02).to(torch.bfloat16)
    res = torch.randn(64, 4096, device="cuda").to(torch.bfloat16)
    res_rows = torch.arange(63, -1, -1, device="cuda", dtype=torch.int32)
    out = linear(x, w, ws, epilogue=EPI_RESIDUAL, residual=res, res_rows=res_rows, splits=splits)
    o = (x.float() @ w.float().T).to(torch.bfloat16).float()
    ref = (res[res_rows.long()].float() + o).to(torch.bfloat16)
    assert _rel(out, ref) <= 1e-2
    torch.cuda.synchronize()
    ws.check_status()


@pytest.mark.parametrize("splits", [1, 4, 5])
def test_linear_swiglu_interleaved(ws, splits):
    from actfold_b200.kernels import EPI_SWIGLU, linear

    FF, H, m = 512, 1024, 96
    wg = (torch.randn(FF, H, device="cuda") * 0.03).to(torch.bfloat16)
    wu = (torch.randn(FF, H, device="cuda") * 0.03).to(torch.bfloat16)
    w = torch.stack([wg.view(FF // 64, 64, H), wu.view(FF // 64, 64, H)], dim=1).reshape(2 * FF, H).contiguous()
    x = torch.randn(m, H, device="cuda").to(torch.bfloat16)
    out = linear(x, w, ws, epilogue=EPI_SWIGLU, splits=splits)
    g = (x.float() @ wg.float().T).to(torch.bfloat16).float()
    u = (x.float() @ wu.float().T).to(torch.bfloat16).float()
    ref = (g / (1 + torch.exp(-g)) * u).to(torch.bfloat16)
    assert out.shape == (m, FF)
    assert _rel(out, ref) <= 1e-2
    torch.cuda.synchronize()
    ws.check_status()


@pytest.mark.parametrize("splits", [1, 2])
def test_linear_rope_matches_oracle(ws, splits):
    from actfold_b200.kernels import EPI_ROPE, linear
    from oracle.llada import apply_rope, rope_tables
    from oracle.numerics import round_bf16

    H, nh, T, m = 256, 2, 64, 20
    n = 3 * H  # q, k, v heads of 128
    x = torch.randn(m, H, device="cuda").to(torch.bfloat16)
    w = (torch.randn(n, H, device="cuda") * 0.05).to(torch.bfloat16)
    cos, sin = rope_tables(T, 128, 500000.0)
    pos = torch.randint(0, T, (m,), device="cuda", dtype=torch.int32)
    out = linear(x, w, ws, epilogue=EPI_ROPE, rope=(torch.from_numpy(cos).cuda(), torch.from_numpy(sin).cuda(), pos, 2 * H), splits=splits)
    qkv = round_bf16((x.float() @ w.float().T).cpu().numpy())
    p = pos.cpu().numpy()
    q = apply_rope(qkv[:, :H].reshape(m, nh, 128), p, cos, sin).reshape(m, H)
    k = apply_rope(qkv[:, H : 2 * H].reshape(m, nh, 128), p, cos, sin).reshape(m, H)
    ref = np.concatenate([q, k, qkv[:, 2 * H :]], axis=1)
    err = np.abs(out.float().cpu().numpy() - ref).max() / np.abs(ref).max()
    assert err <= 1e-2
    torch.cuda.synchronize()
    ws.check_status()


def test_linear_large_n_like_lm_head(ws):
    from actfold_b200.kernels import linear

    x = torch.randn(48, 4096, device="cuda").to(torch.bfloat16)
    w = (torch.randn(126464, 4096, device="cuda") * 0.02).to(torch.bfloat16)
    out = linear(x, w, ws)
    ref = (x.float() @ w.float().T).to(torch.bfloat16)
    assert _rel(out, ref) <= 1e-2
    torch.cuda.synchronize()
    ws.check_status()


@pytest.mark.parametrize("splits", [1, 0])
def test_linear_tiled_weights(ws, splits):
    from actfold_b200.kernels import EPI_SWIGLU, linear, tile_weight

    x = torch.randn(128, 4096, device="cuda").to(torch.bfloat16)
    w = (torch.randn(2048, 4096, device="cuda") * 0.02).to(torch.bfloat16)
    out = linear(x, tile_weight(w), ws, splits=splits, w_tiled=True, n=2048)
    ref = (x.float() @ w.float().T).to(torch.bfloat16)
    assert _rel(out, ref) <= 1e-2
    out_g = linear(x, tile_weight(w), ws, epilogue=EPI_SWIGLU, splits=splits, w_tiled=True, n=2048)
    g = ref.float().view(128, 16, 2, 64)
    gate, up = g[:, :, 0].reshape(128, 1024), g[:, :, 1].reshape(128, 1024)
    ref_g = (gate / (1 + torch.exp(-gate)) * up).to(torch.bfloat16)
    assert _rel(out_g, ref_g) <= 2e-2
    torch.cuda.synchronize()
    ws.check_status()


@pytest.mark.parametrize("m,valid", [(1024, 1024), (1536, 1100)])
def test_linear_many_tokens_wide_weights(ws, m, valid):
    """Row capacities of 512-token multiples over an output wide enough to fill the GPU with (weight tile,
    token tile) CTAs (the shape that takes 512-token tiles when they are enabled): plain store with a
    dynamic valid count (rows past it untouched) and the SwiGLU epilogue."""
    from actfold_b200.kernels import EPI_SWIGLU, linear, tile_weight

    n = 24576
    g = torch.Generator(device="cuda").manual_seed(m)
    x = torch.randn(m, 4096, device="cuda", generator=g).to(torch.bfloat16)
    w = (torch.randn(n, 4096, device="cuda", generator=g) * 0.02).to(torch.bfloat16)
    wt = tile_weight(w)
    m_dev = torch.tensor([valid], dtype=torch.int32, device="cuda")
    out = torch.full((m, n), 7.0, dtype=torch.bfloat16, device="cuda")
    linear(x, wt, ws, out=out, m_dev=m_dev, w_tiled=True, n=n)
    ref = (x.float() @ w.float().T).to(torch.bfloat16)
    assert _rel(out[:valid], ref[:valid]) <= 1e-2
    assert (out[valid:] == 7.0).all()
    out_g = linear(x, wt, ws, epilogue=EPI_SWIGLU, w_tiled=True, n=n)
    r = ref.float().view(m, n // 128, 2, 64)
    gate, up = r[:, :, 0].reshape(m, n // 2), r[:, :, 1].reshape(m, n // 2)
    ref_g = (gate / (1 + torch.exp(-gate)) * up).to(torch.bfloat16)
    assert _rel(out_g, ref_g) <= 2e-2
    torch.cuda.synchronize()
    ws.check_status()
