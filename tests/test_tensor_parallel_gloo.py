"""Tensor-parallel weight slices, as 2 gloo ranks on CPU (host logic; no kernel runs here).

Each rank slices the tiled weights of a tiny LLaDA-shaped model with
``actfold_b200.tensor_parallel`` and computes one block and the LM head from
its slices in fp32 torch, adding its partial O, down and logit-row-sum
results over the ranks with an all-reduce, exactly where the tensor-parallel
pass does. The sum must equal the whole block / LM head computed from the
unsliced weights (fp32 arithmetic, so only summation order differs: relative
error <= 1e-5), and the slices must be the declared rows and columns.
"""

from __future__ import annotations

import dataclasses
import socket
import traceback
from datetime import timedelta

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from actfold_b200 import workloads as W

DIMS = dataclasses.replace(W.LLADA_TINY, n_heads=4, n_kv_heads=2, ffn=512, vocab=640)


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _untile(t: torch.Tensor) -> torch.Tensor:
    nb, kb, r, c = t.shape
    return t.permute(0, 2, 1, 3).reshape(nb * r, kb * c)


def _rope(x, cos, sin):
    h = x.shape[-1] // 2
    c, s = cos[: x.shape[1]][None, :, None, :], sin[: x.shape[1]][None, :, None, :]
    return torch.cat([x[..., :h] * c - x[..., h:] * s, x[..., h:] * c + x[..., :h] * s], dim=-1)


def _rms(x, w, eps):
    return x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + eps) * w


def _block_parts(blk, d, x, cos, sin, reduce):
    """fp32 block from (possibly sliced) tiled weights; ``reduce`` sums a partial over the ranks."""
    q_dim, kv_dim = d.n_heads * d.head_dim, d.n_kv_heads * d.head_dim
    wqkv = _untile(blk.w_qkv).float()
    a = _rms(x, blk.attn_norm.float(), d.rms_eps)
    qkv = a @ wqkv.T
    B, T = x.shape[:2]
    q = _rope(qkv[..., :q_dim].view(B, T, d.n_heads, d.head_dim), cos, sin)
    k = _rope(qkv[..., q_dim:q_dim + kv_dim].view(B, T, d.n_kv_heads, d.head_dim), cos, sin)
    v = qkv[..., q_dim + kv_dim:].view(B, T, d.n_kv_heads, d.head_dim)
    g = d.n_heads // d.n_kv_heads
    k, v = k.repeat_interleave(g, dim=2), v.repeat_interleave(g, dim=2)
    p = torch.softmax(torch.einsum("bqhd,bkhd->bhqk", q, k) / d.head_dim ** 0.5, dim=-1)
    o = torch.einsum("bhqk,bkhd->bqhd", p, v).reshape(B, T, q_dim)
    h = x + reduce(o @ _untile(blk.w_o).float().T)
    b = _rms(h, blk.ffn_norm.float(), d.rms_eps)
    gu = (b @ _untile(blk.w_gateup).float().T).view(B, T, -1, 2, 64)
    f = (torch.nn.functional.silu(gu[..., 0, :]) * gu[..., 1, :]).reshape(B, T, -1)
    return h + reduce(f @ _untile(blk.w_down).float().T)


def _worker(rank, world, port, q):
    try:
        from actfold_b200.llada import LLaDAModel, rope_tables
        from actfold_b200.tensor_parallel import shard_model, shard_parent_cache, split_range

        dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                                timeout=timedelta(seconds=60))
        w = W.llada_weights_numpy(DIMS, seed=3)
        full = LLaDAModel.from_numpy(DIMS, w, device="cpu", max_pos=16)
        loc = shard_model(full, rank, world)
        d, ld = full.dims, loc.dims
        # The slices are the declared rows / columns of the whole matrices.
        hq = split_range(d.n_heads, rank, world)
        hk = split_range(d.n_kv_heads, rank, world)
        f0, f1 = split_range(d.ffn // 64, rank, world)
        full_qkv = _untile(full.layers[0].w_qkv)
        q_rows = full_qkv[hq[0] * 128: hq[1] * 128]
        k_rows = full_qkv[d.q_dim + hk[0] * 128: d.q_dim + hk[1] * 128]
        v_rows = full_qkv[d.q_dim + d.kv_dim + hk[0] * 128: d.q_dim + d.kv_dim + hk[1] * 128]
        assert torch.equal(_untile(loc.layers[0].w_qkv), torch.cat([q_rows, k_rows, v_rows]))
        assert torch.equal(_untile(loc.layers[0].w_o), _untile(full.layers[0].w_o)[:, hq[0] * 128: hq[1] * 128])
        assert torch.equal(_untile(loc.layers[0].w_gateup), _untile(full.layers[0].w_gateup)[f0 * 128: f1 * 128])
        assert torch.equal(_untile(loc.layers[0].w_down), _untile(full.layers[0].w_down)[:, f0 * 64: f1 * 64])
        v_lo, v_hi = split_range(d.vocab // 128, rank, world)
        assert ld.vocab == (v_hi - v_lo) * 128 and loc.embed.data_ptr() == full.embed.data_ptr()

        def allreduce(t):
            t = t.contiguous()
            dist.all_reduce(t)
            return t

        cos, sin = rope_tables(16, d.head_dim, d.rope_theta, "cpu")
        x = torch.randn(2, 16, d.hidden, generator=torch.Generator().manual_seed(5))
        with torch.no_grad():
            want = _block_parts(full.layers[1], d, x, cos, sin, lambda t: t)
            got = _block_parts(loc.layers[1], ld, x, cos, sin, allreduce)
            assert float((got - want).abs().max() / want.abs().max()) <= 1e-5
            # LM head: this rank's vocabulary rows, and the row sums added over the ranks.
            v0, v1 = split_range(d.vocab // 128, rank, world)
            lg_full = x @ _untile(full.lm_head).float().T
            lg_loc = x @ _untile(loc.lm_head).float().T
            assert torch.allclose(lg_loc, lg_full[..., v0 * 128: v1 * 128], rtol=1e-5, atol=1e-6)
            rs = allreduce(lg_loc.sum(-1))
            assert torch.allclose(rs, lg_full.sum(-1), rtol=1e-4, atol=1e-4)
        # Parent cache slice: this rank's heads' Q/K/V columns and vocabulary columns.
        from actfold_b200.sharding import empty_parent_cache

        pc = empty_parent_cache(d, 8, 0.95, "cpu")
        pc.qkv.copy_(torch.arange(pc.qkv.numel(), dtype=torch.float32).view(pc.qkv.shape).to(pc.qkv.dtype))
        pc.logits.copy_(torch.arange(pc.logits.numel(), dtype=torch.float32).view(pc.logits.shape).to(pc.logits.dtype))
        sp = shard_parent_cache(pc, d, rank, world)
        assert sp.qkv.shape[-1] == ld.q_dim + 2 * ld.kv_dim and sp.logits.shape[-1] == ld.vocab
        assert torch.equal(sp.qkv[..., : ld.q_dim], pc.qkv[..., hq[0] * 128: hq[1] * 128])
        assert sp.layer_in is pc.layer_in and sp.self_stable is pc.self_stable
        q.put((rank, "ok"))
        dist.barrier()
        dist.destroy_process_group()
    except Exception:  # reported to the parent, which fails the test
        q.put((rank, traceback.format_exc()))


def test_tensor_parallel_slices_reproduce_the_whole_block():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    out = {}
    for _ in range(2):
        rank, msg = q.get(timeout=180)
        out[rank] = msg
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    assert out == {0: "ok", 1: "ok"}, out


def test_split_range_and_shape_checks():
    from actfold_b200.tensor_parallel import shard_dims, split_range

    assert [split_range(10, r, 3) for r in range(3)] == [(0, 4), (4, 7), (7, 10)]
    assert split_range(988, 7, 8) == (865, 988)
    assert shard_dims(W.LLADA_8B, 1, 8).vocab in (123 * 128, 124 * 128)
    with pytest.raises(ValueError):
        shard_dims(W.DREAM_7B, 0, 8)  # 4 key/value heads cannot be split 8 ways
