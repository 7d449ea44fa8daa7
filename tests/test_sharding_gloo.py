"""Multi-rank host logic of folded verification, as 2 gloo ranks on CPU.

Covers the child sharding, the parent-cache broadcast (payload bit-exact on
the receiving rank, a shape disagreement raised on every rank instead of a
hang) and the gather of per-child results, in the order the GPU path uses
them over NCCL.
"""

from __future__ import annotations

import os
import socket
import traceback
from datetime import timedelta

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from actfold_b200 import workloads as W
from actfold_b200.sharding import (broadcast_parent_cache, check_parent_cache_agrees, empty_parent_cache,
                                   gather_child_results, shard_children)


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _filled_cache(dims, T, tau, seed):
    pc = empty_parent_cache(dims, T, tau, "cpu")
    g = torch.Generator().manual_seed(seed)
    pc.tokens.copy_(torch.randint(0, dims.vocab, (T,), generator=g))
    for t in (pc.layer_in, pc.qkv, pc.logits):
        t.copy_(torch.randn(t.shape, generator=g).to(torch.bfloat16))
    pc.self_stable.copy_(torch.randint(0, 2, pc.self_stable.shape, generator=g).to(torch.uint8))
    pc.row_sums.copy_(torch.randn(pc.row_sums.shape, generator=g))
    return pc


def _worker(rank, world, port, scenario, q):
    try:
        dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                                timeout=timedelta(seconds=60))
        dims, T, tau = W.LLADA_TINY, 24, 0.95
        if scenario == "broadcast":
            pc = _filled_cache(dims, T, tau, 7) if rank == 0 else empty_parent_cache(dims, T, tau, "cpu")
            broadcast_parent_cache(pc, src=0)
            check_parent_cache_agrees(pc)
            ref = _filled_cache(dims, T, tau, 7)
            for a, b in zip(pc.tensors(), ref.tensors()):
                assert a.dtype == b.dtype and a.shape == b.shape
                assert torch.equal(a.view(torch.int16) if a.dtype == torch.bfloat16 else a,
                                   b.view(torch.int16) if b.dtype == torch.bfloat16 else b)
            q.put((rank, "ok"))
        elif scenario == "mismatch":
            pc = _filled_cache(dims, T, tau, 7) if rank == 0 else empty_parent_cache(dims, T + 1, tau, "cpu")
            try:
                broadcast_parent_cache(pc, src=0)
                q.put((rank, "no error"))
            except ValueError as e:
                q.put((rank, "raised" if "differ between ranks" in str(e) else f"wrong message {e}"))
        elif scenario == "gather":
            C, L = 8, dims.n_layers
            start, count = shard_children(C, rank, world)
            scores = torch.arange(start, start + count, dtype=torch.float32)
            div = torch.stack([torch.arange(start, start + count, dtype=torch.int32) + 100 * l for l in range(L)])
            s_all, d_all = gather_child_results(scores, div)
            assert torch.equal(s_all, torch.arange(C, dtype=torch.float32))
            assert torch.equal(d_all, torch.stack([torch.arange(C, dtype=torch.int32) + 100 * l for l in range(L)]))
            q.put((rank, "ok"))
        elif scenario == "diverged":
            pc = _filled_cache(dims, T, tau, 7 + rank)  # different caches on the two ranks
            try:
                check_parent_cache_agrees(pc)
                q.put((rank, "no error"))
            except ValueError:
                q.put((rank, "raised"))
        elif scenario == "gather_bad":
            L = dims.n_layers
            scores = torch.zeros(4)
            div = torch.zeros((L, 4 if rank == 0 else 3), dtype=torch.int32)
            try:
                gather_child_results(scores, div)
                q.put((rank, "no error"))
            except ValueError as e:
                q.put((rank, "raised" if "disagree" in str(e) else f"wrong message {e}"))
        dist.barrier()
        dist.destroy_process_group()
    except Exception:  # reported to the parent, which fails the test
        q.put((rank, traceback.format_exc()))


def _run(scenario, world=2):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, scenario, q)) for r in range(world)]
    for p in procs:
        p.start()
    out = {}
    for _ in range(world):
        rank, msg = q.get(timeout=120)
        out[rank] = msg
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    return out


def test_shard_children_cover_every_child_once():
    for n in (0, 1, 7, 8, 64, 127, 128):
        for world in (1, 2, 3, 4, 8):
            seen = []
            for r in range(world):
                start, count = shard_children(n, r, world)
                assert count >= 0 and count <= -(-n // world)
                seen.extend(range(start, start + count))
            assert seen == list(range(n))
    with pytest.raises(ValueError):
        shard_children(8, 2, 2)


def test_parent_cache_broadcast_is_bit_exact():
    out = _run("broadcast")
    assert out == {0: "ok", 1: "ok"}, out


def test_parent_cache_shape_mismatch_raises_on_every_rank():
    out = _run("mismatch")
    assert out == {0: "raised", 1: "raised"}, out


def test_gather_child_results_in_global_order():
    out = _run("gather")
    assert out == {0: "ok", 1: "ok"}, out


def test_gather_child_results_unequal_shards():
    # 8 children on 3 ranks: shards of 3, 3 and 2 children.
    out = _run("gather", world=3)
    assert out == {0: "ok", 1: "ok", 2: "ok"}, out


def test_diverged_parent_caches_are_detected_on_every_rank():
    out = _run("diverged")
    assert out == {0: "raised", 1: "raised"}, out


def test_gather_child_results_bad_shapes_raise_on_every_rank():
    out = _run("gather_bad")
    assert out == {0: "raised", 1: "raised"}, out
