"""The tensor-parallel folded pass on 2 GPUs against the one-GPU pass (skipped with fewer GPUs).

Two NCCL ranks each hold a slice of the weights (actfold_b200.tensor_parallel)
and verify the same children; rank r's logits are its vocabulary slice. Each
rank also runs the one-GPU pass with the whole model and compares:

* stable masks equal (the cross-rank fp32 sums add the partial products in
  another order, which can only move rows on the gate boundary: at most one
  mismatch per 10,000 rows is allowed, none is expected with these edits);
* its logits slice: relative error <= 2e-2 of the scale, cosine >= 0.999;
* scores (means over the whole vocabulary) within 2e-2 of the logits' scale.

Shapes: the tiny LLaDA block, and 2 layers of the LLaDA-8B shapes (8 children
x 1024 tokens, d = 16). The ranks run as child processes (NCCL_NVLS_ENABLE=0)
with a 120 s process-group timeout.
"""

from __future__ import annotations

import dataclasses
import math
import os
import socket
import traceback
from datetime import timedelta

import pytest
import torch

from actfold_b200 import workloads as W

pytestmark = pytest.mark.gpu


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _case(name):
    if name == "tiny":
        dims = W.LLADA_TINY
        parent, children = W.llada_tokens(64, 16, 0.5, 4, 4, dims.mask_id, 42)
        return dims, parent, children, 64
    dims = dataclasses.replace(W.LLADA_8B, n_layers=2)
    parent, _ = W.llada_tokens(1024, 256, 0.5, 1, 1, dims.mask_id, seed=42)
    return dims, parent, W.llada_children(parent, 8, 16, dims.mask_id, seed=1000), 1024


def _worker(rank, world, port, name, q):
    try:
        import torch.distributed as dist

        from actfold_b200.llada import LLaDAModel
        from actfold_b200.tensor_parallel import TensorParallelVerifier, split_range

        torch.cuda.set_device(rank)
        dev = torch.device("cuda", rank)
        dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                                timeout=timedelta(seconds=120), device_id=dev)
        dims, parent, children, T = _case(name)
        if name == "tiny":
            model = LLaDAModel.from_numpy(dims, W.llada_weights_numpy(dims, seed=7), device=dev, max_pos=T)
        else:
            model = LLaDAModel.random(dims, seed=1234, device=dev, max_pos=T)
        pc = model.parent_pass(torch.from_numpy(parent).to(dev), tau=0.95)
        ct = torch.from_numpy(children).to(dev)
        ref_scores = torch.empty(children.shape[0], dtype=torch.float32, device=dev)
        ref_logits, ref_plan = model.verify(ct, pc, 0.95, scores=ref_scores)
        ref_masks = ref_plan.stable_masks()
        tp = TensorParallelVerifier(model)
        scores = torch.empty_like(ref_scores)
        logits, plan = tp.verify(ct, tp.shard_parent(pc), 0.95, scores=scores)
        torch.cuda.synchronize()
        plan.check_status()
        masks = plan.stable_masks()
        v0, v1 = split_range(dims.vocab // 128, rank, world)
        want = ref_logits[..., v0 * 128: v1 * 128].double()
        got = logits.double()
        rel = float((got - want).abs().max() / want.abs().max())
        cos = float((got * want).sum() / math.sqrt(float((got * got).sum()) * float((want * want).sum())))
        mism = int((masks != ref_masks).sum())
        scale = float(ref_logits.float().abs().max())
        sdiff = float((scores - ref_scores).abs().max())
        ok = rel <= 2e-2 and cos >= 0.999 and mism <= max(1, masks.numel() // 10000) and sdiff <= 2e-2 * scale
        q.put((rank, "ok" if ok else f"rel {rel} cos {cos} mask mismatches {mism} score diff {sdiff}"))
        del plan, tp
        dist.barrier()
        dist.destroy_process_group()
    except Exception:
        q.put((rank, traceback.format_exc()))


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs 2 GPUs")
@pytest.mark.parametrize("name", ["tiny", "llada8b_2layers"])
def test_tensor_parallel_pass_matches_one_gpu(name):
    import torch.multiprocessing as mp

    os.environ["NCCL_NVLS_ENABLE"] = "0"
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, name, q)) for r in range(2)]
    for p in procs:
        p.start()
    out = {}
    for _ in range(2):
        rank, msg = q.get(timeout=600)
        out[rank] = msg
    for p in procs:
        p.join(timeout=120)
        if p.is_alive():
            p.kill()
    assert out == {0: "ok", 1: "ok"}, out
