"""The tensor-parallel folded pass on 2 to 8 GPUs against the one-GPU pass (skipped with fewer than 2).

The NCCL ranks each hold a slice of the weights (actfold_b200.tensor_parallel)
and verify the same children; rank r's logits are its vocabulary slice. Each
rank also runs the one-GPU pass with the whole model and compares:

* stable masks equal (the cross-rank fp32 sums add the partial products in
  another order, which can only move rows on the gate boundary: at most one
  mismatch per 10,000 rows is allowed, none is expected with these edits);
* its logits slice: relative error <= 2e-2 of the scale, cosine >= 0.999;
* scores (means over the whole vocabulary) within 2e-2 of the logits' scale.

Shapes: the tiny LLaDA block on 2 GPUs, and 2 layers of the LLaDA-8B shapes
(8 children x 1024 tokens, d = 16) on every GPU of the box (2, 4 or 8). Both ways of adding the O / down sums over the ranks
run: through peer memory (the default) and through NCCL all-reduces. The ranks run as child processes (NCCL_NVLS_ENABLE=0)
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


def _worker(rank, world, port, name, sums, q):
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
        tp = TensorParallelVerifier(model, sums=sums)
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
        tp.release()
        del plan, tp
        dist.barrier()
        dist.destroy_process_group()
    except Exception:
        q.put((rank, traceback.format_exc()))


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs 2 GPUs")
@pytest.mark.parametrize("sums", ["peer", "nccl"])
@pytest.mark.parametrize("name", ["tiny", "llada8b_2layers"])
def test_tensor_parallel_pass_matches_one_gpu(name, sums):
    import torch.multiprocessing as mp

    os.environ["NCCL_NVLS_ENABLE"] = "0"
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    # The tiny model has 2 heads; the LLaDA-8B layers split over every GPU of the box (2, 4 or 8).
    world = 2 if name == "tiny" else max(w for w in (2, 4, 8) if w <= torch.cuda.device_count())
    procs = [ctx.Process(target=_worker, args=(r, world, port, name, sums, q)) for r in range(world)]
    for p in procs:
        p.start()
    out = {}
    for _ in range(world):
        rank, msg = q.get(timeout=600)
        out[rank] = msg
    for p in procs:
        p.join(timeout=120)
        if p.is_alive():
            p.kill()
    assert out == {r: "ok" for r in range(world)}, out


@pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a GPU")
@pytest.mark.parametrize("name", ["tiny", "llada8b_2layers"])
def test_peer_sum_one_rank_matches_plain_pass(name):
    """The peer-memory sum kernels on one rank (its own exchange buffer only): the push kernel, the launch
    counters, the flags and the consumers' bounded waits run as on N ranks. One rank's slice is the sum of
    its k-splits in split order, as the hook path's local split sum is, so logits, masks and scores are
    bit-identical to a one-rank tensor-parallel plan whose hook sums nothing, over eager runs and graph
    replays (the flags keep counting across passes); scores within 1e-5 (their row sums are added by
    atomics)."""
    from actfold_b200.llada import FoldPlan, LLaDAModel

    dev = torch.device("cuda", 0)
    dims, parent, children, T = _case(name)
    if name == "tiny":
        model = LLaDAModel.from_numpy(dims, W.llada_weights_numpy(dims, seed=7), device=dev, max_pos=T)
    else:
        model = LLaDAModel.random(dims, seed=1234, device=dev, max_pos=T)
    pc = model.parent_pass(torch.from_numpy(parent).to(dev), tau=0.95)
    ct = torch.from_numpy(children).to(dev)
    m_cap, child_cap = LLaDAModel.capacity_and_bound(ct, pc, (pc.tau,) * dims.n_layers)

    def one_rank_plan():
        p = FoldPlan(model, pc, ct.shape[0], m_cap, 0.95, partial_always=True)
        p.set_tensor_parallel(dims.vocab, dims.vocab, lambda kind, layer, t: None)
        p.set_child_cap(child_cap)
        return p

    ref_plan = one_rank_plan()
    ref_scores = torch.empty(children.shape[0], dtype=torch.float32, device=dev)
    ref_logits = torch.empty((ct.shape[0], T, dims.vocab), dtype=torch.bfloat16, device=dev)
    ref_plan.run(ct, ref_logits, ref_scores)
    ref_masks = ref_plan.stable_masks()

    plan = one_rank_plan()
    buf = torch.zeros(plan.peer_bytes(1) + 256, dtype=torch.uint8, device=dev)
    plan.set_peer_sum(0, 1, [(buf.data_ptr() + 255) // 256 * 256])
    logits = torch.empty_like(ref_logits)
    scores = torch.empty_like(ref_scores)
    for _ in range(2):
        logits.fill_(0)
        plan.run(ct, logits, scores)
        torch.cuda.synchronize()
        plan.check_status()
        assert torch.equal(logits, ref_logits)
        assert torch.equal(plan.stable_masks(), ref_masks)
        torch.testing.assert_close(scores, ref_scores, rtol=1e-5, atol=0)  # row sums are added by atomics
    graph = plan.capture(ct, logits, scores)
    for _ in range(3):
        logits.fill_(0)
        graph.replay()
    torch.cuda.synchronize()
    plan.check_status()
    assert torch.equal(logits, ref_logits)
    torch.testing.assert_close(scores, ref_scores, rtol=1e-5, atol=0)
