"""Child sharding and parent-cache exchange for folded verification on several GPUs.

One process per GPU. The children of one parent are independent units of
work, so they are split into contiguous blocks, one per rank, and no data-path
collective is needed. The one exchange is the parent's per-layer activation
cache: one rank runs the dense parent pass and broadcasts the cache, and every
rank then verifies its own children against it. Per-child results can be
gathered afterwards.

The same calls work over NCCL (CUDA tensors) and gloo (CPU tensors, used by
the tests). Every rank takes the same collective steps in the same order, on
the error paths too: a shape disagreement is detected collectively and raised
on every rank rather than leaving some ranks waiting in a broadcast.
"""

from __future__ import annotations

import torch
import torch.distributed as dist

from actfold_b200.llada import ParentCache
from actfold_b200.workloads import ModelDims

_HEADER = 8  # T, L+1, H, qkv width, V, dtype codes (layer_in, logits), tau bits


def shard_children(n_children: int, rank: int, world: int) -> tuple[int, int]:
    """(first child, count) of `rank`'s contiguous block of ceil(n / world) children."""
    if n_children < 0 or world < 1 or not 0 <= rank < world:
        raise ValueError(f"shard_children: bad arguments n={n_children} rank={rank} world={world}")
    per = -(-n_children // world)
    start = min(rank * per, n_children)
    return start, min(per, n_children - start)


def empty_parent_cache(dims: ModelDims, seq: int, tau: float, device: torch.device | str) -> ParentCache:
    """Receive buffers of a parent cache for `dims` and `seq` tokens."""
    L, H = dims.n_layers, dims.hidden
    return ParentCache(
        torch.empty(seq, dtype=torch.int64, device=device),
        torch.empty((L + 1, seq, H), dtype=torch.bfloat16, device=device),
        torch.empty((L, seq, dims.q_dim + 2 * dims.kv_dim), dtype=torch.bfloat16, device=device),
        torch.empty((seq, dims.vocab), dtype=torch.bfloat16, device=device),
        torch.empty((L, seq), dtype=torch.uint8, device=device),
        torch.empty((seq,), dtype=torch.float32, device=device),
        float(tau),
    )


def _header(pc: ParentCache) -> torch.Tensor:
    tau_bits = int(torch.tensor([pc.tau], dtype=torch.float32).view(torch.int32).item())
    return torch.tensor(
        [pc.seq, pc.layer_in.shape[0], pc.layer_in.shape[2], pc.qkv.shape[2], pc.logits.shape[1],
         int(pc.layer_in.dtype == torch.bfloat16), int(pc.logits.dtype == torch.bfloat16), tau_bits],
        dtype=torch.int64,
    )


def broadcast_parent_cache(pc: ParentCache, src: int = 0, group: dist.ProcessGroup | None = None) -> ParentCache:
    """Broadcast `pc` from rank `src` into every rank's `pc` buffers (in place).

    A header with the cache's shapes, dtypes and tau goes first; if any rank's
    buffers disagree with it, every rank raises ValueError before the payload
    is sent.
    """
    dev = pc.tokens.device
    hdr = _header(pc).to(dev)
    mine = hdr.clone()
    dist.broadcast(hdr, src=src, group=group)
    ok = torch.tensor([int(torch.equal(hdr, mine))], dtype=torch.int32, device=dev)
    dist.all_reduce(ok, op=dist.ReduceOp.MIN, group=group)
    if int(ok.item()) != 1:
        raise ValueError(f"broadcast_parent_cache: parent cache shapes differ between ranks (source header {hdr.tolist()}, "
                         f"this rank {mine.tolist()})")
    for t in pc.tensors():
        # Every tensor moves as its bytes (uint8 is supported by every backend).
        dist.broadcast(t.view(torch.uint8), src=src, group=group)
    return pc


def gather_child_results(scores: torch.Tensor, div_count: torch.Tensor, group: dist.ProcessGroup | None = None
                         ) -> tuple[torch.Tensor, torch.Tensor]:
    """All-gather every rank's per-child scores [c] and divergent counts [L, c] (equal c on all ranks).

    Returns (scores [world * c], div_count [L, world * c]) in rank order, i.e. in
    global child order for the contiguous shards of `shard_children`.
    """
    world = dist.get_world_size(group)
    s_all = [torch.empty_like(scores) for _ in range(world)]
    d_all = [torch.empty_like(div_count) for _ in range(world)]
    dist.all_gather(s_all, scores.contiguous(), group=group)
    dist.all_gather(d_all, div_count.contiguous(), group=group)
    return torch.cat(s_all), torch.cat(d_all, dim=-1)
