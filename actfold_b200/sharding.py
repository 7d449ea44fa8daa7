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
    pc.contents_changed()
    return pc


def parent_cache_checksum(pc: ParentCache) -> torch.Tensor:
    """Two int64 checksums per array of the cache (sum of its 32-bit words, and of every other word)."""
    out = []
    for t in pc.tensors():
        b = t.contiguous().view(torch.uint8).reshape(-1)
        pad = (-b.numel()) % 4
        if pad:
            b = torch.cat([b, b.new_zeros(pad)])
        w = b.view(torch.int32)
        out += [w.sum(dtype=torch.int64), w[::2].sum(dtype=torch.int64)]
    return torch.stack(out)


def check_parent_cache_agrees(pc: ParentCache, group: dist.ProcessGroup | None = None) -> None:
    """Raise ValueError on every rank unless all ranks hold bit-identical parent caches (by checksum)."""
    mine = parent_cache_checksum(pc)
    allc = [torch.empty_like(mine) for _ in range(dist.get_world_size(group))]
    dist.all_gather(allc, mine, group=group)
    if any(not torch.equal(c, allc[0]) for c in allc):
        raise ValueError("parent cache differs between ranks after the broadcast")


def gather_child_results(scores: torch.Tensor, div_count: torch.Tensor, group: dist.ProcessGroup | None = None
                         ) -> tuple[torch.Tensor, torch.Tensor]:
    """All-gather every rank's per-child scores [c_r] and divergent counts [L, c_r].

    Ranks may hold different child counts c_r (``shard_children`` gives the last
    ranks fewer children when C is not a multiple of the world size). The
    counts are gathered first; every rank then sends its rows padded to the
    largest count, so all ranks take part in equal-sized collectives, and the
    padding is dropped. A rank whose layer count differs raises ValueError on
    every rank. Returns (scores [sum c_r], div_count [L, sum c_r]) in rank
    order, i.e. in global child order for the contiguous shards of
    ``shard_children``.
    """
    world = dist.get_world_size(group)
    dev = scores.device
    # A malformed call is reported on every rank, after the first collective,
    # so no rank is left waiting in the next one.
    ok = int(scores.dim() == 1 and div_count.dim() == 2 and div_count.shape[1] == scores.shape[0])
    meta = torch.tensor([scores.shape[0], div_count.shape[0] if div_count.dim() == 2 else -1, ok],
                        dtype=torch.int64, device=dev)
    metas = [torch.empty_like(meta) for _ in range(world)]
    dist.all_gather(metas, meta, group=group)
    if not all(int(m[2]) for m in metas):
        raise ValueError(f"gather_child_results: scores [c] and div_count [L, c] disagree on some rank "
                         f"(this rank: scores {tuple(scores.shape)}, div_count {tuple(div_count.shape)})")
    counts = [int(m[0]) for m in metas]
    layers = {int(m[1]) for m in metas}
    if len(layers) != 1:
        raise ValueError(f"gather_child_results: ranks disagree on the layer count ({sorted(layers)})")
    cmax = max(counts)
    L = div_count.shape[0]
    s_pad = torch.zeros(cmax, dtype=scores.dtype, device=dev)
    s_pad[: scores.shape[0]] = scores
    d_pad = torch.zeros((L, cmax), dtype=div_count.dtype, device=dev)
    d_pad[:, : div_count.shape[1]] = div_count
    s_all = [torch.empty_like(s_pad) for _ in range(world)]
    d_all = [torch.empty_like(d_pad) for _ in range(world)]
    dist.all_gather(s_all, s_pad, group=group)
    dist.all_gather(d_all, d_pad, group=group)
    return (torch.cat([s[:c] for s, c in zip(s_all, counts)]),
            torch.cat([d[:, :c] for d, c in zip(d_all, counts)], dim=-1))
