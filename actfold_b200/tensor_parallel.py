"""Tensor-parallel folded verification: one batch of children, the weights split over the ranks.

Child sharding (``actfold_b200.sharding``) gives each GPU its own children,
but every GPU still streams all of the weights each pass, so a fixed batch of
children cannot be verified faster than one GPU's weight-read time. Here every
rank holds a slice of each layer instead (Megatron-style):

* attention: the rows of Wq / Wk / Wv of its heads (query and key/value heads
  split evenly) and the matching columns of Wo;
* FFN: a contiguous run of the gate / up rows (in the 64-row units of the
  interleaved layout) and the matching columns of Wdown;
* LM head: a contiguous run of the vocabulary rows (in 128-row tiles, split
  as evenly as the tiles allow);
* the embedding table, the norms and the residual stream stay whole.

Every rank runs the same folded pass on its slices (``af_fold_set_tensor_parallel``):
gate decisions, compaction and norms are computed redundantly on identical
data; the O and down projections leave fp32 partial sums that are added over
the ranks before the row kernel that adds the residual, and the fresh logits'
row sums are added after the LM head so the scores are means over the whole
vocabulary. Each rank's logits are its vocabulary slice of the full [C, T, V]
logits.

The O and down sums (two per layer) go through peer memory (``sums="peer"``):
every rank maps the other ranks' exchange buffers (CUDA IPC over NVLink), a
kernel after each projection stores this rank's sum into every rank's buffer
and raises a flag there, and the row kernel that consumes the sum waits for the
flags (bounded) and adds the ranks' slices in rank order. ``sums="nccl"`` runs
an NCCL all-reduce per sum instead. Each rank sends its whole partial to every
other rank on the peer path, (N - 1) x 2 MB per sum at 128 rows, against about
2 x 2 MB for NCCL's all-reduce, so the default (``sums="auto"``) takes peer
memory on 2 ranks and NCCL on more (measured on B200: 4.59 against 5.08 ms per
pass on 2 GPUs, 5.54 against 4.63 ms on 8). The row sums after the LM head (one
per pass) use ``torch.distributed.all_reduce`` in both modes.

The parent cache is whole on every rank apart from the per-head K/V columns
and the logits, which are sliced the same way (``shard_parent_cache``).
"""

from __future__ import annotations

import dataclasses

import torch

from actfold_b200.llada import FoldPlan, LLaDABlock, LLaDAModel, ParentCache, round_capacity


def split_range(n: int, rank: int, world: int) -> tuple[int, int]:
    """[lo, hi) of ``rank``'s share of ``n`` units (the first ``n % world`` ranks take one more)."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"split_range: bad rank {rank} of {world}")
    q, r = divmod(n, world)
    lo = rank * q + min(rank, r)
    return lo, lo + q + (1 if rank < r else 0)


def _check(dims, world: int) -> None:
    if dims.n_heads % world or dims.n_kv_heads % world:
        raise ValueError(f"{world} ranks must divide the {dims.n_heads} query and {dims.n_kv_heads} key/value heads")
    if (dims.ffn // 64) % world:
        raise ValueError(f"{world} ranks must divide the {dims.ffn // 64} 64-row FFN units")


def shard_dims(dims, rank: int, world: int):
    """The layer shapes one rank computes (hidden size unchanged, vocabulary = its LM-head rows)."""
    _check(dims, world)
    v_lo, v_hi = split_range(dims.vocab // 128, rank, world)
    return dataclasses.replace(dims, n_heads=dims.n_heads // world, n_kv_heads=dims.n_kv_heads // world,
                               ffn=dims.ffn // world, vocab=(v_hi - v_lo) * 128)


def shard_block(blk: LLaDABlock, dims, rank: int, world: int) -> LLaDABlock:
    """One rank's slice of a block's tiled weights ([n/128, k/64, 128, 64]); copies, so each is contiguous."""
    _check(dims, world)
    hd = dims.head_dim // 128  # 128-row tiles per head
    h_lo, h_hi = (x * hd for x in split_range(dims.n_heads, rank, world))
    k_lo, k_hi = (x * hd for x in split_range(dims.n_kv_heads, rank, world))
    qt, kvt = dims.q_dim // 128, dims.kv_dim // 128
    qkv = torch.cat([blk.w_qkv[h_lo:h_hi], blk.w_qkv[qt + k_lo: qt + k_hi], blk.w_qkv[qt + kvt + k_lo: qt + kvt + k_hi]])
    w_o = blk.w_o[:, 2 * h_lo: 2 * h_hi]  # 64-column k-tiles of Wo: two per 128-wide head
    f_lo, f_hi = split_range(dims.ffn // 64, rank, world)  # 64-row FFN units = 128-row gate/up tiles = 64-col down tiles
    return LLaDABlock(blk.attn_norm, qkv.contiguous(), w_o.contiguous(), blk.ffn_norm,
                      blk.w_gateup[f_lo:f_hi].contiguous(), blk.w_down[:, f_lo:f_hi].contiguous(), tiled=True)


def shard_model(model: LLaDAModel, rank: int, world: int) -> LLaDAModel:
    """One rank's tensor-parallel slice of ``model`` (the embedding table is shared, not copied)."""
    d = model.dims
    v_lo, v_hi = split_range(d.vocab // 128, rank, world)
    if d.vocab % 128:
        raise ValueError("the vocabulary must be a multiple of 128 rows to shard the LM head")
    layers = [shard_block(b, d, rank, world) for b in model.layers]
    return LLaDAModel(shard_dims(d, rank, world), model.embed, layers, model.final_norm,
                      model.lm_head[v_lo:v_hi].contiguous(), max_pos=model.max_pos, lm_head_tiled=True)


def shard_parent_cache(pc: ParentCache, dims, rank: int, world: int) -> ParentCache:
    """The parent cache as one rank's pass reads it: its heads' Q/K/V columns and its vocabulary's logits."""
    _check(dims, world)
    hd = dims.head_dim
    h_lo, h_hi = (x * hd for x in split_range(dims.n_heads, rank, world))
    k_lo, k_hi = (x * hd for x in split_range(dims.n_kv_heads, rank, world))
    q, kv = dims.q_dim, dims.kv_dim
    qkv = torch.cat([pc.qkv[..., h_lo:h_hi], pc.qkv[..., q + k_lo: q + k_hi], pc.qkv[..., q + kv + k_lo: q + kv + k_hi]],
                    dim=-1).contiguous()
    v_lo, v_hi = split_range(dims.vocab // 128, rank, world)
    logits = pc.logits[:, v_lo * 128: v_hi * 128].contiguous()
    return ParentCache(pc.tokens, pc.layer_in, qkv, logits, pc.self_stable, pc.row_sums, pc.tau)


class TensorParallelVerifier:
    """Folded verification of one child batch with this rank's weight slice; call it on every rank.

    ``model`` is the whole model (its parent pass fills the parent cache on
    every rank); ``group`` is the torch.distributed group of the ranks that
    split the weights (NCCL for CUDA tensors).
    """

    def __init__(self, model: LLaDAModel, group=None, sums: str = "auto") -> None:
        import torch.distributed as dist

        if sums not in ("auto", "peer", "nccl"):
            raise ValueError(f"sums must be 'auto', 'peer' or 'nccl', not {sums!r}")
        self.dist = dist
        self.group = group
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        if sums == "auto":
            sums = "peer" if self.world == 2 else "nccl"
        self.sums = sums if self.world > 1 else "nccl"  # one rank: the sums are the identity
        self.full = model
        self.local = shard_model(model, self.rank, self.world)
        self._plans: dict = {}
        self._exchanges: list[PeerExchange] = []

    def shard_parent(self, pc: ParentCache) -> ParentCache:
        return shard_parent_cache(pc, self.full.dims, self.rank, self.world)

    def _sum(self, kind: int, layer: int, t: torch.Tensor) -> None:
        if self.world > 1:
            self.dist.all_reduce(t, op=self.dist.ReduceOp.SUM, group=self.group)

    def plan(self, pc_local: ParentCache, child_tokens: torch.Tensor, tau: float) -> FoldPlan:
        C, T = child_tokens.shape
        m_cap, child_cap = LLaDAModel.capacity_and_bound(child_tokens, pc_local, (pc_local.tau,) * self.local.dims.n_layers)
        key = (id(pc_local), C, m_cap, float(tau))
        p = self._plans.get(key)
        if p is None:
            p = FoldPlan(self.local, pc_local, C, m_cap, tau, partial_always=True)
            p.set_tensor_parallel(self.full.dims.vocab, self.full.dims.vocab, self._sum)
            if self.sums == "peer":  # every rank makes its plan in the same call, so the exchange is collective
                ex = PeerExchange(p.peer_bytes(self.world), self.local.device, self.group)
                p.set_peer_sum(self.rank, self.world, ex.ptrs)
                p.peer_exchange = ex  # this rank's buffer lives as long as the plan
                self._exchanges.append(ex)
            self._plans = {key: p}
        p.set_child_cap(child_cap)
        return p

    def verify(self, child_tokens: torch.Tensor, pc_local: ParentCache, tau: float,
               logits: torch.Tensor | None = None, scores: torch.Tensor | None = None) -> tuple[torch.Tensor, FoldPlan]:
        """(this rank's logits [C, T, V_rank], plan); ``scores`` [C] (optional) get the whole-vocabulary means."""
        child_tokens = child_tokens.to(self.local.device, torch.int64).contiguous()
        plan = self.plan(pc_local, child_tokens, tau)
        if logits is None:
            logits = torch.empty((child_tokens.shape[0], pc_local.seq, self.local.dims.vocab), dtype=torch.bfloat16,
                                 device=self.local.device)
        plan.run(child_tokens, logits, scores)
        return logits, plan

    def release(self) -> None:
        """Unmap the other ranks' exchange buffers of every plan made so far.

        Collective: every rank calls it, with no pass in flight; plans (and
        graphs captured from them) made by this verifier must not run after it.
        """
        for ex in self._exchanges:
            ex.close()
        self._exchanges = []
        self._plans = {}


# Mappings of other processes' allocations, shared by every exchange that
# lands in the same allocation (an allocation is mapped once per process):
# handle bytes -> [mapping base, users].
_IPC_MAPS: dict[bytes, list] = {}


class PeerExchange:
    """This rank's zero-filled exchange buffer and the other ranks' buffers mapped into this process (CUDA IPC).

    Collective over ``group``: the handles are all-gathered, every rank maps
    the others' buffers, and a barrier after the zero fill makes sure that no
    rank's first store reaches a buffer that is still being cleared.
    """

    def __init__(self, nbytes: int, device: torch.device, group=None) -> None:
        import ctypes as C

        import torch.distributed as dist

        from actfold_b200 import _lib
        from actfold_b200.llada import _bind_late

        self.lib = _bind_late()
        self.group = group
        rank, world = dist.get_rank(group), dist.get_world_size(group)
        self.closed = False
        self.buf = torch.zeros(nbytes + 256, dtype=torch.uint8, device=device)
        own = (self.buf.data_ptr() + 255) // 256 * 256
        handle = (C.c_char * 64)()
        off = C.c_int64()
        _lib.check(self.lib.af_ipc_export(C.c_void_p(own), handle, C.byref(off)), "af_ipc_export")
        entries: list = [None] * world
        dist.all_gather_object(entries, (bytes(handle.raw), int(off.value)), group=group)
        self.ptrs: list[int] = []
        self._bases: list[bytes] = []  # handles of the mappings this exchange uses
        err = None
        try:
            for q, (h, o) in enumerate(entries):
                if q == rank:
                    self.ptrs.append(own)
                    continue
                m = _IPC_MAPS.get(h)
                if m is None:
                    ptr, base = C.c_void_p(), C.c_void_p()
                    _lib.check(self.lib.af_ipc_import(C.create_string_buffer(h, 64), 0, C.byref(ptr), C.byref(base)),
                               "af_ipc_import")
                    m = _IPC_MAPS[h] = [int(base.value), 0]
                m[1] += 1
                self._bases.append(h)
                self.ptrs.append(m[0] + int(o))
        except Exception as exc:  # reported on every rank below, so that no rank runs with a partial mapping
            err = exc
        oks: list = [None] * world
        dist.all_gather_object(oks, err is None, group=group)
        if not all(oks):
            self._unmap()
            self.closed = True
            raise err or RuntimeError("peer-memory sums: another rank could not map the exchange buffers")
        torch.cuda.synchronize(device)
        dist.barrier(group=group)

    def close(self) -> None:
        """Unmap the other ranks' buffers (collective; this rank's own buffer stays allocated)."""
        import torch.distributed as dist

        if self.closed:
            return
        torch.cuda.synchronize(self.buf.device)
        dist.barrier(group=self.group)  # no rank still stores into a buffer that is about to be unmapped
        self._unmap()
        self.closed = True

    def _unmap(self) -> None:
        from actfold_b200 import _lib

        for h in self._bases:
            m = _IPC_MAPS[h]
            m[1] -= 1
            if m[1] == 0:
                del _IPC_MAPS[h]
                _lib.check(self.lib.af_ipc_close(m[0]), "af_ipc_close")
        self._bases = []


__all__ = ["PeerExchange", "TensorParallelVerifier", "shard_block", "shard_dims", "shard_model", "shard_parent_cache", "split_range",
           "round_capacity"]
