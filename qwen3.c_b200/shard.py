"""Multi-GPU sharding of the attention block (host side).

One process per GPU; torch.distributed carries the single exchange each
sharded step needs (NCCL over NVLink on GPUs, gloo in the CPU tests).  The
reference has no multi-GPU path: this module and the two collectives it
issues are new, and all arithmetic stays in the library's kernels.

* Sequence shards (long-context decode).  Rank r holds cache positions
  ``seq_chunk(L, world, r)`` of the sequence, stored compactly from row 0 of
  its own context.  Two exchanges are available:

  - ``mode="peer"``: one launch per layer (``q3a_attn_seqshard``) whose
    kernel stores each KV head's (o, lse) straight into every rank's receive
    buffer over NVLink (buffers mapped once with ``q3a_peer_export`` /
    ``q3a_peer_open``; the handles travel through one all_gather_object) and
    merges once all ranks' rows have arrived;
  - ``mode="nccl"``: each rank writes its chunk's normalised output and
    log2-sum-exp into one packed row ``[n_heads*hd | n_heads]``
    (``q3a_attn_partial``); one NCCL all-gather gives every rank all rows, and
    ``q3a_lse_combine_packed`` merges them into the full xb on every rank.
* KV-head shards (batched decode, prefill).  Rank r holds KV heads
  ``kv_heads(n_kv, world, r)`` and their query heads; attention needs no
  exchange, and one all-gather of the head slices rebuilds xb (or a prefill
  output): ``HeadSliceGather`` through NCCL, or ``PeerHeadGather``, one
  ``q3a_gather_cols`` launch that stores each rank's columns straight into
  every rank's registered buffer over NVLink.
"""
from __future__ import annotations

from typing import Callable, Optional


def seq_chunk(total: int, world: int, rank: int) -> tuple[int, int]:
    """Positions [t0, t1) of a ``total``-long sequence held by ``rank``:
    contiguous, in rank order, sizes differing by at most one."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} of world {world}")
    if total < 0:
        raise ValueError(f"length {total}")
    return rank * total // world, (rank + 1) * total // world


def kv_heads(n_kv: int, world: int, rank: int) -> tuple[int, int]:
    """(first KV head, count) held by ``rank``; the heads split evenly."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} of world {world}")
    if n_kv % world != 0:
        raise ValueError(f"{n_kv} KV heads do not split over {world} ranks")
    per = n_kv // world
    return rank * per, per


def packed_width(n_heads: int, hd: int) -> int:
    """Floats per rank in the all-gathered (o, lse) row."""
    return n_heads * hd + n_heads


def _all_gather(dist, out, inp, group):
    """All-gather of equal contiguous rows into ``out`` [world, ...]."""
    if dist.get_backend(group) == "nccl":
        dist.all_gather_into_tensor(out, inp, group=group)
    else:  # gloo: list form, into views of the same buffer
        dist.all_gather(list(out.unbind(0)), inp, group=group)


def open_peer_set(ctx, *, world: int, rank: int, group=None) -> None:
    """Exports this rank's peer buffer and maps every rank's
    (``q3a_peer_export`` / ``q3a_peer_open``; the IPC handles travel through
    one ``all_gather_object``).  Sequence shards exchange their (o, lse)
    words in it; KV-head shards their partial wo products
    (``q3a_wo_residual`` / ``q3a_attn_sublayer``)."""
    import torch.distributed as dist
    handle = ctx.peer_export(world)
    handles = [handle]
    if world > 1:
        handles = [None] * world
        dist.all_gather_object(handles, handle, group=group)
    ctx.peer_open(rank, world, handles)


class SeqShardDecode:
    """One decode step of a sequence sharded over the ranks of ``group``.

    ``partial(o, lse, q, seq, layer, t0, t1)`` and ``combine(xb, parts, n)``
    default to the context's ``attn_partial`` / ``lse_combine_packed``; the
    CPU tests pass the oracle's arithmetic instead to check this module's
    chunking, packing and gather order on gloo ranks.
    """

    def __init__(self, torch, ctx=None, *, world: int, rank: int, group=None,
                 n_heads: int = 32, hd: int = 128, device=None, mode: str = "nccl",
                 partial: Optional[Callable] = None, combine: Optional[Callable] = None):
        import torch.distributed as dist
        self.dist = dist
        self.world, self.rank, self.group = world, rank, group
        if mode not in ("nccl", "peer"):
            raise ValueError(f"mode {mode!r}")
        self.mode = mode
        self.ctx = ctx
        if mode == "peer":
            open_peer_set(ctx, world=world, rank=rank, group=group)
        self.nq = n_heads * hd
        self.width = packed_width(n_heads, hd)
        self.send = torch.zeros(self.width, dtype=torch.float32, device=device)
        self.recv = torch.zeros(world, self.width, dtype=torch.float32, device=device)
        self.partial = partial if partial is not None else ctx.attn_partial
        self.combine = combine if combine is not None else ctx.lse_combine_packed

    def __call__(self, xb, q, seq: int, layer: int, n_local: int):
        """xb <- attention of q over all ranks' chunks; this rank's chunk is
        rows [0, n_local) of its own cache (slot ``seq``, layer ``layer``)."""
        if self.mode == "peer":
            self.ctx.attn_seqshard(xb, q, seq, layer, n_local)
            return
        if self.world == 1:  # one shard: no exchange
            self.partial(self.recv[0, : self.nq], self.recv[0, self.nq:], q, seq, layer, 0, n_local)
        else:
            self.partial(self.send[: self.nq], self.send[self.nq:], q, seq, layer, 0, n_local)
            _all_gather(self.dist, self.recv, self.send, self.group)
        self.combine(xb, self.recv, self.world)


class HeadSliceGather:
    """All-gather of KV-head-sharded xb slices: rank r computed the columns of
    its query heads, ``xb[:, c0:c1]``; afterwards every rank holds all of xb."""

    def __init__(self, torch, *, world: int, rank: int, rows: int, n_heads: int = 32,
                 hd: int = 128, group=None, device=None, dtype=None):
        import torch.distributed as dist
        self.dist = dist
        self.world, self.rank, self.group = world, rank, group
        if n_heads % world != 0:
            raise ValueError(f"{n_heads} query heads do not split over {world} ranks")
        self.w = n_heads // world * hd
        dtype = dtype if dtype is not None else torch.float32
        self.send = torch.zeros(rows, self.w, dtype=dtype, device=device)
        self.recv = torch.zeros(world, rows, self.w, dtype=dtype, device=device)

    def __call__(self, xb):
        """xb [rows, n_heads*hd], this rank's slice filled, others rebuilt."""
        c0 = self.rank * self.w
        self.send.copy_(xb[:, c0:c0 + self.w])
        _all_gather(self.dist, self.recv, self.send, self.group)
        for r in range(self.world):
            if r != self.rank:
                xb[:, r * self.w:(r + 1) * self.w].copy_(self.recv[r])


class PeerHeadGather:
    """All-gather of KV-head-sharded column slices over peer memory: ``buf``
    (a device tensor, registered once on every rank) holds row-major
    matrices [rows, n_heads*hd]; rank r computed the columns of its query
    heads; ``gather(t)`` for a matrix view ``t`` inside ``buf`` gives every
    rank all columns of ``t`` (one ``q3a_gather_cols`` launch)."""

    def __init__(self, torch, ctx, *, world: int, rank: int, buf, group=None, n_heads: int = 32,
                 hd: int = 128):
        import torch.distributed as dist
        if n_heads % world != 0:
            raise ValueError(f"{n_heads} query heads do not split over {world} ranks")
        self.ctx, self.world, self.rank = ctx, world, rank
        self.buf = buf
        handle = ctx.peer_register(buf, buf.numel() * buf.element_size())
        handles = [handle]
        if world > 1:
            handles = [None] * world
            dist.all_gather_object(handles, handle, group=group)
        ctx.peer_register_open(rank, world, handles)
        self.w = n_heads // world * hd

    def __call__(self, t):
        """t: a [rows, n_heads*hd] view of ``buf`` with contiguous rows."""
        es = t.element_size()
        off = t.data_ptr() - self.buf.data_ptr()
        self.ctx.gather_cols(off, t.shape[0], t.stride(0) * es, self.rank * self.w * es, self.w * es)
