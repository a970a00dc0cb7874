"""Host logic of the multi-GPU sharding (qwen3.c_b200/shard.py) on gloo ranks.

Two CPU processes exchange through torch.distributed (gloo, 127.0.0.1) with
the oracle's arithmetic standing in for the kernels, so the chunk bounds,
the packed (o, lse) row, the gather order and the head-slice reassembly are
checked without a GPU.  Parity: the sharded results equal the oracle's
single-process attention (the reference's own loop, cpu/main.c:1331-1353)
to fp32 rounding.
"""
import os
import socket
import sys

import numpy as np
import pytest

import q3a_oracle as orc
import shard
from shapes import HD, HKV, HQ, KV_DIM, KV_MUL, normwise

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_seq_chunk_covers_the_sequence_in_order():
    for total in (0, 1, 7, 1000, 131072):
        for world in (1, 2, 3, 4, 8):
            cuts = [shard.seq_chunk(total, world, r) for r in range(world)]
            assert cuts[0][0] == 0 and cuts[-1][1] == total
            for (a0, a1), (b0, b1) in zip(cuts, cuts[1:]):
                assert a1 == b0
            sizes = [b - a for a, b in cuts]
            assert max(sizes) - min(sizes) <= 1
    with pytest.raises(ValueError):
        shard.seq_chunk(10, 2, 2)


def test_kv_heads_split_evenly():
    assert [shard.kv_heads(8, 4, r) for r in range(4)] == [(0, 2), (2, 2), (4, 2), (6, 2)]
    assert shard.kv_heads(8, 1, 0) == (0, 8)
    with pytest.raises(ValueError):
        shard.kv_heads(8, 3, 0)
    assert shard.packed_width(32, 128) == 32 * 129


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _worker(rank, world, port, kind, q):
    try:
        for p in (os.path.join(ROOT, "oracle"), os.path.join(ROOT, "qwen3.c_b200"),
                  os.path.join(ROOT, "tests")):
            sys.path.insert(0, p)
        import torch
        import torch.distributed as dist
        import q3a_oracle as orc
        import shard
        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        dist.init_process_group("gloo", rank=rank, world_size=world)
        if kind == "seq":
            err = _seq_case(torch, orc, shard, rank, world)
        elif kind == "peer_gather":
            err = _peer_gather_case(torch, shard, rank, world)
        else:
            err = _head_case(torch, orc, shard, rank, world)
        dist.barrier()
        dist.destroy_process_group()
        q.put((rank, err, None))
    except Exception as e:  # reported to the parent, which fails the test
        q.put((rank, None, repr(e)))


def _seq_case(torch, orc, shard, rank, world):
    L = 1000
    kc = orc.randn(L * KV_DIM, 5, 1)  # the whole sequence, as every rank can regenerate it
    vc = orc.randn(L * KV_DIM, 5, 2)
    q = orc.randn(HQ * HD, 5, 3)
    t0, t1 = shard.seq_chunk(L, world, rank)

    def partial(o, lse, qv, seq, layer, a, b):
        # this rank's rows [a, b) are global positions [t0 + a, t0 + b)
        ro, rl = orc.attn_partial(qv.numpy(), kc, vc, 0, t0 + a, t0 + b, HQ, KV_MUL, HD, KV_DIM)
        o.copy_(torch.from_numpy(ro))
        lse.copy_(torch.from_numpy(rl))

    def combine(xb, parts, n):
        p = parts.numpy()
        out, _ = orc.lse_merge(p[:, :HQ * HD].copy(), p[:, HQ * HD:].copy(), HQ, HD)
        xb.copy_(torch.from_numpy(out))

    dec = shard.SeqShardDecode(torch, world=world, rank=rank, partial=partial, combine=combine)
    xb = torch.zeros(HQ * HD)
    dec(xb, torch.from_numpy(q), 0, 0, t1 - t0)
    ref = orc.attn_decode(q, kc, vc, 0, L - 1, HQ, KV_MUL, HD, KV_DIM, L)
    return normwise(xb.numpy(), ref)


def _head_case(torch, orc, shard, rank, world):
    lens = [70, 300, 129]
    B = len(lens)
    xb = torch.zeros(B, HQ * HD)
    ref = np.zeros((B, HQ * HD), np.float32)
    h0, nh = shard.kv_heads(HKV, world, rank)
    c0, c1 = h0 * KV_MUL * HD, (h0 + nh) * KV_MUL * HD
    for b, L in enumerate(lens):
        kc = orc.randn(L * KV_DIM, 40 + b, 1)
        vc = orc.randn(L * KV_DIM, 40 + b, 2)
        q = orc.randn(HQ * HD, 40 + b, 3)
        full = orc.attn_decode(q, kc, vc, 0, L - 1, HQ, KV_MUL, HD, KV_DIM, L)
        ref[b] = full
        xb[b, c0:c1] = torch.from_numpy(full[c0:c1])  # this rank's heads only
    g = shard.HeadSliceGather(torch, world=world, rank=rank, rows=B)
    g(xb)
    return normwise(xb.numpy(), ref)


def _peer_gather_case(torch, shard, rank, world):
    """PeerHeadGather's host side with a stand-in context: the registered
    handles travel to every rank in rank order, and a gather of a matrix view
    inside the buffer asks for this rank's column slice at the right byte
    offsets.  Returns 0.0 when every check holds."""

    class FakeCtx:
        def __init__(self):
            self.opened = None
            self.calls = []

        def peer_register(self, buf, nbytes):
            assert nbytes == buf.numel() * buf.element_size()
            return bytes([rank]) * 136

        def peer_register_open(self, r, w, handles):
            self.opened = (r, w, list(handles))

        def gather_cols(self, off, rows, row_bytes, col0, col_bytes):
            self.calls.append((off, rows, row_bytes, col0, col_bytes))

    ctx = FakeCtx()
    buf = torch.zeros(3, 40, HQ * HD, dtype=torch.bfloat16)
    g = shard.PeerHeadGather(torch, ctx, world=world, rank=rank, buf=buf)
    assert ctx.opened == (rank, world, [bytes([r]) * 136 for r in range(world)])
    g(buf[2])
    es = 2
    w = HQ * HD // world
    assert ctx.calls == [(2 * 40 * HQ * HD * es, 40, HQ * HD * es, rank * w * es, w * es)]
    return 0.0


@pytest.mark.parametrize("kind", ["seq", "head", "peer_gather"])
def test_sharded_exchange_on_two_gloo_ranks(kind):
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    world = 2
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, kind, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = [q.get(timeout=180) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
    for rank, err, exc in res:
        assert exc is None, f"rank {rank}: {exc}"
        assert err < 1e-5, f"rank {rank}: normwise {err}"
