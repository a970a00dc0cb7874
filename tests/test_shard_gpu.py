"""GPU parity of the multi-GPU sharding layouts, through the C-ABI library.

On one GPU, several contexts stand in for the ranks: each holds what one
rank would hold (a compact chunk of the sequence, or a range of KV heads),
and the exchange is done by hand in the layout the all-gather produces.  A
real two-process NCCL run follows when the box has two GPUs.

Tolerances as in tests/shapes.py: fp32 cache normwise 2e-4, bf16 cache
max-abs 1e-2 against the oracle (the reference's attention loop,
cpu/main.c:1331-1353) fed the same bf16-rounded K/V.
"""
import os
import socket
import sys

import numpy as np
import pytest

import q3a_oracle as orc
import q3attn
import shard
from shapes import EPS, HD, HKV, HQ, KV_DIM, KV_MUL, THETA, TOL_BF16_ABS, TOL_F32_NORMWISE, normwise

pytestmark = pytest.mark.gpu
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def check_close(got, ref, bf16, what=""):
    if bf16:
        err = float(np.abs(np.float64(got) - np.float64(ref)).max())
        assert err <= TOL_BF16_ABS, f"{what}: max-abs {err}"
    else:
        err = normwise(got, ref)
        assert err <= TOL_F32_NORMWISE, f"{what}: normwise {err}"


@pytest.mark.parametrize("bf16", [False, True])
@pytest.mark.parametrize("world", [1, 3, 4])
def test_sequence_shards_compact_chunks(bf16, world):
    """Each 'rank' context stores only its chunk, from row 0; packed (o, lse)
    rows merged by q3a_lse_combine_packed equal one pass over the sequence."""
    L = 4001
    kc, vc, _, _ = orc.make_cache(90 + world, 0, L, HKV, HD, L, bf16=bf16)
    q = orc.randn(HQ * HD, 90 + world, 9)
    ref = orc.attn_decode(q, kc, vc, 0, L - 1, HQ, KV_MUL, HD, KV_DIM, L)
    W = shard.packed_width(HQ, HD)
    parts = np.zeros((world, W), np.float32)
    dt = q3attn.KV_BF16 if bf16 else q3attn.KV_F32
    for r in range(world):
        t0, t1 = shard.seq_chunk(L, world, r)
        with q3attn.Context(n_layers=1, max_seq=t1 - t0, kv_dtype=dt) as ctx:
            ctx.kv_load(0, 0, 0, t1 - t0, kc[t0 * KV_DIM:t1 * KV_DIM], vc[t0 * KV_DIM:t1 * KV_DIM])
            o = np.zeros(HQ * HD, np.float32)
            lse = np.zeros(HQ, np.float32)
            ctx.attn_partial(o, lse, q, 0, 0, 0, t1 - t0)
            parts[r, :HQ * HD] = o
            parts[r, HQ * HD:] = lse
    with q3attn.Context(n_layers=1, max_seq=64, kv_dtype=dt) as ctx:
        xb = np.zeros(HQ * HD, np.float32)
        ctx.lse_combine_packed(xb, parts, world)
        check_close(xb, ref, bf16, f"packed combine, {world} shards")
        # the dense-array entry point gives the same bits
        xd = np.zeros(HQ * HD, np.float32)
        ctx.lse_combine(xd, np.ascontiguousarray(parts[:, :HQ * HD]),
                        np.ascontiguousarray(parts[:, HQ * HD:]), world)
        assert np.array_equal(xd, xb)


@pytest.mark.parametrize("bf16", [False, True])
def test_packed_combine_device_mode(bf16):
    import torch
    dev = torch.device("cuda:0")
    L, world = 3000, 2
    kc, vc, _, _ = orc.make_cache(77, 0, L, HKV, HD, L, bf16=bf16)
    q = orc.randn(HQ * HD, 77, 9)
    ref = orc.attn_decode(q, kc, vc, 0, L - 1, HQ, KV_MUL, HD, KV_DIM, L)
    dt = q3attn.KV_BF16 if bf16 else q3attn.KV_F32
    with q3attn.Context(n_layers=1, max_seq=L, kv_dtype=dt, ptr_mode=q3attn.PTR_DEVICE) as ctx:
        ctx.kv_load(0, 0, 0, L, torch.from_numpy(kc).to(dev), torch.from_numpy(vc).to(dev))
        parts = torch.zeros(world, shard.packed_width(HQ, HD), device=dev)
        qd = torch.from_numpy(q).to(dev)
        for r in range(world):
            t0, t1 = shard.seq_chunk(L, world, r)
            ctx.attn_partial(parts[r, :HQ * HD], parts[r, HQ * HD:], qd, 0, 0, t0, t1)
        xb = torch.zeros(HQ * HD, device=dev)
        ctx.lse_combine_packed(xb, parts, world)
        ctx.sync()
        check_close(xb.cpu().numpy(), ref, bf16, "device-mode packed combine")


@pytest.mark.parametrize("bf16", [False, True])
@pytest.mark.parametrize("world", [2, 4])
def test_kv_head_shards_batched_ragged(bf16, world):
    """Each 'rank' context holds 8/world KV heads; the batched fused step
    writes that rank's xb columns; together they equal the oracle block."""
    lens = [1, 300, 77, 1500]
    B = len(lens)
    qw = np.ones(HD, np.float32)
    kw = np.ones(HD, np.float32)
    caches, refs, qs, ks, vs = [], [], [], [], []
    for i, L in enumerate(lens):
        pos = L - 1
        kc, vc, _, _ = orc.make_cache(500 + i, 0, pos, HKV, HD, 2048, bf16=bf16)
        q = orc.randn(HQ * HD, 500 + i, 3)
        k = orc.randn(KV_DIM, 500 + i, 4)
        v = orc.randn(KV_DIM, 500 + i, 5)
        qq, kk = q.copy(), k.copy()
        orc.rmsnorm_head(qq, qw, HQ, HD, EPS)
        orc.rmsnorm_head(kk, kw, HKV, HD, EPS)
        orc.rope(qq, HQ, HD, pos, THETA)
        orc.rope(kk, HKV, HD, pos, THETA)
        kr = kc.copy()
        vr = vc.copy()
        kr[pos * KV_DIM:(pos + 1) * KV_DIM] = orc.bf16_round(kk) if bf16 else kk
        vr[pos * KV_DIM:(pos + 1) * KV_DIM] = orc.bf16_round(v) if bf16 else v
        refs.append(orc.attn_decode(qq, kr, vr, 0, pos, HQ, KV_MUL, HD, KV_DIM, 2048))
        caches.append((kc, vc))
        qs.append(q)
        ks.append(k)
        vs.append(v)
    dt = q3attn.KV_BF16 if bf16 else q3attn.KV_F32
    xb = np.zeros((B, HQ * HD), np.float32)
    for r in range(world):
        h0, nh = shard.kv_heads(HKV, world, r)
        with q3attn.Context(n_layers=1, max_seq=2048, n_seqs=B, kv_dtype=dt,
                            kv_head_begin=h0, kv_head_count=nh) as ctx:
            for i, L in enumerate(lens):
                pos = L - 1
                if pos > 0:
                    # full rows in, as the reference's k/v buffers: the
                    # context keeps its own heads' columns
                    kc, vc = caches[i]
                    ctx.kv_load(i, 0, 0, pos, kc[: pos * KV_DIM], vc[: pos * KV_DIM])
            part = np.zeros((B, HQ * HD), np.float32)
            ctx.attn_layer_batched(part, np.stack(qs), np.stack(ks), np.stack(vs), qw, kw, 0,
                                   list(range(B)), [L - 1 for L in lens])
            c0, c1 = h0 * KV_MUL * HD, (h0 + nh) * KV_MUL * HD
            xb[:, c0:c1] = part[:, c0:c1]
    for i in range(B):
        check_close(xb[i], refs[i], bf16, f"seq {i} len {lens[i]}, {world} head shards")


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _nccl_worker(rank, world, port, out_q):
    try:
        for p in (os.path.join(ROOT, "oracle"), os.path.join(ROOT, "qwen3.c_b200"),
                  os.path.join(ROOT, "tests")):
            sys.path.insert(0, p)
        import datetime
        import torch
        import torch.distributed as dist
        import q3a_oracle as orc
        import q3attn
        import shard
        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        os.environ["NCCL_NVLS_ENABLE"] = "0"
        dev = torch.device(f"cuda:{rank}")
        torch.cuda.set_device(dev)
        dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev,
                                timeout=datetime.timedelta(seconds=60))
        L = 20000
        kc, vc, _, _ = orc.make_cache(123, 0, L, HKV, HD, L, bf16=True)
        qv = orc.randn(HQ * HD, 123, 9)
        t0, t1 = shard.seq_chunk(L, world, rank)
        with q3attn.Context(n_layers=1, max_seq=t1 - t0, kv_dtype=q3attn.KV_BF16,
                            ptr_mode=q3attn.PTR_DEVICE, device=rank) as ctx:
            st = torch.cuda.current_stream(dev)
            ctx.set_stream(st.cuda_stream)
            ctx.kv_load(0, 0, 0, t1 - t0, torch.from_numpy(kc[t0 * KV_DIM:t1 * KV_DIM]).to(dev),
                        torch.from_numpy(vc[t0 * KV_DIM:t1 * KV_DIM]).to(dev))
            dec = shard.SeqShardDecode(torch, ctx, world=world, rank=rank, device=dev)
            xb = torch.zeros(HQ * HD, device=dev)
            dec(xb, torch.from_numpy(qv).to(dev), 0, 0, t1 - t0)
            torch.cuda.synchronize(dev)
            ctx.check_device_error()
            got = xb.cpu().numpy()
        dist.barrier()
        dist.destroy_process_group()
        ref = orc.attn_decode(qv, kc, vc, 0, L - 1, HQ, KV_MUL, HD, KV_DIM, L)
        out_q.put((rank, float(np.abs(np.float64(got) - ref).max()), None))
    except Exception as e:  # reported to the parent, which fails the test
        out_q.put((rank, None, repr(e)))


def test_sequence_shards_over_nccl_two_gpus():
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_nccl_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = [q.get(timeout=300) for _ in range(2)]
    for p in procs:
        p.join(timeout=60)
    for rank, err, exc in res:
        assert exc is None, f"rank {rank}: {exc}"
        assert err <= TOL_BF16_ABS, f"rank {rank}: max-abs {err}"

