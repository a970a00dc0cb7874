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


@pytest.mark.parametrize("world", [2, 4])
def test_kv_head_shards_prefill(world):
    """q3a_prefill on KV-head-sharded contexts: each writes its query heads'
    columns (host mode keeps the rest); together they equal the oracle."""
    S = 200
    seed = 61
    qraw = orc.randn(S * HQ * HD, seed, 3)
    kc, vc, kraw, vraw = orc.make_cache(seed, 0, S, HKV, HD, S, bf16=True)
    qw = np.ones(HD, np.float32)
    q = qraw.copy()
    for s_ in range(S):
        row = q[s_ * HQ * HD:(s_ + 1) * HQ * HD]
        orc.rmsnorm_head(row, qw, HQ, HD, EPS)
        orc.rope(row, HQ, HD, s_, THETA)
    ref = orc.prefill_causal(orc.bf16_round(q), kc, vc, 0, S, HQ, KV_MUL, HD, KV_DIM, S)
    out = np.full((S, HQ * HD), np.nan, np.float32)
    for r in range(world):
        h0, nh = shard.kv_heads(HKV, world, r)
        with q3attn.Context(n_layers=1, max_seq=S, kv_dtype=q3attn.KV_BF16,
                            kv_head_begin=h0, kv_head_count=nh) as ctx:
            ctx.prefill(out, q3attn.OUT_F32, qraw, kraw, vraw, qw, qw, 0, 0, 0, S)
    assert np.all(np.isfinite(out))
    err = float(np.abs(np.float64(out.reshape(-1)) - ref).max())
    assert err <= TOL_BF16_ABS, f"{world} head shards: max-abs {err}"


@pytest.mark.parametrize("bf16", [False, True])
def test_peer_seqshard_one_rank(bf16):
    """The peer-memory path with one rank (no cross-GPU wait): partial decode,
    store of the packed row into its own buffer, flag, merge; repeated calls
    alternate the buffer halves and give the same result."""
    import torch
    dev = torch.device("cuda:0")
    L = 5000
    kc, vc, _, _ = orc.make_cache(808, 0, L, HKV, HD, L, bf16=bf16)
    q = orc.randn(HQ * HD, 808, 9)
    ref = orc.attn_decode(q, kc, vc, 0, L - 1, HQ, KV_MUL, HD, KV_DIM, L)
    dt = q3attn.KV_BF16 if bf16 else q3attn.KV_F32
    with q3attn.Context(n_layers=1, max_seq=L, kv_dtype=dt, ptr_mode=q3attn.PTR_DEVICE) as ctx:
        ctx.kv_load(0, 0, 0, L, torch.from_numpy(kc).to(dev), torch.from_numpy(vc).to(dev))
        h = ctx.peer_export(1)
        assert len(h) == q3attn.IPC_HANDLE_BYTES
        ctx.peer_open(0, 1, [h])
        ctx.set_deterministic(True)  # repeated calls compared bit for bit
        qd = torch.from_numpy(q).to(dev)
        outs = []
        for _ in range(3):
            xb = torch.zeros(HQ * HD, device=dev)
            ctx.attn_seqshard(xb, qd, 0, 0, L)
            ctx.sync()
            ctx.check_device_error()
            outs.append(xb.cpu().numpy())
        for o in outs:
            check_close(o, ref, bf16, "peer seqshard, one rank")
        assert all(np.array_equal(o, outs[0]) for o in outs)


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


@pytest.mark.parametrize("world", [2, 4, 8])
@pytest.mark.parametrize("mode", ["nccl", "peer"])
def test_sequence_shards_over_gpus(tmp_path, mode, world):
    """`world` ranks launched the way bench.py --gpus N is (torchrun, one
    process per GPU); the exchange is an NCCL all-gather or the peer-memory
    stores of q3a_attn_seqshard; each rank checks its combined xb against the
    oracle and writes the error to a file."""
    import subprocess
    import torch
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    env = dict(os.environ, NCCL_NVLS_ENABLE="0", SHARD_TEST_OUT=str(tmp_path), SHARD_MODE=mode)
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node",
           str(world), "--master-addr", "127.0.0.1", "--master-port", str(_free_port()),
           os.path.join(ROOT, "tests", "nccl_seq_shard.py")]
    r = subprocess.run(cmd, env=env, timeout=240, capture_output=True, text=True)
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-2000:]
    for rank in range(world):
        err = float(open(os.path.join(tmp_path, f"rank{rank}.txt")).read())
        assert err <= TOL_BF16_ABS, f"rank {rank}: max-abs {err}"


@pytest.mark.parametrize("world", [2, 4, 8])
def test_peer_head_gather(tmp_path, world):
    """q3a_gather_cols over `world` GPUs (torchrun, one process per GPU):
    every rank ends with every rank's column slice, bit-exact, over repeated
    calls on two matrices of one registered buffer."""
    import subprocess
    import torch
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    env = dict(os.environ, NCCL_NVLS_ENABLE="0", SHARD_TEST_OUT=str(tmp_path))
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node",
           str(world), "--master-addr", "127.0.0.1", "--master-port", str(_free_port()),
           os.path.join(ROOT, "tests", "peer_gather_worker.py")]
    r = subprocess.run(cmd, env=env, timeout=240, capture_output=True, text=True)
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-2000:]
    for rank in range(world):
        bad = int(open(os.path.join(tmp_path, f"rank{rank}.txt")).read())
        assert bad == 0, f"rank {rank}: {bad} slices differ"


@pytest.mark.parametrize("world", [2, 4, 8])
def test_sublayer_over_kv_head_shards(tmp_path, world):
    """The attention sublayer over `world` GPUs holding 8/world KV heads each
    (torchrun, one process per GPU): column-parallel projections and
    attention, row-parallel wo whose partial sums the ranks exchange over
    NVLink inside the kernel.  Every rank's increments match the oracle and
    every rank's x equals rank 0's bit for bit."""
    import subprocess
    import torch
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    env = dict(os.environ, NCCL_NVLS_ENABLE="0", SHARD_TEST_OUT=str(tmp_path))
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node",
           str(world), "--master-addr", "127.0.0.1", "--master-port", str(_free_port()),
           os.path.join(ROOT, "tests", "tp_sublayer_worker.py")]
    r = subprocess.run(cmd, env=env, timeout=300, capture_output=True, text=True)
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-2000:]
    for rank in range(world):
        err, same = open(os.path.join(tmp_path, f"rank{rank}.txt")).read().split()
        assert float(err) <= 3e-2, f"rank {rank}: normwise {err}"
        assert same == "1", f"rank {rank}: x differs from rank 0's"


def test_prefill_to_decode_handoff(tmp_path):
    """Disaggregated prefill and decode on two GPUs: the prompt's KV rows
    travel as one wire blob (q3a_kv_pack -> NCCL send -> q3a_kv_unpack); the
    next token's attention on the decode GPU equals the prefill GPU's bit for
    bit."""
    import subprocess
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    env = dict(os.environ, NCCL_NVLS_ENABLE="0", SHARD_TEST_OUT=str(tmp_path))
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node", "2",
           "--master-addr", "127.0.0.1", "--master-port", str(_free_port()),
           os.path.join(ROOT, "tests", "wire_handoff_worker.py")]
    r = subprocess.run(cmd, env=env, timeout=240, capture_output=True, text=True)
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-2000:]
    a = np.load(os.path.join(tmp_path, "xb0.npy"))
    b = np.load(os.path.join(tmp_path, "xb1.npy"))
    assert np.isfinite(a).all() and np.abs(a).max() > 0
    assert np.array_equal(a.view(np.uint32), b.view(np.uint32))
