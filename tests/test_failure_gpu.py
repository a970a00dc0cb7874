"""Failure detection without a GPU fault: device-side waits run out and the
context stays usable.

The reference stops the process on any error (HIPCHK -> exit(1),
qwen3-8b/gpu/main.c:47-53) and has no device-side waits.  Here every wait of
a kernel on another CTA or another rank is bounded; when the limit passes
the kernel gives up, leaves its output unwritten, sets the device error
flag and returns.  These tests make such waits run out on purpose in the
accepted form: a second rank that never calls, so the words and flags it
would write are never set.  Both "ranks" are contexts on one GPU in one
process (q3a_peer_open_ptrs / q3a_peer_register_open_ptrs); only rank 0 ever
launches, so no two kernels wait on one another.  With the limit lowered to
20 ms the call returns within milliseconds, q3a_check_device_error reports
Q3A_ERR_TIMEOUT, and the same context then decodes correctly.
"""
import time

import numpy as np
import pytest

import q3a_oracle as orc
import q3attn
from shapes import HD, HKV, HQ, KV_DIM, KV_MUL, TOL_BF16_ABS, TOL_F32_NORMWISE, normwise

pytestmark = pytest.mark.gpu

LIMIT_S = 0.02


def _check(got, ref, bf16):
    if bf16:
        assert float(np.abs(np.float64(got) - ref).max()) <= TOL_BF16_ABS
    else:
        assert normwise(got, ref) <= TOL_F32_NORMWISE


def _decode_still_works(ctx, torch, dev, kc, vc, q, L, bf16):
    """A plain split-KV decode on the context after the timeout."""
    ref = orc.attn_decode(q, kc, vc, 0, L - 1, HQ, KV_MUL, HD, KV_DIM, L)
    o = torch.zeros(HQ * HD, device=dev)
    lse = torch.zeros(HQ, device=dev)
    ctx.attn_partial(o, lse, torch.from_numpy(q).to(dev), 0, 0, 0, L)
    ctx.sync()
    ctx.check_device_error()
    _check(o.cpu().numpy(), ref, bf16)


@pytest.mark.parametrize("bf16", [False, True])
def test_sequence_shard_rank_that_never_arrives(bf16):
    import torch
    dev = torch.device("cuda:0")
    L = 3000
    kc, vc, _, _ = orc.make_cache(31, 0, L, HKV, HD, L, bf16=bf16)
    q = orc.randn(HQ * HD, 31, 9)
    dt = q3attn.KV_BF16 if bf16 else q3attn.KV_F32
    with q3attn.Context(n_layers=1, max_seq=L, kv_dtype=dt, ptr_mode=q3attn.PTR_DEVICE) as a, \
            q3attn.Context(n_layers=1, max_seq=64, kv_dtype=dt, ptr_mode=q3attn.PTR_DEVICE) as b:
        a.kv_load(0, 0, 0, L, torch.from_numpy(kc).to(dev), torch.from_numpy(vc).to(dev))
        a.peer_export(2)
        b.peer_export(2)
        # rank 1 (context b) is mapped but never calls q3a_attn_seqshard
        a.peer_open_ptrs(0, 2, [a.peer_buffer(), b.peer_buffer()])
        a.set_wait_limit(LIMIT_S)
        xb = torch.full((HQ * HD,), float("nan"), device=dev)
        qd = torch.from_numpy(q).to(dev)
        torch.cuda.synchronize(dev)
        t0 = time.perf_counter()
        a.attn_seqshard(xb, qd, 0, 0, L)
        a.sync()
        waited = time.perf_counter() - t0
        with pytest.raises(q3attn.Q3AError) as e:
            a.check_device_error()
        assert e.value.code == q3attn.ERR_TIMEOUT
        # the kernel gave up after the lowered limit, not the ~1 s default
        assert waited < 0.5, waited
        # nothing was written for the missing rank's share
        assert torch.isnan(xb).all()
        a.set_wait_limit(0)
        _decode_still_works(a, torch, dev, kc, vc, q, L, bf16)


def test_column_gather_rank_that_never_arrives():
    import torch
    dev = torch.device("cuda:0")
    rows, cols = 64, HQ * HD
    L = 1000
    kc, vc, _, _ = orc.make_cache(32, 0, L, HKV, HD, L)
    q = orc.randn(HQ * HD, 32, 9)
    bufa = torch.zeros(rows, cols, dtype=torch.bfloat16, device=dev)
    bufb = torch.zeros(rows, cols, dtype=torch.bfloat16, device=dev)
    with q3attn.Context(n_layers=1, max_seq=L, ptr_mode=q3attn.PTR_DEVICE) as a, \
            q3attn.Context(n_layers=1, max_seq=64, ptr_mode=q3attn.PTR_DEVICE) as b:
        a.kv_load(0, 0, 0, L, torch.from_numpy(kc).to(dev), torch.from_numpy(vc).to(dev))
        a.peer_register(bufa, bufa.numel() * 2)
        b.peer_register(bufb, bufb.numel() * 2)
        a.peer_register_open_ptrs(0, 2, [bufa.data_ptr(), bufb.data_ptr()],
                                  [a.peer_register_flags(), b.peer_register_flags()])
        a.set_wait_limit(LIMIT_S)
        torch.cuda.synchronize(dev)
        t0 = time.perf_counter()
        a.gather_cols(0, rows, cols * 2, 0, cols)  # rank 0's half of the columns
        a.sync()
        waited = time.perf_counter() - t0
        with pytest.raises(q3attn.Q3AError) as e:
            a.check_device_error()
        assert e.value.code == q3attn.ERR_TIMEOUT
        assert waited < 0.5, waited
        a.set_wait_limit(0)
        _decode_still_works(a, torch, dev, kc, vc, q, L, False)


def test_wait_limit_rejects_bad_values():
    with q3attn.Context(n_layers=1, max_seq=64, ptr_mode=q3attn.PTR_DEVICE) as a:
        for bad in (-1.0, 61.0, float("nan")):
            with pytest.raises(q3attn.Q3AError) as e:
                a.set_wait_limit(bad)
            assert e.value.code == q3attn.ERR_INVALID
        a.set_wait_limit(0.5)
        a.set_wait_limit(0)


def test_wo_exchange_rank_that_never_arrives():
    """Row-parallel wo over two KV-head shards where rank 1 never calls: rank
    0's wo kernel stores its partial sums, waits (bounded) for rank 1's,
    gives up, reports Q3A_ERR_TIMEOUT and leaves x as it was."""
    import torch
    dev = torch.device("cuda:0")
    L = 1000
    kc, vc, _, _ = orc.make_cache(33, 0, L, HKV, HD, L)
    q = orc.randn(HQ * HD, 33, 9)
    dim = 4096
    wo = (torch.randn(dim, HQ * HD, device=dev) * 0.02).half()
    with q3attn.Context(n_layers=1, max_seq=L, ptr_mode=q3attn.PTR_DEVICE,
                        kv_head_begin=0, kv_head_count=4) as a, \
            q3attn.Context(n_layers=1, max_seq=64, ptr_mode=q3attn.PTR_DEVICE,
                           kv_head_begin=4, kv_head_count=4) as b, \
            q3attn.Context(n_layers=1, max_seq=L, ptr_mode=q3attn.PTR_DEVICE) as full:
        a.peer_export(2)
        b.peer_export(2)
        a.peer_open_ptrs(0, 2, [a.peer_buffer(), b.peer_buffer()])
        a.set_wait_limit(LIMIT_S)
        x = torch.randn(dim, device=dev)
        x0 = x.clone()
        xb = torch.randn(HQ * HD, device=dev)
        torch.cuda.synchronize(dev)
        t0 = time.perf_counter()
        a.wo_residual(x, xb, wo)
        a.sync()
        waited = time.perf_counter() - t0
        with pytest.raises(q3attn.Q3AError) as e:
            a.check_device_error()
        assert e.value.code == q3attn.ERR_TIMEOUT
        assert waited < 0.5, waited
        assert torch.equal(x, x0)
        a.set_wait_limit(0)
        full.kv_load(0, 0, 0, L, torch.from_numpy(kc).to(dev), torch.from_numpy(vc).to(dev))
        _decode_still_works(full, torch, dev, kc, vc, q, L, False)
        # the context that timed out still runs its own kernels: the fused
        # block of one token on its KV heads, against the oracle
        from test_decode_gpu import oracle_block, oracle_inputs
        pos = L - 1
        kc2, vc2, q2, k2, v2, qw, kw = oracle_inputs(34, pos, L, False)
        xr, _, _ = oracle_block(kc2, vc2, q2, k2, v2, qw, kw, pos, L, False)
        a.kv_load(0, 0, 0, pos, torch.from_numpy(kc2[:pos * KV_DIM]).to(dev),
                  torch.from_numpy(vc2[:pos * KV_DIM]).to(dev))
        xbd = torch.zeros(1, HQ * HD, device=dev)
        t = lambda arr: torch.from_numpy(arr).to(dev)  # noqa: E731
        a.attn_layer_batched(xbd, t(q2).reshape(1, -1).contiguous(), t(k2).reshape(1, -1).contiguous(),
                             t(v2).reshape(1, -1).contiguous(), t(qw), t(kw), 0, [0], [pos])
        a.sync()
        a.check_device_error()
        held = slice(0, 4 * KV_MUL * HD)
        _check(xbd.cpu().numpy()[0, held], xr[held], False)
