"""q3a_attn_decode_noalloc against q3a_attn_decode, through the C-ABI.

q3a_attn_decode_noalloc serves hosts that must not allocate device memory at
the time they run attention -- an engine whose arena allocator owns all
device memory, a process with a fixed memory budget, code inside a callback
where allocation is forbidden.  It keeps the split-KV scratch in a fixed
array of the library instead of a context.  Its results must equal those of
the context-based entry point on the same inputs, call after call (the
array keeps the previous call's contents, so a second call checks that
nothing stale leaks into it).

This file is named to be collected last; it passes on its own in a fresh
process as well as after the other tests.
"""
import numpy as np
import pytest

import q3a_oracle as orc
import q3attn
from shapes import HD, HKV, HQ, KV_DIM, KV_MUL, TOL_F32_NORMWISE, normwise

pytestmark = pytest.mark.gpu


def _inputs(seed, n_layers, max_seq):
    caches_k, caches_v = [], []
    for layer in range(n_layers):
        kc, vc, _, _ = orc.make_cache(seed, layer, max_seq, HKV, HD, max_seq)
        caches_k.append(kc)
        caches_v.append(vc)
    return np.concatenate(caches_k), np.concatenate(caches_v)


def test_noalloc_matches_context_entry_point_twice():
    import torch
    dev = torch.device("cuda:0")
    torch.cuda.set_device(dev)
    max_seq = 1300
    kc, vc = _inputs(2024, 2, max_seq)
    dk = torch.from_numpy(kc).to(dev)
    dv = torch.from_numpy(vc).to(dev)
    stream = torch.cuda.Stream(device=dev)
    calls = [(0, 650, orc.randn(HQ * HD, 2024, 50)),              # layer 0, pos 650
             (max_seq * KV_DIM, 1299, orc.randn(HQ * HD, 2024, 51))]  # layer 1, last row
    with q3attn.Context(n_layers=1, max_seq=64, ptr_mode=q3attn.PTR_DEVICE) as ctx:
        ctx.set_stream(stream.cuda_stream)
        for loff, pos, q in calls:
            dq = torch.from_numpy(q).to(dev)
            want = torch.zeros(HQ * HD, device=dev)
            got = torch.full((HQ * HD,), float("nan"), device=dev)
            ctx.attn_decode(want, dq, dk, dv, None, loff, pos, HQ, KV_MUL, HD, KV_DIM, max_seq)
            q3attn.attn_decode_noalloc(got, dq, dk, dv, loff, pos, HQ, KV_MUL, HD, KV_DIM,
                                       max_seq, stream.cuda_stream)
            # no bounded wait of the launch expired (reads and clears the
            # fixed array's error word, allocating nothing)
            q3attn.noalloc_check_error(stream.cuda_stream)
            stream.synchronize()
            w = want.cpu().numpy()
            g = got.cpu().numpy()
            assert np.all(np.isfinite(g))
            assert normwise(g, w) <= TOL_F32_NORMWISE
            # and against the CPU oracle
            ref = orc.attn_decode(q, kc, vc, loff, pos, HQ, KV_MUL, HD, KV_DIM, max_seq)
            assert normwise(g, ref) <= TOL_F32_NORMWISE


def test_noalloc_rejects_shapes_beyond_its_scratch():
    import torch
    dev = torch.device("cuda:0")
    buf = torch.zeros(16, device=dev)
    with pytest.raises(q3attn.Q3AError) as e:
        # 32 KV heads: more than the fixed scratch array serves
        q3attn.attn_decode_noalloc(buf, buf, buf, buf, 0, 0, 128, 4, 128, 32 * 128, 1)
    assert e.value.code == q3attn.ERR_INVALID
    assert "16 KV heads" in str(e.value)


def test_noalloc_on_two_devices_in_one_process():
    """The fixed array, its address and the kernel's shared-memory limit are
    per device: one process calls the entry point on device 0, then on
    device 1 (skipped with one GPU), each against the oracle."""
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    max_seq = 700
    kc, vc = _inputs(77, 1, max_seq)
    q = orc.randn(HQ * HD, 77, 52)
    ref = orc.attn_decode(q, kc, vc, 0, max_seq - 1, HQ, KV_MUL, HD, KV_DIM, max_seq)
    for d in (0, 1, 0):
        dev = torch.device(f"cuda:{d}")
        torch.cuda.set_device(dev)
        stream = torch.cuda.Stream(device=dev)
        dk = torch.from_numpy(kc).to(dev)
        dv = torch.from_numpy(vc).to(dev)
        dq = torch.from_numpy(q).to(dev)
        got = torch.full((HQ * HD,), float("nan"), device=dev)
        q3attn.attn_decode_noalloc(got, dq, dk, dv, 0, max_seq - 1, HQ, KV_MUL, HD, KV_DIM,
                                   max_seq, stream.cuda_stream)
        q3attn.noalloc_check_error(stream.cuda_stream)
        g = got.cpu().numpy()
        assert np.all(np.isfinite(g)), f"device {d}"
        assert normwise(g, ref) <= TOL_F32_NORMWISE, f"device {d}"
    torch.cuda.set_device(0)
