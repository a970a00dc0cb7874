"""The KV-cache wire format on the GPU: q3a_kv_pack / q3a_kv_unpack round
trips (fp32 and bf16 caches, device and host pointer modes, a position range
that starts and ends inside pages and inside the bf16 8-row blocks), the
device checksum against the host one, a KV-head subset unpacked into a
sharded context, and a corrupted blob refused with the cache untouched.
Round trips are bit-exact: the payload holds the cache's own values."""
import numpy as np
import pytest

import q3attn
from shapes import HD, HKV, KV_DIM

pytestmark = pytest.mark.gpu

L, MS = 3, 1024
POS0, NT = 61, 203          # inside a 64-token page and an 8-row block at both ends


def filled(kv, ptr_mode, **kw):
    ctx = q3attn.Context(n_layers=L, max_seq=MS, n_seqs=2, kv_dtype=kv, ptr_mode=ptr_mode, **kw)
    for l in range(L):
        ctx.kv_synth(0, l, 0, MS, 4321 + l, 1, 2)
    return ctx


def read(torch, ctx, seq, layer, pos0, n, nkv, dev):
    if ctx.cfg.ptr_mode == q3attn.PTR_DEVICE:
        k = torch.zeros(n * nkv * HD, device=dev)
        v = torch.zeros(n * nkv * HD, device=dev)
        ctx.kv_read(seq, layer, pos0, n, k, v)
        ctx.sync()
        return k.cpu().numpy(), v.cpu().numpy()
    k = np.zeros(n * nkv * HD, np.float32)
    v = np.zeros(n * nkv * HD, np.float32)
    ctx.kv_read(seq, layer, pos0, n, k, v)
    return k, v


@pytest.mark.parametrize("kv", [q3attn.KV_F32, q3attn.KV_BF16])
@pytest.mark.parametrize("mode", [q3attn.PTR_DEVICE, q3attn.PTR_HOST])
def test_pack_unpack_round_trip(kv, mode):
    import torch
    dev = torch.device("cuda:0")
    src = filled(kv, mode)
    dst = q3attn.Context(n_layers=L, max_seq=MS, n_seqs=2, kv_dtype=kv, ptr_mode=mode)
    try:
        nbytes = src.kv_wire_bytes(2, NT)
        es = 2 if kv == q3attn.KV_BF16 else 4
        assert nbytes == 64 + 2 * HKV * 2 * NT * HD * es
        if mode == q3attn.PTR_DEVICE:
            b = torch.zeros(nbytes, dtype=torch.uint8, device=dev)
        else:
            b = np.zeros(nbytes, np.uint8)
        src.kv_pack(0, 1, 2, POS0, NT, b)
        src.sync()
        host = b.cpu().numpy() if mode == q3attn.PTR_DEVICE else b
        q3attn.kv_wire_check(host)          # the device checksum equals the host one
        dst.kv_unpack(1, b)
        dst.sync()
        for l in (1, 2):
            ka, va = read(torch, src, 0, l, POS0, NT, HKV, dev)
            kb, vb = read(torch, dst, 1, l, POS0, NT, HKV, dev)
            assert np.array_equal(ka.view(np.uint32), kb.view(np.uint32)), f"layer {l} K"
            assert np.array_equal(va.view(np.uint32), vb.view(np.uint32)), f"layer {l} V"
        # rows outside the blob's range stay as they were (zero)
        k0, _ = read(torch, dst, 1, 1, 0, POS0, HKV, dev)
        assert not k0.any()
        k3, _ = read(torch, dst, 1, 0, 0, MS, HKV, dev)
        assert not k3.any()
    finally:
        src.close()
        dst.close()


def test_head_subset_into_sharded_context():
    import torch
    dev = torch.device("cuda:0")
    src = filled(q3attn.KV_BF16, q3attn.PTR_DEVICE)
    dst = q3attn.Context(n_layers=L, max_seq=MS, n_seqs=2, kv_dtype=q3attn.KV_BF16,
                         ptr_mode=q3attn.PTR_DEVICE, kv_head_begin=2, kv_head_count=3)
    try:
        b = torch.zeros(src.kv_wire_bytes(L, NT), dtype=torch.uint8, device=dev)
        src.kv_pack(0, 0, L, POS0, NT, b)
        dst.kv_unpack(0, b)
        dst.sync()
        ka, va = read(torch, src, 0, 2, POS0, NT, HKV, dev)
        kb, vb = read(torch, dst, 0, 2, POS0, NT, 3, dev)
        ka = ka.reshape(NT, HKV, HD)[:, 2:5].reshape(-1)
        va = va.reshape(NT, HKV, HD)[:, 2:5].reshape(-1)
        assert np.array_equal(ka, kb) and np.array_equal(va, vb)
        # and a blob of heads 2..4 cannot fill a context holding heads 0..7
        sub = torch.zeros(dst.kv_wire_bytes(1, NT), dtype=torch.uint8, device=dev)
        dst.kv_pack(0, 0, 1, POS0, NT, sub)
        with pytest.raises(q3attn.Q3AError, match="heads"):
            src.kv_unpack(1, sub)
    finally:
        src.close()
        dst.close()


def test_corrupted_blob_leaves_cache_untouched():
    import torch
    dev = torch.device("cuda:0")
    src = filled(q3attn.KV_F32, q3attn.PTR_DEVICE)
    dst = q3attn.Context(n_layers=L, max_seq=MS, n_seqs=2, ptr_mode=q3attn.PTR_DEVICE)
    try:
        b = torch.zeros(src.kv_wire_bytes(1, NT), dtype=torch.uint8, device=dev)
        src.kv_pack(0, 0, 1, POS0, NT, b)
        src.sync()
        b[64 + 12345] ^= 1
        torch.cuda.synchronize()
        with pytest.raises(q3attn.Q3AError, match="checksum"):
            dst.kv_unpack(0, b)
        k, v = read(torch, dst, 0, 0, 0, MS, HKV, dev)
        assert not k.any() and not v.any()
        # a bf16 blob does not go into an fp32 context
        bf = filled(q3attn.KV_BF16, q3attn.PTR_DEVICE)
        try:
            b2 = torch.zeros(bf.kv_wire_bytes(1, 8), dtype=torch.uint8, device=dev)
            bf.kv_pack(0, 0, 1, 0, 8, b2)
            with pytest.raises(q3attn.Q3AError, match="dtype"):
                dst.kv_unpack(0, b2)
        finally:
            bf.close()
    finally:
        src.close()
        dst.close()
