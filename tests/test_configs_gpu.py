"""Parity at the full sizes of BASELINE.json configs[3] and configs[4].

one new query over a 131072-row bf16 cache, through the two
entry points the sequence-sharded decode uses on one GPU --
q3a_attn_seqshard with one rank (the launch bench.py's long_ctx leg times)
and q3a_attn_partial over the whole range (output and log-sum-exp).

the bench's own ragged draw (64 sequences, lengths from
U[512, 32768], numpy PCG64 seed 2024, bench.ragged_lengths) in one fused
q3a_attn_layer_batched step; the shortest, the longest and six more
sequences are checked against the oracle, the others hold seeded device
rows so the launch is the bench's.

Oracle: the reference's attention loop (qwen3-8b/cpu-multicore/main.c:
1346-1369) fed the same bf16-rounded K/V; tolerance max-abs 1e-2 (bf16
cache).
"""
import os
import sys

import numpy as np
import pytest

import q3a_oracle as orc
import q3attn
from shapes import EPS, HD, HKV, HQ, KV_DIM, KV_MUL, THETA, TOL_BF16_ABS

pytestmark = pytest.mark.gpu
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _maxabs(got, ref):
    return float(np.abs(np.float64(got) - np.float64(ref)).max())


def test_long_context_131072_rows():
    import torch
    dev = torch.device("cuda:0")
    L = 131072
    kc, vc, _, _ = orc.make_cache(4242, 0, L, HKV, HD, L, bf16=True)
    q = orc.randn(HQ * HD, 4242, 3)
    ref = orc.attn_decode(q, kc, vc, 0, L - 1, HQ, KV_MUL, HD, KV_DIM, L)
    ref_o, ref_lse = orc.attn_partial(q, kc, vc, 0, 0, L, HQ, KV_MUL, HD, KV_DIM)
    with q3attn.Context(n_layers=1, max_seq=L, kv_dtype=q3attn.KV_BF16,
                        ptr_mode=q3attn.PTR_DEVICE) as ctx:
        dk = torch.from_numpy(kc).to(dev)
        dv = torch.from_numpy(vc).to(dev)
        ctx.kv_load(0, 0, 0, L, dk, dv)
        del dk, dv
        qd = torch.from_numpy(q).to(dev)
        # the long_ctx launch of bench.py at N=1, in the default (balanced)
        # split and in the deterministic one, whose repeated calls are
        # bitwise identical
        ctx.peer_open(0, 1, [ctx.peer_export(1)])
        for det in (False, True):
            ctx.set_deterministic(det)
            outs = []
            for _ in range(2):
                xb = torch.full((HQ * HD,), float("nan"), device=dev)
                ctx.attn_seqshard(xb, qd, 0, 0, L)
                ctx.sync()
                ctx.check_device_error()
                outs.append(xb.cpu().numpy())
            if det:
                assert np.array_equal(outs[0], outs[1])
            for o in outs:
                err = _maxabs(o, ref)
                assert err <= TOL_BF16_ABS, f"seqshard over {L} rows (deterministic {det}): max-abs {err}"
        ctx.set_deterministic(False)
        # the partial entry point over the whole range: o and its lse
        o = torch.zeros(HQ * HD, device=dev)
        lse = torch.zeros(HQ, device=dev)
        ctx.attn_partial(o, lse, qd, 0, 0, 0, L)
        ctx.sync()
        ctx.check_device_error()
        assert _maxabs(o.cpu().numpy(), ref_o) <= TOL_BF16_ABS
        assert _maxabs(lse.cpu().numpy(), ref_lse) <= 1e-3


def test_ragged_batch_bench_draw():
    import torch
    sys.path.insert(0, ROOT)
    from bench import ragged_lengths
    dev = torch.device("cuda:0")
    lens = [int(x) for x in ragged_lengths()]
    B = len(lens)
    assert B == 64
    order = sorted(range(B), key=lambda b: lens[b])
    rng = np.random.default_rng(7)
    middle = [b for b in order[1:-1]]
    checked = sorted({order[0], order[-1], *rng.choice(middle, size=6, replace=False).tolist()})
    Lmax = max(lens)
    ones = np.ones(HD, np.float32)
    q = np.stack([orc.randn(HQ * HD, 600 + b, 3) for b in range(B)])
    k = np.stack([orc.randn(KV_DIM, 600 + b, 4) for b in range(B)])
    v = np.stack([orc.randn(KV_DIM, 600 + b, 5) for b in range(B)])
    refs = {}
    with q3attn.Context(n_layers=1, max_seq=Lmax, n_seqs=B, kv_dtype=q3attn.KV_BF16,
                        ptr_mode=q3attn.PTR_DEVICE) as ctx:
        kraw = torch.empty(Lmax * KV_DIM, device=dev)
        vraw = torch.empty(Lmax * KV_DIM, device=dev)
        w = torch.ones(HD, device=dev)
        for b, L in enumerate(lens):
            n = L - 1
            if b in checked:
                kc, vc, _, _ = orc.make_cache(600 + b, 0, n, HKV, HD, L, bf16=True)
                ctx.kv_load(b, 0, 0, n, torch.from_numpy(kc[: n * KV_DIM]).to(dev),
                            torch.from_numpy(vc[: n * KV_DIM]).to(dev))
                # oracle: the block at pos n with the new row bf16-rounded as
                # the cache stores it
                qq, kk = q[b].copy(), k[b].copy()
                orc.rmsnorm_head(qq, ones, HQ, HD, EPS)
                orc.rmsnorm_head(kk, ones, HKV, HD, EPS)
                orc.rope(qq, HQ, HD, n, THETA)
                orc.rope(kk, HKV, HD, n, THETA)
                kc[n * KV_DIM:(n + 1) * KV_DIM] = orc.bf16_round(kk)
                vc[n * KV_DIM:(n + 1) * KV_DIM] = orc.bf16_round(v[b])
                refs[b] = orc.attn_decode(qq, kc, vc, 0, n, HQ, KV_MUL, HD, KV_DIM, L)
                del kc, vc
            else:
                ctx.randn(kraw, q3attn.OUT_F32, n * KV_DIM, 5151, 1000 + 2 * b)
                ctx.randn(vraw, q3attn.OUT_F32, n * KV_DIM, 5151, 1001 + 2 * b)
                ctx.kv_append(b, 0, 0, n, kraw, vraw, w)
        ctx.sync()
        xb = torch.full((B, HQ * HD), float("nan"), device=dev)
        ctx.attn_layer_batched(xb, torch.from_numpy(q).to(dev), torch.from_numpy(k).to(dev),
                               torch.from_numpy(v).to(dev), w, w, 0, list(range(B)),
                               [L - 1 for L in lens])
        ctx.sync()
        ctx.check_device_error()
        got = xb.cpu().numpy()
    assert np.all(np.isfinite(got))
    for b in checked:
        err = _maxabs(got[b], refs[b])
        assert err <= TOL_BF16_ABS, f"sequence {b} (length {lens[b]}): max-abs {err}"
