"""GPU parity of the decode path (q3a_attn_layer, q3a_attn_decode, batched,
partial + combine, KV append) against the CPU oracle and the golden vectors,
all through the C-ABI library.

Tolerances (stated in tests/shapes.py): fp32 cache normwise max relative
error <= 2e-4; bf16 cache max-abs <= 1e-2 against the reference fed the same
bf16-rounded K/V.
"""
import json
import os

import numpy as np
import pytest

import q3a_oracle as orc
import q3attn
from shapes import (EPS, HD, HKV, HQ, KV_DIM, KV_MUL, THETA, TOL_BF16_ABS, TOL_F32_NORMWISE,
                    elementwise_floor, normwise)

pytestmark = pytest.mark.gpu

GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def check_close(got, ref, bf16, what=""):
    if bf16:
        err = float(np.abs(np.float64(got) - np.float64(ref)).max())
        assert err <= TOL_BF16_ABS, f"{what}: max-abs {err}"
    else:
        err = normwise(got, ref)
        assert err <= TOL_F32_NORMWISE, f"{what}: normwise {err} (elementwise w/ floor " \
                                        f"{elementwise_floor(got, ref)})"
    return err


def oracle_inputs(seed, pos, max_seq, bf16, unit=True):
    if unit:
        qw = np.ones(HD, np.float32)
        kw = np.ones(HD, np.float32)
    else:
        qw = (1.0 + 0.25 * orc.randn(HD, seed, 6)).astype(np.float32)
        kw = (1.0 + 0.25 * orc.randn(HD, seed, 7)).astype(np.float32)
    kc, vc, _, _ = orc.make_cache(seed, 0, pos, HKV, HD, max_seq, kw=kw, bf16=bf16)
    q = orc.randn(HQ * HD, seed, 3)
    k = orc.randn(KV_DIM, seed, 4)
    v = orc.randn(KV_DIM, seed, 5)
    return kc, vc, q, k, v, qw, kw


def oracle_block(kc, vc, q, k, v, qw, kw, pos, max_seq, bf16):
    q = q.copy()
    k = k.copy()
    kc = kc.copy()
    vc = vc.copy()
    orc.rmsnorm_head(q, qw, HQ, HD, EPS)
    orc.rmsnorm_head(k, kw, HKV, HD, EPS)
    orc.rope(q, HQ, HD, pos, THETA)
    orc.rope(k, HKV, HD, pos, THETA)
    ks, vs = (orc.bf16_round(k), orc.bf16_round(v)) if bf16 else (k, v)
    kc[pos * KV_DIM:(pos + 1) * KV_DIM] = ks
    vc[pos * KV_DIM:(pos + 1) * KV_DIM] = vs
    xb = orc.attn_decode(q, kc, vc, 0, pos, HQ, KV_MUL, HD, KV_DIM, max_seq)
    return xb, q, k


def run_layer_host(ctx, kc, vc, q, k, v, qw, kw, pos, layer=0):
    if pos > 0:
        ctx.kv_load(0, layer, 0, pos, kc[: pos * KV_DIM], vc[: pos * KV_DIM])
    xb = np.zeros(HQ * HD, np.float32)
    qq, kk = q.copy(), k.copy()
    ctx.attn_layer(xb, qq, kk, v, qw, kw, layer, pos)
    return xb, qq, kk


@pytest.fixture(scope="module")
def ctx_f32():
    with q3attn.Context(n_layers=2, max_seq=8256, kv_dtype=q3attn.KV_F32) as c:
        yield c


@pytest.fixture(scope="module")
def ctx_bf16():
    with q3attn.Context(n_layers=2, max_seq=8256, kv_dtype=q3attn.KV_BF16) as c:
        yield c


@pytest.mark.parametrize("pos", [0, 1, 63, 64, 65, 127, 1023, 1024])
@pytest.mark.parametrize("bf16", [False, True])
def test_attn_layer_matches_oracle(ctx_f32, ctx_bf16, pos, bf16):
    ctx = ctx_bf16 if bf16 else ctx_f32
    max_seq = pos + 1
    kc, vc, q, k, v, qw, kw = oracle_inputs(4000 + pos, pos, max_seq, bf16, unit=(pos % 2 == 0))
    xr, qr, kr = oracle_block(kc, vc, q, k, v, qw, kw, pos, max_seq, bf16)
    xb, qq, kk = run_layer_host(ctx, kc, vc, q, k, v, qw, kw, pos)
    check_close(xb, xr, bf16, f"xb pos {pos}")
    # q and k are normalised and rotated in place, as the reference does
    assert normwise(qq, qr) < 1e-6
    assert normwise(kk, kr) < 1e-6
    ctx.check_device_error()


def test_attn_layer_matches_golden_vectors(ctx_f32, ctx_bf16):
    """Straight against the outputs of the reference's own compiled code."""
    meta = json.load(open(os.path.join(GOLD, "manifest.json")))
    cases = meta["files"]["decode_block.npz"]["cases"]
    g = np.load(os.path.join(GOLD, "decode_block.npz"))
    for i, case in enumerate(cases):
        bf16 = case["bf16"]
        ctx = ctx_bf16 if bf16 else ctx_f32
        pos = case["pos"]
        kc, vc, q, k, v, qw, kw = oracle_inputs(case["seed"], pos, case["max_seq"], bf16,
                                                unit=case["unit_gains"])
        xb, qq, kk = run_layer_host(ctx, kc, vc, q, k, v, qw, kw, pos)
        check_close(xb, g[f"c{i}_xb_mc"], bf16, f"golden case {i}")
        check_close(xb, g[f"c{i}_xb_la"], bf16, f"golden case {i} (launch_attn)")
        assert normwise(qq, g[f"c{i}_q_out"]) < 1e-6
        assert normwise(kk, g[f"c{i}_k_out"]) < 1e-6


@pytest.mark.parametrize("bf16", [False, True])
def test_attn_layer_8k(ctx_f32, ctx_bf16, bf16):
    ctx = ctx_bf16 if bf16 else ctx_f32
    pos = 8191
    kc, vc, q, k, v, qw, kw = oracle_inputs(77, pos, pos + 1, bf16)
    xr, _, _ = oracle_block(kc, vc, q, k, v, qw, kw, pos, pos + 1, bf16)
    xb, _, _ = run_layer_host(ctx, kc, vc, q, k, v, qw, kw, pos, layer=1)
    check_close(xb, xr, bf16, "8K")


def test_device_pointer_mode_matches_host_mode():
    import torch
    pos = 300
    kc, vc, q, k, v, qw, kw = oracle_inputs(5, pos, pos + 1, False, unit=False)
    xr, qr, kr = oracle_block(kc, vc, q, k, v, qw, kw, pos, pos + 1, False)
    with q3attn.Context(n_layers=1, max_seq=1024, ptr_mode=q3attn.PTR_DEVICE) as ctx:
        dev = torch.device("cuda:0")
        t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(dev)
        ctx.kv_load(0, 0, 0, pos, t(kc[: pos * KV_DIM]), t(vc[: pos * KV_DIM]))
        xb = torch.zeros(HQ * HD, device=dev)
        qd, kd = t(q), t(k)
        ctx.attn_layer(xb, qd, kd, t(v), t(qw), t(kw), 0, pos)
        ctx.sync()
        check_close(xb.cpu().numpy(), xr, False, "device mode")
        assert normwise(qd.cpu().numpy(), qr) < 1e-6
        assert normwise(kd.cpu().numpy(), kr) < 1e-6


@pytest.mark.parametrize("mode", [q3attn.PTR_HOST, q3attn.PTR_DEVICE])
def test_launch_attn_signature(mode):
    """q3a_attn_decode over a caller-owned position-major cache, layer 1 of 2."""
    import torch
    max_seq, pos = 700, 650
    kc0, vc0, _, _ = orc.make_cache(9, 0, max_seq, HKV, HD, max_seq)
    kc1, vc1, _, _ = orc.make_cache(9, 1, max_seq, HKV, HD, max_seq)
    kc = np.concatenate([kc0, kc1])
    vc = np.concatenate([vc0, vc1])
    q = orc.randn(HQ * HD, 9, 40)
    loff = max_seq * KV_DIM
    xr = orc.attn_decode(q, kc, vc, loff, pos, HQ, KV_MUL, HD, KV_DIM, max_seq)
    with q3attn.Context(n_layers=1, max_seq=64, ptr_mode=mode) as ctx:
        if mode == q3attn.PTR_HOST:
            xb = np.zeros(HQ * HD, np.float32)
            ctx.attn_decode(xb, q, kc, vc, None, loff, pos, HQ, KV_MUL, HD, KV_DIM, max_seq)
            got = xb
        else:
            dev = torch.device("cuda:0")
            xb = torch.zeros(HQ * HD, device=dev)
            ctx.attn_decode(xb, torch.from_numpy(q).to(dev), torch.from_numpy(kc).to(dev),
                            torch.from_numpy(vc).to(dev), None, loff, pos, HQ, KV_MUL, HD,
                            KV_DIM, max_seq)
            ctx.sync()
            got = xb.cpu().numpy()
    check_close(got, xr, False, "launch_attn")


@pytest.mark.parametrize("bf16", [False, True])
def test_batched_ragged_matches_oracle(bf16):
    lens = [1, 64, 100, 701, 2000, 65]
    n_seqs = len(lens) + 1
    with q3attn.Context(n_layers=1, max_seq=2048, n_seqs=n_seqs,
                        kv_dtype=q3attn.KV_BF16 if bf16 else q3attn.KV_F32) as ctx:
        refs, qs, ks, vs = [], [], [], []
        qw = np.ones(HD, np.float32)
        kw = np.ones(HD, np.float32)
        seq_ids = [n_seqs - 1 - i for i in range(len(lens))]  # slots in reverse order
        pos = [L - 1 for L in lens]
        for i, L in enumerate(lens):
            kc, vc, q, k, v, _, _ = oracle_inputs(600 + i, pos[i], L, bf16)
            if pos[i] > 0:
                ctx.kv_load(seq_ids[i], 0, 0, pos[i], kc[: pos[i] * KV_DIM], vc[: pos[i] * KV_DIM])
            xr, _, _ = oracle_block(kc, vc, q, k, v, qw, kw, pos[i], L, bf16)
            refs.append(xr)
            qs.append(q)
            ks.append(k)
            vs.append(v)
        xb = np.zeros((len(lens), HQ * HD), np.float32)
        qa, ka, va = np.stack(qs), np.stack(ks), np.stack(vs)
        ctx.attn_layer_batched(xb, qa, ka, va, qw, kw, 0, seq_ids, pos)
        for i in range(len(lens)):
            check_close(xb[i], refs[i], bf16, f"seq {i} len {lens[i]}")
        # the appended rows are in the cache of the right slot
        kr = np.zeros(KV_DIM, np.float32)
        vr = np.zeros(KV_DIM, np.float32)
        ctx.kv_read(seq_ids[3], 0, pos[3], 1, kr, vr)
        assert normwise(vr, orc.bf16_round(vs[3]) if bf16 else vs[3]) == 0.0


@pytest.mark.parametrize("bf16", [False, True])
def test_partial_and_combine(bf16):
    """Sequence-shard steps: per-chunk (o, lse) then the log-sum-exp merge."""
    L = 5000
    with q3attn.Context(n_layers=1, max_seq=L, kv_dtype=q3attn.KV_BF16 if bf16 else q3attn.KV_F32) as ctx:
        kc, vc, _, _ = orc.make_cache(31, 0, L, HKV, HD, L, bf16=bf16)
        ctx.kv_load(0, 0, 0, L, kc, vc)
        q = orc.randn(HQ * HD, 31, 9)
        xr = orc.attn_decode(q, kc, vc, 0, L - 1, HQ, KV_MUL, HD, KV_DIM, L)
        cuts = [0, 1, 1250, 2500, 2500, 3777, L]
        o = np.zeros((len(cuts) - 1, HQ * HD), np.float32)
        lse = np.zeros((len(cuts) - 1, HQ), np.float32)
        for j, (a, b) in enumerate(zip(cuts[:-1], cuts[1:])):
            ctx.attn_partial(o[j], lse[j], q, 0, 0, a, b)
            if b > a:
                ro, rl = orc.attn_partial(q, kc, vc, 0, a, b, HQ, KV_MUL, HD, KV_DIM)
                check_close(o[j], ro, bf16, f"chunk {j}")
                assert np.abs(lse[j] - rl).max() < 1e-3
            else:
                assert np.all(lse[j] == -np.inf)
        xb = np.zeros(HQ * HD, np.float32)
        ctx.lse_combine(xb, o, lse, len(cuts) - 1)
        check_close(xb, xr, bf16, "combined")


@pytest.mark.parametrize("bf16", [False, True])
def test_kv_append_matches_oracle(bf16):
    n, pos0 = 300, 17
    with q3attn.Context(n_layers=3, max_seq=512, kv_dtype=q3attn.KV_BF16 if bf16 else q3attn.KV_F32) as ctx:
        kraw = orc.randn(n * KV_DIM, 3, 1)
        vraw = orc.randn(n * KV_DIM, 3, 2)
        kw = (1.0 + 0.25 * orc.randn(HD, 3, 7)).astype(np.float32)
        ctx.kv_append(0, 2, pos0, n, kraw, vraw, kw)
        kr = np.zeros(n * KV_DIM, np.float32)
        vr = np.zeros(n * KV_DIM, np.float32)
        ctx.kv_read(0, 2, pos0, n, kr, vr)
        kref = np.zeros(n * KV_DIM, np.float32)
        for t in range(n):
            row = kraw[t * KV_DIM:(t + 1) * KV_DIM].copy()
            orc.rmsnorm_head(row, kw, HKV, HD, EPS)
            orc.rope(row, HKV, HD, pos0 + t, THETA)
            kref[t * KV_DIM:(t + 1) * KV_DIM] = row
        if bf16:
            kref = orc.bf16_round(kref)
            assert np.array_equal(vr, orc.bf16_round(vraw))
            assert np.abs(kr - kref).max() <= 2 ** -7  # one bf16 ulp at |k| < 2
        else:
            assert np.array_equal(vr, vraw)
            assert normwise(kr, kref) < 1e-6
        # other layers untouched
        z = np.ones(KV_DIM, np.float32)
        ctx.kv_read(0, 1, pos0, 1, z, z.copy())
        assert np.all(z == 0)


def test_randn_matches_oracle_stream():
    import torch
    n = 1 << 16
    with q3attn.Context(n_layers=1, max_seq=64) as ctx:
        d = torch.empty(n, device="cuda:0")
        ctx.randn(d, q3attn.OUT_F32, n, 1234, 5, 1000)
        ctx.sync()
        got = d.cpu().numpy()
    ref = orc.randn(n, 1234, 5, 1000)
    assert np.abs(got - ref).max() < 1e-5


def test_errors_are_reported_not_fatal(ctx_f32):
    xb = np.zeros(HQ * HD, np.float32)
    q = np.zeros(HQ * HD, np.float32)
    k = np.zeros(KV_DIM, np.float32)
    w = np.ones(HD, np.float32)
    with pytest.raises(q3attn.Q3AError) as e:
        ctx_f32.attn_layer(xb, q, k, k, w, w, 0, 10 ** 6)
    assert e.value.code == q3attn.ERR_INVALID
    with pytest.raises(q3attn.Q3AError):
        ctx_f32.attn_layer(xb, q, k, k, w, w, 5, 0)
    # the context is still usable afterwards
    ctx_f32.attn_layer(xb, q + 1.0, k + 1.0, k, w, w, 0, 0)
    ctx_f32.check_device_error()


def test_launch_count_advances(ctx_f32):
    n0 = ctx_f32.launch_count()
    xb = np.zeros(HQ * HD, np.float32)
    q = orc.randn(HQ * HD, 1, 1)
    k = orc.randn(KV_DIM, 1, 2)
    w = np.ones(HD, np.float32)
    ctx_f32.attn_layer(xb, q, k, k, w, w, 0, 3)
    assert ctx_f32.launch_count() == n0 + 1  # the whole block is one kernel


@pytest.mark.parametrize("bf16", [False, True])
def test_batched_linear_schedule(bf16):
    """More (sequence, kv head) groups than SMs: the linear unit schedule,
    where CTAs cross group boundaries, must give the same results."""
    rng = np.random.default_rng(5)
    n = 20                                  # 160 groups > 148 SMs
    lens = [int(x) for x in rng.integers(1, 300, size=n)]
    lens[0], lens[1] = 1, 299
    with q3attn.Context(n_layers=1, max_seq=320, n_seqs=n,
                        kv_dtype=q3attn.KV_BF16 if bf16 else q3attn.KV_F32) as ctx:
        qw = np.ones(HD, np.float32)
        refs, qs, ks, vs = [], [], [], []
        pos = [L - 1 for L in lens]
        for i, L in enumerate(lens):
            kc, vc, q, k, v, _, _ = oracle_inputs(900 + i, pos[i], L, bf16)
            if pos[i] > 0:
                ctx.kv_load(i, 0, 0, pos[i], kc[: pos[i] * KV_DIM], vc[: pos[i] * KV_DIM])
            refs.append(oracle_block(kc, vc, q, k, v, qw, qw, pos[i], L, bf16)[0])
            qs.append(q)
            ks.append(k)
            vs.append(v)
        xb = np.zeros((n, HQ * HD), np.float32)
        ctx.attn_layer_batched(xb, np.stack(qs), np.stack(ks), np.stack(vs), qw, qw, 0,
                               list(range(n)), pos)
        for i in range(n):
            check_close(xb[i], refs[i], bf16, f"seq {i} len {lens[i]}")
        ctx.check_device_error()
