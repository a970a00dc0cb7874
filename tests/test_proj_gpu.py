"""GPU parity of q3a_attn_layer_proj: the q/k/v projections with fp16
weights (mm_f16, qwen3-8b/cpu/main.c:1206-1213 called at 1315-1317) fused
with the block's QK-RMSNorm, RoPE and KV append, then the decode attention,
against the CPU oracle (orc_mm_f16, pinned bit for bit to the reference's own
mm_f16 by tests/test_oracle_golden.py) and the oracle block.

Tolerances: the kernel adds each row's products per thread, over a warp,
then over eight warps in order, where the reference adds them in one
sequential fp32 sum, so q, k and v agree to fp32 rounding: normwise max
relative error <= 1e-5.  xb: the decode tolerances of
tests/shapes.py (fp32 cache normwise 2e-4, bf16 cache max-abs 1e-2).
"""
import numpy as np
import pytest

import q3a_oracle as orc
import q3attn
from shapes import EPS, HD, HKV, HQ, KV_DIM, KV_MUL, THETA, TOL_BF16_ABS, TOL_F32_NORMWISE, normwise

pytestmark = pytest.mark.gpu

DIM = 4096          # Qwen3-8B model width
TOL_PROJ = 1e-5     # q, k, v: normwise against the sequential fp32 sums


def _weights(seed):
    wq = orc.proj_weights(seed, HQ * HD, DIM)
    wk = orc.proj_weights(seed + 1, KV_DIM, DIM)
    wv = orc.proj_weights(seed + 2, KV_DIM, DIM)
    return wq, wk, wv


def _oracle_step(x, wq, wk, wv, qw, kw, kc, vc, pos, max_seq, bf16):
    """The reference block from the layer input: projections, norm, RoPE,
    cache write at pos (kc, vc updated in place), attention over 0..pos."""
    q = orc.mm_f16(x, wq)
    k = orc.mm_f16(x, wk)
    v = orc.mm_f16(x, wv)
    orc.rmsnorm_head(q, qw, HQ, HD, EPS)
    orc.rmsnorm_head(k, kw, HKV, HD, EPS)
    orc.rope(q, HQ, HD, pos, THETA)
    orc.rope(k, HKV, HD, pos, THETA)
    ks, vs = (orc.bf16_round(k), orc.bf16_round(v)) if bf16 else (k, v)
    kc[pos * KV_DIM:(pos + 1) * KV_DIM] = ks
    vc[pos * KV_DIM:(pos + 1) * KV_DIM] = vs
    xb = orc.attn_decode(q, kc, vc, 0, pos, HQ, KV_MUL, HD, KV_DIM, max_seq)
    return xb, q, k, v


def _check_xb(got, ref, bf16, what):
    if bf16:
        err = float(np.abs(np.float64(got) - np.float64(ref)).max())
        assert err <= TOL_BF16_ABS, f"{what}: max-abs {err}"
    else:
        err = normwise(got, ref)
        assert err <= TOL_F32_NORMWISE, f"{what}: normwise {err}"


@pytest.fixture(scope="module")
def weights():
    import torch
    dev = torch.device("cuda:0")
    wq, wk, wv = _weights(7100)
    dw = [torch.from_numpy(w.view(np.uint16).astype(np.int16)).view(torch.float16).to(dev)
          for w in (wq, wk, wv)]
    return (wq, wk, wv), dw


@pytest.mark.parametrize("bf16", [False, True])
@pytest.mark.parametrize("det", [False, True])
def test_proj_steps_match_oracle(weights, bf16, det):
    """Consecutive tokens over two layers (projection of layer l, decode of
    layer l, then layer l + 1, ...), each step against the oracle block.  The
    decode after the projection streams the rows below pos before its
    dependency wait in the balanced schedule (det False); the deterministic
    schedule waits first."""
    import torch
    dev = torch.device("cuda:0")
    (wq, wk, wv), (dq, dk, dv) = weights
    n_layers, pos0, steps = 2, 1021, 4
    max_seq = pos0 + steps
    qw = (1.0 + 0.25 * orc.randn(HD, 7200, 6)).astype(np.float32)
    kw = (1.0 + 0.25 * orc.randn(HD, 7200, 7)).astype(np.float32)
    caches = [orc.make_cache(7300 + l, l, pos0, HKV, HD, max_seq, kw=kw, bf16=bf16)[:2]
              for l in range(n_layers)]
    kv = q3attn.KV_BF16 if bf16 else q3attn.KV_F32
    with q3attn.Context(n_layers=n_layers, max_seq=max_seq, kv_dtype=kv,
                        ptr_mode=q3attn.PTR_DEVICE) as ctx:
        ctx.set_deterministic(det)
        for l, (kc, vc) in enumerate(caches):
            ctx.kv_load(0, l, 0, pos0, torch.from_numpy(kc[:pos0 * KV_DIM]).to(dev),
                        torch.from_numpy(vc[:pos0 * KV_DIM]).to(dev))
        dqw = torch.from_numpy(qw).to(dev)
        dkw = torch.from_numpy(kw).to(dev)
        for s in range(steps):
            pos = pos0 + s
            for l in range(n_layers):
                x = orc.randn(DIM, 7400 + 10 * s + l, 8)
                kc, vc = caches[l]
                xr, qr, kr, vr = _oracle_step(x, wq, wk, wv, qw, kw, kc, vc, pos, max_seq, bf16)
                xb = torch.full((HQ * HD,), float("nan"), device=dev)
                q = torch.full((HQ * HD,), float("nan"), device=dev)
                k = torch.full((KV_DIM,), float("nan"), device=dev)
                v = torch.full((KV_DIM,), float("nan"), device=dev)
                ctx.attn_layer_proj(xb, q, k, v, torch.from_numpy(x).to(dev), dq, dk, dv,
                                    dqw, dkw, l, pos)
                ctx.sync()
                ctx.check_device_error()
                what = f"step {s} layer {l} (bf16 {bf16}, det {det})"
                assert normwise(q.cpu().numpy(), qr) <= TOL_PROJ, what + ": q"
                assert normwise(k.cpu().numpy(), kr) <= TOL_PROJ, what + ": k"
                assert normwise(v.cpu().numpy(), vr) <= TOL_PROJ, what + ": v"
                _check_xb(xb.cpu().numpy(), xr, bf16, what)
        # the appended rows, read back from the paged cache
        for l, (kc, vc) in enumerate(caches):
            rk = torch.zeros(steps * KV_DIM, device=dev)
            rv = torch.zeros(steps * KV_DIM, device=dev)
            ctx.kv_read(0, l, pos0, steps, rk, rv)
            ctx.sync()
            tol = 1e-2 if bf16 else 1e-5
            assert normwise(rk.cpu().numpy(), kc[pos0 * KV_DIM:]) <= tol
            assert normwise(rv.cpu().numpy(), vc[pos0 * KV_DIM:]) <= tol


def test_proj_first_token_and_optional_outputs(weights):
    """pos 0 (nothing in the cache before the token) with k and v outputs
    omitted; repeated calls at one position give the same result."""
    import torch
    dev = torch.device("cuda:0")
    (wq, wk, wv), (dq, dk, dv) = weights
    qw = np.ones(HD, np.float32)
    kw = np.ones(HD, np.float32)
    kc = np.zeros(KV_DIM, np.float32)
    vc = np.zeros(KV_DIM, np.float32)
    x = orc.randn(DIM, 7500, 8)
    xr, qr, _, _ = _oracle_step(x, wq, wk, wv, qw, kw, kc, vc, 0, 1, False)
    with q3attn.Context(n_layers=1, max_seq=64, ptr_mode=q3attn.PTR_DEVICE) as ctx:
        outs = []
        for _ in range(2):
            xb = torch.zeros(HQ * HD, device=dev)
            q = torch.zeros(HQ * HD, device=dev)
            ctx.attn_layer_proj(xb, q, None, None, torch.from_numpy(x).to(dev), dq, dk, dv,
                                torch.from_numpy(qw).to(dev), torch.from_numpy(kw).to(dev), 0, 0)
            ctx.sync()
            ctx.check_device_error()
            outs.append(xb.cpu().numpy())
            assert normwise(q.cpu().numpy(), qr) <= TOL_PROJ
            _check_xb(outs[-1], xr, False, "pos 0")
        assert np.array_equal(outs[0], outs[1])


def test_proj_rejects_bad_arguments(weights):
    import torch
    dev = torch.device("cuda:0")
    _, (dq, dk, dv) = weights
    t = lambda n: torch.zeros(n, device=dev)  # noqa: E731
    with q3attn.Context(n_layers=1, max_seq=64) as host_ctx:  # host-pointer context
        with pytest.raises(q3attn.Q3AError):
            host_ctx.attn_layer_proj(t(HQ * HD), t(HQ * HD), None, None, t(DIM), dq, dk, dv,
                                     t(HD), t(HD), 0, 0)
    with q3attn.Context(n_layers=1, max_seq=64, ptr_mode=q3attn.PTR_DEVICE) as ctx:
        with pytest.raises(q3attn.Q3AError):  # dim not a multiple of 8
            ctx.attn_layer_proj(t(HQ * HD), t(HQ * HD), None, None, t(1004), dq, dk, dv,
                                t(HD), t(HD), 0, 0)
        with pytest.raises(q3attn.Q3AError):  # dim above 8192
            ctx.attn_layer_proj(t(HQ * HD), t(HQ * HD), None, None, t(8200), dq, dk, dv,
                                t(HD), t(HD), 0, 0)
        with pytest.raises(q3attn.Q3AError):  # pos outside the cache
            ctx.attn_layer_proj(t(HQ * HD), t(HQ * HD), None, None, t(DIM), dq, dk, dv,
                                t(HD), t(HD), 0, 64)
        with pytest.raises(q3attn.Q3AError):  # misaligned input
            ctx.attn_layer_proj(t(HQ * HD), t(HQ * HD), None, None, t(DIM + 1)[1:], dq, dk,
                                dv, t(HD), t(HD), 0, 0)


@pytest.mark.parametrize("dim", [4096, 5120, 2560])
def test_qkv_proj_alone_matches_oracle(weights, dim):
    """q3a_qkv_proj: q, k, v and the appended cache row, no attention.  Widths
    of Qwen3-8B (4096), -14B/-32B (5120: 640 pieces of 16 bytes, three rows
    per stage) and -4B (2560: six rows per stage)."""
    import torch
    dev = torch.device("cuda:0")
    if dim == DIM:
        (wq, wk, wv), (dq, dk, dv) = weights
    else:
        wq = orc.proj_weights(7800, HQ * HD, dim)
        wk = orc.proj_weights(7801, KV_DIM, dim)
        wv = orc.proj_weights(7802, KV_DIM, dim)
        dq, dk, dv = [torch.from_numpy(w.view(np.uint16).astype(np.int16)).view(torch.float16)
                      .to(dev) for w in (wq, wk, wv)]
    qw = (1.0 + 0.25 * orc.randn(HD, 7600, 6)).astype(np.float32)
    kw = (1.0 + 0.25 * orc.randn(HD, 7600, 7)).astype(np.float32)
    for bf16 in (False, True):
        kv = q3attn.KV_BF16 if bf16 else q3attn.KV_F32
        with q3attn.Context(n_layers=3, max_seq=4096, kv_dtype=kv,
                            ptr_mode=q3attn.PTR_DEVICE) as ctx:
            for layer, pos in ((2, 4095), (0, 17)):
                x = orc.randn(dim, 7700 + pos, 8)
                q_r = orc.mm_f16(x, wq)
                k_r = orc.mm_f16(x, wk)
                v_r = orc.mm_f16(x, wv)
                orc.rmsnorm_head(q_r, qw, HQ, HD, EPS)
                orc.rmsnorm_head(k_r, kw, HKV, HD, EPS)
                orc.rope(q_r, HQ, HD, pos, THETA)
                orc.rope(k_r, HKV, HD, pos, THETA)
                q = torch.zeros(HQ * HD, device=dev)
                k = torch.zeros(KV_DIM, device=dev)
                v = torch.zeros(KV_DIM, device=dev)
                ctx.qkv_proj(q, k, v, torch.from_numpy(x).to(dev), dq, dk, dv,
                             torch.from_numpy(qw).to(dev), torch.from_numpy(kw).to(dev), layer, pos)
                rk = torch.zeros(KV_DIM, device=dev)
                rv = torch.zeros(KV_DIM, device=dev)
                ctx.kv_read(0, layer, pos, 1, rk, rv)
                ctx.sync()
                ctx.check_device_error()
                assert normwise(q.cpu().numpy(), q_r) <= TOL_PROJ
                assert normwise(k.cpu().numpy(), k_r) <= TOL_PROJ
                assert normwise(v.cpu().numpy(), v_r) <= TOL_PROJ
                tol = 1e-2 if bf16 else 1e-5
                assert normwise(rk.cpu().numpy(), k_r) <= tol
                assert normwise(rv.cpu().numpy(), v_r) <= tol


def test_qkv_proj_sharded_context(weights):
    """A context holding KV heads [2, 5) projects only their rows: q heads
    8..19 and KV heads 2..4 at their places in the full-width outputs (the
    other entries untouched), and appends only its heads' rows."""
    import torch
    dev = torch.device("cuda:0")
    (wq, wk, wv), (dq, dk, dv) = weights
    b, n = 2, 3
    qw = (1.0 + 0.25 * orc.randn(HD, 7900, 6)).astype(np.float32)
    kw = (1.0 + 0.25 * orc.randn(HD, 7900, 7)).astype(np.float32)
    pos, layer = 777, 1
    x = orc.randn(DIM, 7901, 8)
    q_r = orc.mm_f16(x, wq)
    k_r = orc.mm_f16(x, wk)
    v_r = orc.mm_f16(x, wv)
    orc.rmsnorm_head(q_r, qw, HQ, HD, EPS)
    orc.rmsnorm_head(k_r, kw, HKV, HD, EPS)
    orc.rope(q_r, HQ, HD, pos, THETA)
    orc.rope(k_r, HKV, HD, pos, THETA)
    with q3attn.Context(n_layers=2, max_seq=1024, ptr_mode=q3attn.PTR_DEVICE,
                        kv_head_begin=b, kv_head_count=n) as ctx:
        q = torch.full((HQ * HD,), 7.0, device=dev)
        k = torch.full((KV_DIM,), 7.0, device=dev)
        v = torch.full((KV_DIM,), 7.0, device=dev)
        ctx.qkv_proj(q, k, v, torch.from_numpy(x).to(dev), dq, dk, dv,
                     torch.from_numpy(qw).to(dev), torch.from_numpy(kw).to(dev), layer, pos)
        rk = torch.zeros(n * HD, device=dev)
        rv = torch.zeros(n * HD, device=dev)
        ctx.kv_read(0, layer, pos, 1, rk, rv)
        ctx.sync()
        ctx.check_device_error()
        qh, kh, vh = q.cpu().numpy(), k.cpu().numpy(), v.cpu().numpy()
    qs = slice(b * KV_MUL * HD, (b + n) * KV_MUL * HD)
    ks = slice(b * HD, (b + n) * HD)
    assert normwise(qh[qs], q_r[qs]) <= TOL_PROJ
    assert normwise(kh[ks], k_r[ks]) <= TOL_PROJ
    assert normwise(vh[ks], v_r[ks]) <= TOL_PROJ
    for a in (np.delete(qh, np.r_[qs]), np.delete(kh, np.r_[ks]), np.delete(vh, np.r_[ks])):
        assert (a == 7.0).all()
    assert normwise(rk.cpu().numpy(), k_r[ks]) <= 1e-5
    assert normwise(rv.cpu().numpy(), v_r[ks]) <= 1e-5
