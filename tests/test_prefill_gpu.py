"""GPU parity of the causal prefill (tcgen05 kernel) against the CPU oracle.

The reference defines prefill as its decode step run once per prompt
position (qwen3-8b/cpu/main.c:1481-1499); the oracle does exactly that
(orc_prefill_causal) on the same bf16-rounded Q, K, V the kernel reads, and
the bf16 tolerance (max-abs 1e-2) applies.
"""
import json
import os

import numpy as np
import pytest

import q3a_oracle as orc
import q3attn
from shapes import EPS, HD, HKV, HQ, KV_DIM, KV_MUL, THETA, TOL_BF16_ABS

pytestmark = pytest.mark.gpu

GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def _torch():
    import torch
    return torch


def prepped_q(seed, pos0, S, qw=None):
    """Raw q rows -> QK-RMSNorm -> RoPE at pos0+s (oracle), then bf16 values."""
    if qw is None:
        qw = np.ones(HD, np.float32)
    qraw = orc.randn(S * HQ * HD, seed, 3)
    q = qraw.copy()
    for s in range(S):
        row = q[s * HQ * HD:(s + 1) * HQ * HD]
        orc.rmsnorm_head(row, qw, HQ, HD, EPS)
        orc.rope(row, HQ, HD, pos0 + s, THETA)
    return qraw, orc.bf16_round(q)


def max_abs(a, b):
    return float(np.abs(np.float64(a) - np.float64(b)).max())


@pytest.mark.parametrize("pos0,S", [(0, 128), (0, 1), (0, 64), (0, 200), (64, 300), (37, 129)])
def test_prefill_attn_matches_oracle(pos0, S):
    torch = _torch()
    dev = torch.device("cuda:0")
    n_tok = pos0 + S
    kc, vc, _, _ = orc.make_cache(700 + S, 0, n_tok, HKV, HD, n_tok, bf16=True)
    _, q = prepped_q(700 + S, pos0, S)
    ref = orc.prefill_causal(q, kc, vc, pos0, S, HQ, KV_MUL, HD, KV_DIM, n_tok)
    with q3attn.Context(n_layers=2, max_seq=1024, kv_dtype=q3attn.KV_BF16,
                        ptr_mode=q3attn.PTR_DEVICE) as ctx:
        ctx.kv_load(0, 1, 0, n_tok, torch.from_numpy(kc).to(dev), torch.from_numpy(vc).to(dev))
        qb = torch.from_numpy(q).to(dev).to(torch.bfloat16)
        out = torch.full((S, HQ * HD), float("nan"), device=dev)
        ctx.prefill_attn(out, q3attn.OUT_F32, qb, 0, 1, pos0, S)
        ctx.sync()
        ctx.check_device_error()
        got = out.cpu().numpy().reshape(-1)
    assert np.all(np.isfinite(got))
    err = max_abs(got, ref)
    assert err <= TOL_BF16_ABS, f"prefill pos0={pos0} S={S}: max-abs {err}"


def test_prefill_attn_bf16_output_and_host_mode():
    torch = _torch()
    pos0, S = 0, 160
    kc, vc, _, _ = orc.make_cache(31, 0, S, HKV, HD, S, bf16=True)
    _, q = prepped_q(31, pos0, S)
    ref = orc.prefill_causal(q, kc, vc, pos0, S, HQ, KV_MUL, HD, KV_DIM, S)
    with q3attn.Context(n_layers=1, max_seq=256, kv_dtype=q3attn.KV_BF16) as ctx:  # host mode
        ctx.kv_load(0, 0, 0, S, kc, vc)
        qb = torch.from_numpy(q).to(torch.bfloat16).contiguous()   # host bf16
        out = torch.zeros((S, HQ * HD), dtype=torch.bfloat16)
        ctx.prefill_attn(out, q3attn.OUT_BF16, qb, 0, 0, pos0, S)
        got = out.float().numpy().reshape(-1)
    assert max_abs(got, ref) <= TOL_BF16_ABS + 1e-2 * 0  # bf16 output rounding included


def test_prefill_full_path_matches_oracle():
    """q3a_prefill: raw q/k/v -> norm + RoPE -> append -> causal attention;
    then the cache holds the rows the oracle builds."""
    torch = _torch()
    dev = torch.device("cuda:0")
    pos0, S = 0, 333
    seed = 77
    qw = (1.0 + 0.25 * orc.randn(HD, seed, 6)).astype(np.float32)
    kw = (1.0 + 0.25 * orc.randn(HD, seed, 7)).astype(np.float32)
    qraw, q = prepped_q(seed, pos0, S, qw)
    kc, vc, kraw, vraw = orc.make_cache(seed, 0, S, HKV, HD, S, kw=kw, bf16=True)
    ref = orc.prefill_causal(q, kc, vc, pos0, S, HQ, KV_MUL, HD, KV_DIM, S)
    with q3attn.Context(n_layers=1, max_seq=512, kv_dtype=q3attn.KV_BF16,
                        ptr_mode=q3attn.PTR_DEVICE) as ctx:
        t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(dev)
        out = torch.zeros((S, HQ * HD), device=dev)
        ctx.prefill(out, q3attn.OUT_F32, t(qraw), t(kraw), t(vraw), t(qw), t(kw), 0, 0, pos0, S)
        kr = torch.zeros(S * KV_DIM, device=dev)
        vr = torch.zeros(S * KV_DIM, device=dev)
        ctx.kv_read(0, 0, 0, S, kr, vr)
        ctx.sync()
        got = out.cpu().numpy().reshape(-1)
        kr = kr.cpu().numpy()
        vr = vr.cpu().numpy()
    assert np.array_equal(vr, vc[: S * KV_DIM])
    assert np.abs(kr - kc[: S * KV_DIM]).max() <= 2 ** -7  # one bf16 ulp at |k| < 2
    err = max_abs(got, ref)
    assert err <= TOL_BF16_ABS, f"full prefill: max-abs {err}"


def test_prefill_matches_golden_vectors():
    """Against outputs of the reference's own compiled functions."""
    torch = _torch()
    dev = torch.device("cuda:0")
    meta = json.load(open(os.path.join(GOLD, "manifest.json")))["files"]["prefill.npz"]["cases"]
    g = np.load(os.path.join(GOLD, "prefill.npz"))
    heads = g["heads"]
    for i, case in enumerate(meta):
        seed, pos0, S = case["seed"], case["pos0"], case["S"]
        n_tok = pos0 + S
        kc, vc, _, _ = orc.make_cache(seed, 0, n_tok, HKV, HD, n_tok, bf16=True)
        _, q = prepped_q(seed, pos0, S)
        with q3attn.Context(n_layers=1, max_seq=256, kv_dtype=q3attn.KV_BF16,
                            ptr_mode=q3attn.PTR_DEVICE) as ctx:
            ctx.kv_load(0, 0, 0, n_tok, torch.from_numpy(kc).to(dev), torch.from_numpy(vc).to(dev))
            out = torch.zeros((S, HQ * HD), device=dev)
            ctx.prefill_attn(out, q3attn.OUT_F32, torch.from_numpy(q).to(dev).to(torch.bfloat16),
                             0, 0, pos0, S)
            ctx.sync()
            got = out.cpu().numpy().reshape(S, HQ, HD)[:, heads, :]
        assert max_abs(got, g[f"p{i}_out_heads"]) <= TOL_BF16_ABS, f"golden prefill case {i}"


def test_prefill_2048_matches_oracle_sampled_rows():
    """configs[2] size: S = 2048 against the oracle on a sample of rows."""
    torch = _torch()
    dev = torch.device("cuda:0")
    S = 2048
    kc, vc, _, _ = orc.make_cache(2048, 0, S, HKV, HD, S, bf16=True)
    _, q = prepped_q(2048, 0, S)
    rows = np.array([0, 1, 63, 64, 127, 128, 1000, 1500, 2046, 2047])
    with q3attn.Context(n_layers=1, max_seq=S, kv_dtype=q3attn.KV_BF16,
                        ptr_mode=q3attn.PTR_DEVICE) as ctx:
        ctx.kv_load(0, 0, 0, S, torch.from_numpy(kc).to(dev), torch.from_numpy(vc).to(dev))
        out = torch.zeros((S, HQ * HD), device=dev)
        ctx.prefill_attn(out, q3attn.OUT_F32, torch.from_numpy(q).to(dev).to(torch.bfloat16),
                         0, 0, 0, S)
        ctx.sync()
        ctx.check_device_error()
        got = out.cpu().numpy()
    qd = HQ * HD
    for r in rows:
        ref = orc.attn_decode(q[r * qd:(r + 1) * qd].copy(), kc, vc, 0, int(r), HQ, KV_MUL, HD,
                              KV_DIM, S)
        assert max_abs(got[r], ref) <= TOL_BF16_ABS, f"row {r}"


@pytest.mark.parametrize("nh,pos0,S", [(1, 0, 2048), (2, 0, 2048), (1, 100, 1948)])
def test_prefill_split_items_match_oracle_sampled_rows(nh, pos0, S):
    """Contexts holding 1 or 2 KV heads (the per-rank share of KV-head
    sharding over 8 or 4 GPUs): the kernel cuts the long causal items into
    parts merged by prefill_combine_kernel.  pos0 = 100 puts rows before the
    start of later parts (rows that see no key in such a part).  Sampled rows
    of the context's heads against the oracle."""
    torch = _torch()
    dev = torch.device("cuda:0")
    n_tok = pos0 + S
    kc, vc, _, _ = orc.make_cache(5000 + nh, 0, n_tok, HKV, HD, n_tok, bf16=True)
    _, q = prepped_q(5000 + nh, pos0, S)
    h0 = 2  # first KV head of the context
    c0, c1 = h0 * KV_MUL * HD, (h0 + nh) * KV_MUL * HD
    rows = np.array([0, 1, 27, 28, 127, 128, 129, 700, 1023, 1500, S - 2, S - 1])
    with q3attn.Context(n_layers=1, max_seq=n_tok, kv_dtype=q3attn.KV_BF16,
                        ptr_mode=q3attn.PTR_DEVICE, kv_head_begin=h0, kv_head_count=nh) as ctx:
        ctx.kv_load(0, 0, 0, n_tok, torch.from_numpy(kc).to(dev), torch.from_numpy(vc).to(dev))
        out = torch.zeros((S, HQ * HD), device=dev)
        n0 = ctx.launch_count()
        ctx.prefill_attn(out, q3attn.OUT_F32, torch.from_numpy(q).to(dev).to(torch.bfloat16),
                         0, 0, pos0, S)
        ctx.sync()
        ctx.check_device_error()
        launches = ctx.launch_count() - n0
        got = out.cpu().numpy()
    assert launches == 2, "expected the split kernel and its combine launch"
    qd = HQ * HD
    for r in rows:
        ref = orc.attn_decode(q[r * qd:(r + 1) * qd].copy(), kc, vc, 0, pos0 + int(r), HQ,
                              KV_MUL, HD, KV_DIM, n_tok)
        assert np.all(np.isfinite(got[r, c0:c1])), f"row {r}"
        assert max_abs(got[r, c0:c1], ref[c0:c1]) <= TOL_BF16_ABS, f"nh {nh} row {r}"
