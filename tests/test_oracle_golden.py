"""Pins the CPU oracle (oracle/q3a_oracle.c) to the reference.

The golden vectors in tests/golden/ were produced by the reference's own
functions compiled from its sources (tests/golden/make_golden.py).  The oracle
restates the same arithmetic in the same order, so QK-RMSNorm, RoPE, softmax
and the cpu-multicore attention agree bit for bit; launch_attn
(qwen3-8b/xdna2/main.c:2724) normalises by a reciprocal and agrees to a few
ulps.  CPU only.
"""
import json
import os

import numpy as np
import pytest

import q3a_oracle as orc
from shapes import EPS, HD, HKV, HQ, KV_DIM, KV_MUL, THETA, normwise

GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def _load(name):
    return np.load(os.path.join(GOLD, name))


def _manifest():
    with open(os.path.join(GOLD, "manifest.json")) as f:
        return json.load(f)


def test_norm_rope_softmax_bit_exact():
    g = _load("norm_rope.npz")
    y = g["x"].copy()
    orc.rmsnorm_head(y, g["w"], HQ, HD, EPS)
    assert np.array_equal(y, g["norm_out"])
    for i, p in enumerate(g["rope_pos"]):
        z = g["norm_out"].copy()
        orc.rope(z, HQ, HD, int(p), THETA)
        assert np.array_equal(z, g["rope_out"][i]), f"rope at pos {p}"
    s = g["softmax_in"].copy()
    orc.lib().orc_softmax(orc._ptr(s), s.size)
    assert np.array_equal(s, g["softmax_out"])


def _oracle_block(case):
    seed, pos, unit, bf16 = case["seed"], case["pos"], case["unit_gains"], case["bf16"]
    max_seq = case["max_seq"]
    if unit:
        qw = np.ones(HD, np.float32)
        kw = np.ones(HD, np.float32)
    else:
        qw = (1.0 + 0.25 * orc.randn(HD, seed, 6)).astype(np.float32)
        kw = (1.0 + 0.25 * orc.randn(HD, seed, 7)).astype(np.float32)
    kc = np.zeros(max_seq * KV_DIM, np.float32)
    vc = np.zeros(max_seq * KV_DIM, np.float32)
    kraw = orc.randn(pos * KV_DIM, seed, 1)
    vraw = orc.randn(pos * KV_DIM, seed, 2)
    for t in range(pos):
        row = kraw[t * KV_DIM:(t + 1) * KV_DIM].copy()
        orc.rmsnorm_head(row, kw, HKV, HD, EPS)
        orc.rope(row, HKV, HD, t, THETA)
        kc[t * KV_DIM:(t + 1) * KV_DIM] = row
    vc[: pos * KV_DIM] = vraw
    if bf16:
        kc = orc.bf16_round(kc)
        vc = orc.bf16_round(vc)
    q = orc.randn(HQ * HD, seed, 3)
    k = orc.randn(KV_DIM, seed, 4)
    v = orc.randn(KV_DIM, seed, 5)
    chk = sum(np.float64(a).sum() + np.abs(np.float64(a)).sum()
              for a in (q, k, v, kraw, vraw, qw, kw))
    if bf16:
        # bf16 cache: the appended k/v are stored rounded (after norm/rope)
        orc.rmsnorm_head(q, qw, HQ, HD, EPS)
        orc.rmsnorm_head(k, kw, HKV, HD, EPS)
        orc.rope(q, HQ, HD, pos, THETA)
        orc.rope(k, HKV, HD, pos, THETA)
        kc[pos * KV_DIM:(pos + 1) * KV_DIM] = orc.bf16_round(k)
        vc[pos * KV_DIM:(pos + 1) * KV_DIM] = orc.bf16_round(v)
        xb = orc.attn_decode(q, kc, vc, 0, pos, HQ, KV_MUL, HD, KV_DIM, max_seq)
    else:
        xb = orc.attn_block(q, k, v, qw, kw, kc, vc, 0, pos, HQ, HKV, HD, max_seq, EPS, THETA)
    return xb, q, k, chk


@pytest.mark.parametrize("i", range(12))
def test_decode_block_matches_reference(i):
    cases = _manifest()["files"]["decode_block.npz"]["cases"]
    case = cases[i]
    g = _load("decode_block.npz")
    xb, q, k, chk = _oracle_block(case)
    assert chk == pytest.approx(float(g[f"c{i}_inputs_checksum"]), rel=1e-12), "generator drift"
    assert np.array_equal(q, g[f"c{i}_q_out"])
    assert np.array_equal(k, g[f"c{i}_k_out"])
    # cpu-multicore normalisation: bit-identical
    assert np.array_equal(xb, g[f"c{i}_xb_mc"]), normwise(xb, g[f"c{i}_xb_mc"])
    # launch_attn (multiply by 1/sum): a few ulps
    assert normwise(xb, g[f"c{i}_xb_la"]) < 1e-6


def test_prefill_matches_reference():
    meta = _manifest()["files"]["prefill.npz"]["cases"]
    g = _load("prefill.npz")
    heads = g["heads"]
    for i, case in enumerate(meta):
        seed, pos0, S = case["seed"], case["pos0"], case["S"]
        n_tok = pos0 + S
        kc, vc, kraw, vraw = orc.make_cache(seed, 0, n_tok, HKV, HD, n_tok, bf16=True)
        # make_cache uses streams layer*16+1/2 = 1/2 for layer 0, as the fixture
        qraw = orc.randn(S * HQ * HD, seed, 3)
        chk = sum(np.float64(a).sum() + np.abs(np.float64(a)).sum() for a in (qraw, kraw, vraw))
        assert chk == pytest.approx(float(g[f"p{i}_inputs_checksum"]), rel=1e-12)
        q = qraw.copy()
        qw = np.ones(HD, np.float32)
        for s in range(S):
            row = q[s * HQ * HD:(s + 1) * HQ * HD]
            orc.rmsnorm_head(row, qw, HQ, HD, EPS)
            orc.rope(row, HQ, HD, pos0 + s, THETA)
        q = orc.bf16_round(q)
        out = orc.prefill_causal(q, kc, vc, pos0, S, HQ, KV_MUL, HD, KV_DIM, n_tok)
        sel = out.reshape(S, HQ, HD)[:, heads, :]
        assert np.array_equal(sel, g[f"p{i}_out_heads"])


def test_generator_statistics():
    x = orc.randn(1 << 20, 1234, 0)
    assert abs(float(x.mean())) < 5e-3
    assert abs(float(x.std()) - 1.0) < 5e-3
    # element i is independent of how the stream is split
    a = orc.randn(1000, 7, 3)
    b = np.concatenate([orc.randn(333, 7, 3, 0), orc.randn(667, 7, 3, 333)])
    assert np.array_equal(a, b)


def test_lse_merge_equals_single_pass():
    """Chunked partials merged by log-sum-exp equal one pass over the cache."""
    L = 700
    kc = orc.randn(L * KV_DIM, 11, 1)
    vc = orc.randn(L * KV_DIM, 11, 2)
    q = orc.randn(HQ * HD, 11, 3)
    ref = orc.attn_decode(q, kc, vc, 0, L - 1, HQ, KV_MUL, HD, KV_DIM, L)
    cuts = [0, 1, 64, 300, 301, 700]
    parts = [orc.attn_partial(q, kc, vc, 0, a, b, HQ, KV_MUL, HD, KV_DIM)
             for a, b in zip(cuts[:-1], cuts[1:])]
    o = np.stack([p[0] for p in parts])
    lse = np.stack([p[1] for p in parts])
    out, _ = orc.lse_merge(o, lse, HQ, HD)
    assert normwise(out, ref) < 1e-5
    # an empty chunk contributes nothing
    oe, le = orc.attn_partial(q, kc, vc, 0, 5, 5, HQ, KV_MUL, HD, KV_DIM)
    assert np.all(le == -np.inf) and np.all(oe == 0)
    out2, _ = orc.lse_merge(np.concatenate([o, oe[None]]), np.concatenate([lse, le[None]]), HQ, HD)
    assert normwise(out2, ref) < 1e-5


@pytest.mark.skipif(not orc.ref_available(), reason="reference library not built here")
@pytest.mark.parametrize("pos", [0, 5, 257])
def test_oracle_vs_compiled_reference_random(pos):
    """Fresh random cases straight against the compiled reference."""
    R = orc.ref()
    max_seq = pos + 3
    kc = orc.randn(max_seq * KV_DIM, 99 + pos, 1)
    vc = orc.randn(max_seq * KV_DIM, 99 + pos, 2)
    q = orc.randn(HQ * HD, 99 + pos, 3)
    att = np.zeros(HQ * max_seq, np.float32)
    xr = np.zeros(HQ * HD, np.float32)
    R.q3ref_attn_mc(orc._ptr(xr), orc._ptr(q), orc._ptr(kc), orc._ptr(vc), orc._ptr(att), 0, pos,
                    HQ, KV_MUL, HD, KV_DIM, max_seq)
    xo = orc.attn_decode(q, kc, vc, 0, pos, HQ, KV_MUL, HD, KV_DIM, max_seq)
    assert np.array_equal(xo, xr)


def test_mm_f16_matches_reference():
    """mm_f16 (the projections' fp16 GEMV) bit for bit against the reference's
    own outputs: seeded weights, and every fp16 bit pattern."""
    g = _load("projection.npz")
    for i, case in enumerate(_manifest()["files"]["projection.npz"]["cases"]):
        w = orc.proj_weights(case["seed"], case["d"], case["n"], case["scale"])
        x = orc.randn(case["n"], case["seed"], 201)
        ck = sum(np.float64(a).sum() + np.abs(np.float64(a)).sum()
                 for a in (x, w.astype(np.float32)))
        assert ck == float(g[f"m{i}_inputs_checksum"])
        o = orc.mm_f16(x, w)
        assert np.array_equal(o.view(np.uint32), g[f"m{i}_out"].view(np.uint32))
    w = orc.all_f16_patterns()
    o = orc.mm_f16(np.ones(1024, np.float32), w)
    assert np.array_equal(o.view(np.uint32), g["patterns_rowsum"].view(np.uint32))
    conv = orc.mm_f16(np.ones(1, np.float32), w.reshape(65536, 1))
    assert np.array_equal(conv.view(np.uint32), g["patterns_value"].view(np.uint32))
    # the conversion alone agrees with numpy's fp16 -> fp32 on every number
    # (by value: the sum starts at +0, so -0 comes out as +0)
    ref = w.reshape(-1).astype(np.float32)
    fin = ~np.isnan(ref)
    assert np.array_equal(conv[fin], ref[fin])
    assert np.isnan(conv[~fin]).all()


def test_rmsnorm_matches_reference():
    """The layer input's RMSNorm bit for bit against the reference's rmsnorm
    (run on one thread: the single-core build's summation order)."""
    g = _load("projection.npz")
    seed = int(g["rmsnorm_seed"])
    x = (orc.randn(4096, seed, 202) * 3.0).astype(np.float32)
    w = (1.0 + 0.25 * orc.randn(4096, seed, 203)).astype(np.float32)
    o = orc.rmsnorm(x, w, EPS)
    assert np.array_equal(o.view(np.uint32), g["rmsnorm_out"].view(np.uint32))
