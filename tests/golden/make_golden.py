"""Generates the golden vectors in tests/golden/ by running the REFERENCE's own
CPU functions, compiled from its sources into oracle/_ref/libq3ref.so
(oracle/Makefile, target `ref`).  Inputs come from the seeded generator of
the oracle (oracle/q3a_oracle.c: orc_randn), so each fixture stores seeds and
shapes plus a checksum of the generated inputs, and the reference outputs.

The reference ships no golden vectors, known-answer tests or fixtures, so
these are the pin for the oracle: tests/test_oracle_golden.py checks the C
restatement against them.

Run (in a container that has the reference tree and a built oracle/_ref):
    python tests/golden/make_golden.py
"""
from __future__ import annotations

import json
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, os.path.join(ROOT, "oracle"))
import q3a_oracle as orc  # noqa: E402

HQ, HKV, HD = 32, 8, 128
KV_DIM = HKV * HD
KV_MUL = HQ // HKV
EPS, THETA = 1e-6, 5e6
SEED = 1234


def _p(a):
    return orc._ptr(a)


def checksum(*arrs) -> float:
    return float(sum(np.float64(a).sum() + np.abs(np.float64(a)).sum() for a in arrs))


def ref_cache(seed, n_tok, max_seq, kw, bf16):
    """Cache rows 0..n_tok-1 prepared with the reference's rmsnorm_head_inplace
    and apply_rope (cpu-multicore), position-major [max_seq][kv_dim]."""
    R = orc.ref()
    kc = np.zeros(max_seq * KV_DIM, np.float32)
    vc = np.zeros(max_seq * KV_DIM, np.float32)
    kraw = orc.randn(n_tok * KV_DIM, seed, 1)
    vraw = orc.randn(n_tok * KV_DIM, seed, 2)
    for t in range(n_tok):
        row = kraw[t * KV_DIM:(t + 1) * KV_DIM].copy()
        R.q3ref_rmsnorm_head(_p(row), _p(kw), HKV, HD, EPS)
        R.q3ref_rope(_p(row), HKV, HD, t, THETA)
        kc[t * KV_DIM:(t + 1) * KV_DIM] = row
    vc[: n_tok * KV_DIM] = vraw
    if bf16:
        kc = orc.bf16_round(kc)
        vc = orc.bf16_round(vc)
    return kc, vc, kraw, vraw


def ref_block(seed, pos, max_seq, unit_gains, bf16):
    """One decode step of the reference block (qwen3-8b/cpu/main.c:1319-1353)
    with the reference's functions; cache rows 0..pos-1 pre-filled."""
    R = orc.ref()
    if unit_gains:
        qw = np.ones(HD, np.float32)
        kw = np.ones(HD, np.float32)
    else:
        qw = (1.0 + 0.25 * orc.randn(HD, seed, 6)).astype(np.float32)
        kw = (1.0 + 0.25 * orc.randn(HD, seed, 7)).astype(np.float32)
    kc, vc, kraw, vraw = ref_cache(seed, pos, max_seq, kw, bf16)
    q = orc.randn(HQ * HD, seed, 3)
    k = orc.randn(KV_DIM, seed, 4)
    v = orc.randn(KV_DIM, seed, 5)
    inputs_sum = checksum(q, k, v, kraw, vraw, qw, kw)
    R.q3ref_rmsnorm_head(_p(q), _p(qw), HQ, HD, EPS)
    R.q3ref_rmsnorm_head(_p(k), _p(kw), HKV, HD, EPS)
    R.q3ref_rope(_p(q), HQ, HD, pos, THETA)
    R.q3ref_rope(_p(k), HKV, HD, pos, THETA)
    if bf16:
        k_store = orc.bf16_round(k)
        v_store = orc.bf16_round(v)
    else:
        k_store, v_store = k, v
    R.q3ref_launch_kv_write(_p(k_store), _p(v_store), _p(kc[pos * KV_DIM:]),
                            _p(vc[pos * KV_DIM:]), KV_DIM)
    att = np.zeros(HQ * max_seq, np.float32)
    xb_mc = np.zeros(HQ * HD, np.float32)
    xb_la = np.zeros(HQ * HD, np.float32)
    R.q3ref_attn_mc(_p(xb_mc), _p(q), _p(kc), _p(vc), _p(att), 0, pos, HQ, KV_MUL, HD,
                    KV_DIM, max_seq)
    R.q3ref_launch_attn(_p(xb_la), _p(q), _p(kc), _p(vc), _p(att), 0, pos, HQ, KV_MUL,
                        HD, KV_DIM, max_seq)
    return dict(xb_mc=xb_mc, xb_la=xb_la, q_out=q, k_out=k, qw=qw, kw=kw,
                inputs_checksum=np.float64(inputs_sum))


def main():
    if not orc.ref_available():
        raise SystemExit("oracle/_ref/libq3ref.so is not built (make -C oracle ref REF=...)")
    R = orc.ref()
    meta = {"generator": "orc_randn (splitmix64 counter -> xorshift64* -> Box-Muller)",
            "seed": SEED, "shape": {"Hq": HQ, "Hkv": HKV, "hd": HD},
            "eps": EPS, "theta": THETA, "files": {}}

    # 1. QK-RMSNorm and RoPE: inputs stored, reference outputs stored.
    x = orc.randn(HQ * HD, SEED, 100)
    w = (1.0 + 0.25 * orc.randn(HD, SEED, 101)).astype(np.float32)
    norm_out = x.copy()
    R.q3ref_rmsnorm_head(_p(norm_out), _p(w), HQ, HD, EPS)
    rope_pos = np.array([0, 1, 63, 64, 65, 127, 1023, 1024, 2047, 8191, 131071], np.int32)
    rope_out = np.zeros((len(rope_pos), HQ * HD), np.float32)
    for i, p in enumerate(rope_pos):
        y = norm_out.copy()
        R.q3ref_rope(_p(y), HQ, HD, int(p), THETA)
        rope_out[i] = y
    sm_in = orc.randn(1025, SEED, 102) * 3.0
    sm_out = sm_in.copy()
    R.q3ref_softmax(_p(sm_out), sm_in.size)
    np.savez(os.path.join(HERE, "norm_rope.npz"), x=x, w=w, norm_out=norm_out,
             rope_pos=rope_pos, rope_out=rope_out, softmax_in=sm_in, softmax_out=sm_out)
    meta["files"]["norm_rope.npz"] = "rmsnorm_head_inplace / apply_rope / softmax of qwen3-8b/cpu-multicore/main.c"

    # 2. Decode block (fp32 cache, reference layout), full Qwen3-8B head shape.
    cases = []
    arrays = {}
    max_seq = 1040
    specs = [(p, True, False) for p in (0, 1, 63, 64, 65, 127, 1023, 1024)]
    specs += [(200, False, False), (64, True, True), (1024, True, True), (333, False, True)]
    for i, (pos, unit, bf16) in enumerate(specs):
        seed = SEED + 17 * i
        r = ref_block(seed, pos, max_seq, unit, bf16)
        cases.append({"seed": seed, "pos": pos, "unit_gains": unit, "bf16": bf16,
                      "max_seq": max_seq})
        for k_, v_ in r.items():
            arrays[f"c{i}_{k_}"] = v_
    np.savez(os.path.join(HERE, "decode_block.npz"), **arrays)
    meta["files"]["decode_block.npz"] = {
        "what": "one decode step of qwen3-8b/cpu/main.c:1319-1353 with the reference's "
                "functions; xb_mc = cpu-multicore normalisation, xb_la = launch_attn "
                "(qwen3-8b/xdna2/main.c:2724)",
        "cases": cases}

    # 3. Causal prefill as decode steps at pos0..pos0+S-1 (bf16-rounded q/k/v).
    pre_cases = []
    pre_arrays = {}
    heads = np.array([0, 5, 31], np.int32)
    for i, (pos0, S) in enumerate([(0, 48), (16, 32)]):
        seed = SEED + 1000 + i
        n_tok = pos0 + S
        ms = n_tok
        kw = np.ones(HD, np.float32)
        kc, vc, kraw, vraw = ref_cache(seed, n_tok, ms, kw, True)
        qraw = orc.randn(S * HQ * HD, seed, 3)
        q = qraw.copy()
        qw = np.ones(HD, np.float32)
        for s in range(S):
            row = q[s * HQ * HD:(s + 1) * HQ * HD]
            R.q3ref_rmsnorm_head(_p(row), _p(qw), HQ, HD, EPS)
            R.q3ref_rope(_p(row), HQ, HD, pos0 + s, THETA)
        q = orc.bf16_round(q)
        out = np.zeros((S, HQ * HD), np.float32)
        att = np.zeros(HQ * ms, np.float32)
        for s in range(S):
            xb = np.zeros(HQ * HD, np.float32)
            R.q3ref_attn_mc(_p(xb), _p(q[s * HQ * HD:]), _p(kc), _p(vc), _p(att), 0,
                            pos0 + s, HQ, KV_MUL, HD, KV_DIM, ms)
            out[s] = xb
        sel = out.reshape(S, HQ, HD)[:, heads, :].copy()
        pre_cases.append({"seed": seed, "pos0": pos0, "S": S})
        pre_arrays[f"p{i}_out_heads"] = sel
        pre_arrays[f"p{i}_inputs_checksum"] = np.float64(checksum(qraw, kraw, vraw))
    pre_arrays["heads"] = heads
    np.savez(os.path.join(HERE, "prefill.npz"), **pre_arrays)
    meta["files"]["prefill.npz"] = {
        "what": "causal prefill = reference decode attention at pos0..pos0+S-1 "
                "(qwen3-8b/cpu/main.c:1481-1499), bf16-rounded q/k/v, heads subset",
        "cases": pre_cases}

    proj_golden(meta)
    with open(os.path.join(HERE, "manifest.json"), "w") as f:
        json.dump(meta, f, indent=1)
    print("wrote golden vectors to", HERE)


def proj_golden(meta):
    """4. The fp16 GEMV of the q/k/v projections (mm_f16,
    qwen3-8b/cpu-multicore/main.c:1213-1221) run by the reference."""
    R = orc.ref()
    arrays = {}
    cases = []
    for i, (n, d) in enumerate([(4096, 64), (1024, 48)]):
        seed = SEED + 2000 + i
        w = orc.proj_weights(seed, d, n)
        x = orc.randn(n, seed, 201)
        o = np.zeros(d, np.float32)
        R.q3ref_mm_f16(_p(o), _p(x), _p(w.view(np.uint16)), n, d)
        arrays[f"m{i}_out"] = o
        arrays[f"m{i}_inputs_checksum"] = np.float64(checksum(x, w.astype(np.float32)))
        cases.append({"seed": seed, "n": n, "d": d, "scale": 0.02})
    # every fp16 value: rows of all 65536 patterns against x = 1, and the
    # conversion alone (n = 1, x = [1])
    w = orc.all_f16_patterns()
    o = np.zeros(64, np.float32)
    R.q3ref_mm_f16(_p(o), _p(np.ones(1024, np.float32)), _p(w.view(np.uint16)), 1024, 64)
    arrays["patterns_rowsum"] = o
    conv = np.zeros(65536, np.float32)
    R.q3ref_mm_f16(_p(conv), _p(np.ones(1, np.float32)),
                   _p(np.ascontiguousarray(w.reshape(65536, 1)).view(np.uint16)), 1, 65536)
    arrays["patterns_value"] = conv
    # the layer input's RMSNorm (rmsnorm, run on one OpenMP thread)
    seed = SEED + 2100
    x = (orc.randn(4096, seed, 202) * 3.0).astype(np.float32)
    w = (1.0 + 0.25 * orc.randn(4096, seed, 203)).astype(np.float32)
    o = np.zeros(4096, np.float32)
    R.q3ref_rmsnorm(_p(o), _p(x), _p(w), 4096, EPS)
    arrays["rmsnorm_seed"] = np.int64(seed)
    arrays["rmsnorm_out"] = o
    np.savez(os.path.join(HERE, "projection.npz"), **arrays)
    meta["files"]["projection.npz"] = {
        "what": "mm_f16 (qwen3-8b/cpu-multicore/main.c:1213-1221) run by the reference: "
                "seeded weights (orc_randn * scale rounded to fp16) and x = orc_randn, and "
                "every fp16 bit pattern (row sums against x = 1; each value alone); rmsnorm "
                "(cpu-multicore/main.c:1171-1178 on one OpenMP thread) of x = 3 orc_randn "
                "(stream 202) with gains 1 + 0.25 orc_randn (stream 203)",
        "cases": cases}


if __name__ == "__main__":
    if sys.argv[1:] == ["projection"]:  # only the projection fixture
        if not orc.ref_available():
            raise SystemExit("oracle/_ref/libq3ref.so is not built (make -C oracle ref REF=...)")
        with open(os.path.join(HERE, "manifest.json")) as f:
            m = json.load(f)
        proj_golden(m)
        with open(os.path.join(HERE, "manifest.json"), "w") as f:
            json.dump(m, f, indent=1)
    else:
        main()
