"""The C host harness (qwen3.c_b200/lib/q3a_harness): a C program built
against include/q3attn.h alone, whose per-layer call is the binding a
maintainer adds to the reference's forward(), runs the block on the GPU through the
host-pointer API.  Its layer-0 call is checked against the oracle and
against the reference's own compiled launch_attn (oracle/_ref) on the cache
rows the library holds, read back by the harness with q3a_kv_read.

Tolerances as in tests/shapes.py (fp32 cache: normwise 2e-4; bf16 cache:
max-abs 1e-2 against the reference fed the same bf16-rounded K/V).
"""
import json
import os
import subprocess

import numpy as np
import pytest

import q3a_oracle as orc
from shapes import EPS, HD, HKV, HQ, KV_DIM, KV_MUL, THETA, TOL_BF16_ABS, TOL_F32_NORMWISE, normwise

pytestmark = pytest.mark.gpu
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HARNESS = os.path.join(ROOT, "qwen3.c_b200", "lib", "q3a_harness")


def _load(d, name):
    return np.fromfile(os.path.join(d, name + ".f32"), dtype=np.float32)


@pytest.mark.parametrize("kv", ["f32", "bf16"])
def test_c_harness_layer_matches_oracle_and_reference(tmp_path, kv):
    assert os.path.exists(HARNESS), "build it: make -C qwen3.c_b200"
    ctx_len, seed = 1000, 4321
    r = subprocess.run([HARNESS, "--layers", "2", "--ctx", str(ctx_len), "--kv", kv, "--steps", "2",
                        "--warmup", "1", "--seed", str(seed), "--dump", str(tmp_path)],
                       capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stderr
    line = json.loads(r.stdout.strip().splitlines()[-1])
    assert line["layers"] == 2 and line["ctx"] == ctx_len and line["kv"] == kv
    assert line["us_per_layer"] > 0 and line["launches"] == 2 * 2
    pos = ctx_len - 1
    q_in, k_in, v_in = _load(tmp_path, "q_in"), _load(tmp_path, "k_in"), _load(tmp_path, "v_in")
    # the harness's host generator is the oracle's integer stream and transform
    assert np.array_equal(q_in, orc.randn(HQ * HD, seed, 3))
    assert np.array_equal(v_in, orc.randn(KV_DIM, seed, 5))
    kc = np.zeros(ctx_len * KV_DIM, np.float32)
    vc = np.zeros(ctx_len * KV_DIM, np.float32)
    kc[: pos * KV_DIM] = _load(tmp_path, "kc")
    vc[: pos * KV_DIM] = _load(tmp_path, "vc")
    w = np.ones(HD, np.float32)
    # the block of the reference: norm + RoPE of q and k, KV write, attention
    q, k = q_in.copy(), k_in.copy()
    orc.rmsnorm_head(q, w, HQ, HD, EPS)
    orc.rmsnorm_head(k, w, HKV, HD, EPS)
    orc.rope(q, HQ, HD, pos, THETA)
    orc.rope(k, HKV, HD, pos, THETA)
    bf16 = kv == "bf16"
    kc[pos * KV_DIM:] = orc.bf16_round(k) if bf16 else k
    vc[pos * KV_DIM:] = orc.bf16_round(v_in) if bf16 else v_in
    ref = orc.attn_decode(q, kc, vc, 0, pos, HQ, KV_MUL, HD, KV_DIM, ctx_len)
    xb = _load(tmp_path, "xb")
    if bf16:
        assert float(np.abs(np.float64(xb) - ref).max()) <= TOL_BF16_ABS
    else:
        assert normwise(xb, ref) <= TOL_F32_NORMWISE
    # q and k come back normalised and rotated in place, as in the reference
    assert normwise(_load(tmp_path, "q_out"), q) <= 1e-5
    assert normwise(_load(tmp_path, "k_out"), k) <= 1e-5
    if orc.ref_available():
        # the reference's own compiled attention (xdna2 launch_attn) on the
        # same rows
        R = orc.ref()
        P = orc._ptr
        xr = np.zeros(HQ * HD, np.float32)
        att = np.zeros(HQ * ctx_len, np.float32)
        R.q3ref_launch_attn(P(xr), P(q), P(kc), P(vc), P(att), 0, pos, HQ, KV_MUL, HD, KV_DIM,
                            ctx_len)
        if bf16:
            assert float(np.abs(np.float64(xb) - xr).max()) <= TOL_BF16_ABS
        else:
            assert normwise(xb, xr) <= TOL_F32_NORMWISE
