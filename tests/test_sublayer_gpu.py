"""GPU parity of the attention sublayer's consumer side and of the whole
sublayer: q3a_wo_residual (x += wo . xb, qwen3-8b/cpu/main.c:1355-1356) and
q3a_attn_sublayer (rmsnorm -> q/k/v projections -> QK-norm, RoPE, append ->
attention -> wo -> residual, main.c:1313-1356) against the oracle's
restatement of the same steps (orc_rmsnorm, orc_mm_f16, orc_rmsnorm_head,
orc_rope, orc_attn_decode; each pinned to the reference by
tests/test_oracle_golden.py).

Tolerances are on the sublayer's increment d = x_new - x_old (x_old is
exact on both sides):
- wo alone, d = wo . xb: normwise 1e-5 (fp32 sums in another order);
- whole sublayer, fp32 cache: normwise 1e-3 (the attention's 2e-4 carried
  through wo);
- whole sublayer, bf16 cache: normwise 3e-2 (the bf16 attention tolerance,
  max-abs 1e-2 on xb, carried through wo).
"""
import numpy as np
import pytest

import q3a_oracle as orc
import q3attn
from shapes import EPS, HD, HKV, HQ, KV_DIM, KV_MUL, THETA, normwise

pytestmark = pytest.mark.gpu

DIM = 4096
TOL_WO = 1e-5
TOL_SUB_F32 = 1e-3
TOL_SUB_BF16 = 3e-2


def to_dev_f16(torch, w, dev):
    return torch.from_numpy(w.view(np.uint16).astype(np.int16)).view(torch.float16).to(dev)


def sublayer_weights(seed, dim=DIM):
    """Seeded attention-sublayer weights of a model of width dim (Qwen3-8B:
    4096; Qwen3-4B: 2560), fp16 matrices and fp32 gains."""
    return dict(
        att=(1.0 + 0.1 * orc.randn(dim, seed, 9)).astype(np.float32),
        wq=orc.proj_weights(seed, HQ * HD, dim),
        wk=orc.proj_weights(seed + 1, KV_DIM, dim),
        wv=orc.proj_weights(seed + 2, KV_DIM, dim),
        wo=orc.proj_weights(seed + 3, dim, HQ * HD),
        qn=(1.0 + 0.25 * orc.randn(HD, seed, 6)).astype(np.float32),
        kn=(1.0 + 0.25 * orc.randn(HD, seed, 7)).astype(np.float32),
    )


def oracle_sublayer(x, W, kc, vc, pos, max_seq, bf16):
    """x + attention sublayer of one token at pos; kc, vc (position-major
    [max_seq][kv_dim]) get row pos."""
    xn = orc.rmsnorm(x, W["att"], EPS)
    q = orc.mm_f16(xn, W["wq"])
    k = orc.mm_f16(xn, W["wk"])
    v = orc.mm_f16(xn, W["wv"])
    orc.rmsnorm_head(q, W["qn"], HQ, HD, EPS)
    orc.rmsnorm_head(k, W["kn"], HKV, HD, EPS)
    orc.rope(q, HQ, HD, pos, THETA)
    orc.rope(k, HKV, HD, pos, THETA)
    ks, vs = (orc.bf16_round(k), orc.bf16_round(v)) if bf16 else (k, v)
    kc[pos * KV_DIM:(pos + 1) * KV_DIM] = ks
    vc[pos * KV_DIM:(pos + 1) * KV_DIM] = vs
    xb = orc.attn_decode(q, kc, vc, 0, pos, HQ, KV_MUL, HD, KV_DIM, max_seq)
    return x + orc.mm_f16(xb, W["wo"])


@pytest.fixture(scope="module")
def weights():
    import torch
    dev = torch.device("cuda:0")
    W = sublayer_weights(8100)
    D = {k: (to_dev_f16(torch, v, dev) if v.dtype == np.float16 else torch.from_numpy(v).to(dev))
         for k, v in W.items()}
    return W, D


def test_wo_residual_matches_oracle(weights):
    import torch
    dev = torch.device("cuda:0")
    W, D = weights
    xb = orc.randn(HQ * HD, 8200, 1)
    x0 = orc.randn(DIM, 8200, 2)
    ref = x0 + orc.mm_f16(xb, W["wo"])
    with q3attn.Context(n_layers=1, max_seq=64, ptr_mode=q3attn.PTR_DEVICE) as ctx:
        outs = []
        for _ in range(2):
            x = torch.from_numpy(x0).to(dev)
            ctx.wo_residual(x, torch.from_numpy(xb).to(dev), D["wo"])
            ctx.sync()
            ctx.check_device_error()
            outs.append(x.cpu().numpy())
        assert normwise(outs[0] - x0, ref - x0) <= TOL_WO
        assert np.array_equal(outs[0], outs[1])


@pytest.mark.parametrize("bf16", [False, True])
def test_sublayer_steps_match_oracle(weights, bf16):
    """Two layers x three tokens, the residual stream carried from sublayer
    to sublayer as in forward(); every step against the oracle."""
    import torch
    dev = torch.device("cuda:0")
    W, D = weights
    n_layers, pos0, steps = 2, 700, 3
    max_seq = pos0 + steps
    caches = [orc.make_cache(8300 + l, l, pos0, HKV, HD, max_seq, kw=W["kn"], bf16=bf16)[:2]
              for l in range(n_layers)]
    kv = q3attn.KV_BF16 if bf16 else q3attn.KV_F32
    tol = TOL_SUB_BF16 if bf16 else TOL_SUB_F32
    with q3attn.Context(n_layers=n_layers, max_seq=max_seq, kv_dtype=kv,
                        ptr_mode=q3attn.PTR_DEVICE) as ctx:
        for l, (kc, vc) in enumerate(caches):
            ctx.kv_load(0, l, 0, pos0, torch.from_numpy(kc[:pos0 * KV_DIM]).to(dev),
                        torch.from_numpy(vc[:pos0 * KV_DIM]).to(dev))
        x_ref = orc.randn(DIM, 8400, 1)
        xd = torch.from_numpy(x_ref).to(dev)
        for s in range(steps):
            for l in range(n_layers):
                kc, vc = caches[l]
                x_old = x_ref
                x_ref = oracle_sublayer(x_old, W, kc, vc, pos0 + s, max_seq, bf16)
                ctx.attn_sublayer(xd, D["att"], D["wq"], D["wk"], D["wv"], D["qn"], D["kn"],
                                  D["wo"], l, pos0 + s)
                ctx.sync()
                ctx.check_device_error()
                got = xd.cpu().numpy()
                err = normwise(got - x_old, x_ref - x_old)
                assert err <= tol, f"step {s} layer {l}: normwise {err}"
                # continue from the oracle's x so that errors do not compound
                xd.copy_(torch.from_numpy(x_ref))


def test_sharded_wo_needs_peer_set(weights):
    import torch
    dev = torch.device("cuda:0")
    _, D = weights
    with q3attn.Context(n_layers=1, max_seq=64, ptr_mode=q3attn.PTR_DEVICE,
                        kv_head_begin=2, kv_head_count=2) as ctx:
        with pytest.raises(q3attn.Q3AError):
            ctx.wo_residual(torch.zeros(DIM, device=dev), torch.zeros(HQ * HD, device=dev),
                            D["wo"])


def test_sublayer_at_qwen3_4b_width():
    """Width 2560 (Qwen3-4B: 32 query heads, 8 KV heads of 128): six rows per
    projection stage, wo of 2560 rows x 4096 columns; one layer, two tokens."""
    import torch
    dev = torch.device("cuda:0")
    dim = 2560
    W = sublayer_weights(8600, dim)
    D = {k: (to_dev_f16(torch, v, dev) if v.dtype == np.float16 else torch.from_numpy(v).to(dev))
         for k, v in W.items()}
    pos0, steps = 300, 2
    max_seq = pos0 + steps
    kc, vc = orc.make_cache(8700, 0, pos0, HKV, HD, max_seq, kw=W["kn"])[:2]
    with q3attn.Context(n_layers=1, max_seq=max_seq, ptr_mode=q3attn.PTR_DEVICE) as ctx:
        ctx.kv_load(0, 0, 0, pos0, torch.from_numpy(kc[:pos0 * KV_DIM]).to(dev),
                    torch.from_numpy(vc[:pos0 * KV_DIM]).to(dev))
        x_ref = orc.randn(dim, 8800, 1)
        xd = torch.from_numpy(x_ref).to(dev)
        for s in range(steps):
            x_old = x_ref
            x_ref = oracle_sublayer(x_old, W, kc, vc, pos0 + s, max_seq, False)
            ctx.attn_sublayer(xd, D["att"], D["wq"], D["wk"], D["wv"], D["qn"], D["kn"], D["wo"],
                              0, pos0 + s)
            ctx.sync()
            ctx.check_device_error()
            err = normwise(xd.cpu().numpy() - x_old, x_ref - x_old)
            assert err <= TOL_SUB_F32, f"step {s}: normwise {err}"
            xd.copy_(torch.from_numpy(x_ref))
