"""q3a_graph_begin / end / launch: a token step recorded as one CUDA graph
(the attention sublayer of two layers, and two decode layers) and replayed
gives the same bits as the same calls run one by one (deterministic
schedule on both sides)."""
import numpy as np
import pytest

import q3attn
from shapes import HD, HQ, KV_DIM
from test_sublayer_gpu import DIM, sublayer_weights, to_dev_f16

pytestmark = pytest.mark.gpu


def make_ctx(torch, dev, n_layers, pos):
    ctx = q3attn.Context(n_layers=n_layers, max_seq=pos + 8, ptr_mode=q3attn.PTR_DEVICE)
    ctx.set_deterministic(True)
    for l in range(n_layers):
        ctx.kv_synth(0, l, 0, pos, 555 + l, 1, 2)
    ctx.sync()
    return ctx


def test_sublayer_step_as_graph():
    import torch
    dev = torch.device("cuda:0")
    W = sublayer_weights(8100)
    D = {k: (to_dev_f16(torch, v, dev) if v.dtype == np.float16 else torch.from_numpy(v).to(dev))
         for k, v in W.items()}
    n_layers, pos = 2, 300
    x0 = torch.randn(DIM, device=dev, generator=torch.Generator(device=dev).manual_seed(7))

    def step(ctx, x):
        for l in range(n_layers):
            ctx.attn_sublayer(x, D["att"], D["wq"], D["wk"], D["wv"], D["qn"], D["kn"], D["wo"],
                              l, pos)

    eager = make_ctx(torch, dev, n_layers, pos)
    xe = x0.clone()
    step(eager, xe)
    eager.sync()
    eager.check_device_error()

    ctx = make_ctx(torch, dev, n_layers, pos)
    try:
        xg = x0.clone()
        step(ctx, xg)  # first calls allocate their scratch: before recording
        ctx.sync()
        torch.cuda.synchronize()
        ctx.graph_begin()
        step(ctx, xg)
        g = ctx.graph_end()
        try:
            for _ in range(2):
                xg.copy_(x0)
                torch.cuda.synchronize()
                ctx.graph_launch(g)
                ctx.sync()
                ctx.check_device_error()
                assert torch.equal(xg, xe)
        finally:
            ctx.graph_destroy(g)
    finally:
        ctx.close()
        eager.close()


def test_decode_layers_as_graph():
    import torch
    dev = torch.device("cuda:0")
    n_layers, pos = 2, 1000
    gen = torch.Generator(device=dev).manual_seed(11)
    q = torch.randn(n_layers, HQ * HD, device=dev, generator=gen)
    k = torch.randn(n_layers, KV_DIM, device=dev, generator=gen)
    v = torch.randn(n_layers, KV_DIM, device=dev, generator=gen)
    w = torch.ones(HD, device=dev)

    def step(ctx, xb, qq, kk):
        for l in range(n_layers):
            ctx.attn_layer(xb[l], qq[l], kk[l], v[l], w, w, l, pos)

    eager = make_ctx(torch, dev, n_layers, pos)
    xe, qe, ke = torch.zeros(n_layers, HQ * HD, device=dev), q.clone(), k.clone()
    step(eager, xe, qe, ke)
    eager.sync()

    ctx = make_ctx(torch, dev, n_layers, pos)
    try:
        xg, qg, kg = torch.zeros_like(xe), q.clone(), k.clone()
        torch.cuda.synchronize()
        ctx.graph_begin()
        step(ctx, xg, qg, kg)
        g = ctx.graph_end()
        try:
            for _ in range(2):
                qg.copy_(q)
                kg.copy_(k)
                xg.zero_()
                torch.cuda.synchronize()
                ctx.graph_launch(g)
                ctx.sync()
                ctx.check_device_error()
                assert torch.equal(xg, xe) and torch.equal(qg, qe)
        finally:
            ctx.graph_destroy(g)
    finally:
        ctx.close()
        eager.close()


def test_host_mode_cannot_record():
    with q3attn.Context(n_layers=1, max_seq=64) as ctx:
        with pytest.raises(q3attn.Q3AError):
            ctx.graph_begin()
