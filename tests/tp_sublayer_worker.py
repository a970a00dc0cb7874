"""Worker of test_shard_gpu.py::test_sublayer_over_kv_head_shards, run under
torchrun (one process per GPU): rank r holds KV heads kv_heads(8, world, r)
of a two-layer context; every rank passes the same residual stream x and the
same weights to q3a_attn_sublayer, which projects, attends and multiplies
by wo for the held heads only and sums the ranks' partial wo products over
NVLink peer memory inside the wo kernel.  Each rank writes the largest
normwise error of its sublayer increments against the oracle, and whether
its x equals rank 0's bit for bit at every step."""
import datetime
import os
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
for p in ("qwen3.c_b200", "tests", "oracle"):
    sys.path.insert(0, os.path.join(ROOT, p))

import numpy as np  # noqa: E402
import torch  # noqa: E402
import torch.distributed as dist  # noqa: E402

import q3a_oracle as orc  # noqa: E402
import q3attn  # noqa: E402
import shard  # noqa: E402
from shapes import HD, HKV, KV_DIM, normwise  # noqa: E402
from test_sublayer_gpu import DIM, oracle_sublayer, sublayer_weights, to_dev_f16  # noqa: E402


def main():
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    local = int(os.environ["LOCAL_RANK"])
    dev = torch.device(f"cuda:{local}")
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", device_id=dev, timeout=datetime.timedelta(seconds=60))
    W = sublayer_weights(8100)
    D = {k: (to_dev_f16(torch, v, dev) if v.dtype == np.float16 else torch.from_numpy(v).to(dev))
         for k, v in W.items()}
    n_layers, pos0, steps = 2, 700, 2
    max_seq = pos0 + steps
    caches = [orc.make_cache(8300 + l, l, pos0, HKV, HD, max_seq, kw=W["kn"], bf16=True)[:2]
              for l in range(n_layers)]
    kv0, nkv = shard.kv_heads(HKV, world, rank)
    worst, same = 0.0, True
    st = torch.cuda.Stream(dev)
    with q3attn.Context(n_layers=n_layers, max_seq=max_seq, kv_dtype=q3attn.KV_BF16,
                        ptr_mode=q3attn.PTR_DEVICE, device=local, kv_head_begin=kv0,
                        kv_head_count=nkv) as ctx:
        ctx.set_stream(st.cuda_stream)
        shard.open_peer_set(ctx, world=world, rank=rank)
        for l, (kc, vc) in enumerate(caches):
            ctx.kv_load(0, l, 0, pos0, torch.from_numpy(kc[:pos0 * KV_DIM]).to(dev),
                        torch.from_numpy(vc[:pos0 * KV_DIM]).to(dev))
        st.synchronize()
        x_ref = orc.randn(DIM, 8400, 1)
        xd = torch.from_numpy(x_ref).to(dev)
        torch.cuda.synchronize(dev)
        for s in range(steps):
            for l in range(n_layers):
                kc, vc = caches[l]
                x_old = x_ref
                x_ref = oracle_sublayer(x_old, W, kc, vc, pos0 + s, max_seq, True)
                with torch.cuda.stream(st):
                    ctx.attn_sublayer(xd, D["att"], D["wq"], D["wk"], D["wv"], D["qn"], D["kn"],
                                      D["wo"], l, pos0 + s)
                st.synchronize()
                ctx.check_device_error()
                got = xd.clone()
                worst = max(worst, normwise(got.cpu().numpy() - x_old, x_ref - x_old))
                ref0 = got.clone()
                dist.broadcast(ref0, 0)
                same = same and bool(torch.equal(got, ref0))
                xd.copy_(torch.from_numpy(x_ref))
                torch.cuda.synchronize(dev)
        dist.barrier()
    dist.destroy_process_group()
    with open(os.path.join(os.environ["SHARD_TEST_OUT"], f"rank{rank}.txt"), "w") as f:
        f.write(f"{worst!r} {int(same)}")


if __name__ == "__main__":
    main()
