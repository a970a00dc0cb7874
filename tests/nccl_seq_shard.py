"""Worker of test_shard_gpu.py::test_sequence_shards_over_gpus, run
under torchrun (one process per GPU): a 20000-token bf16 sequence split over
the ranks, one decode step through shard.SeqShardDecode (q3a_attn_partial,
NCCL all-gather, q3a_lse_combine_packed; or, with SHARD_MODE=peer, the
peer-memory exchange of q3a_attn_seqshard), compared with the oracle's single
pass (the reference's attention loop, cpu/main.c:1331-1353)."""
import datetime
import os
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
for p in ("oracle", "qwen3.c_b200", "tests"):
    sys.path.insert(0, os.path.join(ROOT, p))

import numpy as np  # noqa: E402
import torch  # noqa: E402
import torch.distributed as dist  # noqa: E402

import q3a_oracle as orc  # noqa: E402
import q3attn  # noqa: E402
import shard  # noqa: E402
from shapes import HD, HKV, HQ, KV_DIM, KV_MUL  # noqa: E402


def main():
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    local = int(os.environ["LOCAL_RANK"])
    dev = torch.device(f"cuda:{local}")
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", device_id=dev, timeout=datetime.timedelta(seconds=60))
    L = 20000
    kc, vc, _, _ = orc.make_cache(123, 0, L, HKV, HD, L, bf16=True)
    qv = orc.randn(HQ * HD, 123, 9)
    t0, t1 = shard.seq_chunk(L, world, rank)
    st = torch.cuda.Stream(dev)
    with q3attn.Context(n_layers=1, max_seq=t1 - t0, kv_dtype=q3attn.KV_BF16,
                        ptr_mode=q3attn.PTR_DEVICE, device=local) as ctx:
        ctx.set_stream(st.cuda_stream)
        ctx.set_deterministic(True)  # the repeated calls are compared bit for bit
        ctx.kv_load(0, 0, 0, t1 - t0, torch.from_numpy(kc[t0 * KV_DIM:t1 * KV_DIM]).to(dev),
                    torch.from_numpy(vc[t0 * KV_DIM:t1 * KV_DIM]).to(dev))
        dec = shard.SeqShardDecode(torch, ctx, world=world, rank=rank, device=dev,
                                   mode=os.environ.get("SHARD_MODE", "nccl"))
        q = torch.from_numpy(qv).to(dev)
        outs = []
        for _ in range(3):  # repeated calls: the peer exchange alternates buffer halves
            xb = torch.zeros(HQ * HD, device=dev)
            torch.cuda.synchronize(dev)
            with torch.cuda.stream(st):
                dec(xb, q, 0, 0, t1 - t0)
            st.synchronize()
            ctx.check_device_error()
            outs.append(xb.cpu().numpy())
        got = outs[-1]
        assert all(np.array_equal(o, got) for o in outs)
    dist.barrier()
    dist.destroy_process_group()
    ref = orc.attn_decode(qv, kc, vc, 0, L - 1, HQ, KV_MUL, HD, KV_DIM, L)
    err = float(np.abs(np.float64(got) - ref).max())
    with open(os.path.join(os.environ["SHARD_TEST_OUT"], f"rank{rank}.txt"), "w") as f:
        f.write(repr(err))


if __name__ == "__main__":
    main()
