"""Worker of test_shard_gpu.py::test_peer_head_gather, run under torchrun (one
process per GPU): a registered buffer holds two [rows, 32*128] bf16 matrices;
each rank fills the columns of its query heads with a pattern of its own and
q3a_gather_cols (shard.PeerHeadGather) makes every rank hold every rank's
columns.  Repeated calls on both matrices exercise the call numbers."""
import datetime
import os
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
for p in ("qwen3.c_b200", "tests"):
    sys.path.insert(0, os.path.join(ROOT, p))

import torch  # noqa: E402
import torch.distributed as dist  # noqa: E402

import q3attn  # noqa: E402
import shard  # noqa: E402


def pattern(torch, rows, width, r, call):
    """Values of rank r's columns at a call: small integers, exact in bf16."""
    i = torch.arange(rows, dtype=torch.float32)[:, None]
    j = torch.arange(width, dtype=torch.float32)[None, :]
    return ((i * 3 + j * 5 + 17 * r + 29 * call) % 251).to(torch.bfloat16)


def main():
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    local = int(os.environ["LOCAL_RANK"])
    dev = torch.device(f"cuda:{local}")
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", device_id=dev, timeout=datetime.timedelta(seconds=60))
    rows, cols = 300, 32 * 128
    w = cols // world
    buf = torch.zeros(2, rows, cols, dtype=torch.bfloat16, device=dev)
    st = torch.cuda.Stream(dev)
    bad = 0
    with q3attn.Context(n_layers=1, max_seq=128, kv_dtype=q3attn.KV_BF16,
                        ptr_mode=q3attn.PTR_DEVICE, device=local) as ctx:
        ctx.set_stream(st.cuda_stream)
        g = shard.PeerHeadGather(torch, ctx, world=world, rank=rank, buf=buf)
        for call in range(4):
            m = buf[call % 2]
            torch.cuda.synchronize(dev)
            m.zero_()
            m[:, rank * w:(rank + 1) * w] = pattern(torch, rows, w, rank, call).to(dev)
            torch.cuda.synchronize(dev)
            with torch.cuda.stream(st):
                g(m)
            st.synchronize()
            ctx.check_device_error()
            for r in range(world):
                want = pattern(torch, rows, w, r, call).to(dev)
                if not torch.equal(m[:, r * w:(r + 1) * w], want):
                    bad += 1
            # every rank has read its result before anyone writes the matrix again
            dist.barrier()
    dist.destroy_process_group()
    with open(os.path.join(os.environ["SHARD_TEST_OUT"], f"rank{rank}.txt"), "w") as f:
        f.write(repr(bad))


if __name__ == "__main__":
    main()
