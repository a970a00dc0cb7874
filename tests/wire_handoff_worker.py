"""Worker of test_shard_gpu.py::test_prefill_to_decode_handoff (two GPUs,
torchrun): rank 0 prefills a prompt into its cache (q3a_prefill), packs the
prompt's KV rows into a wire blob (q3a_kv_pack) and sends the blob to
rank 1 over NCCL; rank 1 unpacks it into its own context (q3a_kv_unpack).
Both ranks then decode the next token with the same inputs in
deterministic mode; each writes its xb, which must agree bit for bit."""
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
from shapes import HD, HQ, KV_DIM  # noqa: E402


def main():
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    local = int(os.environ["LOCAL_RANK"])
    dev = torch.device(f"cuda:{local}")
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", device_id=dev, timeout=datetime.timedelta(seconds=60))
    n_layers, S = 2, 512
    t = lambda a: torch.from_numpy(a).to(dev)  # noqa: E731
    w = torch.ones(HD, device=dev)
    with q3attn.Context(n_layers=n_layers, max_seq=S + 8, kv_dtype=q3attn.KV_BF16,
                        ptr_mode=q3attn.PTR_DEVICE, device=local) as ctx:
        ctx.set_deterministic(True)
        nbytes = ctx.kv_wire_bytes(n_layers, S)
        blob = torch.zeros(nbytes, dtype=torch.uint8, device=dev)
        if rank == 0:
            out = torch.zeros(S, HQ * HD, device=dev)
            for l in range(n_layers):
                q = t(orc.randn(S * HQ * HD, 900 + l, 3))
                k = t(orc.randn(S * KV_DIM, 900 + l, 4))
                v = t(orc.randn(S * KV_DIM, 900 + l, 5))
                ctx.prefill(out, q3attn.OUT_F32, q, k, v, w, w, 0, l, 0, S)
            ctx.kv_pack(0, 0, n_layers, 0, S, blob)
            ctx.sync()
            dist.send(blob, 1)
        else:
            dist.recv(blob, 0)
            torch.cuda.synchronize(dev)
            ctx.kv_unpack(0, blob)
            ctx.sync()
        # the next token on both ranks
        xbs = []
        for l in range(n_layers):
            q = t(orc.randn(HQ * HD, 950 + l, 3))
            k = t(orc.randn(KV_DIM, 950 + l, 4))
            v = t(orc.randn(KV_DIM, 950 + l, 5))
            xb = torch.zeros(HQ * HD, device=dev)
            ctx.attn_layer(xb, q, k, v, w, w, l, S)
            ctx.sync()
            ctx.check_device_error()
            xbs.append(xb.cpu().numpy())
        dist.barrier()
    dist.destroy_process_group()
    np.save(os.path.join(os.environ["SHARD_TEST_OUT"], f"xb{rank}.npy"), np.stack(xbs))


if __name__ == "__main__":
    main()
