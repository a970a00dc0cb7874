#!/usr/bin/env python
"""Benchmark of the Qwen3 GQA attention block on B200.

Headline workload: full-depth decode attention for
one new token, 36 layers x (32 q heads, 8 KV heads, head_dim 128), KV length
8192 (new token at position 8191), fp32 cache.  One step = the 36 layer calls
of q3a_attn_layer (QK-norm + RoPE + KV append + attention, one kernel each).
`value` is HBM GB/s of algorithmic bytes with everything resident in HBM;
`us_per_layer` is the same measurement as time per layer.  `e2e` is the same
metric through the host-pointer C-ABI called from a C host
(qwen3.c_b200/lib/q3a_harness): q, k, v and the norm gains copied in from
host memory and xb, q, k written back, every layer, synchronously.

Extra keys: `bf16` (the bf16-cache variant), `prefill` (configs[2]: causal
prefill of 2048 tokens, TFLOP/s of the dense contraction), `sublayer` (the
attention sublayer from the residual stream: input RMSNorm fused into the
fp16 q/k/v projections with QK-norm, RoPE and the append, the decode, the
wo projection with the residual add; `sublayer.qkv` and `sublayer.wo` are
the two projection kernels alone against the HBM roofline; at N > 1 the
sublayer runs tensor-parallel over KV heads).

--impl reference times the reference's own CPU code (oracle/_ref, compiled
from the reference sources: launch_attn with OpenMP over heads, plus its
rmsnorm_head / rope / kv write) on the same metric, or the oracle port when
the reference library is absent.

Multi-GPU: one process per GPU (torchrun); every rank decodes its own
sequence (weak scaling, no data-path collective), value = all ranks' bytes /
max-over-ranks time.  The sharded legs scale strongly and carry their own
numbers: `long_ctx` (configs[3], sequence-sharded 128K decode; at N > 1 rank
0 also times the same step on one GPU, so the line gives t(1)/t(N)),
`ragged_batch` (configs[4], KV-head sharded) and `prefill` (configs[2],
KV-head sharded).
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "qwen3.c_b200"))

HQ, HKV, HD = 32, 8, 128
KV_DIM = HKV * HD
N_LAYERS = 36
L_CTX = 8192
POS = L_CTX - 1
METRIC = "decode attn µs/layer + HBM GB/s (KV 8K); prefill attn TFLOP/s (2K tok)"
PREFILL_S = 2048
LONG_L = 131072          # configs[3]: sequence-sharded long-context decode
RAGGED_B = 64            # configs[4]: ragged batch, KV lengths U[512, 32768]
RAGGED_LO, RAGGED_HI = 512, 32768


def algo_bytes_per_layer(esize: int) -> int:
    """Bytes the block must move per layer: K and V rows 0..L-2 read from the
    cache, the new K/V row written, and the fp32 vectors (q in/out, xb out,
    k in/out, v in, two norm gains)."""
    cache = 2 * (L_CTX - 1) * KV_DIM * esize + 2 * KV_DIM * esize
    vecs = 3 * HQ * HD * 4 + 3 * KV_DIM * 4 + 2 * HD * 4
    return cache + vecs


def prefill_flops(S: int = PREFILL_S) -> float:
    return 4.0 * HD * HQ * S * (S + 1) / 2.0


def measured_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        return d.get("hbm_gbs", 6650.0), d.get("bf16_tflops", 1590.0), \
            d.get("bf16_tflops_sustained", 1400.0), "measured"
    return 6650.0, 1590.0, 1400.0, "fallback"


def profile_traffic(name: str):
    """Per-launch DRAM bytes of a kernel from a committed ncu summary."""
    p = os.path.join(ROOT, "profiles", "traffic.json")
    if not os.path.exists(p):
        return None
    with open(p) as f:
        return json.load(f).get(name)


# ------------------------------------------------------------------ clocks
class ClockSampler:
    REASONS = {0x4: "sw_power_cap", 0x8: "hw_slowdown", 0x20: "sw_thermal_slowdown",
               0x40: "hw_thermal_slowdown", 0x80: "hw_power_brake_slowdown",
               0x2: "applications_clocks_setting", 0x1: "gpu_idle"}

    def __init__(self, torch_dev: int, period_s: float = 0.005):
        self.samples = []
        self.reasons = set()
        self.max_mhz = None
        self.period = period_s
        self._stop = threading.Event()
        self.h = None
        try:
            import pynvml
            import torch
            pynvml.nvmlInit()
            uuid = str(torch.cuda.get_device_properties(torch_dev).uuid)
            if not uuid.startswith("GPU-"):
                uuid = "GPU-" + uuid
            self.h = pynvml.nvmlDeviceGetHandleByUUID(uuid)
            self.nv = pynvml
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self.h, pynvml.NVML_CLOCK_SM)
        except Exception as e:  # clocks are reported as unavailable
            self.err = repr(e)

    def _run(self):
        nv = self.nv
        while not self._stop.is_set():
            try:
                self.samples.append(nv.nvmlDeviceGetClockInfo(self.h, nv.NVML_CLOCK_SM))
                r = nv.nvmlDeviceGetCurrentClocksEventReasons(self.h)
                for bit, name in self.REASONS.items():
                    if r & bit:
                        self.reasons.add(name)
            except Exception:
                pass
            time.sleep(self.period)

    def __enter__(self):
        if self.h is not None:
            self.t = threading.Thread(target=self._run, daemon=True)
            self.t.start()
        return self

    def __exit__(self, *a):
        if self.h is not None:
            self._stop.set()
            self.t.join()

    def report(self):
        if self.h is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "note": "nvml unavailable"}
        return {"sm_mhz": statistics.median(self.samples) if self.samples else None,
                "sm_max_mhz": self.max_mhz, "reasons": sorted(self.reasons - {"gpu_idle"}),
                "samples": len(self.samples)}


# ------------------------------------------------------------------ dist
def dist_setup():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return world, rank, local


def max_over_ranks(x: float, world: int, dev) -> float:
    if world == 1:
        return x
    import torch
    import torch.distributed as dist
    t = torch.tensor([x], dtype=torch.float64, device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def barrier(world):
    if world > 1:
        import torch.distributed as dist
        dist.barrier()


# ------------------------------------------------------------------ our arm
def fill_cache(ctx, torch, dev, seed, n_layers, pos, stream):
    """Layer l: k_t, v_t ~ N(0,1) (streams l*16+1, l*16+2), k normed and
    rotated at t by the library's own append kernel, rows 0..pos-1 (full
    rows of all 8 KV heads; a KV-head-sharded context keeps its own)."""
    import q3attn
    kraw = torch.empty(pos * KV_DIM, device=dev)
    vraw = torch.empty(pos * KV_DIM, device=dev)
    ones = torch.ones(HD, device=dev)
    for l in range(n_layers):
        ctx.randn(kraw, q3attn.OUT_F32, kraw.numel(), seed, l * 16 + 1)
        ctx.randn(vraw, q3attn.OUT_F32, vraw.numel(), seed, l * 16 + 2)
        ctx.kv_append(0, l, 0, pos, kraw, vraw, ones)
    stream.synchronize()


def decode_run(args, torch, dev, local, kv_dtype, seed, world, with_e2e, with_cpu):
    import q3attn
    esize = 4 if kv_dtype == q3attn.KV_F32 else 2
    stream = torch.cuda.Stream(device=dev)
    ctx = q3attn.Context(n_layers=N_LAYERS, max_seq=L_CTX, kv_dtype=kv_dtype,
                         ptr_mode=q3attn.PTR_DEVICE, device=local)
    ctx.set_stream(stream.cuda_stream)
    fill_cache(ctx, torch, dev, seed, N_LAYERS, POS, stream)
    # per-layer new-token inputs (raw projections), streams l*16+3/4/5
    q_raw = torch.empty(N_LAYERS, HQ * HD, device=dev)
    k_raw = torch.empty(N_LAYERS, KV_DIM, device=dev)
    v_in = torch.empty(N_LAYERS, KV_DIM, device=dev)
    for l in range(N_LAYERS):
        ctx.randn(q_raw[l], q3attn.OUT_F32, HQ * HD, seed, l * 16 + 3)
        ctx.randn(k_raw[l], q3attn.OUT_F32, KV_DIM, seed, l * 16 + 4)
        ctx.randn(v_in[l], q3attn.OUT_F32, KV_DIM, seed, l * 16 + 5)
    qw = torch.ones(HD, device=dev)
    kw = torch.ones(HD, device=dev)
    q_w = q_raw.clone()
    k_w = k_raw.clone()
    xb = torch.zeros(N_LAYERS, HQ * HD, device=dev)
    stream.synchronize()

    def step():
        # The block normalises and rotates q and k in place, as the reference
        # does; later steps therefore see already-rotated inputs, which
        # changes values, not work.
        for l in range(N_LAYERS):
            ctx.attn_layer(xb[l], q_w[l], k_w[l], v_in[l], qw, kw, l, POS)

    with torch.cuda.stream(stream):
        for _ in range(args.warmup):
            step()
    stream.synchronize()
    ctx.check_device_error()

    # The timed region (K steps = K x 36 decode launches, nothing else) is one
    # CUDA graph bracketed by two events; event records between the kernels
    # would add their own cost to every launch, so the average launch
    # duration is the bracketed time over the number of launches.
    K = args.steps
    e0 = torch.cuda.Event(enable_timing=True, external=True)
    e1 = torch.cuda.Event(enable_timing=True, external=True)
    g = torch.cuda.CUDAGraph()
    n0 = ctx.launch_count()
    with torch.cuda.graph(g, stream=stream):
        e0.record(stream)
        for kk in range(K):
            step()
        e1.record(stream)
    launches = ctx.launch_count() - n0
    with torch.cuda.stream(stream):
        g.replay()  # untimed replay (instantiation, first-touch)
    torch.cuda.synchronize(dev)
    barrier(world)
    torch.cuda.synchronize(dev)
    with ClockSampler(local) as cs:
        with torch.cuda.stream(stream):
            g.replay()
        torch.cuda.synchronize(dev)
    torch.cuda.synchronize(dev)
    barrier(world)
    ctx.check_device_error()
    t_ms = e0.elapsed_time(e1)
    res = {"t_ms": t_ms, "kernel_us": 1000.0 * t_ms / launches,
           "launches": launches, "clocks": cs.report(),
           "bytes_per_layer": algo_bytes_per_layer(esize), "esize": esize}
    del g

    ctx.close()
    if with_e2e:
        res["e2e"] = e2e_run(args, local, kv_dtype, seed)
    return res


DIM = 4096               # Qwen3-8B model width (rows of the projections' input)
GQA_MUL = HQ // HKV      # query heads per KV head


def proj_bytes(esize: int, nkv: int = HKV) -> int:
    """Algorithmic bytes of one projection launch (qkv_kernel) for nkv held
    KV heads: the fp16 weights of their q, k, v rows ((4 + 1 + 1) x nkv x
    128 rows x 4096 columns), the fp32 input x, the fp32 q written, and the
    new K/V row appended."""
    rows = (GQA_MUL + 2) * nkv * HD
    return rows * DIM * 2 + DIM * 4 + GQA_MUL * nkv * HD * 4 + 2 * nkv * HD * esize


def wo_bytes(nkv: int = HKV) -> int:
    """Algorithmic bytes of one wo launch (wo_kernel) for nkv held KV heads:
    the fp16 columns of their query heads (4096 rows x 4 x nkv x 128), the
    fp32 xb slice read, x read and written."""
    cols = GQA_MUL * nkv * HD
    return DIM * cols * 2 + cols * 4 + 2 * DIM * 4


def sublayer_run(args, torch, dev, local, seed, world, rank):
    """The attention sublayer from the residual stream (the rows after the
    path: producer and consumer of the block): per layer q3a_qkv_proj alone,
    q3a_wo_residual alone, and q3a_attn_sublayer (input RMSNorm fused into the
    q/k/v projections + QK-norm + RoPE + append, decode over 8193 rows of the
    fp32 cache, wo + residual), 36 layers per step.  Weights N(0, 0.02^2) in
    fp16, 36 x 84 MB = 3.0 GB (> L2).  At N > 1 rank r holds KV heads
    kv_heads(8, N, r): its q/k/v rows, its cache heads and its wo columns;
    the wo kernel sums the ranks' partial products over NVLink."""
    import q3attn
    import shard
    kv0, nkv = shard.kv_heads(HKV, world, rank)
    stream = torch.cuda.Stream(device=dev)
    ctx = q3attn.Context(n_layers=N_LAYERS, max_seq=L_CTX, kv_dtype=q3attn.KV_F32,
                         ptr_mode=q3attn.PTR_DEVICE, device=local, kv_head_begin=kv0,
                         kv_head_count=nkv)
    ctx.set_stream(stream.cuda_stream)
    if world > 1:
        shard.open_peer_set(ctx, world=world, rank=rank)
    fill_cache(ctx, torch, dev, seed, N_LAYERS, POS, stream)
    g = torch.Generator(device=dev)
    g.manual_seed(seed)
    with torch.cuda.stream(stream):
        wq = (torch.randn(N_LAYERS, HQ * HD, DIM, device=dev, generator=g) * 0.02).half()
        wk = (torch.randn(N_LAYERS, KV_DIM, DIM, device=dev, generator=g) * 0.02).half()
        wv = (torch.randn(N_LAYERS, KV_DIM, DIM, device=dev, generator=g) * 0.02).half()
        wo = (torch.randn(N_LAYERS, DIM, HQ * HD, device=dev, generator=g) * 0.02).half()
        att = 1.0 + 0.1 * torch.randn(N_LAYERS, DIM, device=dev, generator=g)
        x_in = torch.randn(N_LAYERS, DIM, device=dev, generator=g)
    x = x_in[0].clone()
    qw = torch.ones(HD, device=dev)
    kw = torch.ones(HD, device=dev)
    q = torch.zeros(N_LAYERS, HQ * HD, device=dev)
    xb = torch.randn(N_LAYERS, HQ * HD, device=dev, generator=g)
    stream.synchronize()

    def step_qkv():
        for l in range(N_LAYERS):
            ctx.qkv_proj(q[l], None, None, x_in[l], wq[l], wk[l], wv[l], qw, kw, l, POS)

    def step_wo():
        for l in range(N_LAYERS):
            ctx.wo_residual(x, xb[l], wo[l])

    def step_sub():
        for l in range(N_LAYERS):
            ctx.attn_sublayer(x, att[l], wq[l], wk[l], wv[l], qw, kw, wo[l], l, POS)

    res = {"nkv": nkv}
    for name, step in (("qkv", step_qkv), ("wo", step_wo), ("sublayer", step_sub)):
        with torch.cuda.stream(stream):
            for _ in range(args.warmup):
                step()
        stream.synchronize()
        ctx.check_device_error()
        barrier(world)
        n0 = ctx.launch_count()
        t_ms, clocks = time_graph(torch, dev, local, stream, step, args.steps, world)
        ctx.check_device_error()
        res[name] = {"t_ms": t_ms, "clocks": clocks, "launches": ctx.launch_count() - n0}
    ctx.close()
    del wq, wk, wv, wo
    return res


def prefill_run(args, torch, dev, local, seed, world, rank=0):
    """causal prefill of S=2048 prompt rows per layer, 36 layers,
    bf16 Q/K/V (post QK-norm + RoPE), fp32 softmax and accumulation, bf16
    output.  One step = 36 launches of q3a_prefill_attn (the attention of
    each layer over its cache), timed as one CUDA graph between two events.
    With N > 1 ranks each rank holds 8/N KV heads (and their query heads) and
    one all-gather of the output head slices per layer (q3a_gather_cols:
    every rank stores its columns into every rank's output over NVLink)
    rebuilds the output on every rank (strong scaling)."""
    import q3attn
    import shard
    S = PREFILL_S
    h0, nh = shard.kv_heads(HKV, world, rank)
    stream = torch.cuda.Stream(device=dev)
    ctx = q3attn.Context(n_layers=N_LAYERS, max_seq=S, kv_dtype=q3attn.KV_BF16,
                         ptr_mode=q3attn.PTR_DEVICE, device=local, kv_head_begin=h0,
                         kv_head_count=nh)
    ctx.set_stream(stream.cuda_stream)
    fill_cache(ctx, torch, dev, seed, N_LAYERS, S, stream)
    qf = torch.empty(S * HQ * HD, device=dev)
    qs = []
    for l in range(N_LAYERS):
        ctx.randn(qf, q3attn.OUT_F32, qf.numel(), seed, l * 16 + 3)
        stream.synchronize()
        # the kernel reads prepared (normed, rotated) bf16 rows; N(0,1) rows
        # have the same statistics for timing
        qs.append(qf.to(torch.bfloat16).view(S, HQ * HD).contiguous())
    out = torch.empty(N_LAYERS, S, HQ * HD, dtype=torch.bfloat16, device=dev)
    stream.synchronize()
    # output head slices: one q3a_gather_cols launch per layer (each rank
    # stores its columns into every rank's `out` over NVLink)
    gather = shard.PeerHeadGather(torch, ctx, world=world, rank=rank, buf=out) if world > 1 else None

    def step():
        for l in range(N_LAYERS):
            ctx.prefill_attn(out[l], q3attn.OUT_BF16, qs[l], 0, l, 0, S)
            if gather is not None:
                gather(out[l])

    def step_sharded_out():
        # the same launches without the all-gather: each rank's output keeps
        # its own heads (the layout a head-sharded o-projection consumes)
        for l in range(N_LAYERS):
            ctx.prefill_attn(out[l], q3attn.OUT_BF16, qs[l], 0, l, 0, S)

    with torch.cuda.stream(stream):
        for _ in range(args.warmup):
            step()
    stream.synchronize()
    ctx.check_device_error()
    K = max(1, args.steps // 10)
    n0 = ctx.launch_count()
    t_ms, clocks = time_graph(torch, dev, local, stream, step, K, world)
    launches = ctx.launch_count() - n0
    t_so, launches_so = None, 0
    if world > 1:
        n1 = ctx.launch_count()
        t_so, _ = time_graph(torch, dev, local, stream, step_sharded_out, K, world)
        launches_so = ctx.launch_count() - n1
    ctx.check_device_error()
    ctx.close()
    # a layer is one launch, or two when long items are split (+ the combine
    # kernel), plus the gather launch at N > 1: time per layer uses layers
    return {"t_ms": t_ms, "launches": launches, "layers": K * N_LAYERS,
            "clocks": clocks, "steps": K, "t_ms_sharded_out": t_so, "launches_sharded_out": launches_so}


def time_graph(torch, dev, local, stream, step, K, world):
    """K steps captured as one CUDA graph between two events on `stream`
    (collectives included), replayed once untimed and once timed.  With
    N > 1 a small all-reduce sits in the graph before the first event, so
    every rank's timed region starts once all ranks are there (host launch
    skew between ranks is not counted)."""
    e0 = torch.cuda.Event(enable_timing=True, external=True)
    e1 = torch.cuda.Event(enable_timing=True, external=True)
    align = torch.zeros(1, device=dev)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=stream):
        if world > 1:
            import torch.distributed as dist
            dist.all_reduce(align)
        e0.record(stream)
        for _ in range(K):
            step()
        e1.record(stream)
    with torch.cuda.stream(stream):
        g.replay()
    torch.cuda.synchronize(dev)
    barrier(world)
    with ClockSampler(local) as cs:
        with torch.cuda.stream(stream):
            g.replay()
        torch.cuda.synchronize(dev)
    barrier(world)
    t_ms = e0.elapsed_time(e1)
    del g
    return t_ms, cs.report()


def long_ctx_run(args, torch, dev, local, world, rank):
    """one new token attending to a 131072-token bf16 cache, 36
    layers, the sequence split into contiguous chunks over the ranks.  Per
    layer one launch of q3a_attn_seqshard: split-KV decode of the local
    chunk, each KV head's (o, lse) stored into every rank's receive buffer
    over NVLink, merged on every rank once all have arrived.  Strong scaling:
    the total work is fixed as N grows."""
    import q3attn
    import shard
    t0, t1 = shard.seq_chunk(LONG_L, world, rank)
    n_loc = t1 - t0
    stream = torch.cuda.Stream(device=dev)
    ctx = q3attn.Context(n_layers=N_LAYERS, max_seq=n_loc, kv_dtype=q3attn.KV_BF16,
                         ptr_mode=q3attn.PTR_DEVICE, device=local)
    ctx.set_stream(stream.cuda_stream)
    # each rank's chunk from its own streams; q is the same on every rank
    fill_cache(ctx, torch, dev, 4242 + 7919 * rank, N_LAYERS, n_loc, stream)
    q = torch.empty(N_LAYERS, HQ * HD, device=dev)
    for l in range(N_LAYERS):
        ctx.randn(q[l], q3attn.OUT_F32, HQ * HD, 4242, l * 16 + 3)
    xb = torch.zeros(N_LAYERS, HQ * HD, device=dev)
    stream.synchronize()
    dec = shard.SeqShardDecode(torch, ctx, world=world, rank=rank, device=dev, mode="peer")

    def step():
        for l in range(N_LAYERS):
            dec(xb[l], q[l], 0, l, n_loc)

    with torch.cuda.stream(stream):
        for _ in range(args.warmup):
            step()
    stream.synchronize()
    ctx.check_device_error()
    K = max(2, args.steps // 10)
    n0 = ctx.launch_count()
    t_ms, clocks = time_graph(torch, dev, local, stream, step, K, world)
    launches = (ctx.launch_count() - n0)
    ctx.check_device_error()
    ctx.close()
    return {"t_ms": t_ms, "steps": K, "clocks": clocks, "launches": launches,
            "rows_local": n_loc}


def long_ctx_single(args, torch, dev, local):
    """configs[3] on one GPU (rank 0 alone), for t(1)/t(N) in a multi-GPU run:
    the same per-layer launch with the whole 131072-row sequence local."""
    import q3attn
    import shard
    stream = torch.cuda.Stream(device=dev)
    ctx = q3attn.Context(n_layers=N_LAYERS, max_seq=LONG_L, kv_dtype=q3attn.KV_BF16,
                         ptr_mode=q3attn.PTR_DEVICE, device=local)
    ctx.set_stream(stream.cuda_stream)
    fill_cache(ctx, torch, dev, 4242, N_LAYERS, LONG_L, stream)
    q = torch.empty(N_LAYERS, HQ * HD, device=dev)
    for l in range(N_LAYERS):
        ctx.randn(q[l], q3attn.OUT_F32, HQ * HD, 4242, l * 16 + 3)
    xb = torch.zeros(N_LAYERS, HQ * HD, device=dev)
    stream.synchronize()
    dec = shard.SeqShardDecode(torch, ctx, world=1, rank=0, device=dev, mode="peer")

    def step():
        for l in range(N_LAYERS):
            dec(xb[l], q[l], 0, l, LONG_L)

    with torch.cuda.stream(stream):
        for _ in range(args.warmup):
            step()
    stream.synchronize()
    K = max(2, args.steps // 10)
    t_ms, _ = time_graph(torch, dev, local, stream, step, K, 1)
    ctx.check_device_error()
    ctx.close()
    return t_ms * 1000.0 / (K * N_LAYERS)


def ragged_lengths():
    """configs[4] KV lengths: 64 draws from U[512, 32768] (numpy PCG64, seed
    2024); sequence b attends rows 0..L_b-1, the last being its new token."""
    import numpy as np
    return np.random.default_rng(2024).integers(RAGGED_LO, RAGGED_HI + 1, size=RAGGED_B)


def ragged_run(args, torch, dev, local, world, rank):
    """64 sequences, one new token each, bf16 caches, one fused
    batched launch (QK-norm, RoPE, append, attention) per step; rank r holds
    KV heads kv_heads(8, N, r) of every sequence, writes its query heads'
    columns of xb, and one all-gather of the slices over NVLink
    (q3a_gather_cols) rebuilds xb."""
    import q3attn
    import shard
    lens = ragged_lengths()
    h0, nh = shard.kv_heads(HKV, world, rank)
    stream = torch.cuda.Stream(device=dev)
    ctx = q3attn.Context(n_layers=1, max_seq=RAGGED_HI, n_seqs=RAGGED_B,
                         kv_dtype=q3attn.KV_BF16, ptr_mode=q3attn.PTR_DEVICE, device=local,
                         kv_head_begin=h0, kv_head_count=nh)
    ctx.set_stream(stream.cuda_stream)
    ones = torch.ones(HD, device=dev)
    kraw = torch.empty(RAGGED_HI * KV_DIM, device=dev)
    vraw = torch.empty(RAGGED_HI * KV_DIM, device=dev)
    for b, L in enumerate(lens):
        n = int(L) - 1
        # full rows of every sequence on every rank; each keeps its heads
        ctx.randn(kraw, q3attn.OUT_F32, n * KV_DIM, 5151, 1000 + 2 * b)
        ctx.randn(vraw, q3attn.OUT_F32, n * KV_DIM, 5151, 1001 + 2 * b)
        ctx.kv_append(b, 0, 0, n, kraw, vraw, ones)
    del kraw, vraw
    q = torch.empty(RAGGED_B, HQ * HD, device=dev)
    k = torch.empty(RAGGED_B, KV_DIM, device=dev)
    v = torch.empty(RAGGED_B, KV_DIM, device=dev)
    ctx.randn(q, q3attn.OUT_F32, q.numel(), 5151, 3)
    ctx.randn(k, q3attn.OUT_F32, k.numel(), 5151, 4)
    ctx.randn(v, q3attn.OUT_F32, v.numel(), 5151, 5)
    xb = torch.zeros(RAGGED_B, HQ * HD, device=dev)
    stream.synchronize()
    seq_ids = list(range(RAGGED_B))
    pos = [int(L) - 1 for L in lens]
    gather = shard.PeerHeadGather(torch, ctx, world=world, rank=rank, buf=xb) if world > 1 else None

    def step():
        ctx.attn_layer_batched(xb, q, k, v, ones, ones, 0, seq_ids, pos)
        if gather is not None:
            gather(xb)

    with torch.cuda.stream(stream):
        for _ in range(args.warmup):
            step()
    stream.synchronize()
    ctx.check_device_error()
    K = max(3, args.steps // 5)
    n0 = ctx.launch_count()
    t_ms, clocks = time_graph(torch, dev, local, stream, step, K, world)
    launches = ctx.launch_count() - n0
    ctx.check_device_error()
    ctx.close()
    # all ranks together read every row of K and V once (the new row is
    # written, then read from shared memory)
    total_bytes = int(sum(2 * (int(L) - 1) * KV_DIM * 2 + 2 * KV_DIM * 2 for L in lens))
    return {"t_ms": t_ms, "steps": K, "clocks": clocks, "launches": launches,
            "bytes_per_step": total_bytes, "mean_len": float(lens.mean())}


def e2e_run(args, local, kv_dtype, seed):
    """Same step end to end through the host-pointer C-ABI from a C host:
    qwen3.c_b200/lib/q3a_harness (a C program built against
    include/q3attn.h only) runs 36 layer calls of q3a_attn_layer per step on
    this rank's GPU, every call copying q, k, v and the norm gains in from
    host memory and xb, q, k out, synchronously, and times K steps with
    CLOCK_MONOTONIC after W warm-up steps.  Its caches hold the same seeded
    rows as the device-timed leg (q3a_kv_synth, streams layer*16+1/2)."""
    import subprocess
    exe = os.path.join(ROOT, "qwen3.c_b200", "lib", "q3a_harness")
    if not os.path.exists(exe):
        raise RuntimeError(f"{exe} is missing: build it (make -C qwen3.c_b200)")
    cmd = [exe, "--layers", str(N_LAYERS), "--ctx", str(L_CTX),
           "--kv", "bf16" if kv_dtype == 1 else "f32", "--steps", str(args.steps),
           "--warmup", str(max(3, args.warmup)), "--seed", str(seed), "--device", str(local)]
    r = subprocess.run(cmd, capture_output=True, text=True, timeout=600)
    if r.returncode != 0:
        raise RuntimeError(f"q3a_harness failed: {r.stderr[-500:]}")
    h = json.loads(r.stdout.strip().splitlines()[-1])
    return {"t_ms": h["t_s"] * 1000.0, "h2d_bytes_per_step": h["h2d_bytes_per_step"],
            "d2h_bytes_per_step": h["d2h_bytes_per_step"], "launches": h["launches"],
            "us_per_layer": h["us_per_layer"]}


# ------------------------------------------------------------------ CPU reference
def cpu_reference_sample(n_calls_max: int, budget_s: float, n_layers_sample: int = 4):
    """Times the reference's own CPU block (oracle/_ref, or the oracle port)
    on `n_layers_sample` distinct layer caches at KV 8192, fp32."""
    import ctypes
    import numpy as np
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import q3a_oracle as orc
    use_ref = orc.ref_available()
    kind = "reference" if use_ref else "port"
    caches = []
    for l in range(n_layers_sample):
        kc, vc, _, _ = orc.make_cache(1234, l, POS, HKV, HD, L_CTX)
        caches.append((kc, vc))
    q0 = [orc.randn(HQ * HD, 1234, l * 16 + 3) for l in range(n_layers_sample)]
    k0 = [orc.randn(KV_DIM, 1234, l * 16 + 4) for l in range(n_layers_sample)]
    v0 = [orc.randn(KV_DIM, 1234, l * 16 + 5) for l in range(n_layers_sample)]
    w = np.ones(HD, np.float32)
    att = np.zeros(HQ * L_CTX, np.float32)
    xb = np.zeros(HQ * HD, np.float32)
    P = orc._ptr
    if use_ref:
        R = orc.ref()

        def block(l):
            q = q0[l].copy()
            k = k0[l].copy()
            kc, vc = caches[l]
            R.q3ref_rmsnorm_head(P(q), P(w), HQ, HD, 1e-6)
            R.q3ref_rmsnorm_head(P(k), P(w), HKV, HD, 1e-6)
            R.q3ref_rope(P(q), HQ, HD, POS, 5e6)
            R.q3ref_rope(P(k), HKV, HD, POS, 5e6)
            off = POS * KV_DIM * 4
            R.q3ref_launch_kv_write(P(k), P(v0[l]), ctypes.c_void_p(kc.ctypes.data + off),
                                    ctypes.c_void_p(vc.ctypes.data + off), KV_DIM)
            R.q3ref_launch_attn(P(xb), P(q), P(kc), P(vc), P(att), 0, POS, HQ, HQ // HKV, HD,
                                KV_DIM, L_CTX)
    else:
        def block(l):
            q = q0[l].copy()
            k = k0[l].copy()
            kc, vc = caches[l]
            orc.attn_block(q, k, v0[l], w, w, kc, vc, 0, POS, HQ, HKV, HD, L_CTX)
    block(0)  # warm
    calls = 0
    t0 = time.perf_counter()
    while calls < n_calls_max and (time.perf_counter() - t0) < budget_s:
        block(calls % n_layers_sample)
        calls += 1
    dt = time.perf_counter() - t0
    bytes_ = calls * algo_bytes_per_layer(4)
    threads = int(os.environ.get("OMP_NUM_THREADS", os.cpu_count() or 1))
    return {"value": bytes_ / dt / 1e9, "unit": "GB/s", "cores": min(threads, HQ), "kind": kind,
            "us_per_layer": dt / calls * 1e6, "calls": calls,
            "sample": f"{calls} layer calls of the fp32 block at KV 8192 cycling "
                      f"{n_layers_sample} distinct layer caches (OpenMP over the 32 heads, "
                      f"{threads} threads available)"}


def cpu_sublayer_sample(n_calls_max: int, budget_s: float):
    """Times the reference's own CPU attention sublayer (oracle/_ref:
    rmsnorm, mm_f16 for q, k, v, rmsnorm_head, apply_rope, the KV write,
    launch_attn, mm_f16 for wo, the residual add) at KV 8192, fp32 cache, on
    one layer (fp16 weights N(0, 0.02^2)); the oracle port when the
    reference library is absent."""
    import ctypes
    import numpy as np
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import q3a_oracle as orc
    use_ref = orc.ref_available()
    rng = np.random.default_rng(1234)
    f16 = lambda r, c: (rng.standard_normal((r, c), np.float32) * 0.02).astype(np.float16)  # noqa: E731
    wq, wk, wv, wo = f16(HQ * HD, DIM), f16(KV_DIM, DIM), f16(KV_DIM, DIM), f16(DIM, HQ * HD)
    kc, vc, _, _ = orc.make_cache(1234, 0, POS, HKV, HD, L_CTX)
    x = rng.standard_normal(DIM, np.float32)
    gains = np.ones(DIM, np.float32)
    w = np.ones(HD, np.float32)
    att = np.zeros(HQ * L_CTX, np.float32)
    P = orc._ptr
    R = orc.ref() if use_ref else None
    xn = np.zeros(DIM, np.float32)
    q = np.zeros(HQ * HD, np.float32)
    k = np.zeros(KV_DIM, np.float32)
    v = np.zeros(KV_DIM, np.float32)
    xb = np.zeros(HQ * HD, np.float32)
    xb2 = np.zeros(DIM, np.float32)

    def mm(o, xin, wm):
        if use_ref:
            R.q3ref_mm_f16(P(o), P(xin), P(wm.view(np.uint16)), wm.shape[1], wm.shape[0])
        else:
            o[:] = orc.mm_f16(xin, wm)

    def sublayer():
        if use_ref:
            R.q3ref_rmsnorm(P(xn), P(x), P(gains), DIM, 1e-6)
        else:
            xn[:] = orc.rmsnorm(x, gains)
        mm(q, xn, wq)
        mm(k, xn, wk)
        mm(v, xn, wv)
        if use_ref:
            R.q3ref_rmsnorm_head(P(q), P(w), HQ, HD, 1e-6)
            R.q3ref_rmsnorm_head(P(k), P(w), HKV, HD, 1e-6)
            R.q3ref_rope(P(q), HQ, HD, POS, 5e6)
            R.q3ref_rope(P(k), HKV, HD, POS, 5e6)
            off = POS * KV_DIM * 4
            R.q3ref_launch_kv_write(P(k), P(v), ctypes.c_void_p(kc.ctypes.data + off),
                                    ctypes.c_void_p(vc.ctypes.data + off), KV_DIM)
            R.q3ref_launch_attn(P(xb), P(q), P(kc), P(vc), P(att), 0, POS, HQ, HQ // HKV, HD,
                                KV_DIM, L_CTX)
        else:
            xb[:] = orc.attn_block(q.copy(), k.copy(), v, w, w, kc, vc, 0, POS, HQ, HKV, HD, L_CTX)
        mm(xb2, xb, wo)
        x[:] = x + xb2

    sublayer()  # warm
    calls = 0
    t0 = time.perf_counter()
    while calls < n_calls_max and (time.perf_counter() - t0) < budget_s:
        sublayer()
        calls += 1
    dt = time.perf_counter() - t0
    threads = int(os.environ.get("OMP_NUM_THREADS", os.cpu_count() or 1))
    us = dt / calls * 1e6
    bytes_ = proj_bytes(4) + wo_bytes() + 2 * (POS + 1) * KV_DIM * 4
    return {"value": bytes_ / (us * 1e-6) / 1e9, "unit": "GB/s", "cores": threads,
            "kind": "reference" if use_ref else "port", "us_per_layer": us,
            "sample": f"{calls} calls of one fp32 attention sublayer at KV 8192 (the reference's "
                      f"rmsnorm, mm_f16, rmsnorm_head, apply_rope, KV write, launch_attn; OpenMP, "
                      f"{threads} threads available)"}


def run_reference(args, world, rank):
    if rank != 0:
        return
    # one step = one full-depth pass sample: 4 layer calls on distinct caches
    n_per_step = 4
    cpu = cpu_reference_sample(n_calls_max=n_per_step * (args.steps + args.warmup),
                               budget_s=1e9, n_layers_sample=n_per_step)
    us = cpu["us_per_layer"]
    line = {"metric": METRIC, "value": cpu["value"], "unit": "GB/s", "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": us * N_LAYERS / 1000.0, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": config_dict(args, "f32"), "impl": "reference",
            "us_per_layer": us,
            "cpu_baseline": {k: cpu[k] for k in ("value", "unit", "cores", "kind", "sample")},
            "e2e": {"value": cpu["value"], "unit": "GB/s", "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0},
            "note": "step = 4 reference block calls (rmsnorm_head, rope, kv write, launch_attn) "
                    "on distinct layer caches; ms_per_step scaled to 36 layers"}
    print(json.dumps(line), flush=True)


def config_dict(args, dtype):
    return {"workload": "configs[1]: full-depth decode attention, 36 layers, KV 8192 "
                        f"(new token at pos 8191), {dtype} cache, batch 1 per GPU",
            "model": "Qwen3-8B GQA attention block (Hq=32, Hkv=8, d=128)",
            "global_batch": args.gpus, "seq_len": L_CTX,
            "parallelism": f"replicas{args.gpus}" if args.gpus > 1 else "single",
            "l2": "inputs larger than L2 (36 layer caches cycled per step)"}


def ncu_case(args):
    """A small case for ncu: 2 layers at KV 8192, warmup + steps direct calls
    of q3a_attn_layer alternating the layers (2 x 67 MB fp32 > L2 per pair;
    ncu flushes caches before each captured launch anyway)."""
    import torch
    import q3attn
    dev = torch.device("cuda:0")
    if args.ncu_case == "prefill":
        S = PREFILL_S
        stream = torch.cuda.Stream(device=dev)
        ctx = q3attn.Context(n_layers=1, max_seq=S, kv_dtype=q3attn.KV_BF16,
                             ptr_mode=q3attn.PTR_DEVICE)
        ctx.set_stream(stream.cuda_stream)
        fill_cache(ctx, torch, dev, 1234, 1, S, stream)
        qb = torch.randn(S, HQ * HD, device=dev).to(torch.bfloat16)
        out = torch.empty(S, HQ * HD, dtype=torch.bfloat16, device=dev)
        for _ in range(args.warmup + args.steps):
            ctx.prefill_attn(out, q3attn.OUT_BF16, qb, 0, 0, 0, S)
        stream.synchronize()
        ctx.check_device_error()
        ctx.close()
        print(f"ncu case prefill: {args.warmup + args.steps} launches ok")
        return
    if args.ncu_case == "sublayer":
        # 2 layers of the attention sublayer at KV 8192 (fp32 cache),
        # alternating: the three kernels of q3a_attn_sublayer per call
        stream = torch.cuda.Stream(device=dev)
        ctx = q3attn.Context(n_layers=2, max_seq=L_CTX, ptr_mode=q3attn.PTR_DEVICE)
        ctx.set_stream(stream.cuda_stream)
        fill_cache(ctx, torch, dev, 1234, 2, POS, stream)
        with torch.cuda.stream(stream):
            wq = (torch.randn(2, HQ * HD, DIM, device=dev) * 0.02).half()
            wk = (torch.randn(2, KV_DIM, DIM, device=dev) * 0.02).half()
            wv = (torch.randn(2, KV_DIM, DIM, device=dev) * 0.02).half()
            wo = (torch.randn(2, DIM, HQ * HD, device=dev) * 0.02).half()
            att = torch.ones(2, DIM, device=dev)
            x = torch.randn(DIM, device=dev)
            w = torch.ones(HD, device=dev)
        for i in range(args.warmup + args.steps):
            l = i % 2
            ctx.attn_sublayer(x, att[l], wq[l], wk[l], wv[l], w, w, wo[l], l, POS)
        stream.synchronize()
        ctx.check_device_error()
        ctx.close()
        print(f"ncu case sublayer: {args.warmup + args.steps} calls ok")
        return
    if args.ncu_case == "wo":
        # 2 layers of wo (2 x 34 MB) alternating
        stream = torch.cuda.Stream(device=dev)
        ctx = q3attn.Context(n_layers=1, max_seq=64, ptr_mode=q3attn.PTR_DEVICE)
        ctx.set_stream(stream.cuda_stream)
        with torch.cuda.stream(stream):
            wo = (torch.randn(2, DIM, HQ * HD, device=dev) * 0.02).half()
            xb = torch.randn(2, HQ * HD, device=dev)
            x = torch.randn(DIM, device=dev)
        for i in range(args.warmup + args.steps):
            ctx.wo_residual(x, xb[i % 2], wo[i % 2])
        stream.synchronize()
        ctx.check_device_error()
        ctx.close()
        print(f"ncu case wo: {args.warmup + args.steps} launches ok")
        return
    if args.ncu_case == "qkv":
        # 2 layers of weights (2 x 50 MB) alternating
        stream = torch.cuda.Stream(device=dev)
        ctx = q3attn.Context(n_layers=2, max_seq=64, ptr_mode=q3attn.PTR_DEVICE)
        ctx.set_stream(stream.cuda_stream)
        with torch.cuda.stream(stream):
            wq = (torch.randn(2, HQ * HD, DIM, device=dev) * 0.02).half()
            wk = (torch.randn(2, KV_DIM, DIM, device=dev) * 0.02).half()
            wv = (torch.randn(2, KV_DIM, DIM, device=dev) * 0.02).half()
            x = torch.randn(2, DIM, device=dev)
            w = torch.ones(HD, device=dev)
            q = torch.zeros(2, HQ * HD, device=dev)
        for i in range(args.warmup + args.steps):
            ctx.qkv_proj(q[i % 2], None, None, x[i % 2], wq[i % 2], wk[i % 2], wv[i % 2], w, w,
                         i % 2, 0)
        stream.synchronize()
        ctx.check_device_error()
        ctx.close()
        print(f"ncu case qkv: {args.warmup + args.steps} launches ok")
        return
    kv = q3attn.KV_F32 if args.ncu_case == "decode-f32" else q3attn.KV_BF16
    stream = torch.cuda.Stream(device=dev)
    ctx = q3attn.Context(n_layers=2, max_seq=L_CTX, kv_dtype=kv, ptr_mode=q3attn.PTR_DEVICE)
    ctx.set_stream(stream.cuda_stream)
    fill_cache(ctx, torch, dev, 1234, 2, POS, stream)
    q = torch.randn(2, HQ * HD, device=dev)
    k = torch.randn(2, KV_DIM, device=dev)
    v = torch.randn(2, KV_DIM, device=dev)
    w = torch.ones(HD, device=dev)
    xb = torch.zeros(2, HQ * HD, device=dev)
    stream.synchronize()
    for i in range(args.warmup + args.steps):
        ctx.attn_layer(xb[i % 2], q[i % 2], k[i % 2], v[i % 2], w, w, i % 2, POS)
    stream.synchronize()
    ctx.check_device_error()
    ctx.close()
    print(f"ncu case {args.ncu_case}: {args.warmup + args.steps} launches ok")


# ------------------------------------------------------------------ main
_LINE_OUT = None  # the stream of the one JSON line (the saved stdout at N > 1)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=100)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline leg")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-variants", action="store_true")
    ap.add_argument("--ncu-case", default=None, choices=["decode-f32", "decode-bf16", "prefill", "qkv", "wo", "sublayer"],
                    help="small single-kernel run for ncu captures (2 layers, direct launches)")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    world, rank, local = dist_setup()
    global _LINE_OUT
    if world > 1:
        # libraries (NCCL) may print to stdout; everything but the JSON line
        # goes to stderr, the line to the saved stdout
        _LINE_OUT = os.fdopen(os.dup(1), "w")
        os.dup2(2, 1)
    if args.ncu_case:
        ncu_case(args)
        return
    if args.impl == "reference":
        run_reference(args, world, rank)
        return

    import torch
    dev = torch.device(f"cuda:{local}")
    torch.cuda.set_device(dev)
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=dev)
    import q3attn
    seed = 1234 + 7919 * rank
    hbm_peak, tf_peak, tf_sus, peak_src = measured_peaks()

    main_res = decode_run(args, torch, dev, local, q3attn.KV_F32, seed, world,
                          with_e2e=not args.no_e2e, with_cpu=False)
    t_max = max_over_ranks(main_res["t_ms"], world, dev)
    bpl = main_res["bytes_per_layer"]
    K = args.steps
    value = world * K * N_LAYERS * bpl / (t_max / 1000.0) / 1e9
    us_per_layer = t_max * 1000.0 / (K * N_LAYERS)
    kern_us = main_res["kernel_us"]
    achieved = bpl / (kern_us * 1e-6) / 1e9
    traffic = profile_traffic("decode_f32_8k")
    line = {"metric": METRIC, "value": value, "unit": "GB/s", "n_gpus": world, "steps": K,
            "warmup": args.warmup, "ms_per_step": t_max / K, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": config_dict(args, "f32"), "us_per_layer": us_per_layer,
            "gpu_launches": main_res["launches"], "clocks": main_res["clocks"],
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": hbm_peak, "unit": "GB/s",
                         "frac": achieved / hbm_peak, "traffic": traffic,
                         "kernel": "q3a::decode_kernel<float>",
                         "kernel_us_mean": kern_us,
                         "duration_source": "graph of K x 36 back-to-back launches between two "
                                            "CUDA events on the launch stream, / launches",
                         "peak_source": f"{peak_src} hbm_gbs (MEASURED_PEAKS.json)",
                         "algorithmic_bytes_per_launch": bpl}}
    if "e2e" in main_res:
        e = main_res["e2e"]
        t_e = max_over_ranks(e["t_ms"], world, dev)
        line["e2e"] = {"value": world * K * N_LAYERS * bpl / (t_e / 1000.0) / 1e9, "unit": "GB/s",
                       "h2d_bytes_per_step": e["h2d_bytes_per_step"],
                       "d2h_bytes_per_step": e["d2h_bytes_per_step"],
                       "us_per_layer": t_e * 1000.0 / (K * N_LAYERS),
                       "api": "q3a_attn_layer, host pointers, synchronous per layer, "
                              "called from the C host qwen3.c_b200/lib/q3a_harness",
                       "timer": "CLOCK_MONOTONIC around K steps in the C host",
                       "gpu_launches": e["launches"]}
    if not args.no_variants:
        b = decode_run(args, torch, dev, local, q3attn.KV_BF16, seed, world, with_e2e=False,
                       with_cpu=False)
        tb = max_over_ranks(b["t_ms"], world, dev)
        bb = b["bytes_per_layer"]
        ach_b = bb / (b["kernel_us"] * 1e-6) / 1e9
        line["bf16"] = {"value": world * K * N_LAYERS * bb / (tb / 1000.0) / 1e9, "unit": "GB/s",
                        "us_per_layer": tb * 1000.0 / (K * N_LAYERS),
                        "kernel_us_mean": b["kernel_us"], "achieved": ach_b,
                        "frac": ach_b / hbm_peak, "traffic": profile_traffic("decode_bf16_8k"),
                        "clocks": b["clocks"],
                        "gpu_launches": b["launches"]}
        line["gpu_launches"] += b["launches"]
    if not args.no_variants:
        pr = prefill_run(args, torch, dev, local, seed, world, rank)
        t_p = max_over_ranks(pr["t_ms"], world, dev)
        fl = prefill_flops()
        # every rank processes its 8/N KV heads of each layer: the job
        # computes `layers` whole layers in t_p
        us_l = t_p * 1000.0 / pr["layers"]
        tf = fl * pr["layers"] / (t_p / 1000.0) / 1e12
        line["prefill"] = {"metric": "prefill attn TFLOP/s (2K tok)", "value": tf,
                           "unit": "TFLOP/s", "us_per_layer": us_l,
                           "flops_per_layer": fl, "steps": pr["steps"],
                           # the timed region is milliseconds long (K x 36
                           # launches), a burst: the burst bf16 peak is the
                           # denominator; the sustained-peak fraction is kept
                           # beside it for reference
                           "roofline": {"bound": "tensor", "achieved": tf / world,
                                        "peak": tf_peak, "unit": "TFLOP/s",
                                        "frac": tf / world / tf_peak,
                                        "frac_of_sustained_peak": tf / world / tf_sus,
                                        "timed_region_ms": t_p,
                                        "peak_source": f"{peak_src} bf16_tflops (burst, "
                                                       "MEASURED_PEAKS.json)",
                                        "kernel": "q3a::prefill_kernel",
                                        "traffic": profile_traffic("prefill_2k")},
                           "workload": "configs[2]: causal prefill S=2048, Hq=32, Hkv=8, "
                                       "d=128, bf16 Q/K/V, bf16 out, 36 layers per step",
                           "parallelism": f"kvhead{world}" if world > 1 else "single",
                           "scaling": "strong",
                           "clocks": pr["clocks"], "gpu_launches": pr["launches"]}
        if pr["t_ms_sharded_out"] is not None:
            # kernel time with each rank's output left head-sharded (no gather)
            t_so = max_over_ranks(pr["t_ms_sharded_out"], world, dev)
            line["prefill"]["sharded_out"] = {
                "us_per_layer": t_so * 1000.0 / pr["layers"],
                "value": fl * pr["layers"] / (t_so / 1000.0) / 1e12, "unit": "TFLOP/s",
                "note": "same launches without the all-gather of the output head slices"}
            line["gpu_launches"] += pr["launches_sharded_out"]
        line["gpu_launches"] += pr["launches"]
    if not args.no_variants:
        lc = long_ctx_run(args, torch, dev, local, world, rank)
        t_l = max_over_ranks(lc["t_ms"], world, dev)
        bpl_l = 2 * LONG_L * KV_DIM * 2
        n_lay = lc["steps"] * N_LAYERS
        us_l = t_l * 1000.0 / n_lay
        line["long_ctx"] = {"metric": "decode attn µs/layer (KV 128K, sequence-sharded)",
                            "value": bpl_l * n_lay / (t_l / 1000.0) / 1e9, "unit": "GB/s",
                            "us_per_layer": us_l, "n_gpus": world, "scaling": "strong",
                            "parallelism": f"seq{world}" if world > 1 else "single",
                            "workload": "configs[3]: KV 131072 bf16, batch 1, Hq=32, Hkv=8, "
                                        "d=128, 36 layers per step; per layer one "
                                        "q3a_attn_seqshard launch: split-KV decode of the "
                                        "local chunk, (o, lse) of each KV head stored into "
                                        "every rank over NVLink, merged on every rank",
                            "bytes_per_layer": bpl_l, "rows_per_gpu": lc["rows_local"],
                            "hbm_frac_per_gpu": bpl_l / world / (us_l * 1e-6) / 1e9 / hbm_peak,
                            "clocks": lc["clocks"], "gpu_launches": lc["launches"]}
        line["gpu_launches"] += lc["launches"]
        if world > 1:
            # t(1) of the same step, on rank 0's GPU alone (the others wait)
            barrier(world)
            if rank == 0:
                t1 = long_ctx_single(args, torch, dev, local)
                line["long_ctx"]["us_per_layer_1gpu"] = t1
                line["long_ctx"]["speedup_vs_1gpu"] = t1 / us_l
            barrier(world)
        rg = ragged_run(args, torch, dev, local, world, rank)
        t_r = max_over_ranks(rg["t_ms"], world, dev)
        us_s = t_r * 1000.0 / rg["steps"]
        line["ragged_batch"] = {"metric": "batched ragged decode attn µs/step (64 seqs)",
                                "value": rg["bytes_per_step"] * rg["steps"] / (t_r / 1000.0) / 1e9,
                                "unit": "GB/s", "us_per_step": us_s, "n_gpus": world,
                                "scaling": "strong",
                                "parallelism": f"kvhead{world}" if world > 1 else "single",
                                "workload": "configs[4]: 64 sequences, KV lengths U[512, 32768] "
                                            f"(mean {rg['mean_len']:.0f}), bf16, one fused "
                                            "q3a_attn_layer_batched launch per step + "
                                            "all-gather of the xb head slices over NVLink "
                                            "(q3a_gather_cols)",
                                "bytes_per_step": rg["bytes_per_step"],
                                "hbm_frac_per_gpu": rg["bytes_per_step"] / world / (us_s * 1e-6)
                                / 1e9 / hbm_peak,
                                "clocks": rg["clocks"], "gpu_launches": rg["launches"]}
        line["gpu_launches"] += rg["launches"]
        sb = sublayer_run(args, torch, dev, local, seed, world, rank)
        nkv = sb["nkv"]
        n_lay = args.steps * N_LAYERS
        t_q = max_over_ranks(sb["qkv"]["t_ms"], world, dev)
        t_w = max_over_ranks(sb["wo"]["t_ms"], world, dev)
        t_s = max_over_ranks(sb["sublayer"]["t_ms"], world, dev)
        us_q, us_w, us_s = (t * 1000.0 / n_lay for t in (t_q, t_w, t_s))
        qb, wb = proj_bytes(4, nkv), wo_bytes(nkv)
        cache_b = 2 * (POS + 1) * nkv * HD * 4
        sub_b = qb + cache_b + wb                      # per GPU per layer
        ach_q = qb / (us_q * 1e-6) / 1e9
        ach_w = wb / (us_w * 1e-6) / 1e9
        line["sublayer"] = {
            "metric": "attention sublayer x -> x + attn(x), µs/layer (KV 8K, fp32 cache)",
            "value": world * sub_b * n_lay / (t_s / 1000.0) / 1e9, "unit": "GB/s",
            "us_per_layer": us_s, "bytes_per_layer_per_gpu": sub_b, "n_gpus": world,
            "scaling": "strong",
            "parallelism": f"kvhead{world}" if world > 1 else "single",
            "workload": "Qwen3-8B attention sublayer of one token: rmsnorm fused into the fp16 "
                        "q/k/v projections + QK-norm + RoPE + append (qkv_kernel), decode over "
                        "8193 rows of the fp32 cache, wo + residual (wo_kernel; at N > 1 the "
                        "ranks' partial products summed over NVLink inside it); 36 layers per "
                        "step (q3a_attn_sublayer)",
            "hbm_frac_per_gpu": sub_b / (us_s * 1e-6) / 1e9 / hbm_peak,
            "qkv": {"us_per_layer": us_q, "bytes_per_launch": qb,
                    "roofline": {"bound": "hbm", "achieved": ach_q, "peak": hbm_peak,
                                 "unit": "GB/s", "frac": ach_q / hbm_peak,
                                 "traffic": profile_traffic("qkv_proj") if world == 1 else None,
                                 "kernel": "q3a::qkv_kernel<float,1>",
                                 "duration_source": "graph of K x 36 q3a_qkv_proj launches "
                                                    "between two events, / launches"},
                    "clocks": sb["qkv"]["clocks"], "gpu_launches": sb["qkv"]["launches"]},
            "wo": {"us_per_layer": us_w, "bytes_per_launch": wb,
                   "roofline": {"bound": "hbm", "achieved": ach_w, "peak": hbm_peak,
                                "unit": "GB/s", "frac": ach_w / hbm_peak,
                                "traffic": profile_traffic("wo_residual") if world == 1 else None,
                                "kernel": "q3a::wo_kernel<1>",
                                "duration_source": "graph of K x 36 q3a_wo_residual launches "
                                                   "between two events, / launches"},
                   "clocks": sb["wo"]["clocks"], "gpu_launches": sb["wo"]["launches"]},
            "clocks": sb["sublayer"]["clocks"], "gpu_launches": sb["sublayer"]["launches"]}
        line["gpu_launches"] += (sb["qkv"]["launches"] + sb["wo"]["launches"] +
                                 sb["sublayer"]["launches"])
        if rank == 0 and world == 1 and not args.no_cpu:
            line["sublayer"]["cpu_baseline"] = cpu_sublayer_sample(n_calls_max=20, budget_s=5.0)
    if rank == 0 and world == 1 and not args.no_cpu:
        cpu = cpu_reference_sample(n_calls_max=400, budget_s=15.0)
        line["cpu_baseline"] = {k: cpu[k] for k in ("value", "unit", "cores", "kind", "sample")}
        line["cpu_baseline"]["us_per_layer"] = cpu["us_per_layer"]
    if rank == 0:
        print(json.dumps(line), file=_LINE_OUT or sys.stdout, flush=True)
    if world > 1:
        import torch.distributed as dist
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
