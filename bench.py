#!/usr/bin/env python
"""Benchmark of the GQA decode-attention hot path (config 5 for N > 1).

One step = one Qwen3-4B decode token's attention over all 36 layers: q [1, 32, 128] per layer
against that layer's static KV of L = 8192 keys per GPU, laid out [layer, 2, nkv=8, max_len,
hd=128] bf16 in HBM (1.2 GB per GPU, larger than the 126 MB L2, so consecutive layers never hit in
L2). Inputs are seeded synthetic tensors with the reference's pipeline: N(0,1) -> QK-RMSNorm
(eps 1e-6) -> RoPE (theta 1e6). The 36 calls are captured in one CUDA graph and replayed.

N > 1 (torchrun): the sequence is sharded, context 8192 * N with 8192 keys per rank (weak
scaling, the headline); per layer each rank computes a partial (O, LSE) of its shard and the
partials meet over NVLink (peer stores, or NCCL all-gather) and are merged on every rank. The
``config5`` section measures BASELINE config 5 as specified at every N: a fixed 131072-key
context, 131072 / N keys per rank (strong scaling), both exchanges, with the single-GPU time of
the whole context measured in the same run.

Prints ONE JSON line (rank 0). ``value`` = KV bytes read by all ranks per second (GB/s).
``--impl reference`` times the reference's CPU attention path (the grouped decode of
``cuda_graph_executor.py:180-184``, restated in ``oracle/``) on the host cores instead.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

LAYERS, NH, NKV, HD = 36, 32, 8, 128
THETA, EPS = 1e6, 1e-6


def parse_args():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--ctx", type=int, default=8192, help="keys per GPU")
    ap.add_argument("--long-ctx", type=int, default=131072,
                    help="--workload long: keys per layer (131072 = BASELINE config 5; a "
                    "1/N shard of it times one rank's local decode without the exchange)")
    ap.add_argument("--cpu-sample-s", type=float, default=15.0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--sweep", action="store_true", help="also time L in {128..8192}")
    ap.add_argument("--workload", choices=["decode", "prefill", "paged", "long"], default="decode",
                    help="decode: BASELINE config 2 (+ prefill section); prefill: config 3 only; "
                         "paged: config 4 only; long: the 131072-key decode (config 5 on one "
                         "GPU) only (the default line's paged / long_ctx sections alone)")
    ap.add_argument("--layers", type=int, default=36,
                    help="--workload long: layers of 512 MiB of K+V each (36 as in the model)")
    ap.add_argument("--no-prefill", action="store_true")
    ap.add_argument("--exchange", choices=["p2p", "nccl"], default="p2p",
                    help="N>1: partials cross GPUs by NVLink peer stores (p2p) or an NCCL all-gather")
    ap.add_argument("--prefill-T", type=int, nargs="+", default=[512, 1024, 4096])
    ap.add_argument("--step-timeline", action="store_true",
                    help="print the kernel-by-kernel critical path of one Qwen3-4B-shaped decode "
                         "step (CUPTI timeline; diagnostic, not a bench value)")
    ap.add_argument("--no-stable-prefix", action="store_true",
                    help="decode calls without SOLORT_DECODE_STABLE_PREFIX (keys requested only "
                         "after the previous kernel finished)")
    ap.add_argument("--no-config5", action="store_true",
                    help="skip the 131072-key strong-scaling section (BASELINE config 5)")
    ap.add_argument("--no-extras", action="store_true",
                    help="skip the paged / long-context / tok/s sections of the default line")
    return ap.parse_args()


# ------------------------------------------------------------------------------------------
# clocks during the timed region
# ------------------------------------------------------------------------------------------
class ClockSampler:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.path = None

    def start(self):
        import tempfile

        fd, self.path = tempfile.mkstemp(suffix=".csv")
        os.close(fd)
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-i", str(self.gpu), "-lms", "100"],
                stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None
        time.sleep(0.3)

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        time.sleep(0.2)
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        rows = []
        with open(self.path) as fh:
            for line in fh:
                parts = [p.strip() for p in line.split(",")]
                if len(parts) >= 9 and parts[1].isdigit():
                    rows.append(parts)
        os.unlink(self.path)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"]}
        sm = [int(r[1]) for r in rows]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[5 + i] == "Active"})
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": int(rows[0][2]), "reasons": reasons,
                "samples": len(rows), "power_w_max": max(float(r[3]) for r in rows
                                                         if r[3].replace(".", "").isdigit())}


# ------------------------------------------------------------------------------------------
# synthetic inputs (on the device)
# ------------------------------------------------------------------------------------------
def _rmsnorm(x, eps=EPS):
    d = x.float()
    return (d * (d.pow(2).mean(-1, keepdim=True) + eps).rsqrt()).to(x.dtype)


def _rope(x, pos, dtype):
    import torch

    inv = 1.0 / (THETA ** (torch.arange(0, HD, 2, device=x.device).float() / HD))
    f = pos[:, None].float() * inv[None, :]
    emb = torch.cat([f, f], -1)
    cos, sin = emb.cos().to(dtype), emb.sin().to(dtype)
    while cos.dim() < x.dim():
        cos, sin = cos.unsqueeze(-2), sin.unsqueeze(-2)
    h = HD // 2
    return x * cos + torch.cat([-x[..., h:], x[..., :h]], -1) * sin


def make_inputs(ctx: int, rank: int, world: int, device, seed: int = 2024, layers: int = LAYERS):
    """KV [layers, 2, 8, ctx, 128] for keys [rank*ctx, (rank+1)*ctx) of a ctx*world context, and
    the layers' query [layers, 1, 1, 32, 128] at position ctx*world - 1 (same on every rank)."""
    import torch

    bf = torch.bfloat16
    kv = torch.empty(layers, 2, NKV, ctx, HD, dtype=bf, device=device)
    pos = torch.arange(rank * ctx, (rank + 1) * ctx, device=device)
    g = torch.Generator(device=device)
    for li in range(layers):
        g.manual_seed(seed * 1000 + li * 16 + rank)
        k = torch.randn(ctx, NKV, HD, generator=g, device=device).to(bf)
        v = torch.randn(ctx, NKV, HD, generator=g, device=device).to(bf)
        kv[li, 0] = _rope(_rmsnorm(k), pos, bf).transpose(0, 1)
        kv[li, 1] = v.transpose(0, 1)
    g.manual_seed(seed)
    q = torch.randn(layers, 1, 1, NH, HD, generator=g, device=device).to(bf)
    qpos = torch.full((1,), ctx * world - 1, dtype=torch.int64, device=device)
    q = _rope(_rmsnorm(q), qpos.repeat(1), bf)
    return kv, q, qpos


# ------------------------------------------------------------------------------------------
# CPU baseline / reference arm: the reference's grouped decode on the host cores
# ------------------------------------------------------------------------------------------
def cpu_reference_rate(ctx: int, budget_s: float, threads: int) -> dict:
    import torch

    from oracle import attention as A

    torch.set_num_threads(threads)
    q, k, v = A.make_attention_inputs(7, NH, NKV, HD, 1, ctx, ctx - 1)
    scale = HD ** -0.5
    A.decode_reference_grouped(q[0], k, v, ctx - 1, ctx, scale)  # warm
    n, t0 = 0, time.perf_counter()
    while True:
        A.decode_reference_grouped(q[0], k, v, ctx - 1, ctx, scale)
        n += 1
        el = time.perf_counter() - t0
        if el >= budget_s or n >= 100000:
            break
    per_call = el / n
    gbs = 2 * ctx * NKV * HD * 2 / per_call / 1e9
    return {"value": round(gbs, 3), "unit": "GB/s", "cores": threads, "kind": "port",
            "sample": f"{n} single-layer calls of the reference grouped decode "
                      f"(cuda_graph_executor.py:180-184, restated in oracle/) at L={ctx}, "
                      f"32/8 heads, bf16 on CPU; {per_call * 1e3:.2f} ms/call",
            "ms_per_layer_call": round(per_call * 1e3, 4)}


def run_reference_arm(args) -> None:
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    import torch

    threads = os.cpu_count() or 1
    per_step_budget = max(1.0, args.cpu_sample_s / max(1, args.steps))
    # warmup
    for _ in range(args.warmup):
        cpu_reference_rate(args.ctx, 0.2, threads)
    vals = []
    t0 = time.perf_counter()
    for _ in range(args.steps):
        vals.append(cpu_reference_rate(args.ctx, per_step_budget, threads))
    wall = time.perf_counter() - t0
    value = statistics.median(v["value"] for v in vals)
    ms_layer = statistics.median(v["ms_per_layer_call"] for v in vals)
    line = {
        "impl": "reference",
        "metric": "GQA decode-attn HBM GB/s",
        "value": value, "unit": "GB/s", "n_gpus": args.gpus, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(ms_layer * LAYERS, 3),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (seeded N(0,1) -> QK-RMSNorm -> RoPE theta 1e6)",
        "config": {"workload": f"qwen3-4b decode attention, L={args.ctx}, 32/8 heads, hd 128",
                   "sample": "per step: single-layer calls for a bounded time, x36 layers"},
        "cpu_baseline": {"value": value, "unit": "GB/s", "cores": threads, "kind": "port",
                         "sample": vals[0]["sample"]},
        "e2e": {"value": value, "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "wall_s": round(wall, 2),
        "torch_threads": torch.get_num_threads(),
    }
    print(json.dumps(line), flush=True)


# ------------------------------------------------------------------------------------------
# GPU arm
# ------------------------------------------------------------------------------------------

CONFIG5_KEYS, CONFIG5_LAYERS = 131072, 8


def config5_bench(dev, rank: int, world: int, steps: int) -> dict:
    """BASELINE config 5 as specified: a fixed 131072-key context sharded over the N ranks
    (131072 / N contiguous keys each; strong scaling), CONFIG5_LAYERS layers per step, every
    exchange the library offers for N > 1. Reports the per-layer time (max over ranks), the KV
    bytes of all ranks per second and per rank, and the strong-scaling efficiency T1 / (N * TN)
    against the single-GPU decode of the whole context timed on rank 0 in the same run."""
    import torch
    import torch.distributed as dist

    from solort_b200 import ops

    shard = CONFIG5_KEYS // world
    layers = CONFIG5_LAYERS
    bytes_total = 2 * CONFIG5_KEYS * NKV * HD * 2  # K + V of the whole context, per layer

    def timed(step) -> float:
        s = torch.cuda.Stream(device=dev)
        s.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(s):
            for _ in range(2):
                step()
        torch.cuda.current_stream(dev).wait_stream(s)
        torch.cuda.synchronize(dev)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            step()
        for _ in range(3):
            g.replay()
        torch.cuda.synchronize(dev)
        if world > 1:
            dist.barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(steps):
            g.replay()
        e1.record()
        torch.cuda.synchronize(dev)
        us = e0.elapsed_time(e1) * 1e3 / steps / layers
        if world > 1:
            t = torch.tensor([us], dtype=torch.float64, device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            us = float(t.item())
        del g
        return us

    # single-GPU reference: the whole context on rank 0 alone
    t1 = None
    if rank == 0:
        kv1, q1, qpos1 = make_inputs(CONFIG5_KEYS, 0, 1, dev, seed=55, layers=layers)
        out1 = torch.empty_like(q1)
        ws1 = torch.empty(max(256, ops.decode_workspace_bytes(1, 1, NH, NKV, CONFIG5_KEYS)),
                          dtype=torch.uint8, device=dev)

        def step1():
            for li in range(layers):
                ops.gqa_decode(q1[li], kv1[li, 0], kv1[li, 1], qpos1, kv_layout="HND",
                               out=out1[li], workspace=ws1, stable_prefix=True)

        world_saved, world = world, 1  # time it without cross-rank barriers
        t1 = timed(step1)
        world = world_saved
        del kv1
        torch.cuda.empty_cache()
    res = {"total_keys": CONFIG5_KEYS, "keys_per_rank": shard, "layers": layers,
           "scaling": "strong (fixed context, 1/N of it per rank)",
           "single_gpu_us_per_layer": None if t1 is None else round(t1, 2)}
    if world == 1:
        res["us_per_layer"] = round(t1, 2)
        res["GBs"] = round(bytes_total / (t1 * 1e-6) / 1e9, 1)
        return res
    from solort_b200.sharded import ShardedDecode

    kv, q, qpos = make_inputs(shard, rank, world, dev, seed=55, layers=layers)
    outs = torch.empty_like(q)
    ws = torch.empty(max(256, ops.decode_workspace_bytes(1, 1, NH, NKV, shard),
                         ops.decode_exchange_workspace_bytes(1, 1, NH, NKV, shard)),
                     dtype=torch.uint8, device=dev)
    t1_all = torch.tensor([t1 or 0.0], dtype=torch.float64, device=dev)
    dist.broadcast(t1_all, 0)
    t1 = float(t1_all.item())
    res["single_gpu_us_per_layer"] = round(t1, 2)
    for exchange in ("p2p", "nccl"):
        sd = ShardedDecode(rank, world, num_qo_heads=NH, layers=layers, device=dev,
                           exchange=exchange)

        def stepn():
            for li in range(layers):
                sd.layer(li, q[li], kv[li, 0], kv[li, 1], qpos, rank * shard, outs[li], ws,
                         stable_prefix=True)

        tn = timed(stepn)
        sd.close()
        res[exchange] = {"us_per_layer": round(tn, 2),
                         "GBs_all_ranks": round(bytes_total / (tn * 1e-6) / 1e9, 1),
                         "GBs_per_rank": round(bytes_total / world / (tn * 1e-6) / 1e9, 1),
                         "strong_scaling_efficiency": round(t1 / (world * tn), 3)}
    return res


def run_gpu_arm(args) -> None:
    import torch
    import torch.distributed as dist

    from solort_b200 import ops

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={world}")
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        import datetime

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=dev)
    ctx = args.ctx
    kv, q, qpos = make_inputs(ctx, rank, world, dev)
    bytes_per_layer = 2 * ctx * NKV * HD * 2  # K + V of this rank's keys
    outs = torch.empty_like(q)
    ws = torch.empty(max(256, ops.decode_workspace_bytes(1, 1, NH, NKV, ctx),
                         ops.decode_exchange_workspace_bytes(1, 1, NH, NKV, ctx)), dtype=torch.uint8,
                     device=dev)
    sharded = None
    if world > 1:
        from solort_b200.sharded import ShardedDecode

        sharded = ShardedDecode(rank, world, num_qo_heads=NH, layers=LAYERS, device=dev,
                                exchange=args.exchange)

    # q_pos and every key are written before the graph: the calls may request their keys while
    # the previous layer's kernels finish (SOLORT_DECODE_STABLE_PREFIX), as the runner's do.
    stable = not args.no_stable_prefix

    def step():
        for li in range(LAYERS):
            if sharded is None:
                ops.gqa_decode(q[li], kv[li, 0], kv[li, 1], qpos, kv_layout="HND",
                               out=outs[li], workspace=ws, stable_prefix=stable)
            else:
                sharded.layer(li, q[li], kv[li, 0], kv[li, 1], qpos, rank * ctx, outs[li], ws,
                              stable_prefix=stable)

    # capture one step in a graph (side-stream warm-up first, as the reference does)
    s = torch.cuda.Stream(device=dev)
    s.wait_stream(torch.cuda.current_stream(dev))
    with torch.cuda.stream(s):
        for _ in range(2):
            step()
    torch.cuda.current_stream(dev).wait_stream(s)
    torch.cuda.synchronize(dev)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        step()
    torch.cuda.synchronize(dev)

    # correctness spot check of layer 0 against a torch fp32 evaluation on the device
    graph.replay()
    torch.cuda.synchronize(dev)
    if world == 1:
        _spot_check(q[0], kv[0], outs[0], ctx)

    for _ in range(max(3, args.warmup)):
        graph.replay()
    torch.cuda.synchronize(dev)
    if world > 1:
        dist.barrier()
    clocks = ClockSampler(local)
    if rank == 0:
        clocks.start()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize(dev)
    if world > 1:
        dist.barrier()
    start.record()
    for _ in range(args.steps):
        graph.replay()
    end.record()
    torch.cuda.synchronize(dev)
    if world > 1:
        dist.barrier()
    ms = start.elapsed_time(end) / args.steps
    clk = clocks.stop() if rank == 0 else None
    if world > 1:
        t = torch.tensor([ms], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())

    # e2e through the public API with host buffers: per step, pinned q -> device, the step, the
    # outputs -> pinned host. The step is the captured graph of the 36 per-layer public calls (the
    # reference executor replays its decode step as a CUDA graph); the same calls issued eagerly
    # from Python (prepared ctypes calls on the current stream) are reported beside it.
    q_host = q.cpu().pin_memory()
    out_host = torch.empty_like(q_host).pin_memory()
    calls = []
    if sharded is None:
        calls = [ops.DecodeCall(q[li], kv[li, 0], kv[li, 1], qpos, kv_layout="HND",
                                out=outs[li], workspace=ws, stable_prefix=stable)
                 for li in range(LAYERS)]
    elif args.exchange == "p2p":
        calls = [sharded.prepared_layer(li, q[li], kv[li, 0], kv[li, 1], qpos, rank * ctx,
                                        outs[li], ws, stable_prefix=stable)
                 for li in range(LAYERS)]

    def eager_calls():
        if calls:
            for c in calls:
                c()
        else:
            step()

    def timed_e2e(run) -> float:
        def e2e_step():
            q.copy_(q_host, non_blocking=True)
            run()
            out_host.copy_(outs, non_blocking=True)

        for _ in range(3):
            e2e_step()
        torch.cuda.synchronize(dev)
        if world > 1:
            dist.barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        n = max(5, args.steps // 2)
        e0.record()
        for _ in range(n):
            e2e_step()
        e1.record()
        torch.cuda.synchronize(dev)
        t_ms = e0.elapsed_time(e1) / n
        if world > 1:
            t = torch.tensor([t_ms], dtype=torch.float64, device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            t_ms = float(t.item())
        return t_ms

    e2e_ms = timed_e2e(graph.replay)
    e2e_eager_ms = timed_e2e(eager_calls)

    config5 = None if args.no_config5 else config5_bench(dev, rank, world, max(3, args.steps // 4))

    sweep = None
    if args.sweep and world == 1:
        sweep = _sweep(kv, q, qpos, ws, dev)

    total_bytes = bytes_per_layer * LAYERS * world
    value = total_bytes / (ms / 1e3) / 1e9
    e2e_value = total_bytes / (e2e_ms / 1e3) / 1e9
    e2e_eager_value = total_bytes / (e2e_eager_ms / 1e3) / 1e9
    per_call_us = ms * 1e3 / LAYERS
    peaks = _peaks()
    achieved = bytes_per_layer / (per_call_us * 1e-6) / 1e9
    # Each rank's decode launch is the single-GPU launch of its ctx keys (the exchange changes only
    # where the merge sends the rows), so the same capture gives its traffic.
    traffic, traffic_src = _profiled_traffic("decode", ctx)
    line = {
        "metric": "GQA decode-attn HBM GB/s",
        "value": round(value, 1),
        "unit": "GB/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(ms, 4),
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "bf16",
        "data": "synthetic (seeded N(0,1) -> QK-RMSNorm eps 1e-6 -> RoPE theta 1e6)",
        "config": {
            "workload": "qwen3-4b static-KV single-token decode attention (BASELINE config 2"
                        + (", seq-sharded per config 5)" if world > 1 else ")"),
            "layers": LAYERS, "num_qo_heads": NH, "num_kv_heads": NKV, "head_dim": HD,
            "keys_per_gpu": ctx, "context": ctx * world,
            "kv_layout": "[layer, 2, nkv, max_len, hd] bf16",
            "parallelism": f"seq-shard x{world}" if world > 1 else "single GPU",
            "exchange": (("NVLink peer stores of self-marking words + polling merge kernel"
                          if args.exchange == "p2p"
                          else "NCCL all_gather_into_tensor + lse_merge") if world > 1 else None),
            "l2": "inputs larger than L2: 36 layers x 32 MiB KV per GPU replayed in order",
            "graph": "36 layer calls per CUDA graph replay",
            "stable_prefix": stable,
        },
        "pct_of_8TBs": round(100 * value / world / 8000, 2),
        "roofline": {
            "bound": "hbm",
            "kernel": "one attention call = decode_kernel (split-KV) + merge_kernel (PDL-chained)",
            "achieved": round(achieved, 1),
            "peak": peaks[0],
            "unit": "GB/s",
            "frac": round(achieved / peaks[0], 4),
            "peak_source": peaks[1],
            "algorithmic_bytes_per_launch": bytes_per_layer,
            "us_per_launch": round(per_call_us, 3),
            "traffic": traffic,
            "traffic_source": (f"ncu dram__bytes_read.sum + dram__bytes_write.sum of one "
                               f"decode_kernel launch of this workload"
                               + (" (per rank)" if world > 1 else "") + f" ({traffic_src})"
                               if traffic is not None else "no ncu capture of this shape"),
        },
        "e2e": {"value": round(e2e_value, 1), "unit": "GB/s",
                "h2d_bytes_per_step": q_host.numel() * 2,
                "d2h_bytes_per_step": out_host.numel() * 2,
                "ms_per_step": round(e2e_ms, 4),
                "how": "the CUDA graph of one step's 36 public per-layer calls ("
                       + ("ops.gqa_decode" if world == 1 else "ShardedDecode.layer: decode + "
                          + args.exchange + " exchange + merge")
                       + "), replayed between the pinned H2D of the 36 queries and the D2H of "
                       "the 36 outputs, all inside the timed region",
                "eager": {"value": round(e2e_eager_value, 1), "ms_per_step": round(e2e_eager_ms, 4),
                          "how": ("ops.DecodeCall" if world == 1 else
                                  "ops.ShardedDecodeCall" if calls else "ShardedDecode.layer")
                                 + " per layer issued from Python, same copies"}},
        "gpu_launches": LAYERS * (2 if world == 1 else 3) * args.steps,
        "gpu_launches_note": ("timed region: 36 decode_kernel + 36 merge_kernel launches per step"
                              if world == 1 else
                              "timed region per step: 36 x (decode_kernel + merge_kernel sending "
                              "to every rank + exchange_merge_kernel)" if args.exchange == "p2p"
                              else "timed region per step: 36 x (decode_kernel + merge_kernel + "
                              "lse merge), NCCL all-gather kernels not counted"),
        "clocks": clk,
    }
    if config5 is not None:
        line["config5"] = config5
    if sweep:
        line["sweep"] = sweep
    if world == 1 and not args.no_extras:
        line["paged"] = paged_bench(dev, max(3, args.steps // 4))
        line["long_ctx"] = long_ctx_bench(dev, max(2, args.steps // 10))
        line["decode_tok_s"] = tok_s_bench(dev)
        line["decode_tok_s_qwen3_0.6b"] = tok_s_bench(dev, shape="qwen3-0.6b")
        line["decode_tok_s_single_graph"] = tok_s_bench(dev, single_graph=True)
    if world == 1 and not args.no_prefill:
        line["prefill"] = prefill_bench(dev, args.steps, args.warmup, tuple(args.prefill_T))
        if not args.no_cpu_baseline:
            line["prefill"]["cpu_reference_ms_T512"] = round(cpu_prefill_ms(512, os.cpu_count() or 1), 2)
    if world == 1 and rank == 0 and not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_reference_rate(ctx, args.cpu_sample_s, os.cpu_count() or 1)
    if rank == 0:
        print(json.dumps(line), flush=True)
    del graph
    if sharded is not None:
        sharded.close()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def _spot_check(q, kv, out, ctx):
    import torch

    qf = q[0, 0].float().view(NKV, NH // NKV, HD)
    k = kv[0].float()
    v = kv[1].float()
    s = torch.matmul(qf, k.transpose(1, 2)) * HD ** -0.5
    ref = torch.matmul(torch.softmax(s, -1), v).reshape(NH, HD)
    d = (out[0, 0].float() - ref).abs()
    if d.max().item() > 2e-2 or d.mean().item() > 2e-3:
        raise SystemExit(f"spot check failed: max {d.max().item()} mean {d.mean().item()}")


def _sweep(kv, q, qpos_full, ws, dev):
    import torch

    from solort_b200 import ops

    res = {}
    for L in (128, 512, 1024, 2048, 4096, 8192):
        qpos = torch.full((1,), L - 1, dtype=torch.int64, device=dev)
        out = torch.empty_like(q)

        def step():
            for li in range(LAYERS):
                ops.gqa_decode(q[li], kv[li, 0], kv[li, 1], qpos, kv_layout="HND", out=out[li],
                               workspace=ws, max_kv_len=L, stable_prefix=True)

        step()
        torch.cuda.synchronize(dev)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            step()
        for _ in range(3):
            g.replay()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        n = 20
        for _ in range(n):
            g.replay()
        b.record()
        torch.cuda.synchronize(dev)
        ms = a.elapsed_time(b) / n
        byt = 2 * L * NKV * HD * 2
        res[str(L)] = {"us_per_layer": round(ms * 1e3 / LAYERS, 3),
                       "GBs": round(byt * LAYERS / (ms / 1e3) / 1e9, 1),
                       "l2_resident": L * 4096 * LAYERS <= 100 * 2**20}
        del g
    return res


def prefill_bench(dev, steps: int, warmup: int, lengths=(512, 1024, 4096)) -> dict:
    """causal prefill attention of a Qwen3-4B layer, q [T, 32, 128],
    k/v [T, 8, 128] bf16 (seeded, QK-RMSNorm + RoPE). Calls rotate over input sets that
    together exceed L2. FLOPs (causal, algorithmic) = 2 * T^2 * hd * nh."""
    import torch

    from solort_b200 import ops

    res = {}
    peak, src = _peaks(tensor=True)
    for T in lengths:
        set_bytes = T * (NH + 2 * NKV) * HD * 2
        nsets = max(4, -(-(256 << 20) // set_bytes))
        sets = []
        for i in range(nsets):
            g = torch.Generator(device=dev)
            g.manual_seed(100 + i)
            pos = torch.arange(T, device=dev)
            q = _rope(_rmsnorm(torch.randn(T, NH, HD, generator=g, device=dev).to(torch.bfloat16)),
                      pos, torch.bfloat16)
            k = _rope(_rmsnorm(torch.randn(T, NKV, HD, generator=g, device=dev).to(torch.bfloat16)),
                      pos, torch.bfloat16)
            v = torch.randn(T, NKV, HD, generator=g, device=dev).to(torch.bfloat16)
            sets.append((q, k, v, torch.empty_like(q)))

        def run_all():
            for q, k, v, o in sets:
                ops.gqa_prefill(q, k, v, out=o)

        run_all()
        torch.cuda.synchronize(dev)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            run_all()
        for _ in range(max(3, warmup)):
            graph.replay()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        reps = max(3, steps // 4)
        torch.cuda.synchronize(dev)
        a.record()
        for _ in range(reps):
            graph.replay()
        b.record()
        torch.cuda.synchronize(dev)
        us = a.elapsed_time(b) * 1e3 / (reps * nsets)
        flops = 2.0 * T * T * HD * NH
        tf = flops / (us * 1e-6) / 1e12
        res[str(T)] = {"us_per_call": round(us, 2), "tflops": round(tf, 1),
                       "frac_of_peak": round(tf / peak, 4), "gflop": round(flops / 1e9, 3),
                       "rotating_sets": nsets}
        del graph, sets
    res["peak_tflops"] = peak
    res["peak_source"] = src
    res["kernel"] = ("tcgen05.mma M128 N128, TMEM accumulators, TMA-fed: prefill_kernel (one CTA per "
                     "query tile and head), prefill_items_kernel (persistent, when those items "
                     "outnumber the SMs), prefill_pp_kernel (two query tiles per CTA, >= 16 tiles)")
    return res


def _time_graph(fn, dev, reps: int, warmup: int = 3) -> float:
    """Capture fn() in a CUDA graph, replay, return ms per replay (CUDA events)."""
    import torch

    fn()
    torch.cuda.synchronize(dev)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        fn()
    for _ in range(warmup):
        g.replay()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize(dev)
    a.record()
    for _ in range(reps):
        g.replay()
    b.record()
    torch.cuda.synchronize(dev)
    ms = a.elapsed_time(b) / reps
    del g
    return ms


def paged_bench(dev, reps: int) -> dict:
    """page size 16, context 16384, 36 layers of paged NHD arenas; block tables
    are a seeded permutation of the physical pages; sequences A and B share their first 4096
    tokens (256 pages, as a prefix-cache hit gives them). A verifies K = 4 drafts at 16384..16387
    (each causal over the context and the preceding drafts), B decodes one token at 16383. One
    call per layer processes both sequences."""
    import torch

    from solort_b200 import ops

    P, ctx, K, shared = 16, 16384, 4, 256
    n_a, n_b = ctx + K, ctx
    pages_a = -(-n_a // P)
    pages_b = -(-n_b // P)
    pool = pages_a + pages_b - shared  # 1793 physical pages: A (1025) + B-only (768)
    g = torch.Generator().manual_seed(4)
    perm = torch.randperm(pool, generator=g)
    bt_a = perm[:pages_a]
    bt_b = torch.cat([bt_a[:shared], perm[pages_a: pages_a + pages_b - shared]])
    bt = torch.zeros(2, pages_a, dtype=torch.int32)
    bt[0] = bt_a.to(torch.int32)
    bt[1, :pages_b] = bt_b.to(torch.int32)
    bt = bt.to(dev)
    arenas = []
    gen = torch.Generator(device=dev)
    for li in range(LAYERS):
        gen.manual_seed(500 + li)
        a = torch.randn(pool, 2, P, NKV, HD, generator=gen, device=dev).to(torch.bfloat16)
        arenas.append(a)
    q = torch.zeros(LAYERS, 2, K, NH, HD, dtype=torch.bfloat16, device=dev)
    q.normal_(generator=gen)
    qpos = torch.tensor([ctx, ctx - 1], dtype=torch.int64, device=dev)
    qlens = torch.tensor([K, 1], dtype=torch.int32, device=dev)
    out = torch.empty_like(q)
    ws = torch.empty(ops.decode_workspace_bytes(2, K, NH, NKV, n_a, page_size=P), dtype=torch.uint8,
                     device=dev)

    def step():
        for li in range(LAYERS):
            ops.gqa_decode_paged(q[li], arenas[li], bt, qpos, max_kv_len=n_a, q_lens=qlens,
                                 out=out[li], workspace=ws, stable_prefix=True)

    ms = _time_graph(step, dev, reps)
    per_layer = (n_a + n_b) * NKV * HD * 2 * 2
    unique = (n_a + n_b - shared * P) * NKV * HD * 2 * 2
    us = ms * 1e3 / LAYERS
    return {"us_per_layer": round(us, 3), "GBs": round(per_layer / (us * 1e-6) / 1e9, 1),
            "GBs_unique_bytes": round(unique / (us * 1e-6) / 1e9, 1),
            "bytes_per_layer": per_layer, "unique_bytes_per_layer": unique,
            "workload": "page 16, ctx 16384, seq A K=4 verify + seq B decode, 256 shared pages, "
                        "36 layers x 112 MB arenas"}


def long_ctx_bench(dev, reps: int, ctx: int = 131072, layers: int = 36) -> dict:
    """BASELINE config 5 on one GPU: 32/8 heads, one query at position ctx - 1 over 131072 keys per
    layer (512 MiB of K+V), 36 layers (18 GiB)."""
    import torch

    from solort_b200 import ops

    kv = torch.empty(layers, 2, NKV, ctx, HD, dtype=torch.bfloat16, device=dev)
    gen = torch.Generator(device=dev)
    gen.manual_seed(77)
    kv.normal_(generator=gen)
    q = torch.randn(layers, 1, 1, NH, HD, generator=gen, device=dev).to(torch.bfloat16)
    qpos = torch.full((1,), ctx - 1, dtype=torch.int64, device=dev)
    out = torch.empty_like(q)
    ws = torch.empty(ops.decode_workspace_bytes(1, 1, NH, NKV, ctx), dtype=torch.uint8, device=dev)

    def step():
        for li in range(layers):
            ops.gqa_decode(q[li], kv[li, 0], kv[li, 1], qpos, kv_layout="HND", out=out[li],
                           workspace=ws, stable_prefix=True)

    ms = _time_graph(step, dev, reps)
    byt = 2 * ctx * NKV * HD * 2
    us = ms * 1e3 / layers
    del kv
    traffic, traffic_src = _profiled_traffic("decode", ctx)
    return {"ctx": ctx, "layers": layers, "us_per_layer": round(us, 2),
            "GBs": round(byt / (us * 1e-6) / 1e9, 1),
            "frac_of_measured_hbm": round(byt / (us * 1e-6) / 1e9 / _peaks()[0], 4),
            "kernel": "decode_tc_kernel (tcgen05, TMEM; splits of >= 2048 keys) or decode_kernel, "
                      "+ merge_kernel",
            "algorithmic_bytes_per_launch": byt, "traffic": traffic,
            "traffic_source": traffic_src}


# Random-weight Qwen3 shapes for the end-to-end decode rate: (layers, hidden, intermediate,
# query heads, kv heads); head_dim 128, vocab 151936, tied embeddings.
QWEN3_SHAPES = {"qwen3-4b": (36, 2560, 9728, 32, 8), "qwen3-0.6b": (28, 1024, 3072, 16, 8)}


def _qwen3_4b_runner(dev, max_len: int, shape: str = "qwen3-4b", single_graph: bool = False):
    """A random-weight Qwen3-shaped model (default 4B: 36 layers, hidden 2560, 32/8 heads, hd 128,
    intermediate 9728, vocab 151936) and the engine's CUDA-graph runner over it."""
    import torch
    from transformers import Qwen3Config, Qwen3ForCausalLM

    from solort_b200.runner import GraphQwen3Runner

    layers, hidden, inter, nh, nkv = QWEN3_SHAPES[shape]
    cfg = Qwen3Config(vocab_size=151936, hidden_size=hidden, intermediate_size=inter,
                      num_hidden_layers=layers, num_attention_heads=nh, num_key_value_heads=nkv,
                      head_dim=128, max_position_embeddings=40960, rms_norm_eps=1e-6,
                      tie_word_embeddings=True)
    cfg.rope_parameters = {"rope_type": "default", "rope_theta": 1e6}
    cfg.rope_theta = 1e6
    torch.manual_seed(0)
    with torch.device(dev):
        model = Qwen3ForCausalLM(cfg).to(torch.bfloat16).eval()
    return model, GraphQwen3Runner(model, max_len, single_decode_graph=single_graph)


def tok_s_bench(dev, new_tokens: int = 256, prompt_len: int = 512,
                shape: str = "qwen3-4b", single_graph: bool = False) -> dict:
    """End-to-end greedy decode tok/s of the engine's CUDA-graph runner on a random-weight
    Qwen3-shaped model, the reference microbenchmark's tight loop (decode_gpu_argmax back to
    back, one sync at the end; scripts/microbench_decode.py:80-84)."""
    import torch

    max_len = prompt_len + new_tokens + 16
    model, runner = _qwen3_4b_runner(dev, max_len, shape, single_graph)
    prompt = torch.randint(0, 151936, (prompt_len,), device=dev)
    with torch.no_grad():
        first = int(runner.prefill(prompt).argmax(-1).item())
        cur = first
        for pos in range(prompt_len, prompt_len + new_tokens + 4):  # capture every bucket
            cur = runner.decode_argmax(cur, pos)
        torch.cuda.synchronize(dev)
        t0 = time.perf_counter()
        tok = torch.tensor([first], device=dev)
        for pos in range(prompt_len, prompt_len + new_tokens):
            tok = runner.decode_gpu_argmax(tok, pos)
        tok.item()
        dt = time.perf_counter() - t0
    res = {"tok_s": round(new_tokens / dt, 1), "ms_per_token": round(dt * 1e3 / new_tokens, 3),
           "model": f"random-weight {shape} shape, bf16", "prompt": prompt_len,
           "decode_graphs": "one for every length" if single_graph else "one per length bucket",
           "new_tokens": new_tokens,
           "published_reference_rtx4080_tok_s": {"qwen3-4b": 67.0, "qwen3-0.6b": 160.3}[shape]}
    del runner, model
    torch.cuda.empty_cache()
    return res


def cpu_prefill_ms(T: int, threads: int) -> float:
    import torch

    from oracle import attention as A

    torch.set_num_threads(threads)
    q, k, v = A.make_attention_inputs(3, NH, NKV, HD, T, T, 0)
    A.prefill_reference(q, k, v, HD ** -0.5)
    t0 = time.perf_counter()
    n = 0
    while time.perf_counter() - t0 < 3.0 or n < 2:
        A.prefill_reference(q, k, v, HD ** -0.5)
        n += 1
    return (time.perf_counter() - t0) / n * 1e3


def run_paged_workload(args) -> None:
    """BASELINE config 4 alone, one GPU (the paged path runs as replicas only)."""
    import torch

    dev = torch.device("cuda", int(os.environ.get("LOCAL_RANK", "0")))
    torch.cuda.set_device(dev)
    res = paged_bench(dev, max(3, args.steps))
    peak = _peaks()
    line = {"metric": "paged decode+verify HBM GB/s", "value": res["GBs"], "unit": "GB/s",
            "n_gpus": 1, "steps": max(3, args.steps), "warmup": 3,
            "ms_per_step": round(res["us_per_layer"] * LAYERS / 1e3, 4), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "config": {"workload": "qwen3-4b paged decode + K=4 verify (BASELINE config 4)",
                       "page_size": 16, "ctx": 16384, "layers": LAYERS},
            "frac_of_measured_hbm": round(res["GBs"] / peak[0], 4), "peak_source": peak[1],
            "paged": res}
    print(json.dumps(line), flush=True)


def run_long_workload(args) -> None:
    """The 131072-key decode (BASELINE config 5 on one GPU) alone."""
    import torch

    dev = torch.device("cuda", int(os.environ.get("LOCAL_RANK", "0")))
    torch.cuda.set_device(dev)
    res = long_ctx_bench(dev, max(3, args.steps), ctx=args.long_ctx, layers=args.layers)
    line = {"metric": "long-context decode-attn HBM GB/s", "value": res["GBs"], "unit": "GB/s",
            "n_gpus": 1, "steps": max(3, args.steps), "warmup": 3,
            "ms_per_step": round(res["us_per_layer"] * args.layers / 1e3, 4),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic",
            "config": {"workload": f"qwen3-4b decode over {args.long_ctx} keys (BASELINE config 5"
                                   f"{'' if args.long_ctx == 131072 else ', one shard of it'}, 1 GPU)",
                       "keys": args.long_ctx, "layers": args.layers},
            "peak_source": _peaks()[1], "long_ctx": res}
    print(json.dumps(line), flush=True)


def run_prefill_workload(args) -> None:
    import torch

    dev = torch.device("cuda", int(os.environ.get("LOCAL_RANK", "0")))
    torch.cuda.set_device(dev)
    res = prefill_bench(dev, args.steps, args.warmup, tuple(args.prefill_T))
    T = str(max(args.prefill_T))
    line = {"metric": "prefill attn TFLOP/s", "value": res[T]["tflops"], "unit": "TFLOP/s",
            "n_gpus": 1, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(res[T]["us_per_call"] / 1e3, 4), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "config": {"workload": "qwen3-4b causal prefill attention (BASELINE config 3)",
                       "T": int(T), "num_qo_heads": NH, "num_kv_heads": NKV, "head_dim": HD},
            "prefill": res}
    print(json.dumps(line), flush=True)


# Committed ncu summaries that carry a per-launch DRAM traffic figure for a bench workload.
TRAFFIC_PROFILES = {
    ("decode", 8192): "profiles/decode_splitkv_qwen3-4b_L8192_launches.md",
    ("decode", 131072): "profiles/decode_tc_qwen3-4b_L131072.md",
}


def _profiled_traffic(workload: str, keys: int):
    """DRAM bytes (read + write) of one launch of the dominant kernel for this workload, read
    from the `traffic_per_launch_bytes:` line of its committed ncu summary; (None, None) when no
    capture covers the workload."""
    rel = TRAFFIC_PROFILES.get((workload, keys))
    if rel is None:
        return None, None
    try:
        with open(os.path.join(ROOT, rel)) as fh:
            for ln in fh:
                if ln.startswith("traffic_per_launch_bytes:"):
                    return int(ln.split(":", 1)[1].strip().replace(",", "")), rel
    except OSError:
        pass
    return None, None


def _peaks(tensor: bool = False):
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as fh:
            d = json.load(fh)
        if tensor:
            return float(d["bf16_tflops"]), "measured burst (MEASURED_PEAKS.json bf16_tflops)"
        return float(d["hbm_gbs"]), "measured (MEASURED_PEAKS.json hbm_gbs)"
    except Exception:
        if tensor:
            return 1590.0, "fallback 1.59 PFLOP/s"
        return 6650.0, "fallback 6.65 TB/s"


def step_timeline(dev, prompt_len: int = 512) -> dict:
    """Where one decode step of the Qwen3-4B-shaped runner spends its time: a CUPTI kernel
    timeline (torch.profiler) of three graph replays; since launches overlap under PDL, each
    kernel is charged the growth of the latest end time it causes (its critical-path share).
    Diagnostic only: times taken under the profiler are not bench values."""
    import torch
    from torch.profiler import ProfilerActivity, profile

    model, runner = _qwen3_4b_runner(dev, prompt_len + 64)
    kinds = ("gemv_kernel", "prologue_kernel", "decode_kernel", "merge_kernel")
    with torch.no_grad():
        tok = runner.prefill(torch.randint(0, 151936, (prompt_len,), device=dev)).argmax(-1)
        for i in range(8):
            tok = runner.decode_gpu_argmax(tok.view(1), prompt_len + i)
        torch.cuda.synchronize(dev)
        with profile(activities=[ProfilerActivity.CUDA]) as prof:
            for i in range(3):
                tok = runner.decode_gpu_argmax(tok.view(1), prompt_len + 8 + i)
            torch.cuda.synchronize(dev)
    evs = sorted((e.time_range.start, e.time_range.end, e.name) for e in prof.events()
                 if e.device_type == torch.autograd.DeviceType.CUDA)
    step = evs[len(evs) // 3: 2 * len(evs) // 3]  # the middle replay
    proj = ["qkv", "o", "gate_up", "down"]
    shares, gi, last_end = {}, 0, step[0][0]
    for start, end, name in step:
        kind = next((k for k in kinds if k in name), "other (embedding, argmax, copies)")
        if kind == "gemv_kernel":
            kind = "gemv " + (proj[gi % 4] if gi < 4 * 36 else "lm_head")
            gi += 1
        grow = max(0.0, end - last_end)
        last_end = max(last_end, end)
        n, t = shares.get(kind, (0, 0.0))
        shares[kind] = (n + 1, t + grow)
    total = sum(t for _, t in shares.values())
    mb = {"gemv qkv": 31.46, "gemv o": 20.97, "gemv gate_up": 99.61, "gemv down": 49.81,
          "gemv lm_head": 777.9}
    rows = {k: {"launches": n, "critical_path_us": round(t, 1), "share": round(t / total, 4),
                **({"TBs_on_critical_path": round(mb[k] * n / t, 2)} if k in mb else {})}
            for k, (n, t) in sorted(shares.items(), key=lambda kv: -kv[1][1])}
    del runner, model
    torch.cuda.empty_cache()
    return {"step_us": round(total, 1), "context": prompt_len + 9, "kernels": rows}


def main():
    args = parse_args()
    if args.step_timeline:
        import torch

        print(json.dumps(step_timeline(torch.device("cuda", 0)), indent=1))
        return
    if args.impl == "reference":
        run_reference_arm(args)
    elif args.workload == "prefill":
        run_prefill_workload(args)
    elif args.workload == "paged":
        run_paged_workload(args)
    elif args.workload == "long":
        run_long_workload(args)
    else:
        run_gpu_arm(args)


if __name__ == "__main__":
    main()
