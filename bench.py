#!/usr/bin/env python3
"""Benchmark of the B200 packed-weight matmul path (one JSON line on rank 0).

Default workload (BASELINE.json configs[1] at batch 1): all ternary
projections of one BitNet b1.58 2B-class decoder layer -- fused QKV
3840x2560, O 2560x2560, gate 6912x2560, up 6912x2560, down 2560x6912 --
on synthetic data (ternary p = .25/.5/.25, fp32 N(0,1) activations).

One step = one layer's projections at batch B: quantise the four distinct
fp32 inputs (one grouped K1 launch) and run the five products (one grouped
GEMV launch). Consecutive steps use 30 different layer copies (521 MB of
weights, > 2x the 126 MB L2), so every step streams its weights from HBM.

Arms:
  (default)          the CUDA library (ouroboros_b200 / libouroq.so)
  --impl reference   the reference path on the host CPU: the oracle's
                     threaded restatement, same config / metric / unit
Launch: python bench.py [--gpus N --steps K --warmup W]; N > 1 under
torch.distributed.run (one rank per GPU, NCCL), every rank a replica.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

HIDDEN, FFN = 2560, 6912
LAYER_SHAPES = [("attn_qkv", 3840, HIDDEN), ("attn_output", HIDDEN, HIDDEN),
                ("ffn_gate", FFN, HIDDEN), ("ffn_up", FFN, HIDDEN), ("ffn_down", HIDDEN, FFN)]
# which activation each projection reads: qkv <- attn input, o <- attn out,
# gate/up <- ffn input, down <- ffn hidden
INPUT_OF = [0, 1, 2, 2, 3]
INPUT_K = [HIDDEN, HIDDEN, HIDDEN, FFN]
N_LAYERS = 30
WEIGHT_BYTES_PER_LAYER = sum(m * k // 4 for _, m, k in LAYER_SHAPES)  # 17,367,040
FALLBACK_HBM_GBS = 6650.0


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=3000)
    ap.add_argument("--warmup", type=int, default=30)
    ap.add_argument("--batch", type=int, default=1)
    ap.add_argument("--impl", default="ouroq", choices=["ouroq", "reference"])
    ap.add_argument("--no-pdl", action="store_true")
    return ap.parse_args()


def step_bytes(B: int) -> dict:
    """Algorithmic bytes of one step: what an ideal implementation moves once."""
    w = WEIGHT_BYTES_PER_LAYER
    x_f32 = B * sum(INPUT_K) * 4
    y = B * sum(m for _, m, _ in LAYER_SHAPES) * 4
    return {"step": w + x_f32 + y, "gemv": w + x_f32 + y, "weights": w}


def measured_peak():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        try:
            d = json.loads(p.read_text())
            return float(d["hbm_gbs"]), "measured"
        except Exception:
            pass
    return FALLBACK_HBM_GBS, "fallback"


def profiled_traffic(key: str):
    """Per-launch DRAM bytes of the dominant kernel from the committed ncu summary."""
    p = ROOT / "profiles" / "traffic.json"
    if p.exists():
        try:
            return json.loads(p.read_text()).get(key)
        except Exception:
            return None
    return None


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled while the timed region runs."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.rows = []
        self._stop = threading.Event()
        self._t = None

    def _run(self):
        while not self._stop.is_set():
            try:
                out = subprocess.run(["nvidia-smi", "-i", str(self.index), f"--query-gpu={self.Q}",
                                      "--format=csv,noheader,nounits"], capture_output=True,
                                     text=True, timeout=5).stdout.strip()
                if out:
                    self.rows.append([c.strip() for c in out.split(",")])
            except Exception:
                return
            self._stop.wait(0.1)

    def __enter__(self):
        self._t = threading.Thread(target=self._run, daemon=True)
        self._t.start()
        return self

    def __exit__(self, *a):
        self._stop.set()
        if self._t:
            self._t.join(timeout=10)

    def summary(self):
        if not self.rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"], "samples": 0}
        sm = [float(r[1]) for r in self.rows if r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in self.rows if r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in self.rows for i in range(4)
                          if len(r) > 5 + i and r[5 + i].lower() == "active"})
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": max(mx) if mx else None, "reasons": reasons, "samples": len(self.rows)}


# ---------------------------------------------------------------- data
def make_layer(torch, ctx, oq, gen, device):
    """Random ternary layer packed on the device, uploaded through the C ABI."""
    ws = []
    for _, M, K in LAYER_SHAPES:
        r = torch.randint(0, 4, (M, K), generator=gen, device=device, dtype=torch.uint8)
        codes = (r == 3).to(torch.uint8) * 2 + ((r == 1) | (r == 2)).to(torch.uint8)
        c = codes.view(M, K // 4, 4)
        packed = (c[..., 0] | (c[..., 1] << 2) | (c[..., 2] << 4) | (c[..., 3] << 6)).contiguous()
        nz = torch.count_nonzero(codes != 1).item()
        w_scale = 0.02 * nz / (M * K)  # absmean of W_fp = ternary * 0.02
        ws.append((ctx.upload_device(oq.TERNARY2, packed, M, K, None, w_scale), packed))
    return ws


def cpu_reference_gbs(layer_host, B: int, seconds: float, threads: int):
    """Oracle (threaded restatement) on one layer at batch B; returns GB/s and the sample."""
    from oracle import pyoracle as O
    rng = np.random.default_rng(7)
    xs = [rng.standard_normal((B, k), dtype=np.float32) for k in INPUT_K]
    qs = [O.quantize_act(x) for x in xs]
    nb = step_bytes(B)["step"]
    steps, t0 = 0, time.perf_counter()
    while True:
        for (name, M, K), (packed, ws) in zip(LAYER_SHAPES, layer_host):
            q, s = qs[INPUT_OF[[n for n, _, _ in LAYER_SHAPES].index(name)]]
            O.gemm_tern2_mt(packed, M, K, ws, q, s, threads)
        steps += 1
        dt = time.perf_counter() - t0
        if dt >= seconds:
            break
    return nb * steps / dt / 1e9, steps, dt


# ---------------------------------------------------------------- arms
def run_reference(args, rank):
    if rank != 0:
        return
    from oracle import pyoracle as O
    B = args.batch
    threads = O.hw_threads()
    rng = np.random.default_rng(11)
    layer = []
    for _, M, K in LAYER_SHAPES:
        w = rng.integers(0, 4, size=(M, K), dtype=np.int8)
        w = np.where(w == 0, -1, np.where(w == 3, 1, 0)).astype(np.int8)
        layer.append((O.pack_tern2(w), 0.01))
    # bounded sample: each timed step is one layer pass; steps capped so the run ends in minutes
    per = []
    for _ in range(max(args.warmup, 1)):
        cpu_reference_gbs(layer, B, 0.0, threads)
    total_t, total_steps = 0.0, 0
    for _ in range(max(1, min(args.steps, 50))):
        g, st, dt = cpu_reference_gbs(layer, B, 0.0, threads)
        total_t += dt
        total_steps += st
        per.append(dt)
    gbs = step_bytes(B)["step"] * total_steps / total_t / 1e9
    line = {
        "impl": "reference", "metric": "packed-weight GEMV HBM GB/s (BitNet-2B layer projections)",
        "value": round(gbs, 3), "unit": "GB/s", "n_gpus": args.gpus, "steps": total_steps,
        "warmup": args.warmup, "ms_per_step": round(1e3 * total_t / total_steps, 4),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "int8",
        "data": "synthetic",
        "config": {"workload": f"bitnet2b-layer-projections-b{B}", "batch": B,
                   "shapes": [[m, k] for _, m, k in LAYER_SHAPES], "host_cpu": True},
        "cpu_baseline": {"value": round(gbs, 3), "unit": "GB/s", "cores": threads, "kind": "port",
                         "sample": f"{total_steps} layer passes at batch {B} (oracle int8 GEMV, "
                                   f"{threads} threads, rows chunked as ops.rs:104-105)"},
        "e2e": {"value": round(gbs, 3), "unit": "GB/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def run_ouroq(args, rank, world, local_rank):
    import torch
    import torch.distributed as dist
    import ouroboros_b200 as oq

    device = torch.device("cuda", local_rank)
    torch.cuda.set_device(device)
    ctx = oq.Context(local_rank)
    if args.no_pdl:
        ctx.set_pdl(False)
    B = args.batch
    gen = torch.Generator(device=device)
    gen.manual_seed(1234 + rank)
    layers = [make_layer(torch, ctx, oq, gen, device) for _ in range(N_LAYERS)]
    wts = [[w for w, _ in L] for L in layers]

    # device-resident fp32 inputs per layer (independent synthetic activations)
    xs = [[torch.randn((B, k), generator=gen, device=device) for k in INPUT_K] for _ in range(N_LAYERS)]
    ys = [[torch.empty((B, m), dtype=torch.float32, device=device) for _, m, _ in LAYER_SHAPES]
          for _ in range(2)]
    stream = torch.cuda.Stream(device=device)
    def gemv_group(l, slot):
        # one launch: the four fp32 inputs are quantised in the GEMV prologue
        ctx.gemm_group_f32act(wts[l], [xs[l][INPUT_OF[i]] for i in range(5)], ys[slot],
                              stream=stream)

    def step(i):
        gemv_group(i % N_LAYERS, i % 2)

    # CUDA graph of one pass over the 30 layers (launch-bound loop -> graph replay)
    with torch.cuda.stream(stream):
        for i in range(max(args.warmup, 3)):
            step(i)
    stream.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        for i in range(N_LAYERS):
            step(i)
    def replay(n_passes):
        for _ in range(n_passes):
            graph.replay()

    with torch.cuda.stream(stream):
        replay(max(1, args.warmup // N_LAYERS) + 1)
    stream.synchronize()

    passes = max(1, args.steps // N_LAYERS)
    steps = passes * N_LAYERS
    launches_per_step = 1  # one grouped GEMV launch with the quantisation fused in

    def timed(fn, n):
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize(device)
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        fn(n)
        e1.record(stream)
        e1.synchronize()
        torch.cuda.synchronize(device)
        ms = e0.elapsed_time(e1)
        if world > 1:
            t = torch.tensor([ms], device=device)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            ms = float(t.item())
        return ms

    with ClockSampler(local_rank) as clk:
        with torch.cuda.stream(stream):
            ms = timed(replay, passes)
    clocks = clk.summary()

    nb = step_bytes(B)
    value = nb["step"] * steps * world / (ms / 1e3) / 1e9
    # the fused grouped GEMV is the only kernel of a step: its average launch
    # duration is the timed region (CUDA events on its stream) / launches
    gemv_avg_s = ms / 1e3 / steps
    achieved = nb["gemv"] / gemv_avg_s / 1e9
    peak, peak_kind = measured_peak()

    # ---- e2e through the public API with host buffers (pinned), eager calls
    xh = [[x.cpu().pin_memory() for x in xl] for xl in xs[:4]]
    yh = [torch.empty((B, m), dtype=torch.float32).pin_memory() for _, m, _ in LAYER_SHAPES]
    xd = [torch.empty((B, k), device=device) for k in INPUT_K]
    e2e_steps = min(steps, 600)
    h2d = B * sum(INPUT_K) * 4
    d2h = B * sum(m for _, m, _ in LAYER_SHAPES) * 4

    def e2e(n):
        for i in range(n):
            l = i % N_LAYERS
            for j in range(4):
                xd[j].copy_(xh[i % 4][j], non_blocking=True)
            ctx.gemm_group_f32act(wts[l], [xd[INPUT_OF[k]] for k in range(5)], ys[0],
                                  stream=stream)
            for j in range(5):
                yh[j].copy_(ys[0][j], non_blocking=True)

    with torch.cuda.stream(stream):
        e2e(10)
        stream.synchronize()
        e2e_ms = timed(e2e, e2e_steps)
    e2e_value = nb["step"] * e2e_steps * world / (e2e_ms / 1e3) / 1e9

    # ---- CPU baseline (rank 0, N = 1 only), bounded sample of the same workload
    cpu = None
    if rank == 0 and world == 1:
        from oracle import pyoracle as O
        layer_host = [(p.cpu().numpy(), float(w.w_scale)) for (w, p) in layers[0]]
        threads = O.hw_threads()
        gbs, st, dt = cpu_reference_gbs(layer_host, B, 10.0, threads)
        cpu = {"value": round(gbs, 3), "unit": "GB/s", "cores": threads, "kind": "port",
               "sample": f"{st} layer passes ({dt:.1f} s) at batch {B}: oracle int8 GEMV, "
                         f"{threads} threads"}

    if rank == 0:
        traffic = profiled_traffic(f"gemv_group_b{B}")
        line = {
            "metric": "packed-weight GEMV HBM GB/s (BitNet-2B layer projections)",
            "value": round(value, 2), "unit": "GB/s", "n_gpus": world, "steps": steps,
            "warmup": args.warmup, "ms_per_step": round(ms / steps, 5), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "int8",
            "data": "synthetic (ternary p=.25/.5/.25, fp32 N(0,1) activations, random init)",
            "config": {"workload": f"bitnet2b-layer-projections-b{B}", "batch": B,
                       "shapes": [[m, k] for _, m, k in LAYER_SHAPES],
                       "layers_rotated": N_LAYERS,
                       "l2": f"inputs larger than L2: {N_LAYERS} layer copies = "
                             f"{N_LAYERS * WEIGHT_BYTES_PER_LAYER / 1e6:.0f} MB rotated",
                       "parallelism": f"replicas x{world}", "pdl": not args.no_pdl,
                       "launch": "CUDA graph of 30 steps"},
            "decode_tokens_per_s_ternary_only": round(B * world / (ms / 1e3 / steps * N_LAYERS), 1),
            "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak,
                         "unit": "GB/s", "frac": round(achieved / peak, 4),
                         "traffic": traffic, "peak_kind": f"{peak_kind} (hbm_gbs)",
                         "kernel": "gemv_kernel<kTern2,B> (grouped, 5 jobs, fused quantisation)",
                         "bytes_per_launch": nb["gemv"]},
            "cpu_baseline": cpu,
            "e2e": {"value": round(e2e_value, 2), "unit": "GB/s", "h2d_bytes_per_step": h2d,
                    "d2h_bytes_per_step": d2h,
                    "how": "eager Python calls of the public API, pinned host buffers"},
            "gpu_launches": launches_per_step * steps,
            "clocks": clocks,
        }
        print(json.dumps(line), flush=True)
    del graph
    ctx.close()


def main():
    args = parse()
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        run_reference(args, rank)
        return
    if world > 1:
        import datetime
        import torch
        import torch.distributed as dist
        torch.cuda.set_device(local_rank)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local_rank))
    try:
        run_ouroq(args, rank, world, local_rank)
    finally:
        if world > 1:
            import torch.distributed as dist
            dist.barrier()
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
