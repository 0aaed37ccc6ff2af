#!/usr/bin/env python3
"""Benchmark of the B200 packed-weight matmul path (one JSON line on rank 0).

Default workload (the headline configuration, at batch 1): all ternary
projections of one BitNet b1.58 2B-class decoder layer -- fused QKV
3840x2560, O 2560x2560, gate 6912x2560, up 6912x2560, down 2560x6912 --
on synthetic data (ternary p = .25/.5/.25, fp32 N(0,1) activations).

One step = one pass of the path over one batch: fp32 activations in, fp32
outputs out. At B <= 8 that is ONE launch (grouped GEMV with the per-token
quantisation fused into its prologue); at larger B it is one grouped
quantisation launch followed by one matmul launch per matrix (tcgen05
tensor-core GEMM for ternary weights from B = 16). Consecutive steps cycle
through enough weight copies to exceed twice the 126 MB L2, so every step
streams its weights from HBM.

Other workloads (--workload): c1 (6912x2560), c5-up (28672x8192), c5-down
(8192x28672), c3-4096 / c3-11008 (1-bit sign weights, fp16 group scales,
Walsh-Hadamard block 128 on the activations).

Arms:
  (default)          the CUDA library (ouroboros_b200 / libouroq.so)
  --impl reference   the reference's own CPU algorithm on the host cores, as
                     the oracle restates it (matvec_tl1 / matmul_tl1 on the
                     workload's shapes in PTQ1_0, matvec_qblock for TQ1_0),
                     same config / metric / unit
Launch: python bench.py [--gpus N --steps K --warmup W]; N > 1 under
torch.distributed.run (one rank per GPU, NCCL), every rank a replica with
its own weights (no data-path collective: weak scaling).
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

TERN, SIGN, TL1, TQ1 = 1, 2, 3, 4  # OUROQ_FMT_TERNARY2, _SIGN1G128, _PTQ1_0, _TQ1_0
FMT_NAME = {TERN: "ternary2", SIGN: "sign1g128", TL1: "ptq1_0", TQ1: "tq1_0"}
REF_FMTS = (TL1, TQ1)
HIDDEN, FFN = 2560, 6912
L2_BYTES = 126 * 2**20
FALLBACK_HBM_GBS = 6650.0
FALLBACK_BF16_TFLOPS = 1590.0

# workload -> (description, format, [(name, M, K, input index)], [input widths], hadamard block)
WORKLOADS = {
    "layer": ("bitnet2b-layer-projections", TERN,
              [("attn_qkv", 3840, HIDDEN, 0), ("attn_output", HIDDEN, HIDDEN, 1),
               ("ffn_gate", FFN, HIDDEN, 2), ("ffn_up", FFN, HIDDEN, 2),
               ("ffn_down", HIDDEN, FFN, 3)],
              [HIDDEN, HIDDEN, HIDDEN, FFN], 0),
    "c1": ("ternary-6912x2560", TERN, [("w", 6912, 2560, 0)], [2560], 0),
    "c5-up": ("ternary-28672x8192", TERN, [("ffn_up", 28672, 8192, 0)], [8192], 0),
    "c5-down": ("ternary-8192x28672", TERN, [("ffn_down", 8192, 28672, 0)], [28672], 0),
    "c3-4096": ("sign1-wht128-4096x4096", SIGN, [("w", 4096, 4096, 0)], [4096], 128),
    "c3-11008": ("sign1-wht128-11008x4096", SIGN, [("w", 11008, 4096, 0)], [4096], 128),
    # the BitNet-2B layer in the reference's own shard formats (fp32 activations,
    # no quantisation): the path the reference runs today
    "layer-tq1": ("bitnet2b-layer-projections-tq1_0", TQ1,
                  [("attn_qkv", 3840, HIDDEN, 0), ("attn_output", HIDDEN, HIDDEN, 1),
                   ("ffn_gate", FFN, HIDDEN, 2), ("ffn_up", FFN, HIDDEN, 2),
                   ("ffn_down", HIDDEN, 6912, 3)],
                  [HIDDEN, HIDDEN, HIDDEN, FFN], 0),
    # the whole BitNet-2B decode step (configuration 4): 30 layers, KV context
    # 1024, lm_head, greedy sampling; metric: decode tokens/s
    "decode": ("bitnet2b-decode", TERN, [], [], 0),
    "layer-tl1": ("bitnet2b-layer-projections-ptq1_0", TL1,
                  [("attn_qkv", 3840, HIDDEN, 0), ("attn_output", HIDDEN, HIDDEN, 1),
                   ("ffn_gate", FFN, HIDDEN, 2), ("ffn_up", FFN, HIDDEN, 2),
                   ("ffn_down", HIDDEN, 6912, 3)],
                  [HIDDEN, HIDDEN, HIDDEN, FFN], 0),
}


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=30000)
    ap.add_argument("--warmup", type=int, default=30)
    ap.add_argument("--batch", type=int, default=1)
    ap.add_argument("--workload", default="layer", choices=sorted(WORKLOADS))
    ap.add_argument("--impl", default="ouroq", choices=["ouroq", "reference"])
    ap.add_argument("--no-pdl", action="store_true")
    ap.add_argument("--prefetch", default="off", choices=["on", "off"],
                    help="each step's GEMV launch prefetches the next step's weights into L2 "
                         "(ouroq_set_prefetch), as a decode loop may for its next projection group "
                         "(measured no faster on the layer workload, so off by default)")
    ap.add_argument("--prefetch-ahead", type=int, default=1,
                    help="with --prefetch on: the step whose weights each launch prefetches, counted "
                         "ahead of the current one (1 = the next step)")
    ap.add_argument("--cpu-seconds", type=float, default=10.0,
                    help="bound of the CPU-baseline sample (0 = skip)")
    ap.add_argument("--shard", action="store_true",
                    help="row-shard each matrix over the ranks; single-matrix workloads only")
    ap.add_argument("--transport", default="peer", choices=["peer", "nccl"],
                    help="how --shard moves rows between ranks")
    ap.add_argument("--tokens", type=int, default=256,
                    help="decode workload: tokens generated per sequence in the timed region")
    ap.add_argument("--shard-record", default="on", choices=["on", "off"],
                    help="layer workload: add the row-sharded 8192x28672 sub-record over the ranks")
    ap.add_argument("--decode-tokens", type=int, default=64,
                    help="layer workload: tokens of the configuration-4 decode sub-record (0 = skip)")
    ap.add_argument("--layers", type=int, default=30,
                    help="decode workload: layers (30 = BitNet-2B; fewer only to profile a small case)")
    return ap.parse_args()


def weight_bytes(fmt: int, M: int, K: int) -> int:
    if fmt == TL1:
        return M * (K // 128) * 28
    if fmt == TQ1:
        return M * (K // 256) * 54
    return M * K // 4 if fmt == TERN else M * K // 8 + M * (K // 128) * 2


def step_bytes(wl, B: int) -> dict:
    """Algorithmic bytes of one step: what an ideal implementation moves once
    (weights + scales, the fp32 activations read once, the fp32 outputs)."""
    _, fmt, mats, widths, _ = wl
    w = sum(weight_bytes(fmt, M, K) for _, M, K, _ in mats)
    x_f32 = B * sum(widths) * 4
    x_i8 = B * sum(widths) + 4 * B * len(widths)
    y = B * sum(M for _, M, _, _ in mats) * 4
    ops = 2 * B * sum(M * K for _, M, K, _ in mats)
    return {"step": w + x_f32 + y, "gemm": w + x_i8 + y, "weights": w, "ops": ops}


def n_copies(wl) -> int:
    w = step_bytes(wl, 1)["weights"]
    return max(2, -(-2 * L2_BYTES // w))


def peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        try:
            d = json.loads(p.read_text())
            return float(d["hbm_gbs"]), float(d["bf16_tflops"]), "measured"
        except Exception:
            pass
    return FALLBACK_HBM_GBS, FALLBACK_BF16_TFLOPS, "fallback"


def sustained_bf16():
    """The bf16 rate to hold a tensor-bound kernel against when it is timed
    inside a seconds-long loop (the clocks settle under the power cap): the
    measured sustained figure, else the burst figure of peaks()."""
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        try:
            return float(json.loads(p.read_text())["bf16_tflops_sustained"]), "measured bf16_tflops_sustained"
        except Exception:
            pass
    _, bf16, kind = peaks()
    return bf16, f"{kind} bf16_tflops"


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
        # the first nvidia-smi call forks a process: let it finish before the
        # caller opens its timed region, so the fork is not inside it
        t0 = time.perf_counter()
        while not self.rows and self._t.is_alive() and time.perf_counter() - t0 < 2.0:
            time.sleep(0.01)
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


def gate(torch, replays: int):
    """Hold the current stream on the device for a moment (a spin kernel of
    torch's) before the timed region opens, so that the CPU has submitted the
    whole region (`replays` graph launches) before the GPU reaches its first
    event: the CPU's submit latency then stays out of the measurement."""
    seconds = 2e-3 + 1e-4 * replays
    torch.cuda._sleep(int(seconds * 2.0e9))  # cycles at ~2 GHz


def graph_plan(steps: int, ncop: int, max_passes: int = 64, max_single: int = 4096):
    """Cover exactly `steps` steps with CUDA graphs. Up to `max_single` steps:
    one graph of all of them (the copies rotate inside it), so the timed
    region holds no graph-to-graph boundary. Beyond: a graph of G steps (G a
    multiple of the copy count, so replays keep the rotation) replayed `reps`
    times, then one graph of the remaining `rest` steps (copies 0..rest-1,
    which follow a full pass). Returns (G, reps, rest)."""
    if steps <= max_single:
        return 0, 0, steps
    passes = max(1, min(steps // ncop, max_passes))
    G = passes * ncop
    return G, steps // G, steps % G


# ---------------------------------------------------------------- data
def make_copy(torch, ctx, oq, wl, gen, device):
    """One random copy of the workload's matrices, uploaded through the C ABI.
    Returns [(Weight, packed codes, fp16 scales or None)]."""
    _, fmt, mats, _, _ = wl
    out = []
    for _, M, K, _ in mats:
        if fmt in REF_FMTS:
            # random code bytes (every byte is a valid set of trits), finite f16 scales
            gb = 28 if fmt == TL1 else 54
            ng = M * K // (128 if fmt == TL1 else 256)
            p = torch.randint(0, 256, (ng, gb), generator=gen, device=device,
                              dtype=torch.int32).to(torch.uint8)
            sc = (torch.randn((ng,), generator=gen, device=device) * 0.02).abs().to(torch.float16)
            p[:, gb - 2:] = sc.view(torch.uint8).view(ng, 2)
            p = p.reshape(-1).contiguous()
            out.append((ctx.upload_device(fmt, p, M, K, None, 1.0), p, None))
            continue
        if fmt == TERN:
            r = torch.randint(0, 4, (M, K), generator=gen, device=device, dtype=torch.uint8)
            codes = (r == 3).to(torch.uint8) * 2 + ((r == 1) | (r == 2)).to(torch.uint8)
            c = codes.view(M, K // 4, 4)
            packed = (c[..., 0] | (c[..., 1] << 2) | (c[..., 2] << 4) | (c[..., 3] << 6)).contiguous()
            nz = torch.count_nonzero(codes != 1).item()
            del r, codes, c
            w_scale = 0.02 * nz / (M * K)  # absmean of W_fp = ternary * 0.02
            out.append((ctx.upload_device(oq.TERNARY2, packed, M, K, None, w_scale), packed, None))
        else:
            packed = torch.randint(0, 256, (M, K // 8), generator=gen, device=device,
                                   dtype=torch.int32).to(torch.uint8)
            sc = (torch.randn((M, K // 128), generator=gen, device=device) * 0.02).abs()
            sc = sc.to(torch.float16).view(torch.int16).contiguous()
            out.append((ctx.upload_device(oq.SIGN1G128, packed, M, K, sc, 1.0), packed, sc))
    return out


def cpu_model() -> str:
    """The host CPU's model string (for the CPU lines)."""
    try:
        for line in Path("/proc/cpuinfo").read_text().splitlines():
            if line.startswith("model name"):
                return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"


def cpu_oracle_gbs(wl, host_mats, host_signs, B: int, seconds: float, threads: int):
    """Oracle (threaded int8 restatement) on one copy at batch B, looping until
    `seconds` have passed (at least one pass). Returns GB/s at the median step
    time, passes, seconds, median seconds per step."""
    from oracle import pyoracle as O
    _, fmt, mats, widths, block = wl
    rng = np.random.default_rng(7)
    xs = [rng.standard_normal((B, k), dtype=np.float32) for k in widths]
    nb = step_bytes(wl, B)["step"]
    steps, t0 = 0, time.perf_counter()
    durs, ts = [], t0
    while True:
        if fmt in REF_FMTS:
            # the reference's own algorithm for these formats, restated (threaded like it)
            # (a workload that rotates: rotate_fwd of a copy before each matmul,
            # as Qwen35Stage::wh does). Several tokens of a Tl1 matrix go through
            # matmul_tl1's K-column path (Stage::wmat_batched -> matmul_q,
            # ops.rs:219-230); other formats run one matvec per token there too.
            for (_, M, K, xi), (packed, _) in zip(mats, host_mats):
                xb = xs[xi]
                if block:
                    xb = np.stack([O.rotate_fwd(xb[b], host_signs[xi], block) for b in range(B)])
                if fmt == TL1 and B > 1:
                    O.matmul_tl1_sse(packed, M, K, xb, B, threads)
                    continue
                for b in range(B):
                    if fmt == TL1:
                        O.matvec_tl1_sse(packed, M, K, xb[b], threads)
                    else:
                        O.matvec_tq1(packed, M, K, xb[b], threads)
            steps += 1
            now = time.perf_counter()
            durs.append(now - ts)
            ts = now
            dt = now - t0
            if dt >= seconds:
                break
            continue
        qs = [O.quantize_act(x, host_signs[i] if block else None, block) for i, x in enumerate(xs)]
        for (_, M, K, xi), (packed, aux) in zip(mats, host_mats):
            q, s = qs[xi]
            if fmt == TERN:
                O.gemm_tern2_mt(packed, M, K, aux, q, s, threads)
            else:
                O.gemm_sign1_mt(packed, aux, M, K, q, s, threads)
        steps += 1
        now = time.perf_counter()
        durs.append(now - ts)
        ts = now
        dt = now - t0
        if dt >= seconds:
            break
    med = statistics.median(durs)
    return nb / med / 1e9, steps, dt, med


def host_copy(wl, seed: int):
    """A host-side copy of the workload's matrices for the CPU arms."""
    from oracle import pyoracle as O
    _, fmt, mats, widths, block = wl
    out = []
    for i, (_, M, K, _) in enumerate(mats):
        if fmt in REF_FMTS:
            gb = 28 if fmt == TL1 else 54
            p = O.lcg_bytes(seed + i, M * K // (128 if fmt == TL1 else 256) * gb).reshape(-1, gb)
            p[:, gb - 1] = 0x24  # f16 scales ~ 0.02
            out.append((p.reshape(-1), None))
            continue
        if fmt == TERN:
            w = O.ternary(seed + i, M * K).reshape(M, K)
            out.append((O.pack_tern2(w), float(O.absmean_scale(w, 0.02))))
        else:
            w = O.signs(seed + i, M * K).reshape(M, K)
            out.append((O.pack_sign1(w), O.group_scales(seed + 50 + i, M * (K // 128), 0.02)))
    signs = [O.signs(seed + 100 + j, k).astype(np.float32) for j, k in enumerate(widths)]
    return out, signs


def workload_config(args, wl, world):
    desc, fmt, mats, widths, block = wl
    return {"workload": f"{desc}-b{args.batch}", "batch": args.batch,
            "format": FMT_NAME[fmt],
            "shapes": [[M, K] for _, M, K, _ in mats], "hadamard_block": block,
            "weight_copies_rotated": n_copies(wl),
            "l2": f"inputs larger than L2: {n_copies(wl)} weight copies = "
                  f"{n_copies(wl) * step_bytes(wl, 1)['weights'] / 1e6:.0f} MB rotated",
            "parallelism": f"replicas x{world}"}


# ---------------------------------------------------------------- arms
def run_reference(args, rank):
    if rank != 0:
        return
    from oracle import pyoracle as O
    if args.workload == "decode":
        threads = O.hw_threads()
        v, n, dt = cpu_decode_tokens_per_s(args.batch, 20.0, threads)
        line = {"impl": "reference", "metric": "decode tokens/s", "value": round(v, 3),
                "unit": "tokens/s", "n_gpus": args.gpus, "steps": n, "warmup": 0,
                "ms_per_step": round(1e3 * args.batch / v, 3), "higher_is_better": True,
                "scaling": "weak", "vs_baseline": None, "dtype": "fp32", "data": "synthetic",
                "config": {"workload": f"bitnet2b-decode-b{args.batch}-ctx1024-gen256",
                           "batch": args.batch, "host_cpu": True},
                "cpu_baseline": {"value": round(v, 3), "unit": "tokens/s", "cores": threads,
                                 "kind": "port", "cpu_model": cpu_model(),
                                 "sample": f"{n} single-layer passes of run_layer in the "
                                           f"reference's fp32 order (TQ1_0 matvec_qblock "
                                           f"projections, rmsnorm, RoPE, attend over 1025 "
                                           f"positions, silu) scaled to 30 layers, plus the "
                                           f"lm_head in the reference's matvec_f16 order, "
                                           f"{threads} threads for the matvecs"},
                "e2e": {"value": round(v, 3), "unit": "tokens/s", "h2d_bytes_per_step": 0,
                        "d2h_bytes_per_step": 0}}
        print(json.dumps(line), flush=True)
        return
    wl = WORKLOADS[args.workload]
    B = args.batch
    threads = O.hw_threads()
    # The reference's own algorithm: its shard formats as they are; the
    # TERNARY2 / SIGN1G128 shapes re-encoded as PTQ1_0 groups through
    # matvec_tl1 (ops.rs:294-363, the SSE accumulation order), the path the
    # reference runs for ternary and sign shards.
    ref_wl = wl if wl[1] in REF_FMTS else (wl[0], TL1, wl[2], wl[3], wl[4])
    host_mats, host_signs = host_copy(ref_wl, 11)
    for _ in range(max(min(args.warmup, 3), 1)):
        cpu_oracle_gbs(ref_wl, host_mats, host_signs, B, 0.0, threads)
    total_t, total_steps, durs = 0.0, 0, []
    budget = 60.0  # the whole run stays within minutes
    for _ in range(max(1, args.steps)):
        _, st, dt, _ = cpu_oracle_gbs(ref_wl, host_mats, host_signs, B, 0.0, threads)
        total_t += dt
        total_steps += st
        durs.append(dt / st)
        if total_t >= budget:
            break
    # the same step as the GPU arm's (same shapes and batch), so GB/s counts
    # that arm's algorithmic bytes and the two values compare as step times;
    # the median step after the warm-up
    med = statistics.median(durs)
    gbs = step_bytes(wl, B)["step"] / med / 1e9
    cfg = workload_config(args, wl, 1)
    cfg["host_cpu"] = True
    cfg["reference_format"] = FMT_NAME[ref_wl[1]]
    line = {
        "impl": "reference", "metric": "packed-weight GEMV HBM GB/s",
        "value": round(gbs, 3), "unit": "GB/s", "n_gpus": args.gpus, "steps": total_steps,
        "warmup": args.warmup, "ms_per_step": round(1e3 * med, 4),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "f32",
        "data": "synthetic", "config": cfg,
        "cpu_baseline": {"value": round(gbs, 3), "unit": "GB/s", "cores": threads, "kind": "port",
                         "cpu_model": cpu_model(),
                         "sample": f"median of {total_steps} steps at batch {B} (" + (
                             "the reference's own fp32 algorithm for this format, restated"
                             if wl[1] in REF_FMTS else
                             "the reference's matvec_tl1 in fp32 on the same shapes re-encoded "
                             "as PTQ1_0" + (", rotate_fwd first" if wl[4] else "") +
                             (", matmul_tl1's K-column path for the batch" if B > 1 else "") +
                             "; GB/s on the GPU arm's step bytes") +
                                   f", {threads} threads, rows chunked as ops.rs:104-105; "
                                   f"capped at {budget:.0f} s)"},
        "e2e": {"value": round(gbs, 3), "unit": "GB/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def run_ouroq(args, rank, world, local_rank):
    import torch
    import torch.distributed as dist
    import ouroboros_b200 as oq

    wl = WORKLOADS[args.workload]
    desc, fmt, mats, widths, block = wl
    device = torch.device("cuda", local_rank)
    torch.cuda.set_device(device)
    ctx = oq.Context(local_rank)
    if args.no_pdl:
        ctx.set_pdl(False)
    B = args.batch
    gen = torch.Generator(device=device)
    gen.manual_seed(1234 + rank)
    ncop = n_copies(wl)
    copies = [make_copy(torch, ctx, oq, wl, gen, device) for _ in range(ncop)]
    wts = [[w for w, _, _ in c] for c in copies]
    signs = [torch.where(torch.rand(k, generator=gen, device=device) < 0.5, -1.0, 1.0)
             for k in widths] if block else None

    # device-resident fp32 inputs per copy (independent synthetic activations)
    xs = [[torch.randn((B, k), generator=gen, device=device) for k in widths] for _ in range(ncop)]
    ys = [[torch.empty((B, M), dtype=torch.float32, device=device) for _, M, _, _ in mats]
          for _ in range(2)]
    qs = [[torch.empty((B, k), dtype=torch.int8, device=device) for k in widths] for _ in range(2)]
    sxs = [[torch.empty((B,), dtype=torch.float32, device=device) for _ in widths] for _ in range(2)]
    stream = torch.cuda.Stream(device=device)
    fused = B <= 8 or fmt in REF_FMTS
    mat_signs = [signs[xi] for _, _, _, xi in mats] if block else None
    mat_blocks = [block] * len(mats) if block else None

    def run_step(wl_, xin, yout, qbuf, sbuf):
        if fmt in REF_FMTS:
            # fp32 activations straight into the reference-format kernels, one per matrix
            for j, (_, _, _, xi) in enumerate(mats):
                ctx.gemm_f32act(wl_[j], xin[xi], y=yout[j], stream=stream)
            return
        if fused:
            # one launch: the fp32 inputs are quantised in the GEMV prologue
            if len(mats) > 1:
                ctx.gemm_group_f32act(wl_, [xin[xi] for _, _, _, xi in mats], yout,
                                      signs=mat_signs, blocks=mat_blocks, stream=stream)
            else:
                ctx.gemm_f32act(wl_[0], xin[0], signs=signs[0] if block else None,
                                hadamard_block=block, y=yout[0], stream=stream)
        else:
            ctx.quantize_group(xin, qbuf, sbuf, signs=signs if block else None,
                               blocks=[block] * len(widths) if block else None, stream=stream)
            # the projections as one grouped product (one tensor-core launch for ternary weights)
            ctx.gemm_group(wl_, [qbuf[xi] for _, _, _, xi in mats], [sbuf[xi] for _, _, _, xi in mats],
                           yout, stream=stream)

    prefetch = args.prefetch == "on" and fused and fmt not in REF_FMTS

    def step(i):
        if prefetch:
            ctx.set_prefetch(wts[(i + args.prefetch_ahead) % ncop])
        run_step(wts[i % ncop], xs[i % ncop], ys[i % 2], qs[i % 2], sxs[i % 2])

    def gemm_only(i):
        ctx.gemm_group(wts[i % ncop], [qs[0][xi] for _, _, _, xi in mats], [sxs[0][xi] for _, _, _, xi in mats],
                       ys[i % 2], stream=stream)

    def capture(fn, n):
        """One CUDA graph of steps 0..n-1 (launch-bound loop -> graph replay)."""
        n0 = ctx.launch_count()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=stream):
            for i in range(n):
                fn(i)
        return g, (ctx.launch_count() - n0) / max(n, 1)

    def graphs_for(fn, nsteps):
        """Graphs that run exactly nsteps steps: [(graph, replays)]."""
        G, reps, rest = graph_plan(nsteps, ncop)
        out, per = [], 0.0
        if reps:
            g, per = capture(fn, G)
            out.append((g, reps))
        if rest:
            g, per = capture(fn, rest)
            out.append((g, 1))
        return out, per

    def run_graphs(gs):
        for g, reps in gs:
            for _ in range(reps):
                g.replay()

    def timed(gs):
        """Device time of the graphs gs (exactly their steps), max over ranks.
        A spin kernel queued first keeps the CPU's submission out of the window."""
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize(device)
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        with torch.cuda.stream(stream):
            gate(torch, sum(r for _, r in gs))
            e0.record(stream)
            run_graphs(gs)
            e1.record(stream)
        e1.synchronize()
        torch.cuda.synchronize(device)
        ms = e0.elapsed_time(e1)
        if world > 1:
            t = torch.tensor([ms], device=device)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            ms = float(t.item())
        return ms

    PREFIX = 2  # untimed steps ahead of the timed window, in the same graph

    side = torch.cuda.Stream(device)

    def capture_windowed(fn, n):
        """One CUDA graph: PREFIX untimed steps (the rotation's last copies),
        then steps 0..n-1, with an event-record node on a branch after the
        last untimed step and one after the last timed step. The timed window
        then runs from the end of step -1 to the end of step n-1: exactly n
        steps, opening on a running pipeline (no graph launch inside it). The
        event nodes sit on a side branch, so each step's kernels keep their
        programmatic dependency on the previous step's: an event node on the
        main chain would make the first timed launch wait for its
        predecessor's completion instead of overlapping its tail."""
        e0 = torch.cuda.Event(enable_timing=True, external=True)
        e1 = torch.cuda.Event(enable_timing=True, external=True)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=stream):
            for i in range(-PREFIX, 0):
                fn(i)
            n0 = ctx.launch_count()
            side.wait_stream(stream)
            e0.record(side)
            for i in range(n):
                fn(i)
            side.wait_stream(stream)
            e1.record(side)
            stream.wait_stream(side)
            per = (ctx.launch_count() - n0) / max(n, 1)
        return g, e0, e1, per

    def timed_windowed(gw):
        """Device time between the graph's two event-record nodes, max over ranks."""
        g, e0, e1, _ = gw
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize(device)
        with torch.cuda.stream(stream):
            g.replay()
        torch.cuda.synchronize(device)
        ms = e0.elapsed_time(e1)
        if world > 1:
            t = torch.tensor([ms], device=device)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            ms = float(t.item())
        return ms

    # eager warm-up (allocations, kernel loading), then the graphs of exactly
    # args.steps steps, replayed once untimed with the warm-up
    with torch.cuda.stream(stream):
        for i in range(max(args.warmup, 3)):
            step(i)
    stream.synchronize()
    steps = max(1, args.steps)
    windowed = steps <= 4096
    if windowed:
        gw = capture_windowed(step, steps)
        launches_per_step = gw[3]
        with torch.cuda.stream(stream):
            gw[0].replay()
    else:
        graphs, launches_per_step = graphs_for(step, steps)
        with torch.cuda.stream(stream):
            run_graphs(graphs)
    stream.synchronize()

    with ClockSampler(local_rank) as clk:
        ms = timed_windowed(gw) if windowed else timed(graphs)
    clocks = clk.summary()

    nb = step_bytes(wl, B)
    value = nb["step"] * steps * world / (ms / 1e3) / 1e9
    hbm_peak, bf16_peak, peak_kind = peaks()
    tensor_bound = fmt == TERN and B >= 64
    if fused:
        # the step's kernels are the product itself (the fused grouped GEMV, or one
        # reference-format kernel per matrix): bytes of the step / the timed region
        kern_s = ms / 1e3 / steps
        kern_bytes = nb["step"]
        kernel = ("tl1_colblock_kernel (matmul_tl1's K-column order)" if fmt == TL1 and B > 1
                  else f"{'tl1' if fmt == TL1 else 'tq1'}_matvec_kernel (reference order)"
                  if fmt in REF_FMTS else
                  (f"gemv_stream_kernel<B={B}> (fused quantisation)" if fmt == TERN and B <= 8 and not block
                   else f"gemv_kernel<{'kTern2' if fmt == TERN else 'kSign1'},B={B}> (fused quantisation)"))
    else:
        # matmul launches alone, on pre-quantised activations, timed the same way
        if windowed:
            g2 = capture_windowed(gemm_only, steps)
            with torch.cuda.stream(stream):
                g2[0].replay()
            kms = timed_windowed(g2)
        else:
            g2, _ = graphs_for(gemm_only, steps)
            with torch.cuda.stream(stream):
                run_graphs(g2)
            kms = timed(g2)
        kern_s = kms / 1e3 / steps
        kern_bytes = nb["gemm"]
        kernel = (("gemm_tc_kernel (tcgen05 kind::i8, one grouped launch)" if len(mats) > 1 else "gemm_tc_kernel (tcgen05 kind::i8)") if fmt == TERN and B >= 9
                  else "gemm_sign_tc_kernel (tcgen05 kind::i8, group accumulators)" if B >= 9
                  else "gemv_kernel (8-token chunks)")
        del g2
    if tensor_bound:
        # the matmul launches run back to back for seconds: the sustained rate
        bf16_rate, bf16_kind = sustained_bf16()
        int8_peak = 2.0 * bf16_rate
        achieved = nb["ops"] / kern_s / 1e12
        roof = {"bound": "tensor", "achieved": round(achieved, 1), "peak": round(int8_peak, 1),
                "unit": "TOPS", "frac": round(achieved / int8_peak, 4),
                "peak_kind": f"int8 dense = 2 x {bf16_kind}",
                "ops_per_step": nb["ops"]}
    else:
        achieved = kern_bytes / kern_s / 1e9
        roof = {"bound": "hbm", "achieved": round(achieved, 1), "peak": hbm_peak, "unit": "GB/s",
                "frac": round(achieved / hbm_peak, 4), "peak_kind": f"{peak_kind} (hbm_gbs)",
                "bytes_per_step": kern_bytes}
    roof["traffic"] = profiled_traffic(f"{args.workload}_b{B}")
    roof["kernel"] = kernel

    # ---- e2e: the same steps through the reference-facing host-buffer call
    # (ouroq_matmul_q_group: the step's projections in one synchronous round
    # trip, host fp32 x in, host fp32 y out), page-locked host buffers, timed
    # on the host clock around whole calls (each returns after its copy back).
    # A step's activations sit back to back in one buffer and cross in one
    # copy; its outputs come back in one copy (widths are multiples of 128).
    xoff = np.cumsum([0] + [B * k for k in widths]).tolist()
    yoff = np.cumsum([0] + [B * M for _, M, _, _ in mats]).tolist()
    xh = [torch.cat([x.reshape(-1) for x in xl]).cpu().pin_memory() for xl in xs[:2]]
    yh = torch.empty(yoff[-1], dtype=torch.float32).pin_memory()
    xhv = [[xc[xoff[j]:xoff[j + 1]] for j in range(len(widths))] for xc in xh]
    yhv = [yh[yoff[j]:yoff[j + 1]] for j in range(len(mats))]
    h2d = B * sum(widths) * 4
    d2h = B * sum(M for _, M, _, _ in mats) * 4

    wrapper = None
    if not block:  # the host mirrors take no rotation (rotate_fwd is its own call)
        # The call as a foreign caller binds it (a Rust `extern "C"` block):
        # the pointer arrays built once, then one ouroq_matmul_q_group call a
        # step, its status checked. The Python wrapper's own argument checks
        # and array building are timed separately (`python_wrapper`).
        import ctypes
        nm = len(mats)
        arr = ctypes.c_void_p * nm
        w_arr = [arr(*[w.handle for w in wts[c]]) for c in range(ncop)]
        x_arr = [arr(*[xhv[par][xi].data_ptr() for _, _, _, xi in mats]) for par in range(2)]
        y_arr = arr(*[t.data_ptr() for t in yhv])
        call = ctx.lib.ouroq_matmul_q_group

        def e2e(n):
            for i in range(n):
                st = call(ctx.ctx, nm, w_arr[i % ncop], x_arr[i % 2], B, y_arr)
                if st:
                    ctx._check(st)

        def e2e_wrapper(n):
            for i in range(n):
                ctx.matmul_q_group(wts[i % ncop], [xhv[i % 2][xi] for _, _, _, xi in mats], yhv)
        wrapper = e2e_wrapper
        how = ("ouroq_matmul_q_group called through its C ABI as a foreign caller binds it (one "
               "synchronous call a step, status checked): page-locked host x copied in, the "
               "results stored by the kernel into the page-locked host y (d2h bytes = those "
               "stores); host clock around the calls")
    else:
        xcat = torch.empty(xoff[-1], device=device)
        ycat = torch.empty(yoff[-1], device=device)
        xd = [xcat[xoff[j]:xoff[j + 1]].view(B, k) for j, k in enumerate(widths)]
        yd = [ycat[yoff[j]:yoff[j + 1]].view(B, M) for j, (_, M, _, _) in enumerate(mats)]

        def e2e(n):
            with torch.cuda.stream(stream):
                for i in range(n):
                    xcat.copy_(xh[i % 2], non_blocking=True)
                    run_step(wts[i % ncop], xd, yd, qs[0], sxs[0])
                    yh.copy_(ycat, non_blocking=True)
                stream.synchronize()
        how = ("device API with the rotation fused (the host mirrors take none), page-locked "
               "host buffers: one copy in and one copy out a step, host clock")
    e2e(5)
    torch.cuda.synchronize(device)
    e2e_steps = max(1, min(steps, 2000))
    if world > 1:
        dist.barrier()
    t0 = time.perf_counter()
    e2e(e2e_steps)
    e2e_s = time.perf_counter() - t0
    if world > 1:
        t = torch.tensor([e2e_s], device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_s = float(t.item())
    e2e_value = nb["step"] * e2e_steps * world / e2e_s / 1e9
    wrapper_ms = None
    if wrapper is not None:  # the same calls through the Python wrapper (rank-local figure)
        wrapper(5)
        t0 = time.perf_counter()
        wrapper(e2e_steps)
        wrapper_ms = round(1e3 * (time.perf_counter() - t0) / e2e_steps, 5)

    # ---- CPU baseline (rank 0, N = 1 only), bounded sample of the same workload
    cpu = None
    if rank == 0 and world == 1 and args.cpu_seconds > 0:
        from oracle import pyoracle as O
        host_mats = []
        for w, p, sc in copies[0]:
            aux = (float(w.w_scale) if fmt == TERN else
                   None if fmt in REF_FMTS else sc.cpu().numpy().view(np.uint16))
            host_mats.append((p.cpu().numpy(), aux))
        host_signs = [s.cpu().numpy() for s in signs] if block else None
        threads = O.hw_threads()
        cpu_oracle_gbs(wl, host_mats, host_signs, B, 0.0, threads)  # warm-up
        gbs, st, dt, _ = cpu_oracle_gbs(wl, host_mats, host_signs, B, args.cpu_seconds, threads)
        cpu = {"value": round(gbs, 3), "unit": "GB/s", "cores": threads, "kind": "port",
               "cpu_model": cpu_model(),
               "sample": f"median of {st} steps ({dt:.1f} s) at batch {B}: " + (
                   "the reference's own fp32 algorithm for this format (matvec_tl1 x86 order / "
                   "matvec_qblock), restated" if fmt in REF_FMTS else
                   "oracle int8 quantise + GEMV") + f", {threads} threads"}

    if rank == 0:
        cfg = workload_config(args, wl, world)
        cfg.update({"pdl": not args.no_pdl, "l2_prefetch_of_next_step": prefetch,
                    "prefetch_ahead": args.prefetch_ahead if prefetch else 0,
                    "launch": ("one CUDA graph: 2 untimed steps, then exactly the timed steps "
                               "between two event-record nodes" if windowed else
                               "CUDA graphs of exactly the timed steps, queued behind a spin "
                               "kernel before the first event")})
        line = {
            "metric": "packed-weight GEMV HBM GB/s",
            "value": round(value, 2), "unit": "GB/s", "n_gpus": world, "steps": steps,
            "warmup": args.warmup, "ms_per_step": round(ms / steps, 5), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None,
            "dtype": "f32" if fmt in REF_FMTS else "int8",
            "data": "synthetic (random init weights, fp32 N(0,1) activations)",
            "config": cfg,
            "roofline": roof,
            "cpu_baseline": cpu,
            "e2e": {"value": round(e2e_value, 2), "unit": "GB/s", "h2d_bytes_per_step": h2d,
                    "d2h_bytes_per_step": d2h, "steps": e2e_steps,
                    "ms_per_step": round(1e3 * e2e_s / e2e_steps, 5), "how": how,
                    "python_wrapper_ms_per_step": wrapper_ms},
            "gpu_launches": int(round(launches_per_step * steps)),
            "clocks": clocks,
        }
        if args.workload == "layer":
            line["decode_tokens_per_s_ternary_only"] = round(B * world / (ms / 1e3 / steps * 30), 1)
    if windowed:
        del gw
    else:
        del graphs
    if args.workload == "layer" and B == 1 and args.shard_record == "on":
        try:
            rec = sharded_record(ctx, device, world, rank)
        except Exception as e:  # reported, never fatal to the headline line
            rec = {"error": f"{type(e).__name__}: {e}"[:300]}
        if rank == 0:
            line["sharded"] = rec
    if args.workload == "layer" and B <= 2 and args.decode_tokens > 0:
        rec = decode_record(ctx, device, B, args.decode_tokens, world, rank,
                            min(args.cpu_seconds, 3.0))
        if rank == 0:
            line["decode"] = rec
    if rank == 0:
        print(json.dumps(line), flush=True)
    ctx.close()


def decode_record(ctx, device, B: int, tokens: int, world: int, rank: int, cpu_seconds: float):
    """Configuration 4 as a sub-record of the default line: BitNet-2B-class
    decode (30 layers, KV context 1024, tied F16 lm_head with the greedy
    pick), one CUDA graph per token, `tokens` tokens timed on the device (max
    over ranks); the ternary-matmul share is the same projections replayed
    alone over the step's time. Rank 0 at N = 1 adds the reference's fp32
    run_layer on the host cores (bounded sample) as in run_decode."""
    import torch
    import torch.distributed as dist
    from ouroboros_b200.decode import Decoder
    dec = Decoder(ctx, layers=30, batch=B, context=1024, generate=tokens + 8, device=device,
                  seed=29 + rank)
    n0 = ctx.launch_count()
    g_full = dec.capture(dec.step)
    launches = (ctx.launch_count() - n0) / 3
    g_tern = dec.capture(dec.ternary_only_step)

    def timed(g, n):
        if world > 1:
            dist.barrier()
        dec.pos.fill_(1024)
        torch.cuda.synchronize(device)
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        with torch.cuda.stream(dec.stream):
            gate(torch, n)
            e0.record(dec.stream)
            for _ in range(n):
                g.replay()
            e1.record(dec.stream)
        e1.synchronize()
        ms = e0.elapsed_time(e1)
        if world > 1:
            t = torch.tensor([ms], device=device)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            ms = float(t.item())
        return ms

    timed(g_full, 3)
    ms_full = timed(g_full, tokens)
    ms_tern = timed(g_tern, tokens)
    rec = {"workload": f"bitnet2b-decode-b{B}-ctx1024-30layers", "tokens_timed": tokens,
           "tokens_per_s": round(B * world * tokens / (ms_full / 1e3), 2),
           "us_per_token": round(1e3 * ms_full / tokens, 2),
           "ternary_matmul_share": round(ms_tern / ms_full, 4),
           "gpu_launches_per_token": round(launches, 1),
           "how": "one CUDA graph per decode step (RMSNorm fused into the projection launches, "
                  "RoPE + KV append + GQA attention in one launch, F16 lm_head with the argmax), "
                  "device events, max over ranks"}
    del g_full, g_tern
    dec.free()
    del dec
    torch.cuda.empty_cache()
    if rank == 0 and world == 1 and cpu_seconds > 0:
        from oracle import pyoracle as O
        threads = O.hw_threads()
        v, n, _ = cpu_decode_tokens_per_s(B, cpu_seconds, threads)
        rec["cpu_reference_tokens_per_s"] = round(v, 3)
        rec["cpu_reference_sample"] = (f"{n} single-layer passes of run_layer in the reference's fp32 "
                                       f"order (TQ1_0 projections), scaled to 30 layers + the f16 "
                                       f"lm_head; {threads} host threads")
    return rec


def random_tern2_packed(rng, M: int, K: int) -> np.ndarray:
    """Packed ternary codes [M][K/4] with p(-1, 0, +1) = .25, .5, .25: random
    2-bit fields with the code 3 folded onto 1 (vectorised over bytes)."""
    b = rng.integers(0, 256, size=M * K // 4, dtype=np.uint8)
    for j in range(4):
        three = ((b >> (2 * j)) & 3) == 3
        b[three] ^= np.uint8(2 << (2 * j))
    return b.reshape(M, K // 4)


def sharded_record(ctx, device, world: int, rank: int, steps: int = 200):
    """Configuration 5 row-sharded over the job's ranks (every rank holds M/N
    rows of 8192 x 28672, the down projection of a 70B-class FFN): per
    transport (NCCL in-place all-gather; this library's peer stores over
    NVLink) and batch (1, 16), the local product alone, one isolated call
    (product + gather + sync, end to end on the device) and `steps` calls back
    to back in a CUDA graph (gather i overlapping product i + 1 where the
    stream allows). Device events, max over ranks. At N = 1 the same calls on
    one GPU are the baseline."""
    import torch
    import torch.distributed as dist
    import ouroboros_b200 as oq
    from ouroboros_b200 import shard
    M, K = 8192, 28672
    if world > 1:
        shard.join(ctx)
    else:
        ctx.shard_init(oq.shard_unique_id(), 1, 0)
    # enough copies that this rank's rows exceed twice the L2 (every step streams
    # from HBM); each rank draws only the rows it holds (the rest of the full
    # host matrix is never read)
    row0, rows = oq.shard_rows(M, world, rank)
    ncop = min(40, max(2, -(-2 * L2_BYTES // (rows * K // 4))))
    ws = []
    for c in range(ncop):
        full = np.zeros((M, K // 4), np.uint8)
        full[row0:row0 + rows] = random_tern2_packed(np.random.default_rng(4321 + 1000 * c + rank), rows, K)
        ws.append(ctx.upload_shard(oq.TERNARY2, full, M, K, None, 0.01))
        del full
    stream = torch.cuda.Stream(device=device)
    gen = torch.Generator(device=device)
    gen.manual_seed(99)
    rec = {"shape": [M, K], "ranks": world, "rows_per_rank": M // world, "weight_copies": ncop,
           "steps": steps, "bytes_per_step": M * K // 4,
           "how": "device events around CUDA graphs, max over ranks; local = the rank's rows only; "
                  "single = one call (product + gather) then stream sync; pipelined = calls back to back"}

    def timed(g, reps=1):
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize(device)
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        with torch.cuda.stream(stream):
            gate(torch, reps)
            e0.record(stream)
            for _ in range(reps):
                g.replay()
            e1.record(stream)
        ctx.shard_sync(stream, timeout_ms=60000)
        torch.cuda.synchronize(device)
        ms = e0.elapsed_time(e1)
        if world > 1:
            t = torch.tensor([ms], device=device)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            ms = float(t.item())
        return ms

    def graph(fn, n):
        with torch.cuda.stream(stream):
            for i in range(3):
                fn(i)
        ctx.shard_sync(stream, timeout_ms=60000)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=stream):
            for i in range(n):
                fn(i)
        return g

    for B in (1, 16):
        xs = [torch.randn((B, K), generator=gen, device=device) for _ in range(ncop)]
        ys = [torch.empty((B, M), device=device) for _ in range(2)]
        ylocal = torch.empty((B, M // world), device=device)
        g_local = graph(lambda i: ctx.gemm_f32act(ws[i % ncop], xs[i % ncop], y=ylocal, stream=stream), steps)
        timed(g_local)
        local_us = 1e3 * timed(g_local) / steps
        del g_local
        for tr in ("nccl", "peer"):
            ctx.shard_set_transport(tr)
            step = lambda i: ctx.gemm_sharded(ws[i % ncop], xs[i % ncop], y=ys[i % 2], stream=stream)  # noqa: E731
            g_one = graph(step, 1)
            g_pipe = graph(step, steps)
            timed(g_pipe)
            single = [timed(g_one) for _ in range(5)]
            pipe_us = 1e3 * timed(g_pipe) / steps
            rec[f"b{B}_{tr}"] = {"local_product_us": round(local_us, 3),
                                 "single_call_us": round(1e3 * statistics.median(single), 3),
                                 "pipelined_us_per_step": round(pipe_us, 3),
                                 "pipelined_GBs": round(M * K / 4 / (pipe_us / 1e6) / 1e9, 1)}
            del g_one, g_pipe
        del xs, ys, ylocal
    for w in ws:
        w.free()
    ctx.shard_finalize()
    return rec


def cpu_decode_tokens_per_s(B: int, seconds: float, threads: int):
    """The same decode step on the host cores as the reference computes it
    (run_layer, infer/mod.rs:298-336), bounded: one layer -- rmsnorm, the
    seven projections as TQ1_0 shards through matvec_qblock (dequantise, then
    an fp32 dot in element order, threaded over rows like mt_threads), NeoX
    RoPE of q and k, the KV append, attend over the 1025 cached positions,
    the sub-norm, the residual adds, silu(gate) * up -- every op in the
    reference's fp32 order as the oracle restates it, scaled to 30 layers;
    plus the tied lm_head in the reference's f16 order (an eighth of the
    vocabulary, scaled)."""
    from oracle import pyoracle as O
    rng = np.random.default_rng(5)
    shapes = [(2560, 2560), (640, 2560), (640, 2560), (2560, 2560), (6912, 2560), (6912, 2560),
              (2560, 6912)]
    mats = []
    for i, (M, K) in enumerate(shapes):
        pay = O.lcg_bytes(900 + i, M * (K // 256) * 54).reshape(-1, 54)
        sc = (np.abs(rng.standard_normal(pay.shape[0])) * 0.02).astype(np.float16).view(np.uint16)
        pay[:, 52] = sc & 0xFF
        pay[:, 53] = sc >> 8
        mats.append((pay.reshape(-1), M, K))
    norms = {n: (1 + 0.02 * rng.standard_normal(k)).astype(np.float32)
             for n, k in (("attn", 2560), ("attn_sub", 2560), ("ffn", 2560), ("ffn_sub", 6912))}
    # per sequence the cache as the reference keeps it: [position][kv_dim], the
    # 1024-token context plus the token being decoded (position 1024)
    kc = rng.standard_normal((B, 1025, 640), dtype=np.float32)
    vc = rng.standard_normal((B, 1025, 640), dtype=np.float32)
    # the rows of the tied head that the timed sample reads (an eighth, scaled below)
    emb = (0.02 * rng.standard_normal((16384, 2560), dtype=np.float32)).astype(np.float16)
    x = rng.standard_normal((B, 2560), dtype=np.float32)
    pos, rope_base = 1024, 500000.0

    def rms(v, w):
        return np.stack([O.rmsnorm(v[b], w, 1e-5) for b in range(B)])

    def proj(i, v):
        pay, M, K = mats[i]
        return np.stack([O.matvec_tq1(pay, M, K, v[b], threads) for b in range(B)])

    def layer():
        a = rms(x, norms["attn"])
        q, k, v = (proj(i, a) for i in range(3))
        attn = np.empty((B, 2560), np.float32)
        for b in range(B):
            qr = np.concatenate([O.rope_neox(q[b, h * 128:(h + 1) * 128], pos, 128, rope_base)
                                 for h in range(20)])
            kc[b, pos] = np.concatenate([O.rope_neox(k[b, h * 128:(h + 1) * 128], pos, 128,
                                                     rope_base) for h in range(5)])
            vc[b, pos] = v[b]
            attn[b] = O.attend(qr, kc[b], vc[b], 20, 5)
        h1 = x + proj(3, rms(attn, norms["attn_sub"]))
        f = rms(h1, norms["ffn"])
        u_, g_ = proj(4, f), proj(5, f)
        act = np.stack([O.swiglu(g_[b], u_[b]) for b in range(B)])
        return h1 + proj(6, rms(act, norms["ffn_sub"]))

    t0 = time.perf_counter()
    n = 0
    while True:
        layer()
        n += 1
        if time.perf_counter() - t0 >= seconds:
            break
    t_layer = (time.perf_counter() - t0) / n
    # the tied lm_head as the reference computes it (matvec_f16: one fp32 chain
    # per row, threaded over rows), on an eighth of the vocabulary, scaled
    head = np.ascontiguousarray(emb).view(np.uint16)
    t1 = time.perf_counter()
    for b in range(B):
        O.matvec_half(head, 16384, 2560, x[b], threads=threads)
    t_head = (time.perf_counter() - t1) * (128256 / 16384)
    return B / (30 * t_layer + t_head), n, 30 * t_layer + t_head


def run_decode(args, rank, world, local_rank):
    """Configuration 4: BitNet-2B-class decode, 30 layers, KV context 1024,
    256 generated tokens per sequence (the timed region; --tokens), greedy sampling.
    Every rank decodes its own batch (replicas, weak scaling)."""
    import torch
    import torch.distributed as dist
    import ouroboros_b200 as oq
    from ouroboros_b200.decode import Decoder

    device = torch.device("cuda", local_rank)
    torch.cuda.set_device(device)
    ctx = oq.Context(local_rank)
    B, gen = args.batch, args.tokens
    dec = Decoder(ctx, layers=args.layers, batch=B, context=1024, generate=gen, device=device,
                  seed=17 + rank)
    n0 = ctx.launch_count()
    g_full = dec.capture(dec.step)  # two eager steps, then the captured one
    launches_per_token = (ctx.launch_count() - n0) / 3
    dec.lm_head = False
    g_body = dec.capture(dec.step)
    dec.lm_head = True
    g_tern = dec.capture(dec.ternary_only_step)

    def timed(g, n):
        if world > 1:
            dist.barrier()
        dec.pos.fill_(1024)
        torch.cuda.synchronize(device)
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        with torch.cuda.stream(dec.stream):
            gate(torch, n)
            e0.record(dec.stream)
            for _ in range(n):
                g.replay()
            e1.record(dec.stream)
        e1.synchronize()
        ms = e0.elapsed_time(e1)
        if world > 1:
            t = torch.tensor([ms], device=device)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            ms = float(t.item())
        return ms

    timed(g_full, max(3, min(args.warmup, gen)))
    with ClockSampler(local_rank) as clk:
        ms_full = timed(g_full, gen)
    clocks = clk.summary()
    ms_body = timed(g_body, gen)
    ms_tern = timed(g_tern, gen)
    tok_s = B * world * gen / (ms_full / 1e3)
    tok_s_body = B * world * gen / (ms_body / 1e3)
    # ternary weight bytes streamed per token step (all 30 layers)
    tern_bytes = args.layers * (2 * 2560 * 2560 + 2 * 640 * 2560 + 3 * 6912 * 2560) // 4
    achieved = tern_bytes / (ms_tern / 1e3 / gen) / 1e9
    hbm_peak, _, peak_kind = peaks()

    # e2e: the same step with the sampled token ids read back to the host and
    # fed in again from pinned host memory every step
    tok_h = torch.empty((B,), dtype=torch.long).pin_memory()
    def e2e(n):
        for _ in range(n):
            g_full.replay()
            tok_h.copy_(dec.tokens, non_blocking=True)
            dec.tokens.copy_(tok_h, non_blocking=True)
    if world > 1:
        dist.barrier()
    dec.pos.fill_(1024)
    torch.cuda.synchronize(device)
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(dec.stream):
        e0.record(dec.stream)
        e2e(gen)
        e1.record(dec.stream)
    e1.synchronize()
    e2e_ms = e0.elapsed_time(e1)
    e2e_tok_s = B * world * gen / (e2e_ms / 1e3)

    cpu = None
    if rank == 0 and world == 1 and args.cpu_seconds > 0:
        from oracle import pyoracle as O
        threads = O.hw_threads()
        v, n, dt = cpu_decode_tokens_per_s(B, args.cpu_seconds, threads)
        cpu = {"value": round(v, 3), "unit": "tokens/s", "cores": threads, "kind": "port",
               "cpu_model": cpu_model(),
               "sample": f"{n} single-layer passes at batch {B} of run_layer in the "
                         f"reference's fp32 order (TQ1_0 matvec_qblock projections, rmsnorm, "
                         f"RoPE, attend over 1025 positions, silu) scaled to 30 layers, plus the "
                         f"lm_head in the reference's matvec_f16 order (1/8 of the vocabulary, "
                         f"scaled); {threads} threads for the matvecs"}
    if rank == 0:
        line = {
            "metric": "decode tokens/s", "value": round(tok_s, 2), "unit": "tokens/s",
            "n_gpus": world, "steps": gen, "warmup": max(3, min(args.warmup, gen)),
            "ms_per_step": round(ms_full / gen, 5),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "int8",
            "data": "synthetic (random init BitNet-2B-class weights, random 1024-token KV context)",
            "config": {"workload": f"bitnet2b-decode-b{B}-ctx1024-gen{gen}"
                                   + ("" if args.layers == 30 else f"-{args.layers}layers"),
                       "batch": B, "layers": args.layers, "hidden": 2560, "heads": "20/5x128", "ffn": 6912,
                       "vocab": 128256, "kv": "fp32", "parallelism": f"replicas x{world}",
                       "launch": "one CUDA graph per decode step"},
            "tokens_per_s_without_lm_head": round(tok_s_body, 2),
            "ternary_matmul_share": round(ms_tern / ms_full, 4),
            "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": hbm_peak,
                         "unit": "GB/s", "frac": round(achieved / hbm_peak, 4),
                         "peak_kind": f"{peak_kind} (hbm_gbs)", "traffic": None,
                         "kernel": f"ternary projections of one decode step ({args.layers} layers)",
                         "bytes_per_step": tern_bytes},
            "cpu_baseline": cpu,
            "e2e": {"value": round(e2e_tok_s, 2), "unit": "tokens/s", "h2d_bytes_per_step": 8 * B,
                    "d2h_bytes_per_step": 8 * B,
                    "how": "graph replay per token with the sampled ids copied to pinned host "
                           "memory and back"},
            "gpu_launches": int(round(launches_per_token * gen)),
            "clocks": clocks,
        }
        print(json.dumps(line), flush=True)
    del g_full, g_body, g_tern
    dec.free()
    ctx.close()


def run_sharded(args, rank, world, local_rank):
    """Strong scaling of one large matrix: rank r holds rows [r*M/N, (r+1)*M/N),
    every step computes the local rows and all-gathers the full y on every rank."""
    import torch
    import torch.distributed as dist
    import ouroboros_b200 as oq
    from ouroboros_b200 import shard

    wl = WORKLOADS[args.workload]
    desc, fmt, mats, widths, block = wl
    if len(mats) != 1 or fmt != TERN:
        raise SystemExit("--shard takes a single ternary matrix workload (c1, c5-up, c5-down)")
    _, M, K, _ = mats[0]
    device = torch.device("cuda", local_rank)
    torch.cuda.set_device(device)
    ctx = oq.Context(local_rank)
    if world > 1:
        shard.join(ctx)
    else:
        ctx.shard_init(oq.shard_unique_id(), 1, 0)
    ctx.shard_set_transport(args.transport)
    B = args.batch
    ncop = n_copies(wl)
    rng = np.random.default_rng(4321)
    copies = []
    for _ in range(ncop):  # identical full matrices on every rank (same seed)
        codes = rng.integers(0, 4, size=(M, K), dtype=np.uint8)
        codes[codes == 3] = 1  # p(-1, 0, +1) = .25, .5, .25 as codes 0, 1, 2
        c = codes.reshape(M, K // 4, 4)
        packed = (c[..., 0] | (c[..., 1] << 2) | (c[..., 2] << 4) | (c[..., 3] << 6)).astype(np.uint8)
        w_scale = 0.02 * float(np.count_nonzero(codes != 1)) / (M * K)
        copies.append(ctx.upload_shard(oq.TERNARY2, packed, M, K, None, w_scale))
        del codes, c, packed
    gen = torch.Generator(device=device)
    gen.manual_seed(99)
    xs = [torch.randn((B, K), generator=gen, device=device) for _ in range(ncop)]
    ys = [torch.empty((B, M), dtype=torch.float32, device=device) for _ in range(2)]
    ylocal = torch.empty((B, M // world), dtype=torch.float32, device=device)
    stream = torch.cuda.Stream(device=device)

    def step(i):
        ctx.gemm_sharded(copies[i % ncop], xs[i % ncop], y=ys[i % 2], stream=stream)

    def local(i):
        ctx.gemm_f32act(copies[i % ncop], xs[i % ncop], y=ylocal, stream=stream)

    def capture(fn, n):
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=stream):
            for i in range(n):
                fn(i)
        return g

    def graphs_for(fn, nsteps):
        """Graphs that run exactly nsteps steps, after an eager warm-up."""
        with torch.cuda.stream(stream):
            for i in range(max(args.warmup, 3)):
                fn(i)
        ctx.shard_sync(stream, timeout_ms=60000)
        G, reps, rest = graph_plan(nsteps, ncop)
        out = []
        if reps:
            out.append((capture(fn, G), reps))
        if rest:
            out.append((capture(fn, rest), 1))
        return out

    def timed(gs):
        dist.barrier() if world > 1 else None
        torch.cuda.synchronize(device)
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        with torch.cuda.stream(stream):
            gate(torch, sum(r for _, r in gs))
            e0.record(stream)
            for g, reps in gs:
                for _ in range(reps):
                    g.replay()
            e1.record(stream)
        ctx.shard_sync(stream, timeout_ms=120000)
        torch.cuda.synchronize(device)
        ms = e0.elapsed_time(e1)
        if world > 1:
            t = torch.tensor([ms], device=device)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            ms = float(t.item())
        return ms

    steps = max(1, args.steps)
    g_step = graphs_for(step, steps)
    g_local = graphs_for(local, steps)
    timed(g_step)
    with ClockSampler(local_rank) as clk:
        ms = timed(g_step)
    clocks = clk.summary()
    timed(g_local)
    lms = timed(g_local)

    nb = step_bytes(wl, B)
    value = nb["step"] * steps / (ms / 1e3) / 1e9  # the full matrix once per step, all ranks
    hbm_peak, bf16_peak, peak_kind = peaks()
    local_bytes = nb["weights"] // world + B * K * 4 + B * (M // world) * 4
    achieved = local_bytes / (lms / 1e3 / steps) / 1e9
    if rank == 0:
        line = {
            "metric": "packed-weight GEMV HBM GB/s", "value": round(value, 2), "unit": "GB/s",
            "n_gpus": world, "steps": steps, "warmup": args.warmup,
            "ms_per_step": round(ms / steps, 5), "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "int8",
            "data": "synthetic (random init ternary weights, fp32 N(0,1) activations)",
            "config": {"workload": f"{desc}-b{B}-rowsharded", "batch": B, "shapes": [[M, K]],
                       "rows_per_rank": M // world, "weight_copies_rotated": ncop,
                       "parallelism": f"row-sharded x{world}, " + (
                           "peer stores over NVLink" if args.transport == "peer"
                           else "in-place NCCL all-gather"),
                       "launch": "CUDA graphs of exactly the timed steps"},
            "local_product_us": round(1e3 * lms / steps, 3),
            "gather_and_sync_us": round(1e3 * (ms - lms) / steps, 3),
            "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": hbm_peak,
                         "unit": "GB/s", "frac": round(achieved / hbm_peak, 4),
                         "peak_kind": f"{peak_kind} (hbm_gbs)", "traffic": None,
                         "kernel": "per-rank local product (fused GEMV / tensor-core GEMM)",
                         "bytes_per_rank_step": local_bytes},
            "cpu_baseline": None,
            "gpu_launches": None,
            "clocks": clocks,
        }
        print(json.dumps(line), flush=True)
    del g_step, g_local
    ctx.shard_finalize()
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
        if args.workload == "decode":
            run_decode(args, rank, world, local_rank)
        elif args.shard:
            run_sharded(args, rank, world, local_rank)
        else:
            run_ouroq(args, rank, world, local_rank)
    finally:
        if world > 1:
            import torch.distributed as dist
            dist.barrier()
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
