"""bench.py's one-line JSON contract, checked on the host: the reference arm
(the oracle on the host cores) runs without a GPU and must print every key
the driver reads, with the reference arm's own additions."""
import json
import subprocess
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]


def _run(*args):
    out = subprocess.run([sys.executable, str(ROOT / "bench.py"), *args], cwd=ROOT,
                         capture_output=True, text=True, timeout=600)
    assert out.returncode == 0, out.stderr[-2000:]
    lines = [l for l in out.stdout.splitlines() if l.startswith("{")]
    assert len(lines) == 1, out.stdout[-2000:]
    return json.loads(lines[0])


@pytest.mark.parametrize("workload", ["c1", "layer-tl1"])
def test_reference_arm_line(workload):
    d = _run("--impl", "reference", "--steps", "1", "--warmup", "1", "--workload", workload)
    for key in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step",
                "higher_is_better", "scaling", "vs_baseline", "dtype", "data", "config",
                "cpu_baseline", "e2e"):
        assert key in d, key
    assert d["impl"] == "reference"
    assert d["n_gpus"] == 1 and d["steps"] == 1 and d["warmup"] == 1
    assert d["value"] > 0 and d["unit"] == "GB/s" and d["higher_is_better"] is True
    assert d["config"]["workload"].endswith("-b1")
    cb = d["cpu_baseline"]
    assert cb["value"] == d["value"] and cb["cores"] >= 1 and cb["kind"] in ("port", "reference")
    assert d["e2e"] == {"value": d["value"], "unit": d["unit"], "h2d_bytes_per_step": 0,
                        "d2h_bytes_per_step": 0}


def test_reference_arm_under_torchrun_prints_once():
    # the driver launches both arms with torch.distributed.run for N > 1: rank 0
    # alone runs the host-CPU reference and prints; the other ranks exit 0
    out = subprocess.run(
        [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node", "2",
         "--master-addr", "127.0.0.1", "--master-port", "29617", str(ROOT / "bench.py"),
         "--impl", "reference", "--gpus", "2", "--steps", "1", "--warmup", "1",
         "--workload", "c1"],
        cwd=ROOT, capture_output=True, text=True, timeout=600)
    assert out.returncode == 0, out.stderr[-2000:]
    lines = [l for l in out.stdout.splitlines() if l.startswith("{")]
    assert len(lines) == 1, out.stdout[-2000:]
    d = json.loads(lines[0])
    assert d["impl"] == "reference" and d["n_gpus"] == 2 and d["value"] > 0


def test_algorithmic_bytes_match_the_configs():
    # the per-call byte counts of the benchmark configurations: packed weights
    # (+ fp16 scales), int8 activations + one fp32 scale per token, fp32 outputs
    sys.path.insert(0, str(ROOT))
    import bench
    assert bench.step_bytes(bench.WORKLOADS["c1"], 1)["gemm"] == 4_453_892
    assert bench.step_bytes(bench.WORKLOADS["layer"], 1)["weights"] == 17_367_040
    assert bench.step_bytes(bench.WORKLOADS["c3-4096"], 1)["weights"] == 2_359_296
    assert bench.step_bytes(bench.WORKLOADS["c3-11008"], 1)["weights"] == 6_340_608
    assert bench.step_bytes(bench.WORKLOADS["c5-up"], 1)["weights"] == 58_720_256
    assert bench.step_bytes(bench.WORKLOADS["c5-down"], 1)["weights"] == 58_720_256
    # every step streams from HBM: the rotated copies exceed twice the L2
    for name, wl in bench.WORKLOADS.items():
        if wl[2]:
            assert bench.n_copies(wl) * bench.step_bytes(wl, 1)["weights"] >= 2 * bench.L2_BYTES


@pytest.mark.parametrize("steps", [1, 5, 16, 20, 37, 1000, 30000])
def test_graph_plan_runs_exactly_the_requested_steps(steps):
    # the timed region replays graphs whose steps add up to --steps exactly
    # (the driver checks the printed step count against the one it asked for),
    # and the full-pass graph keeps the weight-copy rotation across replays
    sys.path.insert(0, str(ROOT))
    import bench
    ncop = bench.n_copies(bench.WORKLOADS["layer"])
    G, reps, rest = bench.graph_plan(steps, ncop)
    assert G * reps + rest == steps
    assert G % ncop == 0 and G <= 64 * ncop and rest < max(G, steps + 1)
    if steps <= 4096:
        assert reps == 0 and rest == steps  # one graph, no boundary inside the timed region
