"""The bench line the round driver parses, checked without a GPU: the
reference arm (`bench.py --impl reference`, the C restatement of the
reference's CPU path) runs here, and its line must carry the same metric,
unit and workload as our arm's, the fields the driver reads, and a
cpu_baseline / e2e block describing the run.  The headline arm's own line
needs a GPU and is produced by the GPU runs."""
import json
import os
import subprocess
import sys

import bench

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_reference_arm_line():
    out = subprocess.run(
        [sys.executable, "bench.py", "--impl", "reference", "--steps", "1", "--warmup", "0",
         "--layers", "2"],
        cwd=ROOT, capture_output=True, text=True, timeout=600)
    assert out.returncode == 0, out.stderr[-2000:]
    lines = [l for l in out.stdout.splitlines() if l.startswith("{")]
    assert len(lines) == 1, out.stdout[-2000:]
    d = json.loads(lines[0])
    assert d["impl"] == "reference"
    assert d["metric"] == bench.METRIC and d["unit"] == "tokens/s"
    assert d["higher_is_better"] is True and d["value"] > 0
    assert d["n_gpus"] == 1 and d["steps"] == 1 and d["warmup"] == 0
    assert d["config"]["workload"] == bench.WORKLOAD
    cb = d["cpu_baseline"]
    assert cb["kind"] in ("port", "reference") and cb["cores"] >= 1 and cb["sample"]
    assert cb["value"] == d["value"]
    e2e = d["e2e"]
    assert e2e["value"] == d["value"] and e2e["unit"] == d["unit"]
    assert e2e["h2d_bytes_per_step"] == 0 and e2e["d2h_bytes_per_step"] == 0


def test_defaults_meet_the_timing_rules(monkeypatch):
    """No flags: one GPU, at least 3 warm-up steps, a timed loop of a few
    dozen steps, the headline case with every extra block."""
    monkeypatch.setattr(sys, "argv", ["bench.py"])
    args = bench.parse()
    assert args.gpus == 1 and args.warmup >= 3 and 16 <= args.steps <= 512
    assert args.impl == "ours" and args.case == "decode" and args.extras == "all"


def test_reference_arm_under_torchrun_prints_one_line():
    """Launched as the driver launches N > 1 (torchrun, one process per
    rank): rank 0 alone runs the reference's CPU path and prints the line,
    the other rank exits 0 without work."""
    import socket
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    out = subprocess.run(
        [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node", "2",
         "--master-addr", "127.0.0.1", "--master-port", str(port),
         "bench.py", "--impl", "reference", "--gpus", "2", "--steps", "1", "--warmup", "0",
         "--layers", "2"],
        cwd=ROOT, capture_output=True, text=True, timeout=600)
    assert out.returncode == 0, out.stderr[-2000:]
    lines = [l for l in out.stdout.splitlines() if l.startswith("{")]
    assert len(lines) == 1, out.stdout[-2000:]
    d = json.loads(lines[0])
    assert d["impl"] == "reference" and d["n_gpus"] == 2 and d["value"] > 0
    assert d["metric"] == bench.METRIC and d["config"]["workload"] == bench.WORKLOAD


def test_launch_count_matches_the_committed_launch_lists():
    """gpu_launches is counted, not measured: the rule must reproduce the
    per-step counts of the launch lists in profiles/ (two graph replays of 426
    launches at batch 4; 382 launches in one step at batch 64)."""
    assert bench.decode_launches(42, 4) == 426 // 2
    assert bench.decode_launches(42, 64) == 382
    assert bench.decode_launches(42, 4, "i8") == 213 + 42
    assert bench.decode_launches(42, 4, sampling=True) == 214
