"""The launch planners (mojostream_b200/csrc/ms_plan.h) on the host:
tests/plan_check.cu walks a broad grid of shapes under the library's
context limits and checks every plan's invariants.  Q4 projections: K
covered exactly, the kernel the row count calls for, split-K scratch within
the context's buffers, decode segments within the streaming kernel's
registers, cluster merges of at most 8.  Decode attention: split counts
within the kernel's, splits of at least 8 positions, partial sums within the
scratch, cluster merges only where they can hold every split.  Built with nvcc because the planner's header shares
the kernels' definitions; nothing runs on a GPU."""
import os
import shutil
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.mark.skipif(shutil.which("nvcc") is None, reason="needs nvcc")
def test_plan_invariants(tmp_path):
    exe = tmp_path / "plan_check"
    subprocess.run(["nvcc", "-std=c++17", "-O1", "-Wno-deprecated-gpu-targets",
                    "-I", os.path.join(ROOT, "mojostream_b200", "csrc"),
                    os.path.join(ROOT, "tests", "plan_check.cu"), "-o", str(exe)],
                   check=True, capture_output=True, text=True, timeout=300)
    out = subprocess.run([str(exe)], capture_output=True, text=True, timeout=300)
    assert out.returncode == 0, out.stdout[-2000:] + out.stderr[-2000:]
    assert out.stdout.startswith("ok"), out.stdout
