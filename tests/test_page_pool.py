"""The pooled KV cache's page bookkeeping (mojostream_b200/csrc/ms_pages.h),
checked on the host: tests/page_pool_check.cc drives it through random
calls, releases, prefix shares and resets and checks its invariants after
each, including that a call refused for want of pages leaves no trace."""
import os
import shutil
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.mark.skipif(shutil.which("g++") is None, reason="needs g++")
def test_page_pool_invariants(tmp_path):
    exe = tmp_path / "page_pool_check"
    subprocess.run(["g++", "-std=c++17", "-O1", "-Wall", "-Werror",
                    "-I", os.path.join(ROOT, "mojostream_b200", "csrc"),
                    os.path.join(ROOT, "tests", "page_pool_check.cc"), "-o", str(exe)],
                   check=True, capture_output=True, text=True)
    out = subprocess.run([str(exe)], capture_output=True, text=True, timeout=120)
    assert out.returncode == 0, out.stdout[-2000:] + out.stderr[-2000:]
    assert out.stdout.strip().endswith("ok")
