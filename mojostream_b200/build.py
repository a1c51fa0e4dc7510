"""Build libmojostream_cuda.so in place (nvcc, sm_100a; see csrc/Makefile).

Usage: python -m mojostream_b200.build [--trace]

--trace builds the timeline variant (-DMS_STEP_TRACE: every decode projection
and attention CTA records %globaltimer points and its SM) into
mojostream_b200/_trace/libmojostream_cuda.so, which mojostream_b200.timeline
loads; the product library is untouched.
"""
import os
import subprocess

HERE = os.path.dirname(os.path.abspath(__file__))


TRACE_LIB = os.path.join(HERE, "_trace", "libmojostream_cuda.so")


def build(jobs=4, trace=False):
    cmd = ["make", "-s", f"-j{jobs}", "-C", os.path.join(HERE, "csrc")]
    if trace:
        cmd += ["BUILD=_build/trace", "OUT=../_trace/libmojostream_cuda.so", "EXTRA=-DMS_STEP_TRACE"]
    subprocess.run(cmd, check=True)
    return TRACE_LIB if trace else os.path.join(HERE, "libmojostream_cuda.so")


if __name__ == "__main__":
    import sys
    print(build(trace="--trace" in sys.argv[1:]))
