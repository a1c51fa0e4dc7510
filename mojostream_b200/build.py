"""Build libmojostream_cuda.so in place (nvcc, sm_100a; see csrc/Makefile).

Usage: python -m mojostream_b200.build
"""
import os
import subprocess

HERE = os.path.dirname(os.path.abspath(__file__))


def build(jobs=4):
    subprocess.run(["make", "-s", f"-j{jobs}", "-C", os.path.join(HERE, "csrc")], check=True)
    return os.path.join(HERE, "libmojostream_cuda.so")


if __name__ == "__main__":
    print(build())
