"""mojostream_b200 -- B200 (sm_100a) implementation of MojoStream's Gemma-4 token loop.

The product is libmojostream_cuda.so (C-ABI: include/mojostream_cuda.h).  This
package holds its sources (csrc/), the ctypes binding (_lib), a Python host
(runtime), the reference-named operator interface (reference_api) and the
model descriptions of the benchmark configurations (model).
"""
from ._lib import MsError, lib  # noqa: F401

__all__ = ["MsError", "lib"]
