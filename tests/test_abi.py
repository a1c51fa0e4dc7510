"""The C-ABI library loads and exports every symbol include/*.h declares
(no device calls: this runs without a GPU)."""
import ctypes
import glob
import os
import re

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_symbols():
    names = set()
    for h in glob.glob(os.path.join(ROOT, "include", "*.h")):
        src = open(h).read()
        names |= set(re.findall(r"^MS_API\s+[\w\s\*]+?\b(ms_\w+)\s*\(", src, flags=re.M))
    return names


@pytest.fixture(scope="module")
def cdll():
    from mojostream_b200 import _lib
    if not os.path.exists(_lib.LIB_PATH):
        from mojostream_b200 import build
        build.build()
    return ctypes.CDLL(_lib.LIB_PATH)


def test_header_declares_the_abi():
    names = declared_symbols()
    for must in ["ms_init", "ms_q4_gemm", "ms_layer_forward", "ms_forward", "ms_lm_head",
                 "ms_embed", "ms_kv_create", "ms_model_create", "ms_generate", "ms_prefill"]:
        assert must in names


def test_library_exports_every_declared_symbol(cdll):
    missing = [n for n in sorted(declared_symbols()) if not hasattr(cdll, n)]
    assert not missing, missing


def test_binding_covers_the_header():
    from mojostream_b200 import _lib
    assert declared_symbols() == set(_lib.SIGNATURES)


def test_binding_loads_and_answers_without_a_device(cdll):
    from mojostream_b200 import _lib
    L = _lib.lib()
    assert L.ms_abi_version() == 1
    assert L.ms_status_string(4) == b"capacity exceeded"
    h = ctypes.c_void_p()
    # no GPU here (or a bad ordinal): a clean error code, no crash
    assert L.ms_init(9999, ctypes.byref(h)) != 0


def test_exports_only_the_abi(cdll):
    import subprocess
    from mojostream_b200 import _lib
    out = subprocess.run(["nm", "-D", "--defined-only", _lib.LIB_PATH], capture_output=True,
                         text=True).stdout
    syms = {l.split()[-1] for l in out.splitlines() if " T " in l}
    assert syms == declared_symbols(), syms ^ declared_symbols()
