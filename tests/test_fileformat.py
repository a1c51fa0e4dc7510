"""The .mojostream reader (ms_file_check, through the library without a
device) and the host-side writer, pinned by files the reference's own
writers produced (tests/golden/make_files.py): create_fake_model.py (format
1), convert.py (format 2, layer-typed) and export_lm_head.py (lm_head v2)."""
import gzip
import hashlib
import json
import os
import struct

import numpy as np
import pytest

from mojostream_b200 import fileformat as ff
from mojostream_b200._lib import MsError
from mojostream_b200.model import LayerSpec, ModelSpec

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
META = json.load(open(os.path.join(GOLDEN, "files.json")))
HEADER_KEYS = ["format_tag", "n_layers", "hidden", "kv_dim", "ffn_dim", "n_heads", "n_kv_heads",
               "n_tensors", "file_size"]


@pytest.fixture(scope="module")
def lib_built():
    from mojostream_b200 import _lib
    if not os.path.exists(_lib.LIB_PATH):
        from mojostream_b200 import build
        build.build()


def golden(tmp_path, name):
    p = tmp_path / name.replace(".gz", "")
    p.write_bytes(gzip.decompress(open(os.path.join(GOLDEN, name), "rb").read()))
    return str(p)


@pytest.mark.parametrize("name", ["fake_demo", "convert_small"])
def test_reference_files_pass_the_guards(tmp_path, lib_built, name):
    info = ff.file_check(golden(tmp_path, name + ".mojostream.gz"))
    m = META[name]
    for k in HEADER_KEYS + ["sliding_kv_dim", "full_kv_dim", "ple_dim", "sliding_window"]:
        if k in m:
            assert info[k] == m[k], k
    assert info["data_start"] == 4096 and info["data_end"] <= info["file_size"]


@pytest.mark.parametrize("name", ["fake_demo", "convert_small"])
def test_tensors_are_what_the_reference_wrote(tmp_path, name):
    path = golden(tmp_path, name + ".mojostream.gz")
    info, entries = ff.read_header(path)
    _, w = ff.read_mojostream(path)
    for (layer, typ, rows, cols, scale, sha), e in zip(META[name]["tensors"], entries):
        assert e[:4] == (layer, typ, rows, cols)
        assert np.float32(e[4]) == np.float32(scale)
        if typ:
            assert hashlib.sha256(w.layers[layer].mats[typ - 1].tobytes()).hexdigest() == sha
            assert e[6] % 4096 == 0


def golden_spec(path, full_every):
    info, entries = ff.read_header(path)
    return ff.spec_from_file(path, full_every=full_every), info


@pytest.mark.parametrize("name,full_every", [("fake_demo", 0), ("convert_small", 3)])
def test_writer_reproduces_the_reference_files(tmp_path, name, full_every):
    path = golden(tmp_path, name + ".mojostream.gz")
    spec, info = golden_spec(path, full_every)
    _, w = ff.read_mojostream(path)
    out = str(tmp_path / "rewritten.mojostream")
    ff.write_mojostream(out, spec, w, format_tag=info["format_tag"],
                        sliding_window=info["sliding_window"], ple_dim=info["ple_dim"],
                        kv_shared_layers=info["kv_shared_layers"])
    assert open(out, "rb").read() == open(path, "rb").read()


def test_lm_head_v2_is_what_the_exporter_wrote(tmp_path):
    path = golden(tmp_path, "lm_head_v2.bin.gz")
    m = META["lm_head_v2"]
    lm = ff.read_lm_head(path, m["hidden"])
    assert lm["version"] == 2 and lm["vocab"] == m["vocab"]
    assert np.array_equal(lm["bos"], np.array(m["bos"], np.float32))
    assert np.array_equal(lm["gamma"], np.array(m["gamma"], np.float32))
    assert hashlib.sha256(lm["lm_head"].tobytes()).hexdigest() == m["lm_head_sha"]
    out = str(tmp_path / "lm2.bin")
    ff.write_lm_head(out, lm["lm_head"], lm["gamma"], lm["bos"])
    assert open(out, "rb").read() == open(path, "rb").read()


def test_lm_head_v1_layout(tmp_path):
    """v1 as load_lm_head reads it (lm_head.mojo:72-116): vocab, scale, BOS,
    Q4 [D][V/2]; told from v2 by its size."""
    rng = np.random.default_rng(1)
    q4 = rng.integers(0, 256, size=(64, 16), dtype=np.uint8)
    bos = rng.standard_normal(64).astype(np.float32)
    out = str(tmp_path / "lm1.bin")
    ff.write_lm_head(out, q4=q4, bos=bos, scale=0.03)
    lm = ff.read_lm_head(out, 64)
    assert lm["version"] == 1 and lm["vocab"] == 32
    assert np.array_equal(lm["q4"], q4) and np.array_equal(lm["bos"], bos)
    assert os.path.getsize(out) == 8 + 4 * 64 + 64 * 16


# ---------------------------------------------------------------- guards --

def patched(src, dst, off, fmt, value):
    b = bytearray(open(src, "rb").read())
    struct.pack_into(fmt, b, off, value)
    open(dst, "wb").write(bytes(b))
    return dst


ENTRY = lambda i: 128 + 32 * i  # noqa: E731


@pytest.mark.parametrize("off,fmt,value,needle", [
    (0, "<I", 0x12345678, "magic"),
    (32, "<I", 0, "[ShapeGuard] n_heads = 0"),
    (36, "<I", 3, "[ShapeGuard] n_heads=4 not divisible"),
    (40, "<Q", 25, "[ShapeGuard] n_tensors=25"),
    (16, "<I", 0, "[ShapeGuard] n_layers"),
    (ENTRY(9) + 0, "<I", 0, "layer_id=0 expected=1"),
    (ENTRY(10) + 4, "<I", 3, "mat_type=3 expected=2"),
    (ENTRY(13) + 8, "<I", 65, "rows=65 expected=64"),
    (ENTRY(18) + 12, "<I", 32, "Layer 2 K: cols=32 expected=64"),
    (ENTRY(3) + 16, "<f", 0.0, "scale=0"),
    (ENTRY(0) + 16, "<f", -1.0, "Layer 0 PLE: scale=-1"),
    (ENTRY(5) + 24, "<Q", 4096 * 3 + 8, "not 4096-aligned"),
    (ENTRY(23) + 24, "<Q", 4096 * 1000, "outside the data region"),
    (ENTRY(1) + 24, "<Q", 0, "outside the data region"),
    (ENTRY(5) + 24, "<Q", 2**64 - 4096, "outside the data region"),  # offset + size wraps
    (ENTRY(17) + 12, "<I", 96, "head_dim 24 gives kv_dim 48"),
    (12, "<I", 7, "format tag 7"),
])
def test_guards_reject_corrupt_files(tmp_path, lib_built, off, fmt, value, needle):
    src = golden(tmp_path, "convert_small.mojostream.gz")
    bad = patched(src, str(tmp_path / "bad.mojostream"), off, fmt, value)
    with pytest.raises(MsError) as e:
        ff.file_check(bad)
    assert e.value.name == "MS_ERR_SHAPE"
    assert needle in str(e.value), str(e.value)


def test_format1_kv_dim_guard_and_io_errors(tmp_path, lib_built):
    src = golden(tmp_path, "fake_demo.mojostream.gz")
    bad = patched(src, str(tmp_path / "bad.mojostream"), 24, "<I", 32)
    with pytest.raises(MsError, match=r"\[ShapeGuard\] kv_dim=32 expected=16"):
        ff.file_check(bad)
    short = str(tmp_path / "short.mojostream")
    open(short, "wb").write(open(src, "rb").read()[:100])
    with pytest.raises(MsError, match="too small"):
        ff.file_check(short)
    trunc = str(tmp_path / "trunc.mojostream")
    open(trunc, "wb").write(open(src, "rb").read()[:40000])
    with pytest.raises(MsError, match="outside the data region"):
        ff.file_check(trunc)
    with pytest.raises(MsError) as e:
        ff.file_check(str(tmp_path / "missing.mojostream"))
    assert e.value.name == "MS_ERR_INVALID_ARG"


def test_layer_typed_e4b_header_passes(tmp_path, lib_built):
    """E4B's dims (head_dim 256 / 512 != hidden / n_heads = 320), which the
    reference's StreamingRunner ShapeGuard rejects, pass the layer-typed check
    (checked on a header + directory with one layer of each kind)."""
    slide = LayerSpec(256, 8, 2, 512, 256, 10240, 1e4)
    full = LayerSpec(512, 8, 2, 0, 128, 10240, 1e6)
    spec = ModelSpec("e4b-2", 2560, [slide, full])

    from mojostream_b200.model import LayerWeights, ModelWeights
    w = ModelWeights([LayerWeights(1.0, [0.01] * 7,
                                   [np.zeros((K, N // 2), np.uint8) for K, N in l.mat_shapes(2560)])
                      for l in spec.layers])
    path = str(tmp_path / "e4b2.mojostream")
    ff.write_mojostream(path, spec, w)
    info = ff.file_check(path)
    assert (info["sliding_kv_dim"], info["full_kv_dim"], info["sliding_window"]) == (512, 1024, 512)
    s2 = ff.spec_from_file(path, full_every=2)
    assert s2.layers == [slide, full]
