#!/usr/bin/env python3
"""Generate the golden fixtures in this directory from the reference's own code.

Runs only where the reference checkout is present (it is read, never written).
It imports the reference's NumPy oracle ``scripts/gen_reference.py`` and its
model generator ``scripts/create_fake_model.py`` and records their outputs as
small ``.npz`` files, so the tests can pin the C oracle (oracle/ms_oracle.c)
and the CUDA library on machines without the reference:

* ``demo_layer0.npz`` -- the reference's validation case
  (scripts/gen_reference.py:179-232): layer 0 of the seed-42 demo model
  (create_fake_model.py:188-281), input seed 1234 x 0.1, batch 4, base_pos 0,
  run through ``forward_layer`` (gen_reference.py:103-174).  The weights are not
  stored: the test regenerates them with the generator's draw order
  (``demo_layer0_weights`` in tests/golden_io.py) and checks them against the
  SHA-256 of the bytes the reference wrote into model.mojostream.
* ``small_layer.npz`` -- ``forward_layer`` on a smaller uniform layer whose
  weights come from a stated seed (for a fast parity case).
* ``ops.npz`` -- the reference's per-op NumPy functions: ``apply_rope_f32``
  at several (heads, head_dim, pos, theta), ``rmsnorm_f32``, ``swiglu_f32``
  and ``dequant_q4``.

Usage:  python tests/golden/make_golden.py [reference_root]
"""
import hashlib
import importlib.util
import os
import shutil
import subprocess
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(HERE))
from golden_io import demo_layer0_weights, small_layer_weights, SMALL_CFG  # noqa: E402


def _load(path, name):
    spec = importlib.util.spec_from_file_location(name, path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def main():
    ref_root = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("MS_REFERENCE_ROOT", "")
    if not ref_root or not os.path.isdir(ref_root):
        sys.exit("reference checkout not given (argument or MS_REFERENCE_ROOT)")
    gen = _load(os.path.join(ref_root, "scripts", "gen_reference.py"), "ref_gen_reference")

    # ---- 1. the reference's own layer-0 validation case ------------------
    tmp = os.path.join(HERE, ".tmp_golden")
    os.makedirs(tmp, exist_ok=True)
    try:
        ms_path = os.path.join(tmp, "model.mojostream")
        ref_path = os.path.join(tmp, "layer0_ref.bin")
        subprocess.run([sys.executable, os.path.join(ref_root, "scripts", "create_fake_model.py"),
                        "--format", "mojostream", "--out", ms_path], check=True,
                       stdout=subprocess.DEVNULL)
        subprocess.run([sys.executable, os.path.join(ref_root, "scripts", "gen_reference.py"),
                        ms_path, ref_path], check=True, stdout=subprocess.DEVNULL)
        ms = gen.parse_mojostream(ms_path)
        sha = {}
        for e in ms["entries"]:
            if e["layer"] == 0 and e["offset"]:
                n = e["rows"] * (e["cols"] // 2)
                sha[e["type"]] = hashlib.sha256(ms["data"][e["offset"]:e["offset"] + n]).hexdigest()
        ple_file = [e["scale"] for e in ms["entries"] if e["layer"] == 0 and e["type"] == 0][0]
        scales_file = [e["scale"] for e in sorted(
            (e for e in ms["entries"] if e["layer"] == 0 and e["type"] > 0), key=lambda e: e["type"])]
        with open(ref_path, "rb") as f:
            raw = f.read()
        magic, ver, hidden, batch = np.frombuffer(raw[:16], dtype="<u4")
        assert magic == 0x42464552 and ver == 1
        n = int(hidden) * int(batch)
        x_in = np.frombuffer(raw[16:16 + 4 * n], dtype="<f4").reshape(batch, hidden)
        x_out = np.frombuffer(raw[16 + 4 * n:16 + 8 * n], dtype="<f4").reshape(batch, hidden)
    finally:
        shutil.rmtree(tmp, ignore_errors=True)

    w = demo_layer0_weights()
    for t in range(1, 8):
        got = hashlib.sha256(w["mats"][t - 1].tobytes()).hexdigest()
        assert got == sha[t], f"regenerated layer-0 tensor {t} differs from the reference file"
    assert np.float32(w["ple"]) == np.float32(ple_file)
    assert np.allclose(np.float32(w["scales"]), np.float32(scales_file), rtol=0, atol=0)
    np.savez_compressed(
        os.path.join(HERE, "demo_layer0.npz"),
        x_in=x_in, x_out=x_out,
        sha256=np.array([sha[t] for t in range(1, 8)]),
        ple=np.float32(ple_file), scales=np.float32(scales_file),
        io_rmse=np.float64(np.sqrt(((x_in.astype(np.float64) - x_out) ** 2).mean())))

    # ---- 2. a smaller uniform layer through the same NumPy forward -------
    sw = small_layer_weights()
    deq = {}
    names = ["Q", "K", "V", "O", "Gate", "Up", "Down"]
    for i, name in enumerate(names):
        raw8 = sw["mats"][i]
        lo = (raw8 & 0x0F).astype(np.float32) - 8.0
        hi = ((raw8 >> 4) & 0x0F).astype(np.float32) - 8.0
        W = np.empty((raw8.shape[0], raw8.shape[1] * 2), dtype=np.float32)
        W[:, 0::2] = lo * np.float32(sw["scales"][i])
        W[:, 1::2] = hi * np.float32(sw["scales"][i])
        deq[name] = W
    deq["ple_scale"] = sw["ple"]
    rng = np.random.default_rng(777)
    xs = (rng.standard_normal((4, SMALL_CFG["hidden"])).astype(np.float32) * 0.5)
    ys = gen.forward_layer(xs, deq, SMALL_CFG, base_pos=0)["final_out"]
    np.savez_compressed(os.path.join(HERE, "small_layer.npz"), x_in=xs, x_out=ys,
                        sha256=np.array([hashlib.sha256(m.tobytes()).hexdigest() for m in sw["mats"]]))

    # ---- 3. per-op fixtures ------------------------------------------------
    out = {}
    rng = np.random.default_rng(2024)
    rope_cases = [(8, 256, 0, 1e4), (8, 256, 7, 1e4), (2, 256, 511, 1e4), (2, 256, 4095, 1e4),
                  (1, 128, 600, 1e6), (1, 128, 8191, 1e6), (16, 64, 403, 1e4), (8, 128, 1000, 1e4)]
    for i, (nh, hd, pos, base) in enumerate(rope_cases):
        x = rng.standard_normal((nh, hd)).astype(np.float32)
        out[f"rope{i}_x"] = x
        out[f"rope{i}_y"] = gen.apply_rope_f32(x, nh, hd, pos, base)
        out[f"rope{i}_args"] = np.array([nh, hd, pos, base], dtype=np.float64)
    x = (rng.standard_normal((4, 2560)) * 3.0).astype(np.float32)
    out["rms_x"], out["rms_y"] = x, gen.rmsnorm_f32(x)
    g = (rng.standard_normal(4096) * 4.0).astype(np.float32)
    u = (rng.standard_normal(4096) * 4.0).astype(np.float32)
    out["swiglu_g"], out["swiglu_u"], out["swiglu_y"] = g, u, gen.swiglu_f32(g, u)
    wq = rng.integers(0, 256, size=(64, 48), dtype=np.uint8)
    fake_ms = {"data": wq.tobytes(), "entries": [
        {"layer": 0, "type": 1, "rows": 64, "cols": 96, "scale": 0.0625, "offset": 0}]}
    # dequant_q4 treats offset 0 as a PLE entry; give it a non-zero offset.
    fake_ms["data"] = b"\x00" * 16 + wq.tobytes()
    fake_ms["entries"][0]["offset"] = 16
    out["deq_w"], out["deq_y"] = wq, gen.dequant_q4(fake_ms, 0, 1)
    np.savez_compressed(os.path.join(HERE, "ops.npz"), **out)
    print("golden fixtures written to", HERE)


if __name__ == "__main__":
    main()
