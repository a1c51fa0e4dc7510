#!/usr/bin/env python3
"""Golden model files written by the reference's own writers.

Runs only where the reference checkout is present (it is read, never
written); the outputs are small gzipped files in this directory that pin the
library's .mojostream reader (ms_file_check / ms_model_load) and the
host-side writer (mojostream_b200/fileformat.py) on any machine:

* ``fake_demo.mojostream.gz`` -- scripts/create_fake_model.py
  ``generate_mojostream`` (format 1, :194-281) with its dimension constants
  set small (hidden 64, kv 16, ffn 128, 2 layers, 8 q / 2 kv heads);
* ``convert_small.mojostream.gz`` -- scripts/convert.py ``convert``
  (format 2, layer-typed dims + Engram header, :425-530) on a synthetic
  3-layer Gemma-4-style checkpoint (hidden 64, 4 / 2 heads, head_dim 16,
  global head_dim 32, layers sliding / sliding / full, window 32) written as
  F32 safetensors;
* ``lm_head_v2.bin.gz`` -- scripts/export_lm_head.py (v2, :160-168) with
  HIDDEN 64 and VOCAB_N 32 on a synthetic BF16 embedding table;
* ``files.json`` -- what the reference put in each file, computed from the
  reference's own functions: header fields, and per tensor (layer, type,
  rows, cols, scale, SHA-256 of the Q4 bytes) -- the format-1 tensors by
  re-drawing the generator's seed-42 stream with its ``pack_row_major``, the
  format-2 tensors with convert.py's ``quantize_q4_blockwise`` on the
  synthetic weights; for the lm_head the BOS row, gamma and the SHA-256 of
  the fp32 matrix.

Usage:  python tests/golden/make_files.py [reference_root]
"""
import contextlib
import gzip
import hashlib
import importlib.util
import io
import json
import os
import shutil
import struct
import sys
import tempfile

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))


def _load(path, name):
    spec = importlib.util.spec_from_file_location(name, path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def _sha(b):
    return hashlib.sha256(bytes(b)).hexdigest()


def _gz(src, name):
    with open(src, "rb") as f, open(os.path.join(HERE, name), "wb") as out:
        out.write(gzip.compress(f.read(), mtime=0))


def _write_safetensors(path, tensors):
    """Minimal safetensors writer (F32 / BF16 given as raw bytes + dtype)."""
    hdr, blobs, off = {}, [], 0
    for name, (dtype, shape, raw) in tensors.items():
        hdr[name] = {"dtype": dtype, "shape": list(shape), "data_offsets": [off, off + len(raw)]}
        blobs.append(raw)
        off += len(raw)
    h = json.dumps(hdr).encode()
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(h)))
        f.write(h)
        for b in blobs:
            f.write(b)


def fake_demo(ref, tmp):
    cf = _load(os.path.join(ref, "scripts", "create_fake_model.py"), "ref_create_fake_model")
    D, KV, F, L, NH, NKV = 64, 16, 128, 2, 8, 2
    cf.G4_D, cf.G4_KV_D, cf.G4_FFN_D, cf.G4_LAYERS = D, KV, F, L
    cf.G4_N_HEADS, cf.G4_N_KV_HEADS = NH, NKV
    cf.GEMMA4_MATRICES = [("Q", D, D), ("K", D, KV), ("V", D, KV), ("O", D, D),
                          ("Gate", D, F), ("Up", D, F), ("Down", F, D)]
    out = os.path.join(tmp, "fake_demo.mojostream")
    with contextlib.redirect_stdout(io.StringIO()):
        cf.generate_mojostream(out)
    # the generator's draw order (:205-219): PLE, then pack_row_major x 7
    rng = np.random.default_rng(42)
    tensors = []
    for layer in range(L):
        ple = float(rng.uniform(0.8, 1.2))
        tensors.append([layer, 0, 1, 0, float(np.float32(ple)), None])
        for t, (_, rows, cols) in enumerate(cf.GEMMA4_MATRICES, start=1):
            scale, data = cf.pack_row_major(rng, rows, cols)
            tensors.append([layer, t, rows, cols, float(np.float32(scale)), _sha(data.tobytes())])
    _gz(out, "fake_demo.mojostream.gz")
    return dict(format_tag=1, n_layers=L, hidden=D, kv_dim=KV, ffn_dim=F, n_heads=NH,
                n_kv_heads=NKV, n_tensors=8 * L, file_size=os.path.getsize(out), tensors=tensors)


def convert_small(ref, tmp):
    cv = _load(os.path.join(ref, "scripts", "convert.py"), "ref_convert")
    D, NH, NKV, HD, GHD, F, L, W = 64, 4, 2, 16, 32, 128, 3, 32
    types = ["sliding_attention", "sliding_attention", "full_attention"]
    src = os.path.join(tmp, "hf")
    os.makedirs(src)
    with open(os.path.join(src, "config.json"), "w") as f:
        json.dump({"model_type": "gemma4", "text_config": {
            "hidden_size": D, "num_hidden_layers": L, "num_attention_heads": NH,
            "num_key_value_heads": NKV, "intermediate_size": F, "head_dim": HD,
            "global_head_dim": GHD, "layer_types": types, "sliding_window": W,
            "hidden_size_per_layer_input": 8, "num_kv_shared_layers": 0}}, f)
    rng = np.random.default_rng(2024)
    pre = "model.language_model.layers."
    tens, fp = {}, {}
    for l in range(L):
        hd = GHD if types[l] == "full_attention" else HD
        q, kv = NH * hd, NKV * hd
        shapes = {"self_attn.q_proj.weight": (q, D), "self_attn.k_proj.weight": (kv, D),
                  "self_attn.v_proj.weight": (kv, D), "self_attn.o_proj.weight": (D, q),
                  "mlp.gate_proj.weight": (F, D), "mlp.up_proj.weight": (F, D),
                  "mlp.down_proj.weight": (D, F)}
        for suf, shp in shapes.items():
            w = (rng.standard_normal(shp) * 0.05).astype(np.float32)
            fp[pre + f"{l}." + suf] = w
            tens[pre + f"{l}." + suf] = ("F32", shp, w.tobytes())
        norm = (1.0 + 0.1 * rng.standard_normal(D)).astype(np.float32)
        fp[pre + f"{l}.input_layernorm.weight"] = norm
        tens[pre + f"{l}.input_layernorm.weight"] = ("F32", (D,), norm.tobytes())
    _write_safetensors(os.path.join(src, "model.safetensors"), tens)
    out = os.path.join(tmp, "convert_small.mojostream")
    with contextlib.redirect_stdout(io.StringIO()):
        cv.convert(src, out, verbose=False)
    # what convert() writes per tensor (:497-523): PLE = mean |norm| (>= 0.001),
    # then quantize_q4_blockwise of the transposed weight
    order = ["self_attn.q_proj.weight", "self_attn.k_proj.weight", "self_attn.v_proj.weight",
             "self_attn.o_proj.weight", "mlp.gate_proj.weight", "mlp.up_proj.weight",
             "mlp.down_proj.weight"]
    tensors = []
    for l in range(L):
        norm = fp[pre + f"{l}.input_layernorm.weight"]
        ple = max(float(np.mean(np.abs(norm))), 0.001)
        tensors.append([l, 0, 1, 0, float(np.float32(ple)), None])
        for t, suf in enumerate(order, start=1):
            wt = fp[pre + f"{l}." + suf].T
            packed, scale = cv.quantize_q4_blockwise(wt, 32)
            tensors.append([l, t, wt.shape[0], wt.shape[1], float(np.float32(scale)),
                            _sha(packed.tobytes())])
    _gz(out, "convert_small.mojostream.gz")
    return dict(format_tag=2, n_layers=L, hidden=D, kv_dim=NKV * HD, ffn_dim=F, n_heads=NH,
                n_kv_heads=NKV, n_tensors=8 * L, file_size=os.path.getsize(out),
                sliding_kv_dim=NKV * HD, full_kv_dim=NKV * GHD, ple_dim=8, sliding_window=W,
                kv_shared_layers=0, tensors=tensors)


def lm_head_v2(ref, tmp):
    H, VN, VT = 64, 32, 40
    work = os.path.join(tmp, "lm")
    wdir = os.path.join(work, "weights", "gemma-4-e4b-raw")
    os.makedirs(wdir)
    with open(os.path.join(wdir, "tokenizer.json"), "w") as f:
        json.dump({"model": {"vocab": {f"tok{i}": i for i in range(VT)}}, "added_tokens": []}, f)
    rng = np.random.default_rng(7)

    def bf16(a):
        u = np.asarray(a, np.float32).view(np.uint32)
        return (u >> 16).astype("<u2")

    emb = bf16(rng.standard_normal((VT, H)) * 0.1)
    gam = bf16(1.0 + 0.1 * rng.standard_normal(H))
    _write_safetensors(os.path.join(wdir, "model.safetensors"), {
        "model.language_model.embed_tokens.weight": ("BF16", (VT, H), emb.tobytes()),
        "model.language_model.norm.weight": ("BF16", (H,), gam.tobytes())})
    src = open(os.path.join(ref, "scripts", "export_lm_head.py")).read()
    src = src.replace("VOCAB_N        = 8192", f"VOCAB_N        = {VN}")
    src = src.replace("HIDDEN         = 2560", f"HIDDEN         = {H}")
    assert f"VOCAB_N        = {VN}" in src and f"HIDDEN         = {H}" in src
    cwd = os.getcwd()
    os.chdir(work)
    try:
        with contextlib.redirect_stdout(io.StringIO()):
            exec(compile(src, "export_lm_head.py", "exec"), {"__name__": "__main__"})
    finally:
        os.chdir(cwd)
    out = os.path.join(work, "lm_head_proto.bin")
    _gz(out, "lm_head_v2.bin.gz")
    w = (emb.astype(np.uint32) << 16).view(np.float32)[:VN]
    g = (gam.astype(np.uint32) << 16).view(np.float32)
    return dict(version=2, vocab=VN, hidden=H, file_size=os.path.getsize(out),
                bos=[float(v) for v in w[2]], gamma=[float(v) for v in g],
                lm_head_sha=_sha(np.ascontiguousarray(w.T, np.float32).tobytes()))


def main(ref):
    tmp = tempfile.mkdtemp()
    try:
        meta = {"fake_demo": fake_demo(ref, tmp), "convert_small": convert_small(ref, tmp),
                "lm_head_v2": lm_head_v2(ref, tmp)}
    finally:
        shutil.rmtree(tmp)
    with open(os.path.join(HERE, "files.json"), "w") as f:
        json.dump(meta, f, indent=1)


if __name__ == "__main__":
    root = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("MS_REFERENCE_ROOT", "")
    if not root or not os.path.isdir(root):
        sys.exit("usage: make_files.py <reference_root> (or MS_REFERENCE_ROOT)")
    main(root)
