"""The reference's model files, host side.

* ``.mojostream`` (reader: src/streaming/mojostream.mojo:95-160): a 128-byte
  header ("MOJOSTRM", version, format tag, n_layers, hidden, kv_dim, ffn_dim,
  n_heads, n_kv_heads, n_tensors, dir_offset, data_start), a directory of
  32-byte entries (layer, type, rows, cols, scale, flags, offset) with one PLE
  entry and seven Q4 matrices (Q, K, V, O, Gate, Up, Down) per layer, and the
  Q4 data, every tensor on a 4096-byte boundary.  Format 1 is the uniform demo
  stack (scripts/create_fake_model.py:194-281); format 2 has layer-typed dims
  and the Engram extension at header byte 64 ("ENGR", version, kv-shared
  layers, sliding kv_dim, full kv_dim, PLE dim, sliding window;
  scripts/convert.py:359-414).
* ``lm_head_proto.bin`` (load_lm_head, src/inference/lm_head.mojo:61-116):
  v2 = vocab, scale 0, version 2, BOS embedding, final gamma, fp32 [D][V]
  (scripts/export_lm_head.py:160-168); v1 = vocab, scale, BOS embedding, Q4
  [D][V/2].

The loader is native (``ms_file_check`` / ``ms_model_load`` in the CUDA
library, ``runtime.Model.load``).  This module writes the formats (tests,
benchmarks, synthetic models) and reads them back in Python for checks.
"""
import struct

import numpy as np

from .model import LayerSpec, LayerWeights, ModelSpec, ModelWeights

MAGIC = b"MOJOSTRM"
ENGRAM_MAGIC = b"ENGR"
HEADER_BYTES = 128
ENTRY_BYTES = 32
PAGE = 4096
PLE, Q, K, V, O, GATE, UP, DOWN = range(8)


def _align(n, a=PAGE):
    return (n + a - 1) // a * a


def _host_u8(a):
    if not isinstance(a, np.ndarray):
        a = a.cpu().numpy()
    return np.ascontiguousarray(a, dtype=np.uint8)


def _host_f32(a):
    if not isinstance(a, np.ndarray):
        a = a.cpu().numpy()
    return np.ascontiguousarray(a, dtype=np.float32)


def write_mojostream(path, spec, weights, format_tag=2, sliding_window=None, ple_dim=0,
                     kv_shared_layers=0):
    """Write a model as a .mojostream file.

    Every layer shares n_heads, n_kv_heads and ffn_dim (single header fields).
    Format 1 needs head_dim = hidden / n_heads on every layer (the demo
    layout); format 2 records kv_dim = the sliding layers' (as convert.py does)
    and the sliding / full kv dims and window in the Engram extension."""
    D, layers = spec.hidden, spec.layers
    l0 = layers[0]
    NH, NKV, F = l0.n_heads, l0.n_kv_heads, l0.ffn_dim
    for l in layers:
        if (l.n_heads, l.n_kv_heads, l.ffn_dim) != (NH, NKV, F):
            raise ValueError("layers differ in n_heads / n_kv_heads / ffn_dim")
    if format_tag == 1 and any(l.head_dim * NH != D for l in layers):
        raise ValueError("format 1 needs head_dim = hidden / n_heads")
    slide = [l for l in layers if l.window > 0]
    full = [l for l in layers if l.window == 0]
    slide_kv = slide[0].kv_dim if slide else 0
    full_kv = full[0].kv_dim if full else 0
    kv_dim = (slide_kv or full_kv) if format_tag == 2 else l0.kv_dim
    win = sliding_window if sliding_window is not None else (slide[0].window if slide else 0)

    n = len(layers)
    n_tensors = 8 * n
    data_start = _align(HEADER_BYTES + ENTRY_BYTES * n_tensors)
    offsets, cur = [], data_start
    for l in layers:
        row = []
        for Kd, Nd in l.mat_shapes(D):
            row.append(cur)
            cur = _align(cur + Kd * (Nd // 2))
        offsets.append(row)

    hdr = struct.pack("<8sIIIIIIIIQQQ", MAGIC, 1, format_tag, n, D, kv_dim, F, NH, NKV,
                      n_tensors, HEADER_BYTES, data_start)
    if format_tag == 2:
        hdr += struct.pack("<4sIIIIII", ENGRAM_MAGIC, 1, kv_shared_layers, slide_kv, full_kv,
                           ple_dim, win)
    hdr += b"\0" * (HEADER_BYTES - len(hdr))
    with open(path, "wb") as f:
        f.write(hdr)
        for i, (l, lw) in enumerate(zip(layers, weights.layers)):
            f.write(struct.pack("<IIIIfIQ", i, PLE, 1, 0, lw.ple, 0, 0))
            for t, (Kd, Nd) in enumerate(l.mat_shapes(D)):
                f.write(struct.pack("<IIIIfIQ", i, t + 1, Kd, Nd, lw.scales[t], 0, offsets[i][t]))
        f.write(b"\0" * (data_start - f.tell()))
        for i, (l, lw) in enumerate(zip(layers, weights.layers)):
            for t, (Kd, Nd) in enumerate(l.mat_shapes(D)):
                assert f.tell() == offsets[i][t]
                raw = _host_u8(lw.mats[t]).tobytes()
                if len(raw) != Kd * (Nd // 2):
                    raise ValueError(f"layer {i} matrix {t}: {len(raw)} bytes, expected "
                                     f"{Kd * (Nd // 2)}")
                f.write(raw)
                f.write(b"\0" * (_align(len(raw)) - len(raw)))


def write_lm_head(path, lm_head=None, final_gamma=None, bos=None, q4=None, scale=0.0):
    """Write lm_head_proto.bin: v2 from an fp32 [D][V] lm_head (final_gamma and
    bos default to ones and column 2), or v1 from Q4 bytes [D][V/2] and their
    scale."""
    with open(path, "wb") as f:
        if q4 is not None:
            q = _host_u8(q4)
            D, V = q.shape[0], 2 * q.shape[1]
            b = _host_f32(bos) if bos is not None else np.zeros(D, np.float32)
            f.write(struct.pack("<If", V, scale))
            f.write(b.tobytes())
            f.write(q.tobytes())
            return
        W = _host_f32(lm_head)
        D, V = W.shape
        g = _host_f32(final_gamma) if final_gamma is not None else np.ones(D, np.float32)
        b = _host_f32(bos) if bos is not None else np.ascontiguousarray(W[:, 2])
        f.write(struct.pack("<IfI", V, 0.0, 2))
        f.write(b.tobytes())
        f.write(g.tobytes())
        f.write(W.tobytes())


def read_header(path):
    """Header fields and directory entries (no tensor data)."""
    with open(path, "rb") as f:
        h = f.read(HEADER_BYTES)
        (magic, version, tag, n_layers, hidden, kv_dim, ffn, nh, nkv, n_tensors, dir_off,
         data_start) = struct.unpack("<8sIIIIIIIIQQQ", h[:64])
        info = dict(magic=magic, version=version, format_tag=tag, n_layers=n_layers,
                    hidden=hidden, kv_dim=kv_dim, ffn_dim=ffn, n_heads=nh, n_kv_heads=nkv,
                    n_tensors=n_tensors, dir_offset=dir_off, data_start=data_start,
                    kv_shared_layers=0, sliding_kv_dim=0, full_kv_dim=0, ple_dim=0,
                    sliding_window=0)
        if h[64:68] == ENGRAM_MAGIC:
            (_, _, info["kv_shared_layers"], info["sliding_kv_dim"], info["full_kv_dim"],
             info["ple_dim"], info["sliding_window"]) = struct.unpack("<4sIIIIII", h[64:92])
        f.seek(HEADER_BYTES)
        d = f.read(ENTRY_BYTES * n_tensors)
    entries = [struct.unpack("<IIIIfIQ", d[i * ENTRY_BYTES:(i + 1) * ENTRY_BYTES])
               for i in range(n_tensors)]
    return info, entries


def read_mojostream(path):
    """(header dict, ModelWeights): PLE scalars, scales and [K][N/2] bytes per
    layer, in the file's order."""
    info, entries = read_header(path)
    data = np.fromfile(path, dtype=np.uint8)
    layers = []
    for l in range(info["n_layers"]):
        e = entries[8 * l:8 * l + 8]
        mats, scales = [], []
        for (_, _, rows, cols, scale, _, off) in e[1:]:
            mats.append(data[off:off + rows * (cols // 2)].reshape(rows, cols // 2).copy())
            scales.append(scale)
        layers.append(LayerWeights(e[0][4], scales, mats))
    return info, ModelWeights(layers)


def read_lm_head(path, hidden):
    """load_lm_head (lm_head.mojo:61-116): dict(version, vocab, scale, bos,
    gamma, lm_head fp32 [D][V] or q4 [D][V/2])."""
    raw = np.fromfile(path, dtype=np.uint8)
    V = int(raw[:4].view(np.uint32)[0])
    scale = float(raw[4:8].view(np.float32)[0])
    D = hidden
    if raw.size >= 12 + 8 * D + 4 * D * V:  # v2, recognised by size as the reference does
        f = raw[12:12 + 4 * (2 * D + D * V)].view(np.float32)
        return dict(version=2, vocab=V, scale=scale, bos=f[:D].copy(), gamma=f[D:2 * D].copy(),
                    lm_head=f[2 * D:].reshape(D, V).copy())
    bos = raw[8:8 + 4 * D].view(np.float32).copy()
    q4 = raw[8 + 4 * D:8 + 4 * D + D * V // 2].reshape(D, V // 2).copy()
    return dict(version=1, vocab=V, scale=scale, bos=bos, gamma=np.ones(D, np.float32), q4=q4)


def spec_from_file(path, lm_head_path=None, full_every=0, window=0, slide_theta=0.0,
                   full_theta=0.0, full_rotary=0):
    """The ModelSpec ms_model_load builds from a file and its options (the same
    rules: format 1 all full attention with head_dim hidden / n_heads; format 2
    head_dim from Q's columns, full iff (layer + 1) % full_every == 0, default
    6)."""
    info, entries = read_header(path)
    typed = info["format_tag"] == 2
    every = full_every or (6 if typed else 1)
    win = window or info["sliding_window"]
    st = slide_theta or 1e4
    ft = full_theta or (1e6 if typed else st)
    NH, NKV, F = info["n_heads"], info["n_kv_heads"], info["ffn_dim"]
    layers = []
    for l in range(info["n_layers"]):
        hd = entries[8 * l + Q][3] // NH if typed else info["hidden"] // NH
        full = (l + 1) % every == 0
        fr = full_rotary or (128 if typed else hd)
        layers.append(LayerSpec(hd, NH, NKV, 0 if full else win, min(fr, hd) if full else hd, F,
                                ft if full else st))
    vocab = 0
    if lm_head_path:
        with open(lm_head_path, "rb") as f:
            vocab = struct.unpack("<I", f.read(4))[0]
    return ModelSpec("file:" + str(path), info["hidden"], layers, vocab)


def file_check(path):
    """ms_file_check through the library (no device): the header as a dict;
    raises MsError with the failed guard's message."""
    import ctypes

    from ._lib import FileInfo, MsError, lib
    info = FileInfo()
    err = ctypes.create_string_buffer(512)
    st = lib().ms_file_check(str(path).encode(), ctypes.byref(info), err, 512)
    if st != 0:
        raise MsError(st, err.value.decode())
    return {name: getattr(info, name) for name, _ in FileInfo._fields_}
