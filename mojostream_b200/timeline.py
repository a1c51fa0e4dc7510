"""Per-CTA timeline of one decode step (profiling tool; needs a GPU).

Usage:
    python -m mojostream_b200.build --trace
    python -m mojostream_b200.timeline [--batch 4] [--prompt 512] [--layers 42] [--out t.npz]

The trace build of the library (-DMS_STEP_TRACE) makes every CTA of the
one-launch decode projection and attention kernels record its op, its SM, its
entry time, the time its dependency on the previous kernel was met and a few
points inside the kernel (%globaltimer, ns).  This script runs the bench's
E4B-shaped decode step once on random weights and prints, per op of a layer
(median over layers):

* rel->end: from the dependency release to the op's last CTA exit (the op's
  share of the step's critical path) and the gap to the next op's release;
* the median CTA's points after the release (projection: inputs loaded,
  quantised, main loop done, halves merged, split-K merged, epilogue done;
  attention: offsets read, positions done, warps combined, cluster barrier,
  share merged);
* how many SMs held one or two CTAs of the op.

The product library is not touched; timings from the trace build are for
finding where the time goes, not bench numbers.
"""
import argparse
import collections
import ctypes
import os
import sys

import numpy as np

from . import _lib
from .build import TRACE_LIB

REC = np.dtype([("key", "<u8"), ("t0", "<u8"), ("t1", "<u8"), ("t2", "<u8"), ("pts", "<u8", (8,)),
                ("cta", "<i4"), ("kind", "<i4"), ("smid", "<i4"), ("pad", "<i4")])
PROJ_POINTS = [(6, "inputs"), (1, "quantised"), (2, "main loop"), (3, "halves"),
               (4, "split-K"), (5, "epilogue")]
ATTN_POINTS = [(0, "offsets"), (1, "positions"), (2, "combined"), (3, "cluster"), (4, "merged")]
LAYER_OPS = ["QKV", "attention", "O", "gate|up", "down"]


def summarize(recs, ops_per_layer=5):
    """Per-op summary of one step's records (a REC array); returns printable lines."""
    ops = [recs[recs["key"] == k] for k in np.unique(recs["key"])]
    ops.sort(key=lambda s: int(s["t1"].min()))
    if not ops:
        return ["no records"]
    per_pos = collections.defaultdict(list)
    for i, s in enumerate(ops):
        rel = np.int64(s["t1"].min())
        end = (s["t2"].astype(np.int64) - rel) / 1e3
        nxt = ((np.int64(ops[i + 1]["t1"].min()) - np.int64(s["t2"].max())) / 1e3
               if i + 1 < len(ops) else np.nan)
        names = PROJ_POINTS if s["kind"][0] == 0 else ATTN_POINTS
        pts = {}
        for k, name in names:
            col = s["pts"][:, k]
            if (col > 0).all():
                pts[name] = float(np.median((col.astype(np.int64) - rel) / 1e3))
        per_sm = collections.Counter(collections.Counter(s["smid"].tolist()).values())
        per_pos[i % ops_per_layer].append(dict(
            ctas=len(s), crit=float(end.max()), gap=nxt, end_med=float(np.median(end)),
            pts=pts, per_sm=per_sm))
    lines = [f"{len(ops)} ops; sum of rel->end {sum(float(((s['t2'].astype(np.int64) - np.int64(s['t1'].min())) / 1e3).max()) for s in ops):.1f} us"]
    for j in range(ops_per_layer):
        rows = per_pos[j]
        name = LAYER_OPS[j] if ops_per_layer == len(LAYER_OPS) else str(j)
        crit = np.median([r["crit"] for r in rows])
        gap = np.nanmedian([r["gap"] for r in rows])
        endm = np.median([r["end_med"] for r in rows])
        keys = rows[0]["pts"].keys()
        pts = ", ".join(f"{k} {np.median([r['pts'][k] for r in rows if k in r['pts']]):.2f}"
                        for k in keys)
        sm = collections.Counter()
        for r in rows:
            sm.update(r["per_sm"])
        sm_txt = ", ".join(f"{n} CTA: {c / len(rows):.0f} SMs" for n, c in sorted(sm.items()))
        lines.append(f"{name:9s} ctas {rows[0]['ctas']:4d}  rel->end {crit:6.2f} us (median CTA "
                     f"{endm:.2f})  gap {gap:.2f}  | {pts} | {sm_txt}")
    return lines


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__.split("\n\n")[0])
    ap.add_argument("--batch", type=int, default=4)
    ap.add_argument("--prompt", type=int, default=512)
    ap.add_argument("--layers", type=int, default=42)
    ap.add_argument("--out", default=None, help="save the raw records (.npz)")
    args = ap.parse_args(argv)
    if not os.path.exists(TRACE_LIB):
        sys.exit(f"{TRACE_LIB} is missing: python -m mojostream_b200.build --trace")
    _lib.LIB_PATH = TRACE_LIB  # before the first call loads the library
    import torch

    from .model import e4b_spec, synth_weights_device
    from .runtime import Context, KVCache, Model

    B, P = args.batch, args.prompt
    spec = e4b_spec(n_layers=args.layers)
    w = synth_weights_device(spec, seed=1234)
    ctx = Context(0)
    model = Model(ctx, spec, w, max_rows=min(B * P, 2048))
    del w
    torch.cuda.empty_cache()
    window = max(l.window for l in spec.layers)
    kv = KVCache(ctx, model, B, ((P + 64 + 63) // 64) * 64, slide_cap=window + min(P, 2048))
    rng = np.random.default_rng(0)
    ids = [int(t) for t in rng.integers(0, spec.vocab, B * P)]
    seq = sum([[s] * P for s in range(B)], [])
    pos = sum([list(range(P)) for _ in range(B)], [])
    first = model.prefill(kv, ids, seq, pos)
    gen = model.generate(kv, first, list(range(B)), [P] * B, 4)
    cur = [int(t) for t in gen[-1]]
    torch.cuda.synchronize()
    lib = ctypes.CDLL(TRACE_LIB)
    fns = [lib.ms_trace_gemv_stream, lib.ms_trace_attn]
    for f in fns:
        f.restype = ctypes.c_int
        f.argtypes = [ctypes.c_void_p, ctypes.c_size_t, ctypes.c_int]
        f(None, 0, 1)
    _, ms = model.generate(kv, cur, list(range(B)), [P + 4] * B, 1, timing=True)
    torch.cuda.synchronize()
    parts = []
    for f in fns:
        buf = np.zeros(1 << 17, dtype=REC)
        n = f(buf.ctypes.data, buf.nbytes, 0)
        if n < 0:
            sys.exit("copying the trace records failed")
        parts.append(buf[:n])
    recs = np.concatenate(parts)
    print(f"decode step {ms:.3f} ms (trace build), batch {B}, {len(recs)} CTA records")
    for line in summarize(recs):
        print(line)
    if args.out:
        np.savez(args.out, records=recs)


if __name__ == "__main__":
    main()
