#!/usr/bin/env python3
"""Benchmark of the Gemma-4 token loop on B200 (one JSON line on rank 0).

Headline workload: the Gemma-4-E4B-shaped random Q4 model (D 2560, 42 layers =
35 sliding (hd 256, window 512) + 7 full (hd 512, 128 rotary dims, theta 1e6),
8 q / 2 KV heads, FFN 10240, fp32 lm_head over a 262144 vocab), 4 independent
sequences, 512-token seeded prompts (TTFT), then greedy decode at batch 4.  A
step = one decode step of the 4 sequences (4 tokens).  Weights (4.66 GB) and KV
are far larger than L2 (126 MB), so no L2 flush is needed between steps.

value : decode tokens/s, device-resident loop (CUDA-graph replays on the
        library stream, CUDA events), max over ranks
e2e   : the same through ms_decode_step with host buffers (per step: ids / seq /
        pos host->device from pinned memory, next ids and the context's error
        word device->host)
--gpus N (torchrun): every rank runs the E4B loop as an independent replica
        (the sequences are independent; no collective on the data path), weak
        scaling; then the 14B-class model runs tensor parallel over the N ranks
        (the "tp" block: heads / FFN columns / vocabulary sharded, all-reduces
        after O and down), strong scaling.  N = 1 gives the TP1 baseline.
Extra blocks of the default line (N = 1): "demo" (the uniform 40-layer demo
        stack of the reference's bench harness), "q4_sweep" (the isolated Q4
        projection over 20 shapes), "long" (batch 64 at 4 K positions).
--impl reference: the reference's CPU algorithm (the C restatement in oracle/,
        since the Mojo reference cannot be built here) on the host cores, full
        decode steps of the same model.
"""
import argparse
import json
import os
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

PROMPT = 512     # set from --prompt / --batch in main()
BATCH = 4
MAX_ROWS = 2048  # rows per prefill call (the model's activation buffers)
METRIC = "decode tokens/s (batch 4), Gemma-4-E4B-shaped Q4 model"
WORKLOAD = "gemma4-e4b decode, batch 4 independent sequences, 512-token prompts"
DTYPE = "int4 weights x fp32 activations (exact int8-limb tensor-core products), fp32 lm_head"


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=64)
    ap.add_argument("--warmup", type=int, default=8)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--layers", type=int, default=42, help="(debug) fewer layers")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--extras", default="all", choices=["all", "none"],
                    help="all: the default line also carries the demo / q4_sweep / long / tp "
                         "blocks; none: the headline decode only (e.g. for profiling)")
    ap.add_argument("--case", default="decode", choices=["decode", "q4", "tp", "load", "demo"],
                    help="q4: the isolated Q4 projection (one shape with --m/--k/--n, else "
                         "the 20-shape sweep); tp: the 14B-class model tensor-parallel over "
                         "the torchrun ranks; demo: the uniform demo stack")
    ap.add_argument("--batch", type=int, default=None,
                    help="sequences (decode: 4, or 64 for the long-context case; tp: 64)")
    ap.add_argument("--prompt", type=int, default=None,
                    help="prompt tokens per sequence (decode: 512, long context: 4096; tp: 1024)")
    ap.add_argument("--temperature", type=float, default=0.0,
                    help="token-loop sampling (default greedy, the north-star mode; the "
                         "reference's e4b loop uses 0.7)")
    ap.add_argument("--penalty", type=float, default=1.0,
                    help="repetition penalty (the reference's e4b loop uses 1.2)")
    ap.add_argument("--kv", default="f32", choices=["f32", "bf16", "i8"],
                    help="KV cache element type (f32: the parity mode; bf16: half the bytes; "
                         "i8: int8 with a scale per position and KV head)")
    ap.add_argument("--kv-fill", default="prefill", choices=["prefill", "seeded"],
                    help="prefill: the prompts run through ms_prefill (TTFT measured); seeded: "
                         "the cache below the prompt length is filled with seeded K / V values "
                         "(ms_kv_write) and no TTFT is measured -- decode-step profiling without "
                         "a long prefill")
    ap.add_argument("--m", type=int, default=None)
    ap.add_argument("--k", type=int, default=2560)
    ap.add_argument("--n", type=int, default=20480)
    ap.add_argument("--copies", type=int, default=8)
    return ap.parse_args()


def dist_setup(args):
    ws = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return ws, rank, local


def main_config(spec, ws):
    """The `config` of the headline line (both arms)."""
    return {
        "workload": WORKLOAD,
        "layers": spec.n_layers, "hidden": spec.hidden, "vocab": spec.vocab,
        "batch": BATCH, "prompt": PROMPT,
        "parallelism": f"replicas x{ws}" if ws > 1 else "single GPU",
        "l2": "weights + lm_head 4.66 GB >> 126 MB L2 (no flush needed)",
        "kv_dtype": "f32", "sampling": "greedy",
    }


# ------------------------------------------------------------------ clocks --
class ClockSampler:
    """nvidia-smi samples (100 ms) of SM clock and throttle reasons."""
    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu):
        self.gpu, self.rows, self.proc = gpu, [], None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={self.Q}",
                 "--format=csv,noheader,nounits", "-lms", "100"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except Exception:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.rows.append([x.strip() for x in line.split(",")])

    def stop(self):
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()
        out = {"sm_mhz": None, "sm_max_mhz": None, "reasons": []}
        rows = [r for r in self.rows if len(r) >= 9]
        if not rows:
            return out
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        out["sm_mhz"] = float(np.median(sm)) if sm else None
        out["sm_max_mhz"] = float(rows[0][2]) if rows[0][2].replace(".", "").isdigit() else None
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = set()
        for r in rows:
            for i, n in enumerate(names):
                if r[5 + i].lower().startswith("active"):
                    reasons.add(n)
        out["reasons"] = sorted(reasons)
        out["samples"] = len(rows)
        return out


# --------------------------------------------------------------- helpers --
def decode_launches(n_layers, batch, kv="f32", sampling=False):
    """Kernels one decode step launches: the embedding; per layer QKV,
    attention, O, gate|up and down, plus the int8 cache's K / V quantiser and,
    from 9 rows up, the activation quantiser before each of the 4 tensor-core
    projections; the lm_head (one ring launch up to 8 rows, else row
    statistics + a tensor-core pass per 64 rows); the sampler when sampling;
    the token feedback."""
    per_layer = 5 + (1 if kv == "i8" else 0) + (4 if batch > 8 else 0)
    lm = 1 if batch <= 8 else 2 * ((batch + 63) // 64)
    return 1 + per_layer * n_layers + lm + (1 if sampling else 0) + 1


def measured_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return float(d["hbm_gbs"]), float(d["bf16_tflops"]), "measured"
    return 6650.0, 1590.0, "fallback"


def profile_traffic(kernel):
    """DRAM bytes per launch of `kernel` from the committed ncu summary, if any."""
    p = os.path.join(ROOT, "profiles", "traffic.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return d.get(kernel)
    return None


def prompts(n_seq, length, vocab, seed=7):
    rng = np.random.default_rng(seed)
    return rng.integers(0, vocab, size=(n_seq, length)).tolist()


class Dist:
    """Barrier and max-over-ranks on the torchrun group (no-ops at N = 1)."""

    def __init__(self, ws):
        self.ws = ws

    def barrier(self):
        import torch
        torch.cuda.synchronize()
        if self.ws > 1:
            import torch.distributed as dist
            dist.barrier()

    def max(self, v):
        if self.ws == 1:
            return v
        import torch
        import torch.distributed as dist
        t = torch.tensor([v], dtype=torch.float64, device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())


def events():
    import torch
    return torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)


def seeded_fill(model, kv, B, P, slide_cap):
    """Seeded K / V values at positions below P of every sequence and layer
    (ms_kv_write; sliding layers: the slots the ring holds), in place of a
    prefill; returns seeded first ids."""
    import torch
    g = torch.Generator(device="cuda").manual_seed(11)
    for l, ls in enumerate(model.spec.layers):
        lo = max(0, P - slide_cap) if ls.window > 0 else 0
        for s in range(B):
            k = torch.randn((P - lo, ls.kv_dim), device="cuda", generator=g)
            v = torch.randn((P - lo, ls.kv_dim), device="cuda", generator=g)
            kv.write(l, s, lo, k, v)
    torch.cuda.synchronize()
    return [int(t) for t in np.random.default_rng(12).integers(0, model.spec.vocab, size=B)]


def decode_loop(model, kv, B, P, args, D, lib_stream, clocks_gpu=None, slide_cap=0):
    """TTFT (B x P prefill + first token), then warm-up and the timed
    device-resident loop (ms_generate), then the same through ms_decode_step
    with host buffers.  Returns a dict of device times (max over ranks).
    With args.kv_fill == "seeded" the cache is filled with seeded values
    instead of the prefill (ttft_ms is then None)."""
    if getattr(args, "kv_fill", "prefill") == "seeded":
        first = seeded_fill(model, kv, B, P, slide_cap)
        ttft_ms = None
    else:
        ids = sum(prompts(B, P, model.spec.vocab), [])
        seq = sum([[s] * P for s in range(B)], [])
        pos = sum([list(range(P)) for _ in range(B)], [])
        n_warm = min(len(ids), MAX_ROWS)
        model.prefill(kv, ids[:n_warm], seq[:n_warm], pos[:n_warm])  # kernel attributes, buffers
        kv.reset()
        D.barrier()
        e0, e1 = events()
        e0.record(lib_stream)
        first = model.prefill(kv, ids, seq, pos)
        e1.record(lib_stream)
        e1.synchronize()
        ttft_ms = D.max(e0.elapsed_time(e1))
    e0, e1 = events()
    seqs = list(range(B))
    gen = model.generate(kv, first, seqs, [P] * B, args.warmup)
    cur = [int(t) for t in gen[-1]]
    D.barrier()
    clocks = ClockSampler(clocks_gpu).start() if clocks_gpu is not None else None
    gen2, dev_ms = model.generate(kv, cur, seqs, [P + args.warmup] * B, args.steps, timing=True)
    D.barrier()
    dev_ms = D.max(dev_ms)
    cur = [int(t) for t in gen2[-1]]
    p2 = P + args.warmup + args.steps
    D.barrier()
    e0.record(lib_stream)
    t0 = time.perf_counter()
    for i in range(args.steps):
        cur = model.decode_step(kv, cur, seqs, [p2 + i] * B)
    e1.record(lib_stream)
    e1.synchronize()
    wall = time.perf_counter() - t0
    e2e_ms = D.max(e0.elapsed_time(e1))
    D.barrier()
    clk = clocks.stop() if clocks else None
    return {"ttft_ms": ttft_ms, "dev_ms": dev_ms, "e2e_ms": e2e_ms, "wall": wall, "clk": clk,
            "first": first}


# ---------------------------------------------------------------- our arm --
def run_ours(args, ws, rank, local):
    import torch
    import torch.distributed as dist

    from mojostream_b200.model import e4b_spec, synth_weights_device
    from mojostream_b200.runtime import Context, KVCache, Model

    torch.cuda.set_device(local)
    if ws > 1:
        dist.init_process_group("nccl", device_id=torch.device("cuda", local),
                                timeout=__import__("datetime").timedelta(seconds=600))
    D = Dist(ws)
    spec = e4b_spec(n_layers=args.layers)
    w = synth_weights_device(spec, seed=1234)
    ctx = Context(local)
    model = Model(ctx, spec, w, max_rows=min(BATCH * PROMPT, MAX_ROWS))
    if args.temperature > 0.01 or args.penalty > 1.0:
        model.set_sampling(args.temperature, args.penalty, 1234)
    del w
    torch.cuda.empty_cache()
    max_pos = ((PROMPT + args.warmup + 2 * args.steps + 8 + 63) // 64) * 64
    # sliding ring: the window plus the rows of one sequence in one prefill call
    window = max(l.window for l in spec.layers)
    slide_cap = window + min(PROMPT, MAX_ROWS)
    kv = KVCache(ctx, model, BATCH, max_pos, slide_cap=slide_cap, dtype=args.kv)
    lib_stream = torch.cuda.ExternalStream(ctx.stream_ptr)
    r = decode_loop(model, kv, BATCH, PROMPT, args, D, lib_stream, clocks_gpu=local,
                    slide_cap=slide_cap)

    # ---- dominant kernels timed alone (CUDA events on their stream) --------
    hbm, tf, peak_kind = measured_peaks()
    x = torch.randn((BATCH, spec.hidden), device="cuda")
    for _ in range(3):
        model.lm_head(x, logits=False)
    torch.cuda.synchronize()
    n_rep = 10
    s0, s1 = events()
    s0.record()
    for _ in range(n_rep):
        model.lm_head(x, logits=False)
    s1.record()
    s1.synchronize()
    lm_ms = s0.elapsed_time(s1) / n_rep
    lm_bytes = 4 * spec.hidden * spec.vocab + 4 * BATCH * spec.hidden
    proj_ms, proj_bytes = time_q4(ctx, BATCH, PROJ["K"], PROJ["N"], PROJ_COPIES, 3, 10)
    proj_gbs = proj_bytes / (proj_ms / 1e3) / 1e9

    q4 = spec.q4_bytes()
    kv_read = BATCH * spec.kv_bytes_per_seq(PROMPT + args.warmup + args.steps // 2, dtype=args.kv)
    step_bytes = q4 + spec.lm_head_bytes() + kv_read
    step_ms = r["dev_ms"] / args.steps
    tokens = BATCH * args.steps * ws
    value = tokens / (r["dev_ms"] / 1000.0)
    e2e_val = tokens / (r["e2e_ms"] / 1000.0)
    launches_per_step = decode_launches(spec.n_layers, BATCH, args.kv,
                                        args.temperature > 0.01 or args.penalty > 1.0)
    cfg = main_config(spec, ws)
    cfg["kv_dtype"] = args.kv
    if args.temperature > 0.01 or args.penalty > 1.0:
        cfg["sampling"] = {"temperature": args.temperature, "penalty": args.penalty}
    cfg["positions"] = [PROMPT + args.warmup, PROMPT + args.warmup + args.steps]
    if args.kv_fill == "seeded":
        cfg["kv_fill"] = "seeded values below the prompt length (no prefill)"

    result = {
        "metric": METRIC,
        "value": round(value, 2),
        "unit": "tokens/s",
        "n_gpus": ws,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(step_ms, 4),
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": DTYPE,
        "data": "synthetic (seeded random Q4 weights, N(0,0.02) fp32 lm_head, seeded token ids)",
        "config": cfg,
        "ttft_ms": round(r["ttft_ms"], 3) if r["ttft_ms"] is not None else None,
        "e2e": {"value": round(e2e_val, 2), "unit": "tokens/s",
                "h2d_bytes_per_step": 3 * 4 * BATCH, "d2h_bytes_per_step": 4 * BATCH + 4,
                "wall_s": round(r["wall"], 4)},
        "gpu_launches": launches_per_step * args.steps,
        "roofline": {
            "kernel": (f"{'gemv_stream_kernel' if BATCH <= 8 else ('gemm_sk_kernel' if BATCH <= 64 else 'gemm_tc_kernel')} "
                       f"(Q4 projection, M {BATCH}, gate|up K 2560 x N 20480)"),
            "bound": "hbm", "achieved": round(proj_gbs, 1), "peak": hbm, "unit": "GB/s",
            "frac": round(proj_gbs / hbm, 4),
            "traffic": profile_traffic("gemv_stream_kernel") if BATCH <= 8 else None,
            "traffic_source": "ncu capture summarised in profiles/ (not this run)",
            "algorithmic_bytes": proj_bytes, "peak_source": peak_kind,
            "launch_ms": round(proj_ms, 5),
        },
        "roofline_lm_head": {
            "kernel": ("lm_ring_kernel (fp32 [2560 x 262144] streamed by 2-D tensor copies, "
                       "argmax fused)" if BATCH <= 8 else
                       "lm_tc_kernel (fp32 [2560 x 262144] split into bf16 hi + lo on the "
                       "tensor cores, argmax fused)"),
            "bound": "hbm", "achieved": round(lm_bytes / (lm_ms / 1e3) / 1e9, 1),
            "peak": hbm, "unit": "GB/s",
            "frac": round(lm_bytes / (lm_ms / 1e3) / 1e9 / hbm, 4),
            "traffic": profile_traffic("lm_ring_kernel" if BATCH <= 8 else "lm_tc_kernel"),
            "traffic_source": "ncu capture summarised in profiles/ (not this run)",
            "algorithmic_bytes": lm_bytes, "peak_source": peak_kind,
            "launch_ms": round(lm_ms, 4),
        },
        "step_roofline": {
            "bytes_per_step": step_bytes,
            "achieved_gbs": round(step_bytes / (step_ms / 1e3) / 1e9, 1),
            "peak": hbm, "frac": round(step_bytes / (step_ms / 1e3) / 1e9 / hbm, 4),
            "note": "Q4 weights + fp32 lm_head + KV read per decode step / step time",
        },
        "clocks": r["clk"],
        "first_ids": r["first"][:8],
    }
    kv.close()
    if args.extras == "all" and ws == 1:
        result["long"] = run_long(args, ctx, model, lib_stream, hbm)
    model.close()
    ctx.close()
    torch.cuda.empty_cache()
    if args.extras == "all":
        if ws == 1:
            result["demo"] = run_demo_block(args, local)
            result["q4_sweep"] = run_q4_sweep(local)
        try:  # a failure here (same shapes on every rank) is reported, not fatal to the line
            result["tp"] = run_tp_block(args, ws, rank, local, D)
        except Exception as e:  # noqa: BLE001
            result["tp"] = {"error": f"{type(e).__name__}: {e}"[:300]}
    if rank == 0 and ws == 1 and not args.no_cpu_baseline:
        result["cpu_baseline"] = cpu_baseline(spec, args)
    if rank == 0:
        print(json.dumps(result), flush=True)
    if ws > 1:
        dist.barrier()
        dist.destroy_process_group()


# --------------------------------------------------- long context block --
def run_long(args, ctx, model, lib_stream, hbm, B=64, P=4096, steps=32, warmup=4):
    """Batch 64 at 4096-token prompts on the same E4B model (a fresh cache):
    TTFT of 262144 prompt tokens, then the decode loop (f32 cache, the
    parity mode); then the decode loop again on a bf16 cache (half the KV
    bytes) and on an int8 cache (a quarter), each filled with seeded values
    instead of a second prefill, since decode timing does not depend on them."""
    import torch

    from mojostream_b200.runtime import KVCache
    spec = model.spec
    window = max(l.window for l in spec.layers)
    max_pos = ((P + warmup + 2 * steps + 8 + 63) // 64) * 64
    kv = KVCache(ctx, model, B, max_pos, slide_cap=window + MAX_ROWS, dtype="f32")
    a = argparse.Namespace(steps=steps, warmup=warmup)
    r = decode_loop(model, kv, B, P, a, Dist(1), lib_stream)
    kv_read = B * spec.kv_bytes_per_seq(P + warmup + steps // 2)
    step_bytes = spec.q4_bytes() + spec.lm_head_bytes() + kv_read
    step_ms = r["dev_ms"] / steps
    kv.close()
    torch.cuda.empty_cache()
    slide_cap = window + MAX_ROWS
    legs = {}
    for dt in ("bf16", "i8"):
        kvb = KVCache(ctx, model, B, max_pos, slide_cap=slide_cap, dtype=dt)
        ab = argparse.Namespace(steps=steps, warmup=warmup, kv_fill="seeded")
        rb = decode_loop(model, kvb, B, P, ab, Dist(1), lib_stream, slide_cap=slide_cap)
        kvb.close()
        torch.cuda.empty_cache()
        b = spec.q4_bytes() + spec.lm_head_bytes() + \
            B * spec.kv_bytes_per_seq(P + warmup + steps // 2, dtype=dt)
        ms = rb["dev_ms"] / steps
        legs[dt] = {"value": round(B * steps / (rb["dev_ms"] / 1e3), 2), "unit": "tokens/s",
                    "ms_per_step": round(ms, 4),
                    "step_roofline": {"bytes_per_step": b, "peak": hbm,
                                      "frac": round(b / (ms / 1e3) / 1e9 / hbm, 4)}}
    legs["bf16"]["note"] = "bf16 cache (K / V rounded on write), seeded values below 4096"
    legs["i8"]["note"] = ("int8 cache (one fp32 scale per position and KV head), seeded "
                          "values below 4096")
    return {
        "metric": "decode tokens/s (batch 64, 4096-token prompts), E4B-shaped Q4 model",
        "value": round(B * steps / (r["dev_ms"] / 1e3), 2), "unit": "tokens/s",
        "ms_per_step": round(step_ms, 4), "steps": steps, "warmup": warmup,
        "ttft_ms": round(r["ttft_ms"], 2),
        "e2e": {"value": round(B * steps / (r["e2e_ms"] / 1e3), 2), "unit": "tokens/s",
                "h2d_bytes_per_step": 12 * B, "d2h_bytes_per_step": 4 * B + 4},
        "step_roofline": {"bytes_per_step": step_bytes, "peak": hbm,
                          "frac": round(step_bytes / (step_ms / 1e3) / 1e9 / hbm, 4),
                          "note": "Q4 + fp32 lm_head + fp32 KV read per step"},
        "config": {"batch": B, "prompt": P, "kv_dtype": "f32",
                   "positions": [P + warmup, P + warmup + steps]},
        "first_ids": r["first"][:4],
        "bf16_kv": legs["bf16"],
        "i8_kv": legs["i8"],
    }


# ------------------------------------------------------------ demo stack --
def run_demo_block(args, local, steps=100, dims="baseline"):
    """The reference's bench harness workload (src/bench/harness.mojo:185-328):
    the uniform 40-layer demo stack, batch = 4 consecutive positions of one
    sequence, one pass over the empty cache (TTFT) then 100 steps with fresh
    seeded rows each step (the harness's x.fill_random(); no embedding, no
    lm_head).  Layer calls through ms_forward (host-launched, like the
    harness's per-layer loop).  dims "baseline": 8 x 128 q / 2 x 128 KV / FFN
    4096; "rx": the reference generator's 16 x 64 / 4 x 64 / 2048 (the shape
    its published 22.0 tokens/s P50 was measured on)."""
    import torch

    from mojostream_b200.model import demo_spec, synth_weights_device
    from mojostream_b200.runtime import Context, KVCache, Model
    torch.cuda.set_device(local)
    out = {}
    for d in ("baseline", "rx"):
        spec = demo_spec(d)
        ctx = Context(local)
        w = synth_weights_device(spec, seed=42)
        model = Model(ctx, spec, w, max_rows=4)
        del w
        kv = KVCache(ctx, model, 1, 4 * (steps + 2) + 64)
        g = torch.Generator(device="cuda").manual_seed(1234)
        xs = torch.randn((steps + 1, 4, spec.hidden), device="cuda", generator=g) * 0.1
        x = torch.empty((4, spec.hidden), device="cuda")
        lib_stream = torch.cuda.ExternalStream(ctx.stream_ptr)
        seq = [0, 0, 0, 0]
        # TTFT: the first 40-layer pass at base position 0
        torch.cuda.synchronize()
        e0, e1 = events()
        with torch.cuda.stream(lib_stream):
            e0.record(lib_stream)
            x.copy_(xs[0])
            model.forward(x, kv, seq, [0, 1, 2, 3])
            e1.record(lib_stream)
        e1.synchronize()
        ttft = e0.elapsed_time(e1)
        times = []
        with torch.cuda.stream(lib_stream):
            for s in range(1, steps + 1):
                a, b = events()
                a.record(lib_stream)
                x.copy_(xs[s])
                model.forward(x, kv, seq, [4 * s + i for i in range(4)])
                b.record(lib_stream)
                times.append((a, b))
        torch.cuda.synchronize()
        ms = np.array([a.elapsed_time(b) for a, b in times])
        kv.close()
        model.close()
        ctx.close()
        out[d] = {
            "tokens_per_s_p50": round(4 / (np.percentile(ms, 50) / 1e3), 1),
            "step_ms_p50": round(float(np.percentile(ms, 50)), 4),
            "step_ms_p95": round(float(np.percentile(ms, 95)), 4),
            "step_ms_p99": round(float(np.percentile(ms, 99)), 4),
            "ttft_ms": round(ttft, 4),
            "q4_bytes_per_step": spec.q4_bytes(),
            "layers": spec.n_layers,
            "dims": {"q_heads": spec.layers[0].n_heads, "kv_heads": spec.layers[0].n_kv_heads,
                     "head_dim": spec.layers[0].head_dim, "ffn": spec.layers[0].ffn_dim},
        }
    out["metric"] = "demo stack step latency (batch 4 = 4 positions of one sequence), 100 steps"
    out["reference_published"] = {"tokens_per_s_p50": 22.0, "step_ms_p50": 181.59,
                                  "step_ms_p95": 212.63, "dims": "rx",
                                  "hardware": "i7-7500U, 4 threads (the reference's README)"}
    return out


# ------------------------------------------------------------ Q4 sweep --
SWEEP = [(1024, 1024), (4096, 4096), (10240, 2560), (2560, 10240)]  # (N, K)


def run_q4_sweep(local, ms=(1, 4, 16, 64, 512)):
    """The isolated Q4 projection over M x (N, K) (ms_q4_gemm, CUDA events,
    weights cycled over >= 256 MB of copies so each launch streams them from
    HBM): GB/s against the copy peak up to M = 64, TFLOP/s against the bf16
    peak at M = 512."""
    import torch

    from mojostream_b200.runtime import Context
    torch.cuda.set_device(local)
    hbm, tf, kind = measured_peaks()
    ctx = Context(local)
    rows = []
    for (N, K) in SWEEP:
        copies = max(2, min(512, (256 << 20) // (K * N // 2) + 1))
        wts = q4_copies(ctx, K, N, copies)
        for M in ms:
            t, nbytes = time_q4_on(wts, M, K, N, 2, 5 if M < 512 else 2)
            row = {"M": M, "N": N, "K": K, "us": round(t * 1e3, 2)}
            if M <= 64:
                gbs = nbytes / (t / 1e3) / 1e9
                row.update({"gbs": round(gbs, 1), "frac_hbm": round(gbs / hbm, 4)})
            else:
                tfl = 2.0 * M * N * K / (t / 1e3) / 1e12
                row.update({"tflops": round(tfl, 1), "frac_tensor": round(tfl / tf, 4)})
            rows.append(row)
        for q in wts:
            q.close()
    ctx.close()
    return {"peak_gbs": hbm, "peak_tflops": tf, "peak_source": kind,
            "bytes": "N*K/2 + 4*M*(K+N) per launch", "points": rows}


# ---------------------------------------------------------- tp block --
def run_tp_block(args, ws, rank, local, D, B=64, P=1024, steps=24, warmup=4):
    """The 14B-class model (D 5120, 48 layers, 40 q / 8 KV heads, FFN 13824,
    V 262144) tensor parallel over the ws ranks: batch 64, 1024-token prompts,
    greedy decode.  value = decode tokens/s of the whole job (every rank
    serves the same tokens: strong scaling)."""
    import torch

    from mojostream_b200.model import b14_spec, synth_weights_device
    from mojostream_b200.runtime import Context, KVCache, Model
    from mojostream_b200.tp import tp_setup
    torch.cuda.set_device(local)
    spec = b14_spec()
    ctx = Context(local)
    if ws > 1:
        tp_setup(ctx)
    w = synth_weights_device(spec, seed=1414)
    model = Model(ctx, spec, w, max_rows=MAX_ROWS)
    del w
    torch.cuda.empty_cache()
    window = max(l.window for l in spec.layers)
    max_pos = ((P + warmup + 2 * steps + 8 + 63) // 64) * 64
    kv = KVCache(ctx, model, B, max_pos, slide_cap=window + P, dtype="f32")
    lib_stream = torch.cuda.ExternalStream(ctx.stream_ptr)
    a = argparse.Namespace(steps=steps, warmup=warmup)
    r = decode_loop(model, kv, B, P, a, D, lib_stream)
    ar_ms = allreduce_ms(ws, B, spec.hidden, 2 * spec.n_layers, D) if ws > 1 else 0.0
    hbm, _, kind = measured_peaks()
    kv_read = B * spec.kv_bytes_per_seq(P + warmup + steps // 2)
    step_bytes = (spec.q4_bytes() + spec.lm_head_bytes() + kv_read) / ws
    step_ms = r["dev_ms"] / steps
    kv.close()
    model.close()
    ctx.close()
    torch.cuda.empty_cache()
    return {
        "metric": f"decode tokens/s (batch {B}), 14B-class Q4 model, tensor parallel",
        "value": round(B * steps / (r["dev_ms"] / 1e3), 2), "unit": "tokens/s",
        "n_gpus": ws, "scaling": "strong", "ms_per_step": round(step_ms, 4),
        "steps": steps, "warmup": warmup, "ttft_ms": round(r["ttft_ms"], 2),
        "e2e": {"value": round(B * steps / (r["e2e_ms"] / 1e3), 2), "unit": "tokens/s",
                "h2d_bytes_per_step": 12 * B, "d2h_bytes_per_step": 4 * B + 4},
        "step_roofline": {"bytes_per_step_per_gpu": int(step_bytes), "peak": hbm,
                          "peak_source": kind,
                          "frac": round(step_bytes / (step_ms / 1e3) / 1e9 / hbm, 4)},
        "allreduce_est": {"ms_per_step": round(ar_ms, 4),
                          "share": round(ar_ms / step_ms, 4) if step_ms else None,
                          "note": "2 x layers standalone NCCL all-reduces of [64, 5120] fp32 "
                                  "on the same ranks (the decode path sums O / down over "
                                  "peer memory inside the projection epilogue instead)"},
        "config": {"workload": "14b-class tensor-parallel decode", "layers": spec.n_layers,
                   "hidden": spec.hidden, "vocab": spec.vocab, "batch": B, "prompt": P,
                   "parallelism": f"tp{ws}", "kv_dtype": "f32"},
        "first_ids": r["first"][:4],
    }


def allreduce_ms(ws, B, Dm, n, D):
    """Device time of n back-to-back NCCL all-reduces of [B, Dm] fp32 (max
    over ranks), the collective volume of one tensor-parallel decode step."""
    import torch
    import torch.distributed as dist
    t = torch.randn((B, Dm), device="cuda")
    for _ in range(3):
        dist.all_reduce(t)
    D.barrier()
    e0, e1 = events()
    e0.record()
    for _ in range(n):
        dist.all_reduce(t)
    e1.record()
    e1.synchronize()
    return D.max(e0.elapsed_time(e1))


# ---------------------------------------------------------- CPU baseline --
def oracle_model(spec, positions, threads, seed=5):
    """The oracle (C restatement of the reference's CPU path) on the seeded
    benchmark weights, with its KV caches filled with seeded values below
    `positions` (a CPU prefill of 4 x 512 tokens would take minutes; decode
    timing does not depend on the cached values)."""
    from mojostream_b200.model import synth_weights
    from oracle import oracle
    wn = synth_weights(spec, seed=1234)
    om = oracle.OracleModel(spec, wn, BATCH, positions + 1024, slide_cap=1024, workers=threads)
    rng = np.random.default_rng(seed)
    for li in range(spec.n_layers):
        k, v = om.kv_arrays(li)
        n = min(positions, k.shape[1])
        k[:, :n] = rng.standard_normal((BATCH, n, k.shape[2]), dtype=np.float32)
        v[:, :n] = rng.standard_normal((BATCH, n, k.shape[2]), dtype=np.float32)
    return om


def oracle_steps(om, n_steps, start_pos, budget_s=None):
    """n_steps full greedy decode steps (embed, every layer, final norm,
    lm_head, argmax) of BATCH sequences; returns (steps done, seconds)."""
    rng = np.random.default_rng(1)
    ids = rng.integers(0, om.spec.vocab, size=BATCH).tolist()
    t0 = time.perf_counter()
    done = 0
    for i in range(n_steps):
        x = om.embed(ids)
        x = om.forward(x, list(range(BATCH)), [start_pos + i] * BATCH)
        ids = om.argmax(om.lm_head(x))
        done += 1
        if budget_s and time.perf_counter() - t0 > budget_s:
            break
    return done, time.perf_counter() - t0


THREAD_NOTE = ("the reference parallelises its Q4 and fp32 matmuls over 64-row blocks "
               "(kernels.mojo:266-267, 670-671), so at batch 4 one thread has work whatever "
               "the thread count offered")


def cpu_baseline(spec, args, budget_s=20.0):
    threads = os.cpu_count() or 1
    om = oracle_model(spec, PROMPT, threads)
    oracle_steps(om, 1, PROMPT)
    done, dt = oracle_steps(om, 1000, PROMPT + 1, budget_s=budget_s)
    step_s = dt / done
    return {"value": round(BATCH / step_s, 4), "unit": "tokens/s", "cores": 1,
            "threads_offered": threads, "kind": "port",
            "sample": f"{done} full decode steps (all {spec.n_layers} layers and the whole "
                      f"lm_head, batch {BATCH}) at positions {PROMPT + 1}+, KV pre-filled with "
                      f"seeded values, {dt:.1f} s; " + THREAD_NOTE}


def run_reference(args, ws, rank, local):
    """The reference's CPU path (C restatement) on the host cores, rank 0 only:
    full decode steps of the same model and batch as our arm."""
    if rank != 0:
        return
    from mojostream_b200.model import e4b_spec
    spec = e4b_spec(n_layers=args.layers)
    threads = os.cpu_count() or 1
    om = oracle_model(spec, PROMPT, threads)
    oracle_steps(om, args.warmup, PROMPT)
    done, dt = oracle_steps(om, args.steps, PROMPT + args.warmup)
    step_s = dt / done
    v = BATCH / step_s
    print(json.dumps({
        "impl": "reference",
        "metric": METRIC,
        "value": round(v, 4), "unit": "tokens/s", "n_gpus": ws, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(1e3 * step_s, 2),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "fp32 activations x int4 weights dequantised to fp32 (the reference's CPU path)",
        "data": "synthetic (seeded random Q4 weights, N(0,0.02) fp32 lm_head, seeded token ids)",
        "config": main_config(spec, 1),
        "cpu_baseline": {"value": round(v, 4), "unit": "tokens/s", "cores": 1,
                         "threads_offered": threads, "kind": "port",
                         "sample": f"{done} full decode steps after {args.warmup} warm-up steps "
                                   f"(KV pre-filled with seeded values below position {PROMPT}); "
                                   + THREAD_NOTE},
        "e2e": {"value": round(v, 4), "unit": "tokens/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }), flush=True)


# ------------------------------------------------------------ Q4 timing --
def q4_copies(ctx, K, N, copies):
    """`copies` distinct seeded Q4 weights [K][N/2] on the device."""
    import torch
    from mojostream_b200.runtime import Q4Weight
    g = torch.Generator(device="cuda").manual_seed(3)
    ws = []
    for _ in range(copies):
        w = torch.randint(0, 256, (K, N // 2), dtype=torch.uint8, device="cuda", generator=g)
        ws.append(Q4Weight(ctx, w, K, N, 0.01))
        del w
    return ws


def time_q4(ctx, M, K, N, copies, warmup, reps):
    """Average time of one ms_q4_gemm launch (CUDA events on the launching
    stream) cycling over `copies` distinct weights, so that the weights
    streamed between two uses of the same one exceed L2.  Returns (ms, bytes
    per launch: packed weights + fp32 input and output rows)."""
    ws = q4_copies(ctx, K, N, copies)
    out = time_q4_on(ws, M, K, N, warmup, reps)
    for q in ws:
        q.close()
    return out


def time_q4_on(ws, M, K, N, warmup, reps):
    import torch
    g = torch.Generator(device="cuda").manual_seed(4)
    x = torch.randn((M, K), device="cuda", generator=g)
    y = torch.empty((M, N), device="cuda")
    for _ in range(warmup):
        for q in ws:
            q.gemm(x, y)  # launched on torch's current stream
    torch.cuda.synchronize()
    e0, e1 = events()
    e0.record()
    for _ in range(reps):
        for q in ws:
            q.gemm(x, y)
    e1.record()
    e1.synchronize()
    ms = e0.elapsed_time(e1) / (reps * len(ws))
    return ms, K * N // 2 + 4 * M * (K + N)


# The projection shape the bench's roofline line is quoted on: the fused
# gate|up matrix of an E4B layer (the largest of a decode step).
PROJ = dict(M=BATCH, K=2560, N=2 * 10240)
PROJ_COPIES = 8   # 8 x 26 MB > L2


def run_q4_case(args):
    """The isolated Q4 projection: one shape (--m/--k/--n, e.g. for ncu
    captures) or, without --m, the 20-shape sweep."""
    import torch
    from mojostream_b200.runtime import Context
    torch.cuda.set_device(0)
    if args.m is None:
        print(json.dumps({"case": "q4_sweep", **run_q4_sweep(0)}), flush=True)
        return
    ctx = Context(0)
    ms, nbytes = time_q4(ctx, args.m, args.k, args.n, args.copies, args.warmup, args.steps)
    hbm, _, kind = measured_peaks()
    print(json.dumps({"case": "q4", "M": args.m, "K": args.k, "N": args.n, "copies": args.copies,
                      "ms": round(ms, 5), "gbs": round(nbytes / ms / 1e6, 1), "peak": hbm,
                      "peak_source": kind, "frac": round(nbytes / ms / 1e6 / hbm, 4)}), flush=True)


def run_load(args):
    """The model-file path (.mojostream + lm_head_proto.bin -> HBM): the E4B
    files written to a temporary directory (so they sit in the page cache),
    then ms_model_load timed; beside it the reference's way of reading a
    .mojostream file, one whole-file read into host memory
    (src/streaming/mojostream.mojo:112-116), timed on the same files."""
    import shutil
    import tempfile

    import torch
    from mojostream_b200 import fileformat as ff
    from mojostream_b200.model import e4b_spec, synth_weights
    from mojostream_b200.runtime import Context, Model
    torch.cuda.set_device(0)
    spec = e4b_spec(n_layers=args.layers)
    tmp = tempfile.mkdtemp(prefix="ms_load_")
    try:
        path, lmp = os.path.join(tmp, "e4b.mojostream"), os.path.join(tmp, "lm_head_proto.bin")
        w = synth_weights(spec, seed=1234)
        ff.write_mojostream(path, spec, w)
        ff.write_lm_head(lmp, w.lm_head, w.final_gamma)
        del w
        file_bytes = os.path.getsize(path) + os.path.getsize(lmp)
        t0 = time.perf_counter()
        for p in (path, lmp):
            with open(p, "rb") as f:
                blob = f.read()
            del blob
        ref_s = time.perf_counter() - t0
        ctx = Context(0)
        runs = []
        for _ in range(max(1, min(args.steps, 5))):
            torch.cuda.synchronize()
            t0 = time.perf_counter()
            m = Model.load(ctx, path, lmp, max_rows=64)
            torch.cuda.synchronize()
            runs.append((time.perf_counter() - t0, m.load_seconds, m.load_bytes))
            m.close()
        wall, stream_s, nbytes = min(runs)
        print(json.dumps({
            "case": "load", "metric": "model file -> HBM GB/s (E4B .mojostream + fp32 lm_head)",
            "value": round(nbytes / stream_s / 1e9, 2), "unit": "GB/s",
            "bytes": nbytes, "stream_s": round(stream_s, 4),
            "e2e": {"value": round(nbytes / wall / 1e9, 2), "unit": "GB/s",
                    "wall_s": round(wall, 4), "note": "Model.load incl. repack"},
            "runs": len(runs), "files": "page cache (written just before)",
            "cpu_baseline": {"value": round(file_bytes / ref_s / 1e9, 2), "unit": "GB/s",
                             "kind": "reference-style whole-file read into host RAM",
                             "cores": 1, "seconds": round(ref_s, 4)},
        }), flush=True)
        ctx.close()
    finally:
        shutil.rmtree(tmp, ignore_errors=True)


def run_tp_case(args, ws, rank, local):
    """The 14B-class tensor-parallel block on its own (--case tp)."""
    import datetime

    import torch
    import torch.distributed as dist
    torch.cuda.set_device(local)
    if ws > 1:
        dist.init_process_group("nccl", device_id=torch.device("cuda", local),
                                timeout=datetime.timedelta(seconds=600))
    D = Dist(ws)
    out = run_tp_block(args, ws, rank, local, D, B=args.batch or 64, P=args.prompt or 1024,
                       steps=args.steps, warmup=args.warmup)
    if rank == 0:
        print(json.dumps(out), flush=True)
    if ws > 1:
        dist.barrier()
        dist.destroy_process_group()


def main():
    global BATCH, PROMPT, METRIC, WORKLOAD
    args = parse()
    ws, rank, local = dist_setup(args)
    if args.case == "decode":
        BATCH = args.batch or BATCH
        PROMPT = args.prompt or PROMPT
        if (BATCH, PROMPT) != (4, 512):
            METRIC = f"decode tokens/s (batch {BATCH}), Gemma-4-E4B-shaped Q4 model"
            WORKLOAD = (f"gemma4-e4b decode, batch {BATCH} independent sequences, "
                        f"{PROMPT}-token prompts")
    if args.case == "q4":
        run_q4_case(args)
    elif args.case == "load":
        run_load(args)
    elif args.case == "demo":
        print(json.dumps({"case": "demo", **run_demo_block(args, local)}), flush=True)
    elif args.case == "tp" and args.impl != "reference":
        run_tp_case(args, ws, rank, local)
    elif args.impl == "reference":
        run_reference(args, ws, rank, local)
    else:
        run_ours(args, ws, rank, local)


if __name__ == "__main__":
    main()
