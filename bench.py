#!/usr/bin/env python3
"""Benchmark of the Gemma-4 token loop on B200 (one JSON line on rank 0).

Workload (default): Gemma-4-E4B-shaped random Q4 model
(D 2560, 42 layers = 35 sliding (hd 256, window 512) + 7 full (hd 512, 128
rotary dims, theta 1e6), 8 q / 2 KV heads, FFN 10240, fp32 lm_head over a
262144 vocab), 4 independent sequences, 512-token seeded prompts (TTFT), then
greedy decode at batch 4.  A step = one decode step of the 4 sequences
(4 tokens).  Weights (4.66 GB) and KV are far larger than L2 (126 MB), so no L2
flush is needed between steps.

value : decode tokens/s, device-resident loop (CUDA-graph replays on the
        library stream, CUDA events), max over ranks
e2e   : the same through ms_decode_step with host buffers (per step: ids / seq /
        pos host->device from pinned memory, next ids device->host)
--gpus N: N independent replicas (one process per GPU, no collective on the
        data path: the sequences are independent), weak scaling.
--impl reference: the reference's CPU algorithm (the C port in oracle/, since
        the Mojo reference cannot be built here) on the host cores.
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


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=256)
    ap.add_argument("--warmup", type=int, default=8)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--layers", type=int, default=42, help="(debug) fewer layers")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--case", default="decode", choices=["decode", "q4", "tp", "load"],
                    help="q4: the isolated Q4 projection (BASELINE configs[1] shapes), "
                         "a small case for profiling; tp: the 14B-class model (configs[4]) "
                         "tensor-parallel over the torchrun ranks")
    ap.add_argument("--batch", type=int, default=None,
                    help="sequences (decode: 4 = configs[2], 64 = configs[3]; tp: 64)")
    ap.add_argument("--prompt", type=int, default=None,
                    help="prompt tokens per sequence (decode: 512, configs[3]: 4096; tp: 1024)")
    ap.add_argument("--temperature", type=float, default=0.0,
                    help="token-loop sampling (default greedy, the north-star mode; the "
                         "reference's e4b loop uses 0.7)")
    ap.add_argument("--penalty", type=float, default=1.0,
                    help="repetition penalty (the reference's e4b loop uses 1.2)")
    ap.add_argument("--kv", default="f32", choices=["f32", "bf16"],
                    help="KV cache element type (f32: the parity mode; bf16: configs[3]'s "
                         "reduced-precision cache)")
    ap.add_argument("--m", type=int, default=4)
    ap.add_argument("--k", type=int, default=2560)
    ap.add_argument("--n", type=int, default=20480)
    ap.add_argument("--copies", type=int, default=8)
    return ap.parse_args()


def dist_setup(args):
    ws = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return ws, rank, local


# ------------------------------------------------------------------ clocks --
class ClockSampler:
    """nvidia-smi samples (200 ms) of SM clock and throttle reasons."""
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


def prompts(seed=7):
    rng = np.random.default_rng(seed)
    return rng.integers(0, 262144, size=(BATCH, PROMPT)).tolist()


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
    kv = KVCache(ctx, model, BATCH, max_pos, slide_cap=window + min(PROMPT, MAX_ROWS),
                 dtype=args.kv)
    lib_stream = torch.cuda.ExternalStream(ctx.stream_ptr)

    def barrier():
        torch.cuda.synchronize()
        if ws > 1:
            dist.barrier()

    def max_over_ranks(v):
        if ws == 1:
            return v
        t = torch.tensor([v], dtype=torch.float64, device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    # ---- TTFT: 4 x 512-token prefill + first token -------------------------
    P = prompts()
    ids = sum(P, [])
    seq = sum([[s] * PROMPT for s in range(BATCH)], [])
    pos = sum([list(range(PROMPT)) for _ in range(BATCH)], [])
    model.prefill(kv, ids, seq, pos)  # warm (kernel attributes, allocations)
    kv.reset()
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(lib_stream)
    first = model.prefill(kv, ids, seq, pos)
    e1.record(lib_stream)
    e1.synchronize()
    ttft_ms = max_over_ranks(e0.elapsed_time(e1))

    # ---- decode: warm-up then the timed device-resident loop ---------------
    seqs = list(range(BATCH))
    p0 = [PROMPT] * BATCH
    gen = model.generate(kv, first, seqs, p0, args.warmup)
    cur = [int(t) for t in gen[-1]]
    p1 = [PROMPT + args.warmup] * BATCH
    barrier()
    clocks = ClockSampler(local)
    clocks.start()
    gen2, dev_ms = model.generate(kv, cur, seqs, p1, args.steps, timing=True)
    barrier()
    dev_ms = max_over_ranks(dev_ms)
    # ---- e2e through host buffers, one ms_decode_step per step -------------
    cur = [int(t) for t in gen2[-1]]
    p2 = [PROMPT + args.warmup + args.steps] * BATCH
    barrier()
    e0.record(lib_stream)
    t0 = time.perf_counter()
    for i in range(args.steps):
        cur = model.decode_step(kv, cur, seqs, [p + i for p in p2])
    e1.record(lib_stream)
    e1.synchronize()
    wall_e2e = time.perf_counter() - t0
    e2e_ms = max_over_ranks(e0.elapsed_time(e1))
    barrier()
    clk = clocks.stop()

    # ---- dominant kernels timed alone (CUDA events on their stream) --------
    hbm, tf, peak_kind = measured_peaks()
    x = torch.randn((BATCH, spec.hidden), device="cuda")
    for _ in range(3):
        model.lm_head(x, logits=False)
    torch.cuda.synchronize()
    n_rep = 10
    s0, s1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
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
    kv_read = BATCH * spec.kv_bytes_per_seq(PROMPT + args.warmup + args.steps // 2)
    if args.kv == "bf16":
        kv_read //= 2
    step_bytes = q4 + spec.lm_head_bytes() + kv_read
    step_ms = dev_ms / args.steps
    tokens = BATCH * args.steps * ws
    value = tokens / (dev_ms / 1000.0)
    e2e_val = tokens / (e2e_ms / 1000.0)
    launches_per_step = 1 + 5 * spec.n_layers + (BATCH + 3) // 4 + 1
    if args.temperature > 0.01 or args.penalty > 1.0:
        launches_per_step += 1  # the sampler after the lm_head

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
        "dtype": "int4 weights x fp32 activations (exact int8-limb tensor-core products), fp32 lm_head",
        "data": "synthetic (seeded random Q4 weights, N(0,0.02) fp32 lm_head, seeded token ids)",
        "config": {
            "workload": WORKLOAD,
            "layers": spec.n_layers, "hidden": spec.hidden, "vocab": spec.vocab,
            "batch": BATCH, "prompt": PROMPT, "positions": [PROMPT + args.warmup,
                                                            PROMPT + args.warmup + args.steps],
            "parallelism": f"replicas x{ws}" if ws > 1 else "single GPU",
            "l2": "weights + lm_head 4.66 GB >> 126 MB L2 (no flush needed)",
            "kv_dtype": args.kv,
            "sampling": ({"temperature": args.temperature, "penalty": args.penalty}
                         if args.temperature > 0.01 or args.penalty > 1.0 else "greedy"),
        },
        "ttft_ms": round(ttft_ms, 3),
        "e2e": {"value": round(e2e_val, 2), "unit": "tokens/s",
                "h2d_bytes_per_step": 3 * 4 * BATCH, "d2h_bytes_per_step": 4 * BATCH,
                "wall_s": round(wall_e2e, 4)},
        "gpu_launches": launches_per_step * args.steps,
        "roofline": {
            "kernel": (f"{'gemv_stream_kernel' if BATCH <= 8 else 'gemm_tc_kernel'} "
                       f"(Q4 projection, M {BATCH}, gate|up K 2560 x N 20480)"),
            "bound": "hbm", "achieved": round(proj_gbs, 1), "peak": hbm, "unit": "GB/s",
            "frac": round(proj_gbs / hbm, 4),
            "traffic": profile_traffic("gemv_stream_kernel") if BATCH <= 8 else None,
            "algorithmic_bytes": proj_bytes, "peak_source": peak_kind,
            "launch_ms": round(proj_ms, 5),
        },
        "roofline_lm_head": {
            "kernel": "lm_head_kernel (fp32 [2560 x 262144], argmax fused)",
            "bound": "hbm", "achieved": round(lm_bytes / (lm_ms / 1e3) / 1e9, 1),
            "peak": hbm, "unit": "GB/s",
            "frac": round(lm_bytes / (lm_ms / 1e3) / 1e9 / hbm, 4),
            "traffic": profile_traffic("lm_head_kernel"),
            "algorithmic_bytes": lm_bytes, "peak_source": peak_kind,
            "launch_ms": round(lm_ms, 4),
        },
        "step_roofline": {
            "bytes_per_step": step_bytes, "achieved_gbs": round(step_bytes / (step_ms / 1e3) / 1e9, 1),
            "peak": hbm, "frac": round(step_bytes / (step_ms / 1e3) / 1e9 / hbm, 4),
            "note": "Q4 weights + fp32 lm_head + KV read per decode step / step time",
        },
        "clocks": clk,
        "first_ids": first[:8],
    }
    if rank == 0 and not args.no_cpu_baseline:
        result["cpu_baseline"] = cpu_baseline(spec)
    if rank == 0:
        print(json.dumps(result), flush=True)
    if ws > 1:
        dist.barrier()
        dist.destroy_process_group()


# ---------------------------------------------------------- CPU baseline --
# The reference's CPU path is timed on a proportional sample of a decode step:
# 6 of the 42 layers (5 sliding + 1 full, the model's own 5:1 pattern) and
# 1/7 of the lm_head columns, i.e. 1/7 of every kind of work in a step; the
# step time is 7 x the sample time.  A full E4B step is ~3 s on one core, so
# the sample keeps the reference arm's K + W steps within a couple of minutes.
SAMPLE_FRAC = 7


def sample_spec(spec):
    from mojostream_b200.model import e4b_spec
    return e4b_spec(n_layers=spec.n_layers // SAMPLE_FRAC, vocab=spec.vocab // SAMPLE_FRAC)


def oracle_sample(spec, positions, seed=5):
    """Oracle model of the sample spec (seeded weights) with KV caches filled
    with seeded values below `positions` (the sample times decode steps, not
    the prefill)."""
    from mojostream_b200.model import synth_weights
    from oracle import oracle
    wn = synth_weights(spec, seed=1234)
    om = oracle.OracleModel(spec, wn, BATCH, positions + 1024, slide_cap=1024)
    rng = np.random.default_rng(seed)
    for li in range(spec.n_layers):
        k, v = om.kv_arrays(li)
        n = min(positions, k.shape[1])
        k[:, :n] = rng.standard_normal((BATCH, n, k.shape[2]), dtype=np.float32)
        v[:, :n] = rng.standard_normal((BATCH, n, k.shape[2]), dtype=np.float32)
    return om


def time_oracle_steps(om, n_steps, start_pos, budget_s=None):
    """Times n_steps sampled decode steps; returns (steps done, seconds)."""
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


SAMPLE_NOTE = ("each step: 6 of 42 layers (5 sliding + 1 full) and 1/7 of the lm_head "
               "columns at batch 4, step time = 7 x sample time; the reference's Q4 "
               "matmul threads over 64-row blocks, so batch 4 runs on 1 thread")


def cpu_baseline(spec, budget_s=20.0):
    sspec = sample_spec(spec)
    om = oracle_sample(sspec, PROMPT)
    time_oracle_steps(om, 1, PROMPT)
    done, dt = time_oracle_steps(om, 1000, PROMPT + 1, budget_s=budget_s)
    step_s = SAMPLE_FRAC * dt / done
    return {"value": round(BATCH / step_s, 4), "unit": "tokens/s", "cores": 1,
            "kind": "port",
            "sample": f"{done} sampled decode steps at positions {PROMPT + 1}+ (KV pre-filled "
                      f"with seeded values), {dt:.1f} s; " + SAMPLE_NOTE}


def run_reference(args, ws, rank, local):
    """The reference's CPU path (C restatement) on the host cores, rank 0 only."""
    if rank != 0:
        return
    from mojostream_b200.model import e4b_spec
    spec = e4b_spec(n_layers=args.layers)
    sspec = sample_spec(spec)
    om = oracle_sample(sspec, PROMPT)
    time_oracle_steps(om, args.warmup, PROMPT)
    done, dt = time_oracle_steps(om, args.steps, PROMPT + args.warmup)
    step_s = SAMPLE_FRAC * dt / done
    v = BATCH / step_s
    print(json.dumps({
        "impl": "reference",
        "metric": METRIC,
        "value": round(v, 4), "unit": "tokens/s", "n_gpus": ws, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(1e3 * step_s, 2),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "fp32", "data": "synthetic (seeded)",
        "config": {"workload": WORKLOAD, "layers": spec.n_layers, "batch": BATCH},
        "cpu_baseline": {"value": round(v, 4), "unit": "tokens/s", "cores": 1, "kind": "port",
                         "sample": f"{done} sampled decode steps; " + SAMPLE_NOTE},
        "e2e": {"value": round(v, 4), "unit": "tokens/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }), flush=True)


def time_q4(ctx, M, K, N, copies, warmup, reps):
    """Average time of one ms_q4_gemm launch (CUDA events on the launching
    stream) cycling over `copies` distinct weights, so that the weights
    streamed between two uses of the same one exceed L2.  Returns (ms, bytes
    per launch: packed weights + fp32 input and output rows)."""
    import torch
    from mojostream_b200.runtime import Q4Weight
    g = torch.Generator(device="cuda").manual_seed(3)
    ws = []
    for _ in range(copies):
        w = torch.randint(0, 256, (K, N // 2), dtype=torch.uint8, device="cuda", generator=g)
        ws.append(Q4Weight(ctx, w, K, N, 0.01))
        del w
    x = torch.randn((M, K), device="cuda", generator=g)
    y = torch.empty((M, N), device="cuda")
    for _ in range(warmup):
        for q in ws:
            q.gemm(x, y)  # launched on torch's current stream
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(reps):
        for q in ws:
            q.gemm(x, y)
    e1.record()
    e1.synchronize()
    ms = e0.elapsed_time(e1) / (reps * copies)
    for q in ws:
        q.close()
    return ms, K * N // 2 + 4 * M * (K + N)


# The projection shape the bench's roofline line is quoted on: the fused
# gate|up matrix of an E4B layer (the largest of a decode step).
PROJ = dict(M=BATCH, K=2560, N=2 * 10240)
PROJ_COPIES = 8   # 8 x 26 MB > L2


def run_q4_case(args):
    """The isolated Q4 projection (a small case, e.g. for ncu captures)."""
    import torch
    from mojostream_b200.runtime import Context
    torch.cuda.set_device(0)
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
        for _ in range(max(1, args.steps)):
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


def run_tp(args, ws, rank, local):
    """14B-class random Q4 model, heads / FFN columns /
    vocabulary sharded over the ranks (one all-reduce after O and after down
    per layer, NCCL inside the library), batch-B prefill of P-token prompts
    then greedy decode.  value = decode tokens/s of the whole job (every rank
    serves the same tokens: strong scaling)."""
    import datetime

    import torch
    import torch.distributed as dist

    from mojostream_b200.model import b14_spec, synth_weights_device
    from mojostream_b200.runtime import Context, KVCache, Model
    from mojostream_b200.tp import tp_setup

    torch.cuda.set_device(local)
    if ws > 1:
        dist.init_process_group("nccl", device_id=torch.device("cuda", local),
                                timeout=datetime.timedelta(seconds=600))
    B, P = args.batch, args.prompt
    spec = b14_spec(n_layers=args.layers if args.layers != 42 else 48)
    ctx = Context(local)
    if ws > 1:
        tp_setup(ctx)
    w = synth_weights_device(spec, seed=1414)
    model = Model(ctx, spec, w, max_rows=2048)
    del w
    torch.cuda.empty_cache()
    window = max(l.window for l in spec.layers)
    max_pos = ((P + args.warmup + 2 * args.steps + 8 + 63) // 64) * 64
    kv = KVCache(ctx, model, B, max_pos, slide_cap=window + P, dtype=args.kv)
    lib_stream = torch.cuda.ExternalStream(ctx.stream_ptr)

    def barrier():
        if ws > 1:
            dist.barrier()
        torch.cuda.synchronize()

    def max_over_ranks(v):
        if ws == 1:
            return v
        t = torch.tensor([v], dtype=torch.float64, device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    rng = np.random.default_rng(77)
    prompts_ = [[int(t) for t in rng.integers(0, spec.vocab, P)] for _ in range(B)]
    ids = sum(prompts_, [])
    seq = sum([[s_] * P for s_ in range(B)], [])
    pos = sum([list(range(P)) for _ in range(B)], [])
    # warm prefill (kernel attributes, NCCL connections), then the timed one
    model.prefill(kv, ids[:P], seq[:P], pos[:P])
    kv.reset()
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(lib_stream)
    first = model.prefill(kv, ids, seq, pos)
    e1.record(lib_stream)
    e1.synchronize()
    ttft_ms = max_over_ranks(e0.elapsed_time(e1))

    seqs = list(range(B))
    gen = model.generate(kv, first, seqs, [P] * B, args.warmup)
    cur = [int(t) for t in gen[-1]]
    barrier()
    clocks = ClockSampler(local)
    clocks.start()
    gen2, dev_ms = model.generate(kv, cur, seqs, [P + args.warmup] * B, args.steps, timing=True)
    barrier()
    dev_ms = max_over_ranks(dev_ms)
    cur = [int(t) for t in gen2[-1]]
    p2 = P + args.warmup + args.steps
    barrier()
    e0.record(lib_stream)
    for i in range(args.steps):
        cur = model.decode_step(kv, cur, seqs, [p2 + i] * B)
    e1.record(lib_stream)
    e1.synchronize()
    e2e_ms = max_over_ranks(e0.elapsed_time(e1))
    barrier()
    clk = clocks.stop()
    hbm, _, peak_kind = measured_peaks()
    tokens = B * args.steps
    step_ms = dev_ms / args.steps
    kv_read = B * spec.kv_bytes_per_seq(P + args.warmup + args.steps // 2)
    if args.kv == "bf16":
        kv_read //= 2
    step_bytes = (spec.q4_bytes() + spec.lm_head_bytes() + kv_read) / ws  # per GPU
    result = {
        "metric": "decode tokens/s (batch %d), 14B-class Q4 model, tensor parallel" % B,
        "value": round(tokens / (dev_ms / 1e3), 2), "unit": "tokens/s", "n_gpus": ws,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(step_ms, 4),
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
        "dtype": "int4 weights x fp32 activations (exact int8-limb tensor-core products), fp32 lm_head",
        "data": "synthetic (seeded random Q4 weights and token ids)",
        "config": {"workload": "14b-class tensor-parallel decode (BASELINE configs[4])",
                   "layers": spec.n_layers, "hidden": spec.hidden, "vocab": spec.vocab,
                   "batch": B, "prompt": P, "parallelism": f"tp{ws}", "kv_dtype": args.kv,
                   "l2": "weights + KV >> 126 MB L2 (no flush needed)"},
        "ttft_ms": round(ttft_ms, 3),
        "e2e": {"value": round(tokens / (e2e_ms / 1e3), 2), "unit": "tokens/s",
                "h2d_bytes_per_step": 12 * B, "d2h_bytes_per_step": 4 * B},
        "step_roofline": {"bytes_per_step_per_gpu": int(step_bytes),
                          "achieved_gbs": round(step_bytes / (step_ms / 1e3) / 1e9, 1),
                          "peak": hbm, "peak_source": peak_kind,
                          "frac": round(step_bytes / (step_ms / 1e3) / 1e9 / hbm, 4)},
        "clocks": clk,
        "first_ids": first[:4],
    }
    if rank == 0:
        print(json.dumps(result), flush=True)
    kv.close()
    model.close()
    ctx.close()
    if ws > 1:
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
    elif args.case == "tp" and args.impl != "reference":
        args.batch = args.batch or 64
        args.prompt = args.prompt or 1024
        run_tp(args, ws, rank, local)
    elif args.impl == "reference":
        run_reference(args, ws, rank, local)
    else:
        run_ours(args, ws, rank, local)


if __name__ == "__main__":
    main()
