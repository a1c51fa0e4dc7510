"""Parity of the CUDA library (through its C-ABI) with the CPU oracle.

Tolerances: per-layer relative RMSE <= 1e-4 (the reference's own validation
threshold, src/tests/validate_layer.mojo:31), final logits <= 1e-3, greedy ids
identical; the Q4 dequant is bit-exact.  Each teacher-forced check feeds the
same input rows to both sides so errors do not compound.
"""
import os

import numpy as np
import pytest

from golden_io import DEMO_CFG, demo_layer0_weights
from parity_util import layer_step, rel_rmse
from mojostream_b200.model import (LayerSpec, LayerWeights, ModelSpec, ModelWeights, e4b_spec,
                                   small_spec, synth_weights)

pytestmark = pytest.mark.gpu
GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


@pytest.fixture(scope="module")
def torch_cuda():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch


@pytest.fixture(scope="module")
def ctx(torch_cuda):
    from mojostream_b200.runtime import Context
    c = Context(0)
    yield c
    c.close()


def to_dev(torch, a):
    return torch.from_numpy(np.ascontiguousarray(a, np.float32)).cuda()


# ---------------------------------------------------------------- Q4 GEMM --

@pytest.mark.parametrize("M", [1, 3, 4, 6, 8, 16, 64, 70])
@pytest.mark.parametrize("K,N", [(1024, 1024), (2560, 512), (512, 2560), (10240, 256)])
def test_q4_gemm_matches_oracle(ctx, torch_cuda, oracle_lib, M, K, N):
    from mojostream_b200.runtime import Q4Weight
    torch = torch_cuda
    rng = np.random.default_rng(M * 7919 + K + N)
    W = rng.integers(0, 256, size=(K, N // 2), dtype=np.uint8)
    A = rng.standard_normal((M, K)).astype(np.float32)
    scale = float(rng.uniform(0.005, 0.02))
    w = Q4Weight(ctx, W, K, N, scale)
    C = torch.zeros((M, N), dtype=torch.float32, device="cuda")
    w.gemm(to_dev(torch, A), C)
    torch.cuda.synchronize()
    ref = oracle_lib.q4_matmul(A, W, N, scale)
    assert rel_rmse(C.cpu().numpy(), ref) < 2e-5
    w.close()


def test_q4_gemm_accumulates_like_the_reference(ctx, torch_cuda, oracle_lib):
    from mojostream_b200.runtime import Q4Weight
    torch = torch_cuda
    rng = np.random.default_rng(1)
    K, N, M = 2560, 2048, 4
    W = rng.integers(0, 256, size=(K, N // 2), dtype=np.uint8)
    A = rng.standard_normal((M, K)).astype(np.float32)
    C0 = rng.standard_normal((M, N)).astype(np.float32)
    w = Q4Weight(ctx, W, K, N, 0.01)
    C = to_dev(torch, C0)
    w.gemm(to_dev(torch, A), C, accumulate=True)
    torch.cuda.synchronize()
    ref = oracle_lib.q4_matmul(A, W, N, 0.01, C=C0)
    assert rel_rmse(C.cpu().numpy(), ref) < 2e-5


def test_q4_dequant_bit_exact(ctx, torch_cuda, oracle_lib):
    """One-hot rows read the dequantised weights back: (nibble - 8) * scale
    must be bit-identical to the reference's dequant_vec."""
    from mojostream_b200.runtime import Q4Weight
    torch = torch_cuda
    rng = np.random.default_rng(2)
    K, N = 128, 256
    W = rng.integers(0, 256, size=(K, N // 2), dtype=np.uint8)
    scale = 0.0137
    w = Q4Weight(ctx, W, K, N, scale)
    for k0 in (0, 64):
        A = np.zeros((64, K), np.float32)
        A[np.arange(64), k0 + np.arange(64)] = 1.0
        C = torch.zeros((64, N), dtype=torch.float32, device="cuda")
        w.gemm(to_dev(torch, A), C)
        torch.cuda.synchronize()
        ref = oracle_lib.dequant(W[k0:k0 + 64], N, scale)
        assert np.array_equal(C.cpu().numpy(), ref)


def test_q4_gemm_rejects_bad_shapes(ctx, torch_cuda):
    from mojostream_b200._lib import MsError
    from mojostream_b200.runtime import Q4Weight
    W = np.zeros((100, 32), np.uint8)
    with pytest.raises(MsError) as e:
        Q4Weight(ctx, W, 100, 64, 1.0)  # K not a multiple of 64
    assert e.value.name == "MS_ERR_SHAPE"
    with pytest.raises(MsError):
        Q4Weight(ctx, np.zeros((64, 4), np.uint8), 64, 8, 1.0)  # N not a multiple of 16


# ------------------------------------------------------------ layer parity --

def uniform_spec(cfg):
    hd = cfg["hidden"] // cfg["n_heads"]
    l = LayerSpec(hd, cfg["n_heads"], cfg["n_kv_heads"], 0, hd, cfg["ffn_dim"], 1e4)
    return ModelSpec("uniform", cfg["hidden"], [l], 0)


def test_reference_validation_case_layer0(ctx, torch_cuda):
    """The reference's own numeric test (validate_layer.mojo): layer 0 of the
    seed-42 demo model vs its NumPy oracle output, rel-RMSE < 1e-4."""
    from mojostream_b200 import reference_api as ra
    from mojostream_b200.runtime import Model
    torch = torch_cuda
    d = np.load(os.path.join(GOLDEN, "demo_layer0.npz"))
    w = demo_layer0_weights()
    spec = uniform_spec(DEMO_CFG)
    model = Model(ctx, spec, ModelWeights([LayerWeights(w["ple"], w["scales"], w["mats"])]),
                  max_rows=4)
    kv = ra.KVCache(ctx, model, 8)
    x = to_dev(torch, d["x_in"])
    cfg = ra.Gemma4Config(1024, 256, 2048, 1, 16, 4)
    ra.gemma4_forward_layer(x, 0, model, kv, cfg, 0)
    torch.cuda.synchronize()
    err = rel_rmse(x.cpu().numpy(), d["x_out"])
    assert err < 1e-4, err


def run_teacher_forced(ctx, torch, oracle_lib, spec, weights, n_seq, max_pos, calls,
                       slide_cap=0, tol=1e-4, kv_dtype="f32"):
    """calls: list of (seq list, pos list).  Every call runs every layer on both
    sides with identical input rows; after each layer the K / V rows the GPU
    wrote are compared with the oracle's and copied into the oracle's cache
    (parity_util.sync_kv_rows), so both sides attend over identical caches.
    The bar is a flat `tol` per layer.  kv_dtype "bf16": the GPU cache holds
    bfloat16 and the oracle rounds its K / V the same way; "i8": int8 with a
    scale per head row, and the oracle stores each row as that cache reads it
    back.  Returns the worst per-layer rel-RMSE."""
    from mojostream_b200.runtime import KVCache, Model
    M = max(len(s) for s, _ in calls)
    model = Model(ctx, spec, weights, max_rows=M)
    kv = KVCache(ctx, model, n_seq, max_pos, slide_cap, dtype=kv_dtype)
    om = oracle_lib.OracleModel(spec, weights, n_seq, max_pos, slide_cap=slide_cap or None,
                                kv_bf16=kv_dtype == "bf16", kv_i8=kv_dtype == "i8")
    rng = np.random.default_rng(11)
    worst, flips, n = 0.0, 0, 0
    for seq, pos in calls:
        x = (rng.standard_normal((len(seq), spec.hidden)) * 2.0).astype(np.float32)
        for l in range(spec.n_layers):
            got, y, f = layer_step(torch, model, kv, om, l, x, seq, pos, kv_dtype)
            flips += f
            err = rel_rmse(got, y)
            worst = max(worst, err)
            n += 1
            assert err < tol, (l, seq, pos, err)
            x = y
    print(f"teacher-forced: {n} layer calls, max rel-RMSE {worst:.3g} (bar {tol:g}), "
          f"{flips} K / V elements rounded differently (synchronised)")
    kv.close()
    model.close()
    return worst


def test_small_hybrid_decode_window_wrap(ctx, torch_cuda, oracle_lib):
    """Sliding (window 64, circular cache) and full layers with partial RoPE;
    3 independent sequences decoded past two window wraps."""
    spec = small_spec(vocab=0, n_layers=6, window=64)
    w = synth_weights(spec, seed=21)
    calls = [([0, 1, 2], [p, p + 5, p + 17]) for p in range(0, 150)]
    run_teacher_forced(ctx, torch_cuda, oracle_lib, spec, w, 3, 256, calls)


def test_rx_demo_batch_is_positions_of_one_sequence(ctx, torch_cuda, oracle_lib):
    """The reference's batch semantics (src/main.mojo:584-592): B rows are the
    consecutive positions base..base+B-1 of one sequence, causal inside the
    batch; RX demo dims (16 x 64 heads, 4 KV heads, FFN 2048)."""
    l = LayerSpec(64, 16, 4, 0, 64, 2048, 1e4)
    spec = ModelSpec("demo-rx-2", 1024, [l, l], 0, (0.04, 0.15))
    w = synth_weights(spec, seed=42)
    calls = [([0] * 4, [b + 4 * s for b in range(4)]) for s in range(12)]
    run_teacher_forced(ctx, torch_cuda, oracle_lib, spec, w, 1, 64, calls)


def test_ragged_rows_and_mixed_sequences(ctx, torch_cuda, oracle_lib):
    spec = small_spec(vocab=0, n_layers=6, window=32)
    w = synth_weights(spec, seed=5)
    calls = [([0], [0]), ([1, 1, 1], [0, 1, 2]), ([0, 1, 2, 0, 2], [1, 3, 0, 2, 1]),
             ([2] * 7, list(range(2, 9)))]
    # sequence 2 writes 7 positions in one call: the sliding ring needs 32 + 7 - 1 slots
    run_teacher_forced(ctx, torch_cuda, oracle_lib, spec, w, 3, 64, calls, slide_cap=48)


def test_large_row_block(ctx, torch_cuda, oracle_lib):
    """M = 70 rows: two m-blocks of the projection kernel (64 + 6)."""
    spec = small_spec(vocab=0, n_layers=2, window=96)
    w = synth_weights(spec, seed=9)
    calls = [([0] * 70, list(range(70)))]
    run_teacher_forced(ctx, torch_cuda, oracle_lib, spec, w, 1, 128, calls, slide_cap=176)


def test_e4b_dims_sliding_and_full_layers(ctx, torch_cuda, oracle_lib):
    """Real E4B layer shapes (hd 256 sliding window 512 / hd 512 full with
    128 rotary dims, theta 1e6): a 640-token prompt in 64-row chunks (the
    sliding ring wraps), then single-row decode steps."""
    spec = e4b_spec(n_layers=6, vocab=0)
    w = synth_weights(spec, seed=4)
    calls = [([0] * 64, list(range(p, p + 64))) for p in range(0, 640, 64)]
    calls += [([0], [640 + i]) for i in range(3)]
    run_teacher_forced(ctx, torch_cuda, oracle_lib, spec, w, 1, 1024, calls, slide_cap=576)


# ------------------------------------------------------------ bf16 KV --

def test_bf16_kv_small_hybrid_decode(ctx, torch_cuda, oracle_lib):
    """bf16 cache (decode kernels, window wraps) against the oracle with its
    K / V rounded to bf16: the fp32 bound of 1e-4 per layer."""
    spec = small_spec(vocab=0, n_layers=6, window=32)
    w = synth_weights(spec, seed=23)
    calls = [([0, 1, 2], [p, p + 3, p + 9]) for p in range(0, 80)]
    run_teacher_forced(ctx, torch_cuda, oracle_lib, spec, w, 3, 128, calls, kv_dtype="bf16")


def test_bf16_kv_e4b_dims_prefill_and_decode(ctx, torch_cuda, oracle_lib):
    """E4B layer shapes with a bf16 cache: 64-row prefill chunks (tensor-core
    projections writing K / V, the prefill attention reading them) past the
    sliding wrap, then decode rows."""
    spec = e4b_spec(n_layers=6, vocab=0)
    w = synth_weights(spec, seed=24)
    calls = [([0] * 64, list(range(p, p + 64))) for p in range(0, 640, 64)]
    calls += [([0], [640 + i]) for i in range(3)]
    run_teacher_forced(ctx, torch_cuda, oracle_lib, spec, w, 1, 1024, calls, slide_cap=576,
                       kv_dtype="bf16")


def test_bf16_kv_changes_results_by_rounding_only(ctx, torch_cuda, oracle_lib):
    """Against the fp32 oracle the bf16 cache moves a layer's output by the
    rounding of K / V (~1e-3 relative), far above fp32 noise and far below
    a wrong result."""
    from mojostream_b200.runtime import KVCache, Model
    torch = torch_cuda
    spec = small_spec(vocab=0, n_layers=2, window=32)
    w = synth_weights(spec, seed=25)
    model = Model(ctx, spec, w, max_rows=16)
    kv = KVCache(ctx, model, 1, 64, slide_cap=48, dtype="bf16")  # 16 rows per call: 32 + 15 slots
    om = oracle_lib.OracleModel(spec, w, 1, 64, slide_cap=48)
    x = (np.random.default_rng(3).standard_normal((16, spec.hidden)) * 2).astype(np.float32)
    for l in range(2):
        xg = to_dev(torch, x)
        model.layer_forward(l, xg, kv, [0] * 16, list(range(16)))
        y = om.layer_forward(l, x, [0] * 16, list(range(16)))
        err = rel_rmse(xg.cpu().numpy(), y)
        assert 1e-6 < err < 1e-2, (l, err)
        x = y
    kv.close()


def test_bf16_kv_greedy_generate_matches_oracle(ctx, torch_cuda, oracle_lib):
    """Greedy generation with a bf16 cache, checked teacher-forced: two
    oracles (K / V rounded to bf16, and fp32) are fed the GPU's own ids.  Every
    GPU id is the bf16 oracle's best, or its bf16-oracle logit is below the best
    by less than twice what the bf16 rounding itself moves those two logits
    (|bf16 - fp32 oracle|): a value within fp32 noise of a bf16 rounding
    boundary rounds differently on the two sides (one bf16 ulp, 2^-8
    relative, in that K / V element), so near-ties scale with the rounding."""
    from mojostream_b200.runtime import KVCache, Model
    spec = small_spec(vocab=4096, n_layers=6, window=32)
    w = synth_weights(spec, seed=77, symmetric=True)
    rng = np.random.default_rng(98)
    prompts = [list(rng.integers(0, 4096, size=n)) for n in (9, 20, 3)]
    steps = 16
    model = Model(ctx, spec, w, max_rows=32)
    kv = KVCache(ctx, model, 3, 128, slide_cap=64, dtype="bf16")
    ids = sum(prompts, [])
    seq = sum([[s] * len(p) for s, p in enumerate(prompts)], [])
    pos = sum([list(range(len(p))) for p in prompts], [])
    first = model.prefill(kv, ids, seq, pos)
    gen = model.generate(kv, first, [0, 1, 2], [len(p) for p in prompts], steps - 1)
    dev = np.vstack([np.array(first)[None, :], gen])

    oms = [oracle_lib.OracleModel(spec, w, 3, 128, slide_cap=64, kv_bf16=b) for b in (True, False)]
    lgs = []
    for om in oms:
        last = [om.forward(om.embed(p), [s] * len(p), list(range(len(p))))[-1]
                for s, p in enumerate(prompts)]
        lgs.append(om.lm_head(np.stack(last)))
    cur = [len(p) for p in prompts]
    exact, near = 0, []
    for st in range(steps):
        lb, lf = lgs
        for r in range(3):
            j, best = int(dev[st, r]), int(np.argmax(lb[r]))
            if j == best:
                exact += 1
                continue
            noise = max(abs(lb[r][best] - lf[r][best]), abs(lb[r][j] - lf[r][j]))
            gap = lb[r][best] - lb[r][j]
            assert gap <= 2 * noise + 1e-4 * abs(lb[r][best]), (st, r, j, best, gap, noise)
            near.append((st, r, float(gap), float(noise)))
        if st + 1 < steps:
            lgs = [om.lm_head(om.forward(om.embed([int(v) for v in dev[st]]), [0, 1, 2], cur))
                   for om in oms]
            cur = [c + 1 for c in cur]
    print(f"bf16 KV greedy ids: {exact} exact, near-ties {near}")
    assert exact >= 0.8 * dev.size, (exact, near)
    assert kv.nbytes * 2 == KVCache(ctx, model, 3, 128, slide_cap=64).nbytes


# ----------------------------------------------- reference runner quirk --

def test_rx_padding_rows_overwrite_the_window(ctx, torch_cuda, oracle_lib):
    """The reference E4B runner's batch: the real token in row 0 at position
    p and three zero rows at p+1..p+3 of the same sequence, every step
    (src/inference/lm_head.mojo:133-143, gemma4_e4b_infer.mojo:45-54).  With
    slide_cap equal to the window their K / V land in slots row 0 still
    attends once p >= window - 3.  The call is rejected by default; with
    ms_kv_allow_window_overwrite the GPU reproduces the runner: every layer
    within 1e-4 of the oracle fed the same rows (which writes every row's
    K / V, then attends by slot, as write_kv_sliding /
    compute_sliding_attention do)."""
    from mojostream_b200._lib import MsError
    from mojostream_b200.runtime import KVCache, Model
    torch = torch_cuda
    spec = small_spec(vocab=0, n_layers=6, window=32)
    w = synth_weights(spec, seed=71)
    model = Model(ctx, spec, w, max_rows=4)
    kv = KVCache(ctx, model, 1, 128, slide_cap=32)
    om = oracle_lib.OracleModel(spec, w, 1, 128, slide_cap=32)
    seq = [0, 0, 0, 0]
    with pytest.raises(MsError) as e:
        model.layer_forward(0, to_dev(torch, np.zeros((4, spec.hidden), np.float32)), kv, seq,
                            [0, 1, 2, 3])
    assert e.value.name == "MS_ERR_CAPACITY"
    kv.allow_window_overwrite(True)
    rng = np.random.default_rng(72)
    worst = 0.0
    for p in range(48):
        x = np.zeros((4, spec.hidden), np.float32)
        x[0] = rng.standard_normal(spec.hidden) * 2.0
        pos = [p, p + 1, p + 2, p + 3]
        for l in range(spec.n_layers):
            got, y, _ = layer_step(torch, model, kv, om, l, x, seq, pos, "f32")
            err = rel_rmse(got, y)
            worst = max(worst, err)
            assert err < 1e-4, (p, l, err)
            x = y
    print(f"runner padding quirk: 48 steps x 6 layers, max rel-RMSE {worst:.3g}")
    kv.close()
    model.close()


# ------------------------------------------------------------ int8 KV --

def test_i8_kv_write_read_bit_exact(ctx, torch_cuda, oracle_lib):
    """ms_kv_write into an int8 cache quantises each head row exactly as the
    oracle's quantiser (int8 q, scale = max|v| / 127; read back as q * scale,
    bit for bit), for sliding (ring) and full layers, rows of very different
    magnitudes and an all-zero row; the cache is about a quarter of fp32."""
    from mojostream_b200.runtime import KVCache, Model
    torch = torch_cuda
    spec = small_spec(vocab=0, n_layers=2, window=32)
    w = synth_weights(spec, seed=51)
    model = Model(ctx, spec, w, max_rows=16)
    kv = KVCache(ctx, model, 2, 96, slide_cap=48, dtype="i8")
    rng = np.random.default_rng(52)
    for l, ls in enumerate(spec.layers):
        n = 40
        k = rng.standard_normal((n, ls.kv_dim)).astype(np.float32)
        v = rng.standard_normal((n, ls.kv_dim)).astype(np.float32)
        k *= np.float32(10.0) ** rng.integers(-6, 6, size=(n, 1)).astype(np.float32)
        k[3] = 0.0
        v[7, : ls.head_dim] = 0.0
        kv.write(l, 1, 20, to_dev(torch, k), to_dev(torch, v))
        kg, vg = kv.read(l, 1, 20, n, ls.kv_dim)
        torch.cuda.synchronize()
        for a, g in ((k, kg), (v, vg)):
            q, s = oracle_lib.quant_i8(a.reshape(-1, ls.head_dim))
            want = (q.astype(np.float32) * s[:, None]).reshape(a.shape)
            assert np.array_equal(g.cpu().numpy(), want), l
    f32 = KVCache(ctx, model, 2, 96, slide_cap=48)
    assert kv.nbytes < 0.3 * f32.nbytes, (kv.nbytes, f32.nbytes)
    f32.close()
    kv.close()
    model.close()


def test_i8_kv_small_hybrid_decode(ctx, torch_cuda, oracle_lib):
    """int8 cache (decode kernel, window wraps) against the oracle holding
    the same int8 values: the fp32 bound of 1e-4 per layer."""
    spec = small_spec(vocab=0, n_layers=6, window=32)
    w = synth_weights(spec, seed=53)
    calls = [([0, 1, 2], [p, p + 3, p + 9]) for p in range(0, 80)]
    run_teacher_forced(ctx, torch_cuda, oracle_lib, spec, w, 3, 128, calls, kv_dtype="i8")


def test_i8_kv_e4b_dims_prefill_and_decode(ctx, torch_cuda, oracle_lib):
    """E4B layer shapes with an int8 cache: 64-row prefill chunks (tensor-core
    projections staging K / V, the quantiser, the prefill attention
    dequantising) past the sliding wrap, then decode rows."""
    spec = e4b_spec(n_layers=6, vocab=0)
    w = synth_weights(spec, seed=54)
    calls = [([0] * 64, list(range(p, p + 64))) for p in range(0, 640, 64)]
    calls += [([0], [640 + i]) for i in range(3)]
    run_teacher_forced(ctx, torch_cuda, oracle_lib, spec, w, 1, 1024, calls, slide_cap=576,
                       kv_dtype="i8")


def test_i8_kv_changes_results_by_quantisation_only(ctx, torch_cuda, oracle_lib):
    """Against the fp32 oracle the int8 cache moves a layer's output by the
    quantisation of K / V (~1e-2 relative), far above fp32 noise and below
    a wrong result."""
    from mojostream_b200.runtime import KVCache, Model
    torch = torch_cuda
    spec = small_spec(vocab=0, n_layers=2, window=32)
    w = synth_weights(spec, seed=55)
    model = Model(ctx, spec, w, max_rows=16)
    kv = KVCache(ctx, model, 1, 64, slide_cap=48, dtype="i8")
    om = oracle_lib.OracleModel(spec, w, 1, 64, slide_cap=48)
    x = (np.random.default_rng(3).standard_normal((16, spec.hidden)) * 2).astype(np.float32)
    for l in range(2):
        xg = to_dev(torch, x)
        model.layer_forward(l, xg, kv, [0] * 16, list(range(16)))
        y = om.layer_forward(l, x, [0] * 16, list(range(16)))
        err = rel_rmse(xg.cpu().numpy(), y)
        assert 1e-5 < err < 5e-2, (l, err)
        x = y
    kv.close()
    model.close()


def test_i8_kv_greedy_generate_matches_oracle(ctx, torch_cuda, oracle_lib):
    """Greedy generation with an int8 cache (prefill, then the captured decode
    loop), replayed on the oracle over the GPU's own cache: the cache the GPU
    ended with (every layer, every written position; no ring wrapped) is
    copied into the oracle, which then runs the prompts and the GPU's ids
    without writing K / V.  With the caches identical only fp32 noise
    separates the two sides: every GPU id is the oracle's best, or (once at
    most) a near-tie within 1e-3 of the best logit; the free-running
    comparison would instead measure the int8 rounding (a value within fp32
    noise of a rounding boundary moves by a whole step, max|row| / 127, on
    one side), which this model turns into logit moves of about 1."""
    from mojostream_b200.runtime import KVCache, Model
    torch = torch_cuda
    spec = small_spec(vocab=4096, n_layers=6, window=32)
    w = synth_weights(spec, seed=57, symmetric=True)
    rng = np.random.default_rng(58)
    prompts = [list(rng.integers(0, 4096, size=n)) for n in (9, 20, 3)]
    steps = 16
    model = Model(ctx, spec, w, max_rows=32)
    kv = KVCache(ctx, model, 3, 128, slide_cap=64, dtype="i8")
    ids = sum(prompts, [])
    seq = sum([[s] * len(p) for s, p in enumerate(prompts)], [])
    pos = sum([list(range(len(p))) for p in prompts], [])
    first = model.prefill(kv, ids, seq, pos)
    gen = model.generate(kv, first, [0, 1, 2], [len(p) for p in prompts], steps - 1)
    dev = np.vstack([np.array(first)[None, :], gen])

    om = oracle_lib.OracleModel(spec, w, 3, 128, slide_cap=64)
    for l, ls in enumerate(spec.layers):
        kb, vb = om.kv_arrays(l)
        for s, p in enumerate(prompts):
            n = len(p) + steps - 1  # positions written: the prompt and steps - 1 decode rows
            kg, vg = kv.read(l, s, 0, n, ls.kv_dim)
            kb[s, :n] = kg.cpu().numpy()
            vb[s, :n] = vg.cpu().numpy()
    om.set_kv_frozen(True)
    last = [om.forward(om.embed(p), [s] * len(p), list(range(len(p))))[-1]
            for s, p in enumerate(prompts)]
    lg = om.lm_head(np.stack(last))
    cur = [len(p) for p in prompts]
    ties = []
    for st in range(steps):
        for r in range(3):
            j, best = int(dev[st, r]), int(np.argmax(lg[r]))
            if j != best:
                gap = float(lg[r][best] - lg[r][j])
                assert gap <= 1e-3 * abs(float(lg[r][best])) + 1e-4, (st, r, j, best, gap)
                ties.append((st, r, gap))
        if st + 1 < steps:
            lg = om.lm_head(om.forward(om.embed([int(v) for v in dev[st]]), [0, 1, 2], cur))
            cur = [c + 1 for c in cur]
    print(f"int8 KV greedy ids over the GPU's cache: {dev.size - len(ties)} of {dev.size} "
          f"identical, near-ties {ties}")
    assert len(ties) <= 1, ties
    assert len(set(dev.ravel().tolist())) >= 4
    kv.close()
    model.close()


# ------------------------------------------------------------- lm_head --

def test_lm_head_logits_and_argmax(ctx, torch_cuda, oracle_lib):
    from mojostream_b200.runtime import Model
    torch = torch_cuda
    spec = small_spec(vocab=32768, n_layers=1)
    spec.hidden = 256
    w = synth_weights(spec, seed=8)
    model = Model(ctx, spec, w, max_rows=6)
    om = oracle_lib.OracleModel(spec, w, 1, 16)
    rng = np.random.default_rng(3)
    x = (rng.standard_normal((6, spec.hidden)) * 3).astype(np.float32)
    logits, am = model.lm_head(to_dev(torch, x))
    torch.cuda.synchronize()
    ref = om.lm_head(x)
    assert rel_rmse(logits.cpu().numpy(), ref) < 1e-5
    assert am.cpu().tolist() == om.argmax(ref)


@pytest.mark.parametrize("M", [2, 12])
def test_argmax_ties_pick_the_first(ctx, torch_cuda, M):
    """temperature_sampling's strict '>' (lm_head.mojo:226-229): among equal
    maxima the smallest index wins, also across CTAs of the kernel (2 rows:
    the CUDA-core kernel; 12 rows: the tensor-core kernel)."""
    from mojostream_b200.runtime import Model
    torch = torch_cuda
    spec = small_spec(vocab=8192, n_layers=1)
    w = synth_weights(spec, seed=1)
    w.lm_head[:] = 0.0
    w.lm_head[:, [700, 5000, 7000]] = 1.0  # three equal maxima in different CTAs
    w.final_gamma[:] = 1.0
    model = Model(ctx, spec, w, max_rows=M)
    x = np.ones((M, spec.hidden), np.float32)
    _, am = model.lm_head(to_dev(torch, x), logits=False)
    torch.cuda.synchronize()
    assert am.cpu().tolist() == [700] * M


@pytest.fixture(scope="module")
def wide_lm_model():
    """hidden 2560 (E4B's D) and 131072 vocabulary columns: 1024 column
    groups, so each persistent CTA of the tensor-core lm_head takes several
    (both tensor-memory accumulators, ring phases wrapping)."""
    l = LayerSpec(64, 4, 2, 0, 64, 512, 1e4)
    spec = ModelSpec("wide-lm", 2560, [l], 131072, (0.02, 0.06))
    return spec, synth_weights(spec, seed=61)


@pytest.mark.parametrize("M", [9, 16, 33, 64, 130])
def test_lm_head_tensor_cores_match_oracle(ctx, torch_cuda, oracle_lib, wide_lm_model, M):
    """Batches of 9+ rows run the lm_head on the tensor cores (operands split
    into bfloat16 hi + lo, three MMAs per k-step, fp32 accumulation).  The
    logits bar is 1e-3 rel-RMSE; the split gives about 1e-5, so the test holds
    it to 1e-4, which a missing low part (about 2e-3) would fail.  Ids equal
    the oracle's, except where its two best logits are closer than 1e-4 of
    their size (then either id)."""
    from mojostream_b200.runtime import Model
    torch = torch_cuda
    spec, w = wide_lm_model
    model = Model(ctx, spec, w, max_rows=M)
    om = oracle_lib.OracleModel(spec, w, 1, 16, workers=8)
    x = (np.random.default_rng(M).standard_normal((M, spec.hidden)) * 3).astype(np.float32)
    logits, am = model.lm_head(to_dev(torch, x))
    torch.cuda.synchronize()
    ref = om.lm_head(x)
    err = rel_rmse(logits.cpu().numpy(), ref)
    print(f"M={M}: logits rel-RMSE {err:.3g}")
    assert err < 1e-4, err
    got = am.cpu().tolist()
    want = om.argmax(ref)
    for r in range(M):
        if got[r] != want[r]:
            top = float(ref[r][want[r]])
            assert top - float(ref[r][got[r]]) <= 1e-4 * abs(top), (r, got[r], want[r])
    _, am2 = model.lm_head(to_dev(torch, x), logits=False)  # argmax without the logits store
    torch.cuda.synchronize()
    assert am2.cpu().tolist() == got
    model.close()


# ---------------------------------------------------------- end to end --

def oracle_generate(om, prompts, steps, with_margins=False):
    """Greedy loop on the oracle: prefill every prompt, then `steps` tokens.
    with_margins: also (top1 - top2, |top1|, runner-up id) per step and row."""
    n = len(prompts)
    last = []
    for s, p in enumerate(prompts):
        x = om.embed(p)
        x = om.forward(x, [s] * len(p), list(range(len(p))))
        last.append(x[-1])

    def pick(lg):
        order = np.argsort(lg, axis=1, kind="stable")
        top = lg[np.arange(n), order[:, -1]]
        second = lg[np.arange(n), order[:, -2]]
        return om.argmax(lg), (top - second, np.abs(top), order[:, -2], lg)

    ids, mg = pick(om.lm_head(np.stack(last)))
    pos = [len(p) for p in prompts]
    out, margins = [ids], [mg]
    for _ in range(steps - 1):
        x = om.embed(ids)
        x = om.forward(x, list(range(n)), pos)
        ids, mg = pick(om.lm_head(x))
        pos = [q + 1 for q in pos]
        out.append(ids)
        margins.append(mg)
    return (np.array(out), margins) if with_margins else np.array(out)


# A greedy flip counts as a tie (not a failure) when the oracle's top-2 logit
# margin is below this fraction of the top logit and the GPU picked an id
# whose oracle logit is within that margin of the best: the choices are
# within fp32 noise of each other.
TIE_REL = 1e-4


def compare_greedy(gen, ref, margins, tie_rel=None):
    """Step-by-step id comparison; after a tie a row's continuation diverges
    legitimately and is not compared further.  Returns (matched, ties)."""
    tie_rel = TIE_REL if tie_rel is None else tie_rel
    steps, n = ref.shape
    alive = [True] * n
    matched, ties = 0, []
    for s in range(steps):
        for r in range(n):
            if not alive[r]:
                continue
            if gen[s, r] == ref[s, r]:
                matched += 1
                continue
            gap, top, runner = margins[s][0][r], margins[s][1][r], margins[s][2][r]
            # the GPU's id must be within the tie margin of the oracle's best
            lg = margins[s][3][r]
            near = lg[ref[s, r]] - lg[gen[s, r]] <= tie_rel * max(top, 1e-30)
            assert gap <= tie_rel * max(top, 1e-30) and (gen[s, r] == runner or near), \
                f"step {s} row {r}: gpu {gen[s, r]} oracle {ref[s, r]} (margin {gap:.3g}, top {top:.3g})"
            ties.append((s, r, float(gap)))
            alive[r] = False
    return matched, ties


def test_prefill_and_greedy_generate_match_oracle(ctx, torch_cuda, oracle_lib):
    """Identical greedy ids over 32 steps (the north-star gate) for 3
    sequences with different prompt lengths."""
    from mojostream_b200.runtime import KVCache, Model
    spec = small_spec(vocab=4096, n_layers=6, window=32)
    w = synth_weights(spec, seed=77, symmetric=True)  # ids must depend on the input
    rng = np.random.default_rng(99)
    prompts = [list(rng.integers(0, 4096, size=n)) for n in (9, 20, 3)]
    steps = 32
    om = oracle_lib.OracleModel(spec, w, 3, 128, slide_cap=64)
    ref, margins = oracle_generate(om, prompts, steps, with_margins=True)
    assert len(set(ref.ravel().tolist())) > 20  # a meaningful id sequence

    model = Model(ctx, spec, w, max_rows=32)
    kv = KVCache(ctx, model, 3, 128, slide_cap=64)
    ids = sum(prompts, [])
    seq = sum([[s] * len(p) for s, p in enumerate(prompts)], [])
    pos = sum([list(range(len(p))) for p in prompts], [])
    first = model.prefill(kv, ids, seq, pos)
    gen = model.generate(kv, first, [0, 1, 2], [len(p) for p in prompts], steps - 1)
    allg = np.vstack([np.array(first)[None, :], gen])
    matched, ties = compare_greedy(allg, ref, margins)
    print(f"greedy ids: {matched} matched, ties {ties}")
    # every id compared matched (compare_greedy asserts a mismatch is a genuine
    # tie, after which that row's continuation legitimately differs); at most
    # one such tie over the 96 picks
    steps, n = ref.shape
    compared = steps * n - sum(steps - 1 - s for s, _, _ in ties)
    assert len(ties) <= 1 and matched == compared - len(ties), (matched, compared, ties)


def test_decode_step_host_buffers_match_generate(ctx, torch_cuda):
    from mojostream_b200.runtime import KVCache, Model
    spec = small_spec(vocab=4096, n_layers=6, window=32)
    w = synth_weights(spec, seed=78, symmetric=True)
    model = Model(ctx, spec, w, max_rows=4)
    kv1 = KVCache(ctx, model, 2, 64)
    kv2 = KVCache(ctx, model, 2, 64)
    ids, pos = [5, 17], [0, 0]
    steps = []
    for _ in range(10):
        ids = model.decode_step(kv1, ids, [0, 1], pos)
        pos = [p + 1 for p in pos]
        steps.append(ids)
    gen = model.generate(kv2, [5, 17], [0, 1], [0, 0], 10)
    assert np.array_equal(gen, np.array(steps))


# ------------------------------------------------------------ host errors --

def test_capacity_and_argument_errors_before_launch(ctx, torch_cuda):
    from mojostream_b200._lib import MsError
    from mojostream_b200.runtime import KVCache, Model
    torch = torch_cuda
    spec = small_spec(vocab=0, n_layers=2, window=16)
    w = synth_weights(spec, seed=2)
    model = Model(ctx, spec, w, max_rows=4)
    kv = KVCache(ctx, model, 2, 32)
    x = torch.zeros((2, spec.hidden), dtype=torch.float32, device="cuda")
    with pytest.raises(MsError) as e:
        model.forward(x, kv, [0, 1], [5, 32])  # position beyond max_pos
    assert e.value.name == "MS_ERR_CAPACITY"
    with pytest.raises(MsError) as e:
        model.forward(x, kv, [0, 2], [0, 0])  # no such sequence
    assert e.value.name == "MS_ERR_INVALID_ARG"
    with pytest.raises(MsError) as e:
        model.forward(x, kv, [1, 1], [3, 3])  # same slot twice
    assert e.value.name == "MS_ERR_INVALID_ARG"
    x5 = torch.zeros((5, spec.hidden), dtype=torch.float32, device="cuda")
    with pytest.raises(MsError) as e:
        model.forward(x5, kv, [0] * 5, list(range(5)))  # more rows than max_rows
    assert e.value.name == "MS_ERR_CAPACITY"
    with pytest.raises(MsError) as e:  # 20 positions of one sequence overrun the 16-slot ring
        big = Model(ctx, spec, w, max_rows=20)
        kvb = KVCache(ctx, big, 1, 64)
        big.forward(torch.zeros((20, spec.hidden), device="cuda"), kvb, [0] * 20, list(range(20)))
    assert e.value.name == "MS_ERR_CAPACITY"
    xu = torch.zeros((3 * spec.hidden + 1,), dtype=torch.float32, device="cuda")[1:]
    with pytest.raises(MsError) as e:
        model.forward(xu.view(3, spec.hidden), kv, [0, 1, 0], [0, 0, 1])
    assert e.value.name == "MS_ERR_ALIGN"
