"""ms_model_load: a model streamed from .mojostream + lm_head_proto.bin
files behaves exactly like the same weights given as arrays (same repacked
bits, so the same ids and logits), and its first layer matches the oracle."""
import os

import numpy as np
import pytest

from mojostream_b200 import fileformat as ff
from mojostream_b200.model import LayerSpec, ModelSpec, small_spec, synth_weights

pytestmark = pytest.mark.gpu


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


def prompts():
    rng = np.random.default_rng(11)
    return [list(rng.integers(3, 4096, size=n)) for n in (7, 13)]


def run_ids(model, torch):
    from mojostream_b200.runtime import KVCache
    kv = KVCache(model.ctx, model, 2, 64, slide_cap=48)
    P = prompts()
    ids, seq = sum(P, []), sum([[s] * len(p) for s, p in enumerate(P)], [])
    pos = sum([list(range(len(p))) for p in P], [])
    first = model.prefill(kv, ids, seq, pos)
    gen = model.generate(kv, first, [0, 1], [len(p) for p in P], 6)
    x = torch.randn((3, model.spec.hidden), device="cuda", generator=torch.Generator(
        device="cuda").manual_seed(5))
    lg, am = model.lm_head(x)
    torch.cuda.synchronize()
    kv.close()
    return np.vstack([np.array(first)[None], gen]), lg.cpu().numpy()


@pytest.mark.parametrize("staging", [0, 65536])
def test_loaded_model_equals_array_model(ctx, torch_cuda, tmp_path, staging):
    from mojostream_b200.runtime import Model
    spec = small_spec(vocab=4096, n_layers=6, window=32)
    w = synth_weights(spec, seed=31, symmetric=True)
    path, lmp = str(tmp_path / "m.mojostream"), str(tmp_path / "lm.bin")
    ff.write_mojostream(path, spec, w)
    ff.write_lm_head(lmp, w.lm_head, w.final_gamma)
    ref = Model(ctx, spec, w, max_rows=32)
    got = Model.load(ctx, path, lmp, max_rows=32, full_rotary=64, staging_bytes=staging)
    assert got.spec.layers == spec.layers
    assert got.weight_bytes == ref.weight_bytes
    data = ff.file_check(path)
    assert got.load_bytes == data["data_end"] - data["data_start"] + 4 * spec.hidden * spec.vocab
    ids_r, lg_r = run_ids(ref, torch_cuda)
    ids_g, lg_g = run_ids(got, torch_cuda)
    assert np.array_equal(ids_r, ids_g)
    assert np.array_equal(lg_r, lg_g)
    print(f"loaded {got.load_bytes / 1e6:.1f} MB in {got.load_seconds * 1e3:.1f} ms")


def test_bos_embeds_as_the_files_vector(ctx, torch_cuda, tmp_path):
    """apply_bos_embedding (lm_head.mojo:133-143): token 2 embeds as the lm_head
    file's BOS vector; every other id as its column."""
    from mojostream_b200.runtime import Model
    spec = small_spec(vocab=4096, n_layers=2, window=32)
    w = synth_weights(spec, seed=32, symmetric=True)
    bos = np.random.default_rng(3).standard_normal(spec.hidden).astype(np.float32)
    path, lmp = str(tmp_path / "m.mojostream"), str(tmp_path / "lm.bin")
    ff.write_mojostream(path, spec, w)
    ff.write_lm_head(lmp, w.lm_head, w.final_gamma, bos)
    m = Model.load(ctx, path, lmp, max_rows=8, full_rotary=64)
    x = m.embed([2, 5, 2]).cpu().numpy()
    assert np.array_equal(x[0], bos) and np.array_equal(x[2], bos)
    assert np.array_equal(x[1], w.lm_head[:, 5])


def test_q4_lm_head_v1_expands_exactly(ctx, torch_cuda, tmp_path):
    """v1 (Q4 lm_head, gamma 1): logits equal an fp32 model whose lm_head is
    (nibble - 8) * scale (kernels.mojo:100-108) and whose gamma is 1."""
    from mojostream_b200.model import ModelWeights
    from mojostream_b200.runtime import Model
    spec = small_spec(vocab=4096, n_layers=2, window=32)
    w = synth_weights(spec, seed=33, symmetric=True)
    rng = np.random.default_rng(4)
    q4 = rng.integers(0, 256, size=(spec.hidden, spec.vocab // 2), dtype=np.uint8)
    scale = np.float32(0.0123)
    lo, hi = (q4 & 15).astype(np.float32) - 8, (q4 >> 4).astype(np.float32) - 8
    W = np.empty((spec.hidden, spec.vocab), np.float32)
    W[:, 0::2], W[:, 1::2] = lo * scale, hi * scale
    path, lmp = str(tmp_path / "m.mojostream"), str(tmp_path / "lm1.bin")
    ff.write_mojostream(path, spec, w)
    ff.write_lm_head(lmp, q4=q4, bos=W[:, 2], scale=float(scale))
    got = Model.load(ctx, path, lmp, max_rows=8, full_rotary=64)
    ref = Model(ctx, spec, ModelWeights(w.layers, W, np.ones(spec.hidden, np.float32)), max_rows=8)
    torch = torch_cuda
    x = torch.randn((4, spec.hidden), device="cuda")
    a, ia = got.lm_head(x)
    b, ib = ref.lm_head(x)
    torch.cuda.synchronize()
    assert torch.equal(a, b) and torch.equal(ia, ib)


def test_format1_demo_file_layer_matches_oracle(ctx, torch_cuda, oracle_lib, tmp_path):
    """A format-1 file (the demo stack's layout, create_fake_model.py): every
    layer full attention, head_dim hidden / n_heads, RoPE theta 1e4."""
    from mojostream_b200.runtime import KVCache, Model
    torch = torch_cuda
    l = LayerSpec(64, 8, 2, 0, 64, 1024, 1e4)
    spec = ModelSpec("demo-file", 512, [l] * 3, 0, (0.04, 0.15))
    w = synth_weights(spec, seed=34)
    path = str(tmp_path / "demo.mojostream")
    ff.write_mojostream(path, spec, w, format_tag=1)
    m = Model.load(ctx, path, max_rows=8)
    assert m.spec.layers == spec.layers
    kv = KVCache(ctx, m, 1, 16)
    x = np.random.default_rng(1234).standard_normal((4, 512)).astype(np.float32) * 0.1
    xd = torch.from_numpy(x).cuda()
    m.layer_forward(0, xd, kv, [0] * 4, [0, 1, 2, 3])
    om = oracle_lib.OracleModel(spec, w, 1, 16)
    ref = om.layer_forward(0, x, [0] * 4, [0, 1, 2, 3])
    got = xd.cpu().numpy()
    err = np.sqrt(((got - ref) ** 2).mean() / (ref ** 2).mean())
    assert err < 1e-4, err
    kv.close()


def test_load_errors_before_any_device_work(ctx, torch_cuda, tmp_path):
    from mojostream_b200._lib import MsError
    from mojostream_b200.runtime import Model
    spec = small_spec(vocab=4096, n_layers=6, window=32)
    w = synth_weights(spec, seed=35)
    path = str(tmp_path / "m.mojostream")
    ff.write_mojostream(path, spec, w)
    # E4B's rule puts the full layer at 5 (0-based); full_every=4 mistypes layer 3
    with pytest.raises(MsError, match="layer 3 is full attention by full_every=4"):
        Model.load(ctx, path, full_every=4)
    b = bytearray(open(path, "rb").read())
    b[0] = 0
    open(path, "wb").write(bytes(b))
    with pytest.raises(MsError, match="magic"):
        Model.load(ctx, path)
    with pytest.raises(MsError):
        Model.load(ctx, str(tmp_path / "missing.mojostream"))
