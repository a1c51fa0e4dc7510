"""Serving requests that come and go: the pooled KV cache (full-attention pages
drawn from one shared pool), slot release and reuse, shared prompt prefixes.

Reference: the cache types of the token loop (KVCache, src/main.mojo:257-301;
HybridKVCache, src/inference/gemma4_e4b.mojo:83-116, with write_kv_sliding /
write_kv_full at :211-249) and the roadmap item they grow into (paged KV
allocator / continuous batching, README.md:487-489).  Every id sequence is
compared with an oracle run of the same request from scratch; the model is
the 6-layer hybrid (sliding window 32 + full layers with partial RoPE) with
symmetric weights, whose ids depend on the input and which is not chaotic, so
greedy ids are compared free-running.
"""
import numpy as np
import pytest

from mojostream_b200.model import small_spec, synth_weights

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


@pytest.fixture(scope="module")
def model_w():
    spec = small_spec(vocab=4096, n_layers=6, window=32)
    return spec, synth_weights(spec, seed=313, symmetric=True)


def oracle_run(oracle_lib, spec, w, prompt, steps, slide_cap):
    """Greedy ids of one request from scratch: the first id after the prompt,
    then `steps` more."""
    om = oracle_lib.OracleModel(spec, w, 1, 512, slide_cap=slide_cap)
    x = om.forward(om.embed(prompt), [0] * len(prompt), list(range(len(prompt))))
    ids = [om.argmax(om.lm_head(x[-1:]))[0]]
    p = len(prompt)
    for _ in range(steps):
        x = om.forward(om.embed([ids[-1]]), [0], [p])
        ids.append(om.argmax(om.lm_head(x))[0])
        p += 1
    return ids


def prompts(lengths, seed):
    rng = np.random.default_rng(seed)
    return [[int(t) for t in rng.integers(0, 4096, size=n)] for n in lengths]


def prefill_rows(prompts_, slots):
    ids, seq, pos = [], [], []
    for p, s in zip(prompts_, slots):
        ids += p
        seq += [s] * len(p)
        pos += list(range(len(p)))
    return ids, seq, pos


def test_pooled_cache_ragged_lengths_match_oracle(ctx, torch_cuda, oracle_lib, model_w):
    """Four requests of 9 / 70 / 3 / 40 prompt tokens share a pool of 24
    pages (384 positions; fixed slots would hold 4 x 256); their greedy ids
    over 12 steps equal the oracle's, and the pool holds exactly the pages
    their lengths need."""
    from mojostream_b200.runtime import KVCache, Model
    spec, w = model_w
    P = prompts([9, 70, 3, 40], 41)
    model = Model(ctx, spec, w, max_rows=128)
    kv = KVCache(ctx, model, 4, 256, slide_cap=112, pool_pages=24)
    assert kv.pages() == (0, 24)
    ids, seq, pos = prefill_rows(P, [0, 1, 2, 3])
    first = model.prefill(kv, ids, seq, pos)
    steps = 12
    gen = model.generate(kv, first, [0, 1, 2, 3], [len(p) for p in P], steps)
    got = np.vstack([np.array(first)[None, :], gen])
    for s, p in enumerate(P):
        ref = oracle_run(oracle_lib, spec, w, p, steps, 112)
        assert list(got[:, s]) == ref, (s, list(got[:, s]), ref)
    need = sum((len(p) + steps - 1) // 16 + 1 for p in P)  # pages up to the last position
    assert kv.pages()[0] == need, (kv.pages(), need)
    kv.close()
    model.close()


@pytest.mark.parametrize("pool_pages", [0, 20])
def test_released_slot_reused_by_a_shorter_request(ctx, torch_cuda, oracle_lib, model_w,
                                                   pool_pages):
    """Slot 0 serves request A (60 prompt tokens + 10 steps), is released, and
    takes request B (a 7-token prompt) in one ms_prefill call together with
    slot 1's next decode row; B's ids and slot 1's continuation equal fresh
    oracle runs.  Fixed slots (pool_pages 0: the slot is reused as it was
    left) and the pooled cache (A's pages go back to the pool)."""
    from mojostream_b200.runtime import KVCache, Model
    spec, w = model_w
    A, B, C = prompts([60, 7, 25], 43)
    model = Model(ctx, spec, w, max_rows=96)
    kv = KVCache(ctx, model, 2, 128, slide_cap=96, pool_pages=pool_pages)
    ids, seq, pos = prefill_rows([A, C], [0, 1])
    first = model.prefill(kv, ids, seq, pos)
    gen = model.generate(kv, first, [0, 1], [len(A), len(C)], 10)
    c_ids = [first[1]] + [int(t) for t in gen[:, 1]]  # slot 1: C so far
    c_pos = len(C) + 10
    kv.release(0)
    if pool_pages:  # only slot 1's pages (positions 0 .. c_pos - 1) remain
        assert kv.pages()[0] == (c_pos - 1) // 16 + 1, kv.pages()
    # B's prompt in slot 0 and C's next row in slot 1, one call
    ids = B + [c_ids[-1]]
    seq = [0] * len(B) + [1]
    pos = list(range(len(B))) + [c_pos]
    first2 = model.prefill(kv, ids, seq, pos)
    gen2 = model.generate(kv, first2, [0, 1], [len(B), c_pos + 1], 8)
    b_got = [first2[0]] + [int(t) for t in gen2[:, 0]]
    c_got = c_ids + [first2[1]] + [int(t) for t in gen2[:, 1]]
    assert b_got == oracle_run(oracle_lib, spec, w, B, 8, 96)
    assert c_got == oracle_run(oracle_lib, spec, w, C, 10 + 1 + 8, 96)
    kv.close()
    model.close()


@pytest.mark.parametrize("pool_pages", [0, 16])
def test_shared_prefix(ctx, torch_cuda, oracle_lib, model_w, pool_pages):
    """A 40-token prefix computed once in slot 0 is shared into slot 1
    (ms_kv_share_prefix: two whole pages by reference, the third copied);
    each slot then continues with its own tokens, and both equal oracle runs
    of prefix + continuation from scratch.  A later write into a shared page
    (ms_kv_write into slot 1 below the prefix end) gets a private copy and
    leaves slot 0's rows alone."""
    from mojostream_b200.runtime import KVCache, Model
    torch = torch_cuda
    spec, w = model_w
    prefix, t0, t1 = prompts([40, 6, 9], 47)
    model = Model(ctx, spec, w, max_rows=64)
    kv = KVCache(ctx, model, 2, 128, slide_cap=96, pool_pages=pool_pages)
    ids, seq, pos = prefill_rows([prefix], [0])
    model.prefill(kv, ids, seq, pos)
    kv.share_prefix(0, 1, 40)
    if pool_pages:
        assert kv.pages()[0] == 4  # 3 pages of slot 0 + slot 1's copy of the third
    rows = t0 + t1
    seq = [0] * len(t0) + [1] * len(t1)
    pos = list(range(40, 40 + len(t0))) + list(range(40, 40 + len(t1)))
    first = model.prefill(kv, rows, seq, pos)
    gen = model.generate(kv, first, [0, 1], [40 + len(t0), 40 + len(t1)], 6)
    for s, t in enumerate((t0, t1)):
        got = [first[s]] + [int(v) for v in gen[:, s]]
        assert got == oracle_run(oracle_lib, spec, w, prefix + t, 6, 96), s
    # copy on write: overwrite position 5 of slot 1 (a shared full-attention page)
    full = [l for l, ls in enumerate(spec.layers) if ls.window == 0][0]
    kvd = spec.layers[full].kv_dim
    k0, _ = kv.read(full, 0, 5, 1, kvd)
    used = kv.pages()[0]
    z = torch.zeros((1, kvd), device="cuda")
    kv.write(full, 1, 5, z, z)
    k0b, _ = kv.read(full, 0, 5, 1, kvd)
    k1b, _ = kv.read(full, 1, 5, 1, kvd)
    torch.cuda.synchronize()
    assert torch.equal(k0, k0b) and not torch.equal(k0, k1b)
    assert float(k1b.abs().max()) == 0.0
    if pool_pages:
        assert kv.pages()[0] == used + 1  # slot 1's private copy of page 0
    kv.close()
    model.close()


@pytest.mark.parametrize("pool_pages", [0, 16])
def test_i8_shared_prefix_copies_scales(ctx, torch_cuda, model_w, pool_pages):
    """int8 cache: a shared prefix (whole pages by reference, the last page
    copied; sliding rings copied) reads back in the new slot bit for bit,
    scales included, and a copy-on-write leaves the source slot alone."""
    from mojostream_b200.runtime import KVCache, Model
    torch = torch_cuda
    spec, w = model_w
    (prefix,) = prompts([40], 49)
    model = Model(ctx, spec, w, max_rows=64)
    kv = KVCache(ctx, model, 2, 128, slide_cap=96, dtype="i8", pool_pages=pool_pages)
    ids, seq, pos = prefill_rows([prefix], [0])
    model.prefill(kv, ids, seq, pos)
    kv.share_prefix(0, 1, 40)
    for l, ls in enumerate(spec.layers):
        a = kv.read(l, 0, 0, 40, ls.kv_dim)
        b = kv.read(l, 1, 0, 40, ls.kv_dim)
        torch.cuda.synchronize()
        assert torch.equal(a[0], b[0]) and torch.equal(a[1], b[1]), l
        assert float(a[0].abs().max()) > 0
    full = [l for l, ls in enumerate(spec.layers) if ls.window == 0][0]
    kvd = spec.layers[full].kv_dim
    k0, _ = kv.read(full, 0, 5, 1, kvd)
    z = torch.full((1, kvd), 0.5, device="cuda")
    kv.write(full, 1, 5, z, z)
    k0b, _ = kv.read(full, 0, 5, 1, kvd)
    k1b, _ = kv.read(full, 1, 5, 1, kvd)
    torch.cuda.synchronize()
    want = float(np.float32(127) * (np.float32(0.5) / np.float32(127)))  # q 127, scale 0.5 / 127
    assert torch.equal(k0, k0b) and bool((k1b == want).all())
    kv.close()
    model.close()


def test_generate_with_a_new_cache_after_one_was_closed(ctx, torch_cuda, oracle_lib, model_w):
    """ms_generate keeps its decode step as a captured graph that holds the
    cache's device pointers.  Caches of different sizes are created, used and
    closed one after another on one model (a new cache can get a closed one's
    host address); each must get its own graph: every run's ids equal the
    oracle's."""
    from mojostream_b200.runtime import KVCache, Model
    spec, w = model_w
    P = prompts([12, 7], 51)
    model = Model(ctx, spec, w, max_rows=32)
    ids, seq, pos = prefill_rows(P, [0, 1])
    refs = [oracle_run(oracle_lib, spec, w, p, 6, 48) for p in P]
    for max_pos in (128, 256, 192):
        kv = KVCache(ctx, model, 2, max_pos, slide_cap=48)
        first = model.prefill(kv, ids, seq, pos)
        gen = model.generate(kv, first, [0, 1], [len(p) for p in P], 6)
        got = np.vstack([np.array(first)[None, :], gen])
        for s in range(2):
            assert list(got[:, s]) == refs[s], (max_pos, s)
        kv.close()
    model.close()


def test_cache_of_a_destroyed_model_is_refused(ctx, torch_cuda, model_w):
    """A cache refers to the model it was made for.  After that model is
    destroyed, a new model (which may get the freed one's host address) must
    refuse the cache before any kernel runs, address reused or not."""
    from mojostream_b200._lib import MsError
    from mojostream_b200.runtime import KVCache, Model
    spec, w = model_w
    a = Model(ctx, spec, w, max_rows=8)
    kv = KVCache(ctx, a, 1, 64, slide_cap=48)
    a.close()
    b = Model(ctx, spec, w, max_rows=8)
    with pytest.raises(MsError) as e:
        b.decode_step(kv, [1], [0], [0])
    assert e.value.name == "MS_ERR_STATE"
    kv.close()
    fresh = KVCache(ctx, b, 1, 64, slide_cap=48)
    assert len(b.decode_step(fresh, [1], [0], [0])) == 1
    fresh.close()
    b.close()


def test_pool_exhaustion_is_an_error_before_launch(ctx, torch_cuda, model_w):
    """A call the pool cannot serve fails before any kernel runs and takes
    nothing: the pages the sequences before the short one got are given
    back, so the host and device block tables stay equal."""
    from mojostream_b200._lib import MsError
    from mojostream_b200.runtime import KVCache, Model
    spec, w = model_w
    model = Model(ctx, spec, w, max_rows=64)
    kv = KVCache(ctx, model, 2, 256, slide_cap=96, pool_pages=4)
    P = prompts([50, 30], 5)
    ids, seq, pos = prefill_rows(P, [0, 1])  # 4 + 2 pages > 4
    with pytest.raises(MsError) as e:
        model.prefill(kv, ids, seq, pos)
    assert e.value.name == "MS_ERR_CAPACITY"
    assert kv.pages()[0] == 0  # the refused call took no pages
    first = model.prefill(kv, P[1], [1] * 30, list(range(30)))  # fits alone
    assert first[1] >= 0
    kv.close()
    model.close()
