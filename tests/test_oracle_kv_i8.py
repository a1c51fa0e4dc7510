"""The int8 KV cache's quantiser in the oracle (oracle/ms_oracle.c
orc_quant_i8), pinned against an independent NumPy restatement of the rule
the GPU cache applies per (position, KV head) row: scale = max|v| / 127,
q = rint(v * (127 / max|v|)) clamped to [-127, 127], read back as q * scale,
every step one IEEE float32 operation.  The reference has no int8 cache (it is
on its roadmap, README.md:487-489), so the rule itself is the specification.
"""
import numpy as np

from oracle import oracle


def numpy_quant(x):
    x = np.asarray(x, np.float32)
    amax = np.abs(x).max(axis=1)
    scale = amax / np.float32(127)
    with np.errstate(divide="ignore"):
        inv = np.where(amax > 0, np.float32(127) / amax, np.float32(0)).astype(np.float32)
    q = np.clip(np.rint(x * inv[:, None]), -127, 127).astype(np.int8)
    return q, scale.astype(np.float32)


def rows(seed):
    rng = np.random.default_rng(seed)
    x = rng.standard_normal((64, 256)).astype(np.float32)
    x *= (np.float32(10.0) ** rng.integers(-20, 20, size=(64, 1))).astype(np.float32)
    x[5] = 0.0                                     # all-zero row
    x[6] = np.float32(-3.5)                        # constant row
    x[7, :] = 0.0
    x[7, 9] = np.float32(1e-30)                    # one tiny value
    x[8] = np.arange(256, dtype=np.float32) - 128  # integer ramp: ties at .5 steps
    return x


def test_quant_matches_numpy_restatement():
    for seed in range(4):
        x = rows(seed)
        q, s = oracle.quant_i8(x)
        qn, sn = numpy_quant(x)
        assert np.array_equal(q, qn) and np.array_equal(s, sn), seed


def test_quant_properties():
    x = rows(9)
    q, s = oracle.quant_i8(x)
    back = q.astype(np.float32) * s[:, None]
    nz = np.abs(x).max(axis=1) > 0
    # the largest magnitude of a row maps to +-127; zero rows to scale 0
    assert (np.abs(q[nz]).max(axis=1) == 127).all()
    assert (s[~nz] == 0).all() and (q[~nz] == 0).all()
    # error at most half a step (plus float rounding)
    err = np.abs(back - x)
    assert (err <= s[:, None] * np.float32(0.5 + 1e-5) + 1e-38).all()
    # idempotent: quantising what the cache reads back gives the same bytes
    q2, s2 = oracle.quant_i8(back)
    assert np.array_equal(q2, q)
    assert np.allclose(s2, s, rtol=1e-6, atol=0)
