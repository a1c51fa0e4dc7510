"""The int8 KV cache's quantiser in the oracle (oracle/ms_oracle.c
orc_quant_i8), pinned against an independent NumPy restatement of the rule
the GPU cache applies per (position, KV head) row: scale = max|v| / 127,
q = rint(v * (127 / max|v|)) clamped to [-127, 127] (fminf(fmaxf()), as on the
GPU), read back as q * scale, every step one IEEE float32 operation; a row
whose max|v| is below 2^-120 (127 / max|v| would overflow) is a zero row.  The reference has no int8 cache (it is
on its roadmap, README.md:487-489), so the rule itself is the specification.
"""
import numpy as np

from oracle import oracle


MIN_AMAX = np.float32(2.0 ** -120)


def numpy_quant(x):
    x = np.asarray(x, np.float32)
    amax = np.abs(x).max(axis=1)
    live = amax >= MIN_AMAX
    scale = np.where(live, amax / np.float32(127), np.float32(0)).astype(np.float32)
    with np.errstate(divide="ignore", over="ignore"):
        inv = np.where(live, np.float32(127) / amax, np.float32(0)).astype(np.float32)
    r = np.fmin(np.fmax(np.rint(x * inv[:, None]), np.float32(-127)), np.float32(127))
    return r.astype(np.int8), scale


def rows(seed):
    rng = np.random.default_rng(seed)
    x = rng.standard_normal((64, 256)).astype(np.float32)
    x *= (np.float32(10.0) ** rng.integers(-20, 20, size=(64, 1))).astype(np.float32)
    x[5] = 0.0                                     # all-zero row
    x[6] = np.float32(-3.5)                        # constant row
    x[7, :] = 0.0
    x[7, 9] = np.float32(1e-30)                    # one tiny value
    x[8] = np.arange(256, dtype=np.float32) - 128  # integer ramp: ties at .5 steps
    x[9] = 0.0
    x[9, 3] = np.float32(1e-38)                    # 127 / amax overflows: a zero row
    x[10] = rng.standard_normal(256).astype(np.float32) * np.float32(2.0 ** -140)  # subnormal
    x[11] = 0.0
    x[11, 0] = MIN_AMAX                            # the smallest row still quantised
    x[11, 1] = -MIN_AMAX / np.float32(2)
    x[12] = 0.0
    x[12, 0] = MIN_AMAX / np.float32(2)            # just below it: a zero row
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
    nz = np.abs(x).max(axis=1) >= MIN_AMAX
    # the largest magnitude of a row maps to +-127; zero and tiny rows to scale 0
    assert (np.abs(q[nz]).max(axis=1) == 127).all()
    assert (s[~nz] == 0).all() and (q[~nz] == 0).all()
    assert (np.abs(x[~nz]) < MIN_AMAX).all()
    # error at most half a step (plus float rounding); a tiny row's error is
    # its own magnitude, below 2^-120
    err = np.abs(back - x)
    assert (err[nz] <= s[nz, None] * np.float32(0.5 + 1e-5) + 1e-38).all()
    # idempotent: quantising what the cache reads back gives the same bytes
    q2, s2 = oracle.quant_i8(back)
    assert np.array_equal(q2, q)
    assert np.allclose(s2, s, rtol=1e-6, atol=0)
