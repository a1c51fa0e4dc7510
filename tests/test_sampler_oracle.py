"""The oracle's restatement of temperature_sampling (src/inference/lm_head.mojo:
198-254) on known answers and against an fp64 inverse-CDF restatement.

The reference seeds its draw with perf_counter_ns (lm_head.mojo:245), so no
run of it can be repeated and it has no golden vectors for this function:
the known answers below are worked by hand from the source lines.
"""
import numpy as np
import pytest

A_LCG = 6364136223846793005
C_LCG = 1442695040888963407


def seed_for_lcg(low31):
    """A seed whose LCG step (lm_head.mojo:246) has the given low 31 bits."""
    return ((low31 - C_LCG) * pow(A_LCG, -1, 2 ** 31)) % (2 ** 31)


def penalised(row, generated, penalty):
    """lm_head.mojo:213-221 in float32, once per history entry."""
    r = np.array(row, np.float32)
    if penalty > 1.0:
        p = np.float32(penalty)
        for t in generated:
            if 0 <= t < r.size:
                r[t] = r[t] / p if r[t] > 0 else r[t] * p
    return r


def exact_cdf(row, temperature):
    """Running sum of softmax(row / T) in float64."""
    z = (row.astype(np.float64) - row.max()) / np.float64(np.float32(temperature))
    e = np.exp(z)
    return np.cumsum(e) / e.sum()


def test_greedy_first_maximum(oracle_lib):
    assert oracle_lib.temperature_sampling(np.array([0.5, 2, 2, -1], np.float32), 0.0, [], 1.0, 0) == 1
    # temperatures at or below 0.01 are greedy (lm_head.mojo:223)
    assert oracle_lib.temperature_sampling(np.array([0.5, 2, 3, -1], np.float32), 0.01, [], 1.0, 0) == 2


def test_repetition_penalty_known_answers(oracle_lib):
    ts = oracle_lib.temperature_sampling
    # positive logits are divided: 2.0 / 1.2 < 1.9
    assert ts(np.array([0.5, 2.0, 1.9, -1.0], np.float32), 0.0, [1], 1.2, 0) == 2
    # once per occurrence: 3 / 1.25 / 1.25 = 1.92 < 2 but 3 / 1.25 = 2.4 > 2
    assert ts(np.array([3.0, 2.0], np.float32), 0.0, [0, 0], 1.25, 0) == 1
    assert ts(np.array([3.0, 2.0], np.float32), 0.0, [0], 1.25, 0) == 0
    # non-positive logits are multiplied: -1.2 < -1.1
    assert ts(np.array([-1.0, -1.1], np.float32), 0.0, [0], 1.2, 0) == 1
    # ids outside the vocabulary are skipped, penalties <= 1 do nothing
    assert ts(np.array([3.0, 2.0], np.float32), 0.0, [7, -3], 1.25, 0) == 0
    assert ts(np.array([1.0, 2.0], np.float32), 0.0, [1], 0.5, 0) == 1


def test_target_of_a_seed(oracle_lib):
    # lm_head.mojo:246-247: low 31 bits of one LCG step over Float32(0x7FFFFFFF)
    for low in (0, 1, 12345, 0x40000000, 0x7FFFFFFF):
        assert oracle_lib.sample_target(seed_for_lcg(low)) == np.float32(low) / np.float32(2 ** 31)
    assert oracle_lib.sample_target(seed_for_lcg(0)) == 0.0
    assert oracle_lib.sample_target(seed_for_lcg(0x7FFFFFFF)) == 1.0


def test_target_zero_returns_the_first_id(oracle_lib):
    # the first running sum is >= 0 whatever its probability (lm_head.mojo:251-253)
    row = np.array([-100.0, 0.0, 0.0], np.float32)
    assert oracle_lib.temperature_sampling(row, 1.0, [], 1.0, seed_for_lcg(0)) == 0


def test_splitmix64_vector(oracle_lib):
    # first output of SplitMix64 from state 0 (Steele, Lea, Flood 2014)
    assert oracle_lib.splitmix64(0) == 0xE220A8397B1DCDAF
    assert oracle_lib.row_seed(0, 0, 0) == 0xE220A8397B1DCDAF


@pytest.mark.parametrize("V,T,pen", [(50, 0.7, 1.2), (1000, 1.0, 1.0), (4099, 2.5, 1.5)])
def test_inverse_cdf_against_float64(oracle_lib, V, T, pen):
    """The fp32 sequential running sum picks the fp64 inverse-CDF id, up to
    targets within 1e-5 of a boundary."""
    rng = np.random.default_rng(V)
    agree = 0
    for trial in range(60):
        row = rng.standard_normal(V).astype(np.float32) * 3
        gen = list(rng.integers(0, V, size=20)) + [int(np.argmax(row))] * 2
        seed = int(rng.integers(0, 2 ** 63))
        j = oracle_lib.temperature_sampling(row, T, gen, pen, seed)
        t = oracle_lib.sample_target(seed)
        cdf = exact_cdf(penalised(row, gen, pen), T)
        lo = cdf[j - 1] if j > 0 else 0.0
        assert lo - 1e-5 <= t <= cdf[j] + 1e-5, (trial, j, t, lo, cdf[j])
        agree += int(np.searchsorted(cdf, t) == j)
    assert agree >= 58
