"""Teacher-forced check of a sampled token loop against the oracle (shared by
the single-GPU and tensor-parallel tests).

The device's ids are fed to the oracle model; at every step the oracle picks
from its own logits with the same history (prompt + tokens so far) and row
seed splitmix64(seed ^ (seq << 32 | pos)) (temperature_sampling,
src/inference/lm_head.mojo:198-254).  A different id is accepted only as fp32
noise: a near-tie of the two best penalised logits (greedy), or a target
within 1e-4 of the device id's fp64 inverse-CDF interval (temperature).
"""
import numpy as np

from test_sampler_oracle import exact_cdf, penalised


def check_sampled_ids(oracle_lib, om, prompts, dev, T, pen, seed, tie_rel=1e-4):
    """dev [steps][n]: row 0 the prefill's first ids, then one row per
    decode step.  Returns (exact, near) counts; asserts on anything else.
    tie_rel: how far (relative to the best) a greedy pick's logit may sit
    below the oracle's best and still count as fp noise."""
    n = len(prompts)
    steps = dev.shape[0]
    hist = [list(map(int, p)) for p in prompts]
    last = []
    for s, p in enumerate(prompts):
        x = om.forward(om.embed(p), [s] * len(p), list(range(len(p))))
        last.append(x[-1])
    logits = om.lm_head(np.stack(last))
    pos = [len(p) - 1 for p in prompts]  # position of the row whose logits are sampled
    exact, near = 0, 0
    for st in range(steps):
        for r in range(n):
            rs = oracle_lib.row_seed(seed, r, pos[r])
            ref = oracle_lib.temperature_sampling(logits[r], T, hist[r], pen, rs)
            j = int(dev[st, r])
            if ref == j:
                exact += 1
                continue
            pl = penalised(logits[r], hist[r], pen)
            if T <= 0.01:
                best = pl[ref]
                assert best - pl[j] <= tie_rel * abs(best), (st, r, j, ref, best - pl[j])
            else:
                cdf = exact_cdf(pl, T)
                t = oracle_lib.sample_target(rs)
                lo = cdf[j - 1] if j > 0 else 0.0
                assert lo - 1e-4 <= t <= cdf[j] + 1e-4, (st, r, j, ref, t)
            near += 1
        ids = [int(v) for v in dev[st]]
        for r in range(n):
            hist[r].append(ids[r])
        pos = [p + 1 for p in pos]
        if st + 1 < steps:
            logits = om.lm_head(om.forward(om.embed(ids), list(range(n)), pos))
    return exact, near
