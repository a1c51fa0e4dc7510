"""The timeline tool's summary (CPU): synthetic per-CTA records of a 2-layer
step, checked for the op order, critical paths, gaps and the SM histogram."""
import numpy as np

from mojostream_b200.timeline import REC, summarize


def synthetic_step(n_layers=2):
    recs = []
    t = 1_000_000
    for layer in range(n_layers):
        for j, (kind, ctas) in enumerate([(0, 144), (1, 128), (0, 140), (0, 160), (0, 140)]):
            key = 0x1000 * (layer * 5 + j + 1)
            for c in range(ctas):
                r = np.zeros((), dtype=REC)
                r["key"], r["kind"], r["cta"], r["smid"] = key, kind, c, c // 2
                r["t0"] = t - 10_000
                r["t1"] = t + (c % 3)             # release at t
                r["t2"] = t + 5_000 + 10 * c      # last CTA ends at t + 5000 + 10 (ctas - 1)
                r["pts"][:] = t + 1_000
                recs.append(r)
            t += 5_000 + 10 * (ctas - 1) + 600    # next op released 0.6 us after this one ends
    return np.array(recs, dtype=REC)


def test_summary_orders_ops_and_reports_critical_paths():
    lines = summarize(synthetic_step())
    assert lines[0].startswith("10 ops")
    assert lines[1].startswith("QKV") and "ctas  144" in lines[1]
    assert "rel->end   6.43 us" in lines[1]          # 5 us + 10 ns x 143
    assert "gap 0.60" in lines[1]
    assert lines[2].startswith("attention") and "offsets 1.00" in lines[2]
    assert "2 CTA: 72 SMs" in lines[1]               # two CTAs per SM in the synthetic placement
