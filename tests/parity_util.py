"""Helpers of the GPU parity tests (test infrastructure).

sync_kv_rows compares the K / V rows a GPU layer call wrote with the oracle's
own rows and then copies the GPU's rows into the oracle's cache, so that the
layer comparison that follows sees identical inputs and identical caches (a
bf16 cache value within fp32 noise of a rounding boundary rounds differently
on the two sides; without the copy that one-ulp difference, 2^-8 of the
element, would be measured as a layer error; an int8 cache value likewise
moves by one quantisation step, max|head row| / 127).
"""
import numpy as np


def rel_rmse(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.sqrt(((a - b) ** 2).mean()) / (np.sqrt((b ** 2).mean()) + 1e-12))


def to_dev(torch, a):
    return torch.from_numpy(np.ascontiguousarray(a, np.float32)).cuda()


def sync_kv_rows(kv, om, layer, seq, pos, mode):
    """The K / V rows the GPU just wrote for (seq, pos) against the oracle's
    own: within 1e-5 of the row's largest magnitude (fp32 noise of the
    projection), plus for mode "bf16" one bfloat16 rounding step of the
    element, for mode "i8" one int8 step of its head row.  The oracle's rows
    are then replaced by the GPU's; returns how many elements differed."""
    ls = om.spec.layers[layer]
    kb, vb = om.kv_arrays(layer)
    flips = 0
    for s, p in zip(seq, pos):
        kg, vg = kv.read(layer, s, p, 1, ls.kv_dim)
        kg, vg = kg.cpu().numpy()[0], vg.cpu().numpy()[0]
        slot = p % kb.shape[1] if ls.window > 0 else p
        for g, o in ((kg, kb[s, slot]), (vg, vb[s, slot])):
            d = np.abs(g.astype(np.float64) - o)
            lim = 1e-5 * float(np.abs(o).max()) + 1e-30
            if mode == "bf16":
                lim = lim + 2.0 ** -7 * np.maximum(np.abs(o), np.abs(g))
            elif mode == "i8":
                step = np.abs(o).reshape(-1, ls.head_dim).max(axis=1) / 127.0
                lim = lim + np.repeat(step * 1.001, ls.head_dim)
            assert (d <= lim).all(), (layer, s, p, float((d / lim).max()))
            flips += int((g != o).sum())
        kb[s, slot] = kg
        vb[s, slot] = vg
    return flips


def layer_step(torch, model, kv, om, layer, x, seq, pos, kv_sync):
    """One layer on both sides from the same rows x; returns (GPU rows,
    oracle rows, K / V elements that rounded differently)."""
    xg = to_dev(torch, x)
    model.layer_forward(layer, xg, kv, seq, pos)
    y = om.layer_forward(layer, x, seq, pos)
    torch.cuda.synchronize()
    flips = 0
    if kv_sync:
        flips = sync_kv_rows(kv, om, layer, seq, pos, kv_sync)
        if flips:
            om.set_kv_frozen(True)
            y = om.layer_forward(layer, x, seq, pos)
            om.set_kv_frozen(False)
    return xg.cpu().numpy(), y, flips
