"""Seeded weights behind the golden fixtures (shared by make_golden.py and the tests).

``demo_layer0_weights`` regenerates layer 0 of the reference's seed-42 demo
model by repeating the draw order of its generator
(scripts/create_fake_model.py:188-213 and pack_row_major :94-97): one
``uniform(0.8, 1.2)`` PLE draw, then per matrix Q, K, V, O, Gate, Up, Down a
``uniform(0.04, 0.15)`` scale draw followed by ``integers(0, 256)`` bytes of
shape ``(rows, cols // 2)``.  The fixture stores the SHA-256 of the bytes the
reference wrote, so a drift in NumPy's generator is caught instead of silently
changing the case.
"""
import numpy as np

DEMO_CFG = {"hidden": 1024, "kv_dim": 256, "ffn_dim": 2048, "n_heads": 16, "n_kv_heads": 4}
SMALL_CFG = {"hidden": 256, "kv_dim": 128, "ffn_dim": 512, "n_heads": 4, "n_kv_heads": 2}


def _shapes(cfg):
    D, KV, F = cfg["hidden"], cfg["kv_dim"], cfg["ffn_dim"]
    return [(D, D), (D, KV), (D, KV), (D, D), (D, F), (D, F), (F, D)]


def _draw_layer(rng, cfg):
    ple = float(rng.uniform(0.8, 1.2))
    scales, mats = [], []
    for rows, cols in _shapes(cfg):
        scales.append(float(rng.uniform(0.04, 0.15)))
        mats.append(rng.integers(0, 256, size=(rows, cols // 2), dtype=np.uint8))
    return {"ple": ple, "scales": scales, "mats": mats}


def demo_layer0_weights():
    """Layer 0 of the reference's seed-42 demo model (RX dims)."""
    return _draw_layer(np.random.default_rng(42), DEMO_CFG)


def small_layer_weights():
    """A smaller uniform layer from seed 4242 (same draw recipe)."""
    return _draw_layer(np.random.default_rng(4242), SMALL_CFG)
