"""Model descriptions and seeded synthetic weights for the token loop.

A model is a hidden size, a list of per-layer specs and an optional fp32
lm_head.  The five benchmark configurations of the project are built here:

* ``demo_spec``  -- the uniform demo stack of bench.mojo (src/main.mojo:230-253),
  either with the benchmark dims (8 q-heads x 128, 2 KV heads, FFN 4096) or the
  reference's own generator dims (16 x 64, 4 KV heads, FFN 2048,
  scripts/create_fake_model.py:59-64);
* ``e4b_spec``   -- Gemma-4-E4B shaped: 35 sliding + 7 full layers, full iff
  (layer + 1) % 6 == 0 (src/inference/gemma4_e4b.mojo:33-63);
* ``b14_spec``   -- a 14B-class Gemma-style stack (5 sliding : 1 full).

Weights use the reference layout: per matrix a uint8 array ``[K][N/2]`` (low
nibble = even column), one fp32 scale per tensor, one PLE scalar per layer;
the lm_head is fp32 ``[D][V]``.  Draws follow the project's synthetic recipe:
Q4 bytes uniform 0..255 (values -8..7), scales uniform in ``scale_range``, PLE
uniform in [0.8, 1.2], final RMSNorm gains N(1, 0.02), lm_head N(0, 0.02^2).
"""
from dataclasses import dataclass, field
from typing import List, Optional

import numpy as np

MAT_NAMES = ["Q", "K", "V", "O", "Gate", "Up", "Down"]


@dataclass
class LayerSpec:
    head_dim: int
    n_heads: int
    n_kv_heads: int
    window: int          # 0 = attend to all cached positions
    rotary_dims: int     # leading dims of each head that RoPE rotates
    ffn_dim: int
    rope_theta: float

    @property
    def q_dim(self):
        return self.n_heads * self.head_dim

    @property
    def kv_dim(self):
        return self.n_kv_heads * self.head_dim

    def mat_shapes(self, D):
        """(K, N) of Q, K, V, O, Gate, Up, Down."""
        q, kv, F = self.q_dim, self.kv_dim, self.ffn_dim
        return [(D, q), (D, kv), (D, kv), (q, D), (D, F), (D, F), (F, D)]

    def q4_bytes(self, D):
        return sum(K * N // 2 for K, N in self.mat_shapes(D))


@dataclass
class ModelSpec:
    name: str
    hidden: int
    layers: List[LayerSpec]
    vocab: int = 0
    scale_range: tuple = (0.005, 0.02)

    @property
    def n_layers(self):
        return len(self.layers)

    def q4_bytes(self):
        return sum(l.q4_bytes(self.hidden) for l in self.layers)

    def lm_head_bytes(self):
        return 4 * self.hidden * self.vocab

    def kv_bytes_per_seq(self, seq_len, slide_cap=None, dtype="f32"):
        """K+V bytes one decode step reads for a sequence of seq_len: fp32,
        bf16, or int8 (a byte per value plus a 4-byte scale per KV head)."""
        total = 0
        for l in self.layers:
            n = min(seq_len, l.window) if l.window > 0 else seq_len
            row = {"f32": 4 * l.kv_dim, "bf16": 2 * l.kv_dim,
                   "i8": l.kv_dim + 4 * l.n_kv_heads}[dtype]
            total += 2 * n * row
        return total


@dataclass
class LayerWeights:
    ple: float
    scales: List[float]
    mats: list           # 7 uint8 arrays (NumPy or torch) [K][N/2]


@dataclass
class ModelWeights:
    layers: List[LayerWeights]
    lm_head: Optional[object] = None      # fp32 [D][V]
    final_gamma: Optional[object] = None  # fp32 [D]
    extra: dict = field(default_factory=dict)


def is_full_layer(layer):
    """gemma4_e4b.mojo:60-63: full attention iff (layer + 1) % 6 == 0."""
    return (layer + 1) % 6 == 0


def demo_spec(dims="baseline", n_layers=40):
    if dims == "baseline":
        l = LayerSpec(128, 8, 2, 0, 128, 4096, 1e4)
        return ModelSpec("demo-baseline", 1024, [l] * n_layers, 0, (0.005, 0.02))
    if dims == "rx":
        l = LayerSpec(64, 16, 4, 0, 64, 2048, 1e4)
        return ModelSpec("demo-rx", 1024, [l] * n_layers, 0, (0.04, 0.15))
    raise ValueError(dims)


def e4b_spec(n_layers=42, vocab=262144):
    slide = LayerSpec(256, 8, 2, 512, 256, 10240, 1e4)
    full = LayerSpec(512, 8, 2, 0, 128, 10240, 1e6)
    layers = [full if is_full_layer(i) else slide for i in range(n_layers)]
    return ModelSpec("gemma4-e4b", 2560, layers, vocab, (0.005, 0.02))


def b14_spec(n_layers=48, vocab=262144):
    slide = LayerSpec(128, 40, 8, 1024, 128, 13824, 1e4)
    full = LayerSpec(128, 40, 8, 0, 128, 13824, 1e6)
    layers = [full if is_full_layer(i) else slide for i in range(n_layers)]
    return ModelSpec("gemma-14b", 5120, layers, vocab, (0.005, 0.02))


def small_spec(vocab=4096, n_layers=6, window=64):
    """A reduced model with both layer types for fast parity tests:
    hidden 256; sliding layers hd 64, full layers hd 128 with partial RoPE."""
    slide = LayerSpec(64, 4, 2, window, 64, 512, 1e4)
    full = LayerSpec(128, 4, 2, 0, 64, 512, 1e6)
    layers = [full if is_full_layer(i) else slide for i in range(n_layers)]
    return ModelSpec("small-hybrid", 256, layers, vocab, (0.02, 0.06))


def _symmetric_bytes(rng, shape):
    """Bytes whose two nibbles are uniform in 1..15 (values -7..7, mean 0)."""
    lo = rng.integers(1, 16, size=shape, dtype=np.uint8)
    hi = rng.integers(1, 16, size=shape, dtype=np.uint8)
    return (lo | (hi << 4)).astype(np.uint8)


def synth_weights(spec, seed=0, symmetric=False):
    """Seeded weights as NumPy arrays (host); fine for models up to a few GB.

    symmetric=False is the benchmark recipe (nibbles uniform 0..15, values
    -8..7 with mean -0.5).  That mean adds the same term to every output
    column, which after a few layers dominates the hidden state, so greedy ids
    stop depending on the input.  symmetric=True draws values -7..7 (mean 0)
    so token-id parity tests see inputs that matter."""
    rng = np.random.default_rng(seed)
    D = spec.hidden
    layers = []
    for l in spec.layers:
        ple = float(rng.uniform(0.8, 1.2))
        scales, mats = [], []
        for K, N in l.mat_shapes(D):
            scales.append(float(rng.uniform(*spec.scale_range)))
            if symmetric:
                mats.append(_symmetric_bytes(rng, (K, N // 2)))
            else:
                mats.append(rng.integers(0, 256, size=(K, N // 2), dtype=np.uint8))
        layers.append(LayerWeights(ple, scales, mats))
    lm = gamma = None
    if spec.vocab:
        lm = (rng.standard_normal((D, spec.vocab), dtype=np.float32) * np.float32(0.02))
        gamma = (1.0 + 0.02 * rng.standard_normal(D)).astype(np.float32)
    return ModelWeights(layers, lm, gamma)


def synth_weights_device(spec, seed=0, device="cuda"):
    """Seeded weights generated directly in device memory (torch), for the
    multi-GB benchmark models.  Same distributions as ``synth_weights`` (a
    different stream: torch's generator)."""
    import torch
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    gh = np.random.default_rng(seed)
    D = spec.hidden
    layers = []
    for l in spec.layers:
        ple = float(gh.uniform(0.8, 1.2))
        scales, mats = [], []
        for K, N in l.mat_shapes(D):
            scales.append(float(gh.uniform(*spec.scale_range)))
            mats.append(torch.randint(0, 256, (K, N // 2), dtype=torch.uint8, device=device,
                                      generator=g))
        layers.append(LayerWeights(ple, scales, mats))
    lm = gamma = None
    if spec.vocab:
        lm = torch.randn((D, spec.vocab), dtype=torch.float32, device=device, generator=g) * 0.02
        gamma = (1.0 + 0.02 * torch.randn(D, dtype=torch.float32, device=device, generator=g))
    return ModelWeights(layers, lm, gamma)
