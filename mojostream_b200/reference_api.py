"""The reference's operator interface for the token loop, on the CUDA library.

Same names, argument meaning and batch semantics as the Mojo functions they
replace, so host code and parity tests read like the reference's own:

* ``matmul_q4_bpack_raw``  -- src/linalg/kernels.mojo:201-267 (accumulates into C)
* ``gemma4_forward_layer`` -- src/main.mojo:538-613 (B rows = positions
  base_pos .. base_pos + B - 1 of one sequence, causal inside the batch)
* ``e4b_forward_layer``    -- src/inference/gemma4_e4b.mojo:459-540 (same rows)
* ``apply_final_norm`` + ``project_lm_head`` -- src/inference/lm_head.mojo:119-168
* ``temperature_sampling`` -- src/inference/lm_head.mojo:198-254 (row 0 of
  the logits, repetition penalty over ``generated``, greedy at T <= 0.01);
  greedy without a penalty is also the argmax ``apply_final_norm_and_project``
  returns

Differences (by design): the reference's kernels check nothing; here shapes and
cache capacity are checked before launch and raise ``MsError``.  Weights are
uploaded and repacked once (``Gemma4Weights`` wraps an ``ms_model``) instead of
being passed per call.  ``temperature_sampling`` leaves the logits unchanged
(the reference rewrites its row in place) and takes the seed of its draw as an
argument (the reference reads perf_counter_ns, which stays the default).
"""
import time
from dataclasses import dataclass

import numpy as np

from . import runtime
from ._lib import MsError  # noqa: F401  (re-exported for callers)


@dataclass
class Gemma4Config:
    """src/main.mojo:230-253."""
    hidden: int
    kv_dim: int
    ffn_dim: int
    n_layers: int
    n_heads: int
    n_kv_heads: int


class KVCache:
    """src/main.mojo:257-301: one sequence, ``cur_len`` advanced by the caller."""

    def __init__(self, ctx, model, max_seq_len, slide_cap=0):
        self.impl = runtime.KVCache(ctx, model, 1, max_seq_len, slide_cap)
        self.max_len = max_seq_len
        self.cur_len = 0

    def is_full(self):
        return self.cur_len >= self.max_len

    def reset(self):
        self.cur_len = 0
        self.impl.reset()


def matmul_q4_bpack_raw(C, A, bq_ptr, packed_cols, scale, workers=0, ctx=None):
    """C[M, N] += A[M, K] . dequant(bq); bq is [K][packed_cols] uint8 (host or
    device), N = 2 * packed_cols.  C and A are CUDA float32 tensors.  ``workers``
    is accepted for signature parity (the GPU decides its own parallelism).

    Given raw bytes, each call uploads and repacks the weight (and, without
    ``ctx``, makes a context) and waits for the result: right for a one-off
    call.  A host loop makes a ``runtime.Q4Weight`` once and passes it as
    ``bq_ptr``: the call then only launches the projection on torch's current
    stream (its scale must equal ``scale``)."""
    K = A.shape[1]
    N = 2 * packed_cols
    if C.shape[1] != N or C.shape[0] != A.shape[0]:
        raise ValueError(f"C is {tuple(C.shape)}, expected ({A.shape[0]}, {N})")
    if isinstance(bq_ptr, runtime.Q4Weight):
        if (bq_ptr.K, bq_ptr.N) != (K, N):
            raise ValueError(f"weight is {bq_ptr.K} x {bq_ptr.N}, expected {K} x {N}")
        if np.float32(scale) != np.float32(bq_ptr.scale):
            raise ValueError(f"scale {scale} differs from the weight's {bq_ptr.scale}")
        bq_ptr.gemm(A, C, accumulate=True)
        return C
    if tuple(bq_ptr.shape) != (K, packed_cols):
        raise ValueError(f"weights are {tuple(bq_ptr.shape)}, expected ({K}, {packed_cols})")
    own = ctx is None
    ctx = ctx or runtime.Context(A.device.index or 0)
    w = runtime.Q4Weight(ctx, bq_ptr, K, N, scale)
    try:
        w.gemm(A, C, accumulate=True)
        if own:
            ctx.sync(current=True)
    finally:
        w.close()
        if own:
            ctx.close()
    return C


def _rows(base_pos, batch):
    return [0] * batch, [base_pos + b for b in range(batch)]


def gemma4_forward_layer(x, layer_id, weights, kv, cfg, base_pos, workers=0):
    """x [B, hidden] CUDA tensor, updated in place; rows are positions
    base_pos + b of the cache's sequence."""
    seq, pos = _rows(base_pos, x.shape[0])
    weights.layer_forward(layer_id, x, kv.impl, seq, pos)
    return x


def e4b_forward_layer(x, layer, w, kv, base_pos, workers=0):
    """Same contract as gemma4_forward_layer for the hybrid (sliding / full) model."""
    return gemma4_forward_layer(x, layer, w, kv, None, base_pos, workers)


def apply_final_norm_and_project(x, weights):
    """apply_final_norm + project_lm_head: returns (logits, greedy ids)."""
    return weights.lm_head(x, logits=True)


Gemma4Weights = runtime.Model


def temperature_sampling(logits, temperature, generated, penalty=1.0, seed=None, ctx=None):
    """lm_head.mojo:198-254 on row 0 of a CUDA float32 logits tensor: returns
    the sampled id (int).  seed: the draw's seed (default perf_counter_ns, as
    the reference)."""
    own = ctx is None
    ctx = ctx or runtime.Context(logits.device.index or 0)
    try:
        if seed is None:
            seed = time.perf_counter_ns()
        out = ctx.sample(logits[:1].contiguous(), [list(generated)], temperature, penalty,
                         [seed & 0xFFFFFFFFFFFFFFFF])
        return int(out.cpu()[0])
    finally:
        if own:
            ctx.close()
