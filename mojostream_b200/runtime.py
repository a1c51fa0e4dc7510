"""Python host of libmojostream_cuda.so: contexts, models, KV caches, calls.

Device memory for activations is handled with torch tensors (plumbing only);
every computation runs in the CUDA library through its C-ABI.
"""
import ctypes

import numpy as np

from . import _lib
from ._lib import check, int_array, lib


def _ptr(t):
    """Data pointer of a torch tensor or NumPy array (kept alive by the caller)."""
    if hasattr(t, "data_ptr"):
        return ctypes.c_void_p(t.data_ptr())
    return ctypes.c_void_p(t.ctypes.data)


def _check_f32(t, what, min_numel=0):
    """A tensor handed to the C-ABI as a bare pointer: the library reads or
    writes min_numel dense fp32 values there, so it must be a contiguous
    float32 CUDA tensor holding at least that many (the library cannot see a
    tensor's size; alignment and device residency it checks itself)."""
    if not getattr(t, "is_cuda", False):
        raise ValueError(f"{what}: a CUDA tensor is needed")
    if str(t.dtype) != "torch.float32":
        raise ValueError(f"{what}: float32 needed, got {t.dtype}")
    if not t.is_contiguous():
        raise ValueError(f"{what}: a contiguous tensor is needed")
    if t.numel() < min_numel:
        raise ValueError(f"{what}: {t.numel()} values, the call uses {min_numel}")


def _check_rows(M, **lists):
    """Per-row lists handed to the C-ABI as bare arrays of M ints: each must
    have exactly M entries (the library reads M of each)."""
    for name, v in lists.items():
        if len(v) != M:
            raise ValueError(f"{name}: {len(v)} entries for {M} rows")


_CUDA_STREAM_LEGACY = 1  # cudaStreamLegacy: the legacy default stream handle


def _stream():
    """torch's current stream as a cudaStream_t.  torch's default stream is
    handle 0, which the C-ABI reads as "the context's stream"; pass the legacy
    default stream handle instead so work stays ordered with torch's."""
    import torch
    s = torch.cuda.current_stream().cuda_stream
    return ctypes.c_void_p(s if s else _CUDA_STREAM_LEGACY)


def tp_unique_id():
    """A fresh tensor-parallel group id (ms_tp_unique_id), made by rank 0."""
    n = lib().ms_tp_unique_id_bytes()
    buf = ctypes.create_string_buffer(n)
    check(lib().ms_tp_unique_id(buf, n))
    return buf.raw


class Context:
    """ms_ctx: one CUDA device, its stream and scratch memory."""

    def __init__(self, device=0):
        h = ctypes.c_void_p()
        st = lib().ms_init(device, ctypes.byref(h))
        if st != 0:
            raise _lib.MsError(st, f"ms_init({device}) failed")
        self.h = h
        self.device = device

    def check(self, status):
        check(status, self.h)

    def sync(self, current=False):
        """ms_sync: wait for the context's stream (current=True: torch's
        current stream, where the wrappers launch) and raise any error the
        kernels recorded."""
        self.check(lib().ms_sync(self.h, _stream() if current else None))

    @property
    def stream_ptr(self):
        """The context's cudaStream_t (as an int)."""
        return lib().ms_ctx_stream(self.h)

    def sample(self, logits, generated, temperature, penalty, seeds):
        """temperature_sampling (lm_head.mojo:198-254) of every row of a CUDA
        fp32 logits tensor [M][V] (ms_sample).  generated: one id list per row
        (the repetition-penalty history); seeds: one uint64 per row (the
        reference draws it from perf_counter_ns).  Returns int32 ids on the
        device."""
        import torch
        M, V = logits.shape
        _check_f32(logits, "logits", M * V)
        hist = [int(t) for g in generated for t in g]
        off = np.zeros(M + 1, np.int32)
        off[1:] = np.cumsum([len(g) for g in generated])
        h = torch.tensor(hist + [0], dtype=torch.int32, device=logits.device)
        o = torch.tensor(off, dtype=torch.int32, device=logits.device)
        sd = torch.tensor(np.asarray(seeds, np.uint64).view(np.int64), dtype=torch.int64,
                          device=logits.device)
        out = torch.empty(M, dtype=torch.int32, device=logits.device)
        self.check(lib().ms_sample(self.h, _ptr(logits), M, V, _ptr(h), _ptr(o),
                                   float(temperature), float(penalty), _ptr(sd), _ptr(out),
                                   _stream()))
        return out

    def tp_init(self, world, rank, unique_id):
        """Join a tensor-parallel group of `world` ranks (ms_tp_init); call
        before creating models.  unique_id: the bytes of tp_unique_id() made
        by rank 0."""
        buf = ctypes.create_string_buffer(bytes(unique_id), len(unique_id))
        self.check(lib().ms_tp_init(self.h, int(world), int(rank), buf))

    @property
    def tp_world(self):
        return lib().ms_tp_world(self.h)

    def close(self):
        if self.h:
            lib().ms_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class Q4Weight:
    """ms_q4_weight: one Q4 matrix repacked for the tensor-core projection."""

    def __init__(self, ctx, w_rx, K, N, scale):
        self.ctx, self.K, self.N, self.scale = ctx, K, N, float(scale)
        h = ctypes.c_void_p()
        ctx.check(lib().ms_q4_weight_create(ctx.h, _ptr(w_rx), K, N, float(scale),
                                            ctypes.byref(h)))
        self.h = h

    def gemm(self, A, C, accumulate=False):
        M = A.shape[0]
        _check_f32(A, "A", M * self.K)
        _check_f32(C, "C", M * self.N)
        self.ctx.check(lib().ms_q4_gemm(self.ctx.h, self.h, _ptr(C), _ptr(A), M,
                                        1 if accumulate else 0, _stream()))
        return C

    def close(self):
        if self.h:
            lib().ms_q4_weight_destroy(self.ctx.h, self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class Model:
    """ms_model built from a ModelSpec and ModelWeights (NumPy or torch)."""

    def __init__(self, ctx, spec, weights, max_rows=4):
        self.ctx, self.spec, self.max_rows = ctx, spec, max_rows
        n = spec.n_layers
        descs = (_lib.LayerDesc * n)()
        keep = []
        for i, (ls, lw) in enumerate(zip(spec.layers, weights.layers)):
            d = descs[i]
            d.head_dim, d.n_heads, d.n_kv_heads = ls.head_dim, ls.n_heads, ls.n_kv_heads
            d.window, d.rotary_dims, d.ffn_dim = ls.window, ls.rotary_dims, ls.ffn_dim
            d.rope_theta, d.ple = ls.rope_theta, lw.ple
            for m in range(7):
                arr = lw.mats[m]
                if isinstance(arr, np.ndarray):
                    arr = np.ascontiguousarray(arr, dtype=np.uint8)
                else:
                    arr = arr.contiguous()
                keep.append(arr)
                d.w[m] = _ptr(arr).value
                d.scale[m] = lw.scales[m]
        md = _lib.ModelDesc()
        md.hidden, md.n_layers = spec.hidden, n
        md.layers = descs
        md.vocab = spec.vocab
        md.max_rows = max_rows
        if spec.vocab:
            lm = weights.lm_head
            lm = np.ascontiguousarray(lm, np.float32) if isinstance(lm, np.ndarray) else lm.contiguous()
            g = weights.final_gamma
            if g is not None:
                g = np.ascontiguousarray(g, np.float32) if isinstance(g, np.ndarray) else g.contiguous()
            keep += [lm, g]
            md.lm_head = _ptr(lm).value
            md.final_gamma = _ptr(g).value if g is not None else None
        h = ctypes.c_void_p()
        ctx.check(lib().ms_model_create(ctx.h, ctypes.byref(md), ctypes.byref(h)))
        self.h = h

    @classmethod
    def load(cls, ctx, path, lm_head_path=None, max_rows=64, full_every=0, window=0,
             slide_theta=0.0, full_theta=0.0, full_rotary=0, staging_bytes=0):
        """ms_model_load: a model from a .mojostream file (and an
        lm_head_proto.bin).  The options cover what the file does not say;
        zeros take the loader's defaults."""
        from . import fileformat
        o = _lib.LoadOpts(full_every, window, slide_theta, full_theta, full_rotary, max_rows,
                          staging_bytes)
        h = ctypes.c_void_p()
        ctx.check(lib().ms_model_load(ctx.h, str(path).encode(),
                                      str(lm_head_path).encode() if lm_head_path else None,
                                      ctypes.byref(o), ctypes.byref(h)))
        self = cls.__new__(cls)
        self.ctx, self.max_rows, self.h = ctx, max_rows, h
        self.spec = fileformat.spec_from_file(path, lm_head_path, full_every, window, slide_theta,
                                              full_theta, full_rotary)
        secs, nbytes = ctypes.c_double(), ctypes.c_uint64()
        lib().ms_load_stats(ctx.h, ctypes.byref(secs), ctypes.byref(nbytes))
        self.load_seconds, self.load_bytes = secs.value, nbytes.value
        return self

    @property
    def weight_bytes(self):
        return lib().ms_model_weight_bytes(self.h)

    def close(self):
        if self.h:
            lib().ms_model_destroy(self.ctx.h, self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    # ---- calls -------------------------------------------------------------
    def layer_forward(self, layer, x, kv, seq, pos):
        """x: CUDA float32 tensor [M][hidden], updated in place."""
        M = x.shape[0]
        _check_f32(x, "x", M * self.spec.hidden)
        _check_rows(M, seq=seq, pos=pos)
        self.ctx.check(lib().ms_layer_forward(self.ctx.h, self.h, layer, _ptr(x), kv.h,
                                              int_array(seq), int_array(pos), M, _stream()))
        return x

    def forward(self, x, kv, seq, pos):
        M = x.shape[0]
        _check_f32(x, "x", M * self.spec.hidden)
        _check_rows(M, seq=seq, pos=pos)
        self.ctx.check(lib().ms_forward(self.ctx.h, self.h, _ptr(x), kv.h, int_array(seq),
                                        int_array(pos), M, _stream()))
        return x

    def embed(self, ids):
        import torch
        x = torch.empty((len(ids), self.spec.hidden), dtype=torch.float32, device="cuda")
        self.ctx.check(lib().ms_embed(self.ctx.h, self.h, int_array(ids), len(ids), _ptr(x),
                                      _stream()))
        return x

    def lm_head(self, x, logits=True):
        import torch
        M = x.shape[0]
        _check_f32(x, "x", M * self.spec.hidden)
        lg = torch.empty((M, self.spec.vocab), dtype=torch.float32, device="cuda") if logits else None
        am = torch.empty(M, dtype=torch.int32, device="cuda")
        self.ctx.check(lib().ms_lm_head(self.ctx.h, self.h, _ptr(x), M,
                                        _ptr(lg) if lg is not None else None, _ptr(am), _stream()))
        return lg, am

    def set_sampling(self, temperature=0.0, penalty=1.0, seed=0):
        """Sampling of decode_step / generate / prefill (ms_set_sampling);
        the defaults are the greedy argmax."""
        self.ctx.check(lib().ms_set_sampling(self.ctx.h, self.h, float(temperature),
                                             float(penalty), int(seed) & 0xFFFFFFFFFFFFFFFF))

    def decode_step(self, kv, ids, seq, pos):
        M = len(ids)
        _check_rows(M, seq=seq, pos=pos)
        out = (ctypes.c_int * M)()
        self.ctx.check(lib().ms_decode_step(self.ctx.h, self.h, kv.h, int_array(ids),
                                            int_array(seq), int_array(pos), M, out))
        return list(out)

    def generate(self, kv, ids, seq, pos, steps, timing=False):
        """Tokens [steps][M] (greedy unless set_sampling chose otherwise); with
        timing=True also the device ms of the loop."""
        M = len(ids)
        _check_rows(M, seq=seq, pos=pos)
        out = (ctypes.c_int * (M * steps))()
        ms = ctypes.c_float(0.0)
        self.ctx.check(lib().ms_generate(self.ctx.h, self.h, kv.h, int_array(ids),
                                         int_array(seq), int_array(pos), M, steps, out,
                                         ctypes.byref(ms)))
        ids_out = np.array(list(out), dtype=np.int64).reshape(steps, M)
        return (ids_out, float(ms.value)) if timing else ids_out

    def prefill(self, kv, ids, seq, pos):
        _check_rows(len(ids), seq=seq, pos=pos)
        first = (ctypes.c_int * kv.n_seq)(*([-1] * kv.n_seq))
        self.ctx.check(lib().ms_prefill(self.ctx.h, self.h, kv.h, int_array(ids),
                                        int_array(seq), int_array(pos), len(ids), first))
        return list(first)


class KVCache:
    """ms_kv: paged cache for n_seq sequences."""

    def __init__(self, ctx, model, n_seq, max_pos, slide_cap=0, dtype="f32", pool_pages=0):
        """dtype "f32" (the parity mode), "bf16" (half the cache bytes) or
        "i8" (int8 with one scale per position and KV head: about a quarter);
        pool_pages > 0: the full-attention layers share a pool of that many
        16-position pages (ms_kv_create_pooled)."""
        self.ctx, self.n_seq, self.max_pos, self.dtype = ctx, n_seq, max_pos, dtype
        self.model = model  # the cache reads its model's layer shapes: keep it alive
        h = ctypes.c_void_p()
        code = {"f32": 0, "bf16": 1, "i8": 2}[dtype]
        if pool_pages:
            ctx.check(lib().ms_kv_create_pooled(ctx.h, model.h, n_seq, max_pos, slide_cap, code,
                                                pool_pages, ctypes.byref(h)))
        else:
            ctx.check(lib().ms_kv_create_typed(ctx.h, model.h, n_seq, max_pos, slide_cap, code,
                                               ctypes.byref(h)))
        self.h = h

    def _kv_dim(self, layer):
        """Values per cached row of `layer` on this rank (its share of the KV
        heads under tensor parallelism); 0 for a layer the model lacks (the
        library reports that)."""
        layers = self.model.spec.layers
        if not 0 <= layer < len(layers):
            return 0
        return layers[layer].kv_dim // max(1, self.ctx.tp_world)

    def release(self, seq):
        """ms_kv_release: slot seq is free for a new request."""
        self.ctx.check(lib().ms_kv_release(self.ctx.h, self.h, seq))

    def share_prefix(self, src, dst, n_pos):
        """ms_kv_share_prefix: slot dst starts with src's first n_pos positions."""
        self.ctx.check(lib().ms_kv_share_prefix(self.ctx.h, self.h, src, dst, n_pos))

    def allow_window_overwrite(self, allow=True):
        """ms_kv_allow_window_overwrite: accept calls whose rows overwrite
        sliding slots other rows of the call still attend (the reference
        E4B runner's zero padding rows)."""
        self.ctx.check(lib().ms_kv_allow_window_overwrite(self.ctx.h, self.h, int(allow)))

    def pages(self):
        """(used, total) full-attention pages."""
        u, t = ctypes.c_int(), ctypes.c_int()
        check(lib().ms_kv_pages(self.h, ctypes.byref(u), ctypes.byref(t)))
        return u.value, t.value

    @property
    def nbytes(self):
        return lib().ms_kv_bytes(self.h)

    def reset(self):
        self.ctx.check(lib().ms_kv_reset(self.ctx.h, self.h))

    def write(self, layer, seq, pos0, k, v):
        """ms_kv_write: rows k, v (fp32 device tensors [n][kv_dim]) become the
        cached K / V of positions pos0 .. pos0 + n - 1 of sequence seq."""
        n = k.shape[0]
        _check_f32(k, "k", n * self._kv_dim(layer))
        _check_f32(v, "v", n * self._kv_dim(layer))
        self.ctx.check(lib().ms_kv_write(self.ctx.h, self.h, layer, seq, pos0, k.shape[0],
                                         _ptr(k), _ptr(v), _stream()))

    def read(self, layer, seq, pos0, n, kv_dim):
        """ms_kv_read: the cached K / V rows of positions pos0 .. pos0 + n - 1
        as two fp32 device tensors [n][kv_dim]."""
        import torch
        if 0 < self._kv_dim(layer) != kv_dim:
            raise ValueError(f"kv_dim {kv_dim}: layer {layer} caches rows of {self._kv_dim(layer)}")
        k = torch.empty((n, kv_dim), dtype=torch.float32, device="cuda")
        v = torch.empty((n, kv_dim), dtype=torch.float32, device="cuda")
        self.ctx.check(lib().ms_kv_read(self.ctx.h, self.h, layer, seq, pos0, n, _ptr(k),
                                        _ptr(v), _stream()))
        return k, v

    def close(self):
        if self.h:
            lib().ms_kv_destroy(self.ctx.h, self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
