"""ctypes front end of the CPU oracle (oracle/ms_oracle.c).

TEST INFRASTRUCTURE ONLY: imported by tests/, by __graft_entry__.smoke() as the
checker and by bench.py's CPU-baseline leg.  The product (mojostream_b200 and
libmojostream_cuda.so) never imports or links it.

The functions take and return NumPy arrays; ``OracleModel`` runs whole layers,
the final norm, the fp32 lm_head, the embedding gather and the greedy pick on a
model described by ``mojostream_b200.model.ModelSpec`` with weights in the
reference layout (Q4 bytes ``[K][N/2]``, fp32 lm_head ``[D][V]``).
"""
import ctypes
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_SO = os.path.join(_HERE, "_build", "libms_oracle.so")
_lib = None

_f32p = ctypes.POINTER(ctypes.c_float)
_u8p = ctypes.POINTER(ctypes.c_uint8)
_i32p = ctypes.POINTER(ctypes.c_int)


class OrcLayer(ctypes.Structure):
    _fields_ = [("head_dim", ctypes.c_int), ("n_heads", ctypes.c_int),
                ("n_kv_heads", ctypes.c_int), ("window", ctypes.c_int),
                ("rotary_dims", ctypes.c_int), ("ffn_dim", ctypes.c_int),
                ("rope_theta", ctypes.c_float), ("ple", ctypes.c_float),
                ("w", _u8p * 7), ("scale", ctypes.c_float * 7)]


class OrcKVLayer(ctypes.Structure):
    _fields_ = [("n_seq", ctypes.c_int), ("cap", ctypes.c_int), ("kv_dim", ctypes.c_int),
                ("k", _f32p), ("v", _f32p), ("bf16", ctypes.c_int), ("frozen", ctypes.c_int),
                ("i8", ctypes.c_int)]


def build():
    """Compile the oracle library (gcc, see oracle/Makefile)."""
    subprocess.run(["make", "-s", "-C", _HERE], check=True)


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(_SO):
            build()
        L = ctypes.CDLL(_SO)
        L.orc_q4_matmul.argtypes = [_f32p, _f32p, _u8p, ctypes.c_int, ctypes.c_int,
                                    ctypes.c_int, ctypes.c_float, ctypes.c_int]
        L.orc_fp32_matmul.argtypes = [_f32p, _f32p, _f32p, ctypes.c_int, ctypes.c_int,
                                      ctypes.c_int, ctypes.c_int]
        L.orc_rmsnorm.argtypes = [_f32p, ctypes.c_int, ctypes.c_int]
        L.orc_rmsnorm_weighted.argtypes = [_f32p, _f32p, ctypes.c_int, ctypes.c_int]
        L.orc_swiglu.argtypes = [_f32p, _f32p, ctypes.c_int]
        L.orc_rope.argtypes = [_f32p, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_float]
        L.orc_rope_inv_freq.argtypes = [_f32p, ctypes.c_int, ctypes.c_float]
        L.orc_dequant.argtypes = [_u8p, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_float]
        L.orc_dequant.restype = ctypes.c_float
        L.orc_attention_row.argtypes = [_f32p, _f32p, _f32p, _f32p, ctypes.c_int, ctypes.c_int,
                                        ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                        ctypes.c_int]
        L.orc_layer_forward.argtypes = [ctypes.POINTER(OrcLayer), ctypes.c_int, _f32p,
                                        ctypes.c_int, _i32p, _i32p,
                                        ctypes.POINTER(OrcKVLayer), ctypes.c_int]
        L.orc_layer_forward.restype = ctypes.c_int
        L.orc_lm_head.argtypes = [_f32p, _f32p, _f32p, _f32p, ctypes.c_int, ctypes.c_int,
                                  ctypes.c_int, ctypes.c_int]
        L.orc_argmax.argtypes = [_f32p, ctypes.c_int]
        L.orc_argmax.restype = ctypes.c_int
        L.orc_embed.argtypes = [_f32p, _f32p, ctypes.c_int, ctypes.c_int, ctypes.c_int]
        L.orc_temperature_sampling.argtypes = [_f32p, ctypes.c_int, ctypes.c_float, _i32p,
                                               ctypes.c_int, ctypes.c_float, ctypes.c_uint64]
        L.orc_temperature_sampling.restype = ctypes.c_int
        L.orc_sample_target.argtypes = [ctypes.c_uint64]
        L.orc_sample_target.restype = ctypes.c_float
        L.orc_quant_i8.argtypes = [_f32p, ctypes.c_int, ctypes.POINTER(ctypes.c_int8), _f32p]
        L.orc_quant_i8_rows.argtypes = [_f32p, ctypes.c_int, ctypes.c_int,
                                        ctypes.POINTER(ctypes.c_int8), _f32p]
        _lib = L
    return _lib


def _p(a, t):
    return a.ctypes.data_as(t)


def _f32(a):
    return np.ascontiguousarray(a, dtype=np.float32)


def q4_matmul(A, W, N, scale, C=None, workers=1):
    """C += A . dequant(W); W is [K][N/2] uint8 (kernels.mojo:201-267)."""
    A = _f32(A)
    M, K = A.shape
    W = np.ascontiguousarray(W, dtype=np.uint8)
    assert W.shape == (K, N // 2)
    C = np.zeros((M, N), np.float32) if C is None else _f32(C).copy()
    lib().orc_q4_matmul(_p(C, _f32p), _p(A, _f32p), _p(W, _u8p), M, K, N, scale, workers)
    return C


def fp32_matmul(A, B, workers=1):
    A, B = _f32(A), _f32(B)
    M, K = A.shape
    N = B.shape[1]
    C = np.zeros((M, N), np.float32)
    lib().orc_fp32_matmul(_p(C, _f32p), _p(A, _f32p), _p(B, _f32p), M, K, N, workers)
    return C


def dequant(W, N, scale):
    K = W.shape[0]
    W = np.ascontiguousarray(W, dtype=np.uint8)
    out = np.empty((K, N), np.float32)
    L = lib()
    for k in range(K):
        for n in range(N):
            out[k, n] = L.orc_dequant(_p(W, _u8p), N, k, n, scale)
    return out


def quant_i8(x):
    """int8 KV cache quantisation of each row of x (one head row per row):
    (q int8 [n][hd], scale fp32 [n]); the row reads back as q * scale."""
    x = _f32(np.atleast_2d(x))
    q = np.empty(x.shape, np.int8)
    s = np.empty(x.shape[0], np.float32)
    lib().orc_quant_i8_rows(_p(x, _f32p), x.shape[0], x.shape[1],
                            q.ctypes.data_as(ctypes.POINTER(ctypes.c_int8)), _p(s, _f32p))
    return q, s


def rmsnorm(x):
    x = _f32(x).copy()
    lib().orc_rmsnorm(_p(x, _f32p), x.shape[0], x.shape[1])
    return x


def rmsnorm_weighted(x, gamma):
    x = _f32(x).copy()
    g = _f32(gamma)
    lib().orc_rmsnorm_weighted(_p(x, _f32p), _p(g, _f32p), x.shape[0], x.shape[1])
    return x


def swiglu(g, u):
    g, u = _f32(g), _f32(u).copy()
    lib().orc_swiglu(_p(g, _f32p), _p(u, _f32p), u.size)
    return u


def rope(x, n_heads, hd, pos, theta):
    x = _f32(x).copy()
    lib().orc_rope(_p(x, _f32p), n_heads, hd, pos, theta)
    return x


def rope_inv_freq(hd, theta):
    out = np.empty(hd // 2, np.float32)
    lib().orc_rope_inv_freq(_p(out, _f32p), hd, theta)
    return out


class OracleModel:
    """Runs a ModelSpec on the CPU with the oracle.  KV caches are owned here.

    ``slide_cap`` is the slot count of circular (sliding-window) caches; the
    reference uses exactly the window (gemma4_e4b.mojo:219-228).  ``kv_bf16``
    keeps K / V rounded to bfloat16 (the GPU's reduced-precision cache);
    ``kv_i8`` keeps each K / V head row as the int8 cache reads it back.
    """

    def __init__(self, spec, weights, n_seq, max_pos, slide_cap=None, workers=1, kv_bf16=False,
                 kv_i8=False):
        self.spec, self.w, self.workers = spec, weights, workers
        self._layers, self._kv, self._keep = [], [], []
        for li, ls in enumerate(spec.layers):
            lw = weights.layers[li]
            L = OrcLayer()
            L.head_dim, L.n_heads, L.n_kv_heads = ls.head_dim, ls.n_heads, ls.n_kv_heads
            L.window, L.rotary_dims, L.ffn_dim = ls.window, ls.rotary_dims, ls.ffn_dim
            L.rope_theta, L.ple = ls.rope_theta, lw.ple
            for m in range(7):
                arr = np.ascontiguousarray(lw.mats[m], dtype=np.uint8)
                self._keep.append(arr)
                L.w[m] = _p(arr, _u8p)
                L.scale[m] = lw.scales[m]
            self._layers.append(L)
            cap = (slide_cap or ls.window) if ls.window > 0 else max_pos
            kvd = ls.n_kv_heads * ls.head_dim
            kb = np.zeros((n_seq, cap, kvd), np.float32)
            vb = np.zeros((n_seq, cap, kvd), np.float32)
            kv = OrcKVLayer()
            kv.n_seq, kv.cap, kv.kv_dim = n_seq, cap, kvd
            kv.k, kv.v = _p(kb, _f32p), _p(vb, _f32p)
            kv.bf16 = 1 if kv_bf16 else 0
            kv.i8 = 1 if kv_i8 else 0
            self._kv.append((kv, kb, vb))

    def kv_arrays(self, layer):
        return self._kv[layer][1], self._kv[layer][2]

    def set_kv_frozen(self, on):
        """While on, layer_forward writes no K / V rows: it attends over the
        cache as it stands (rows copied in from the implementation under test)."""
        for kv, _, _ in self._kv:
            kv.frozen = 1 if on else 0

    def layer_forward(self, layer, x, seq, pos):
        x = _f32(x).copy()
        seq = np.ascontiguousarray(seq, dtype=np.int32)
        pos = np.ascontiguousarray(pos, dtype=np.int32)
        rc = lib().orc_layer_forward(ctypes.byref(self._layers[layer]), self.spec.hidden,
                                     _p(x, _f32p), x.shape[0], _p(seq, _i32p), _p(pos, _i32p),
                                     ctypes.byref(self._kv[layer][0]), self.workers)
        if rc != 0:
            raise ValueError(f"oracle layer_forward rejected the call ({rc})")
        return x

    def forward(self, x, seq, pos):
        for li in range(len(self.spec.layers)):
            x = self.layer_forward(li, x, seq, pos)
        return x

    def embed(self, ids):
        D, V = self.spec.hidden, self.spec.vocab
        W = self.w.lm_head
        x = np.empty((len(ids), D), np.float32)
        for r, t in enumerate(ids):
            row = np.empty(D, np.float32)
            lib().orc_embed(_p(row, _f32p), _p(W, _f32p), D, V, int(t))
            x[r] = row
        return x

    def lm_head(self, x):
        x = _f32(x).copy()
        M = x.shape[0]
        D, V = self.spec.hidden, self.spec.vocab
        logits = np.empty((M, V), np.float32)
        g = _f32(self.w.final_gamma)
        lib().orc_lm_head(_p(logits, _f32p), _p(x, _f32p), _p(g, _f32p),
                          _p(self.w.lm_head, _f32p), M, D, V, self.workers)
        return logits

    @staticmethod
    def argmax(logits):
        logits = _f32(logits)
        return [lib().orc_argmax(_p(np.ascontiguousarray(logits[r]), _f32p), logits.shape[1])
                for r in range(logits.shape[0])]


def temperature_sampling(row, temperature, generated, penalty, seed):
    """lm_head.mojo:198-254 on one logits row (a copy; the reference writes
    its row in place).  Returns the sampled id."""
    r = np.ascontiguousarray(_f32(row)).copy()
    g = np.ascontiguousarray(np.asarray(generated, np.int32))
    return lib().orc_temperature_sampling(_p(r, _f32p), r.size, float(temperature),
                                          _p(g, _i32p), g.size, float(penalty),
                                          int(seed) & 0xFFFFFFFFFFFFFFFF)


def sample_target(seed):
    """The uniform draw of temperature_sampling for a seed (lm_head.mojo:246-247)."""
    return float(lib().orc_sample_target(int(seed) & 0xFFFFFFFFFFFFFFFF))


def splitmix64(z):
    """SplitMix64 (Steele, Lea, Flood 2014): the token loop's per-row seed is
    splitmix64(seed ^ (seq << 32 | pos))."""
    M = 0xFFFFFFFFFFFFFFFF
    z = (z + 0x9E3779B97F4A7C15) & M
    z = ((z ^ (z >> 30)) * 0xBF58476D1CE4E5B9) & M
    z = ((z ^ (z >> 27)) * 0x94D049BB133111EB) & M
    return z ^ (z >> 31)


def row_seed(seed, seq, pos):
    return splitmix64((int(seed) ^ ((int(seq) << 32) | int(pos))) & 0xFFFFFFFFFFFFFFFF)
