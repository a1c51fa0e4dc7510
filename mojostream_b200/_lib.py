"""ctypes binding of libmojostream_cuda.so (C-ABI: include/mojostream_cuda.h).

This is the binding a Python host uses; a Mojo host binds the same symbols
with DLHandle.  There is no fallback: if the library is
missing or does not export a declared symbol, loading fails loudly.
"""
import ctypes
import os

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libmojostream_cuda.so")

MS_OK = 0
STATUS_NAMES = {
    0: "MS_OK", 1: "MS_ERR_INVALID_ARG", 2: "MS_ERR_SHAPE", 3: "MS_ERR_ALIGN",
    4: "MS_ERR_CAPACITY", 5: "MS_ERR_CUDA", 6: "MS_ERR_NCCL", 7: "MS_ERR_OOM",
    8: "MS_ERR_STATE", 9: "MS_ERR_TIMEOUT", 10: "MS_ERR_UNSUPPORTED",
}

_vp = ctypes.c_void_p
_ip = ctypes.POINTER(ctypes.c_int)
_fp = ctypes.POINTER(ctypes.c_float)
_u8p = ctypes.POINTER(ctypes.c_uint8)


class LayerDesc(ctypes.Structure):
    """ms_layer_desc."""
    _fields_ = [("head_dim", ctypes.c_int), ("n_heads", ctypes.c_int),
                ("n_kv_heads", ctypes.c_int), ("window", ctypes.c_int),
                ("rotary_dims", ctypes.c_int), ("ffn_dim", ctypes.c_int),
                ("rope_theta", ctypes.c_float), ("ple", ctypes.c_float),
                ("w", _vp * 7), ("scale", ctypes.c_float * 7)]


class ModelDesc(ctypes.Structure):
    """ms_model_desc."""
    _fields_ = [("hidden", ctypes.c_int), ("n_layers", ctypes.c_int),
                ("layers", ctypes.POINTER(LayerDesc)), ("vocab", ctypes.c_int),
                ("lm_head", _vp), ("final_gamma", _vp), ("max_rows", ctypes.c_int)]


class FileInfo(ctypes.Structure):
    """ms_file_info."""
    _fields_ = [("format_tag", ctypes.c_int), ("n_layers", ctypes.c_int),
                ("hidden", ctypes.c_int), ("kv_dim", ctypes.c_int), ("ffn_dim", ctypes.c_int),
                ("n_heads", ctypes.c_int), ("n_kv_heads", ctypes.c_int),
                ("n_tensors", ctypes.c_uint64), ("data_start", ctypes.c_uint64),
                ("data_end", ctypes.c_uint64), ("file_size", ctypes.c_uint64),
                ("kv_shared_layers", ctypes.c_int), ("sliding_kv_dim", ctypes.c_int),
                ("full_kv_dim", ctypes.c_int), ("ple_dim", ctypes.c_int),
                ("sliding_window", ctypes.c_int)]


class LoadOpts(ctypes.Structure):
    """ms_load_opts."""
    _fields_ = [("full_every", ctypes.c_int), ("window", ctypes.c_int),
                ("slide_theta", ctypes.c_float), ("full_theta", ctypes.c_float),
                ("full_rotary", ctypes.c_int), ("max_rows", ctypes.c_int),
                ("staging_bytes", ctypes.c_size_t)]


# name -> (restype, argtypes); every symbol include/mojostream_cuda.h declares
SIGNATURES = {
    "ms_abi_version": (ctypes.c_int, []),
    "ms_status_string": (ctypes.c_char_p, [ctypes.c_int]),
    "ms_init": (ctypes.c_int, [ctypes.c_int, ctypes.POINTER(_vp)]),
    "ms_destroy": (ctypes.c_int, [_vp]),
    "ms_last_error": (ctypes.c_char_p, [_vp]),
    "ms_sync": (ctypes.c_int, [_vp, _vp]),
    "ms_malloc": (ctypes.c_int, [_vp, ctypes.c_size_t, ctypes.POINTER(_vp)]),
    "ms_free": (ctypes.c_int, [_vp, _vp]),
    "ms_memcpy": (ctypes.c_int, [_vp, _vp, _vp, ctypes.c_size_t, ctypes.c_int, _vp]),
    "ms_q4_weight_create": (ctypes.c_int, [_vp, _vp, ctypes.c_int, ctypes.c_int, ctypes.c_float,
                                           ctypes.POINTER(_vp)]),
    "ms_q4_weight_destroy": (ctypes.c_int, [_vp, _vp]),
    "ms_q4_gemm": (ctypes.c_int, [_vp, _vp, _vp, _vp, ctypes.c_int, ctypes.c_int, _vp]),
    "ms_q4_gemm_noalloc": (ctypes.c_int, [_vp, _vp, _vp, _vp, ctypes.c_int, ctypes.c_int, _vp]),
    "ms_model_create": (ctypes.c_int, [_vp, ctypes.POINTER(ModelDesc), ctypes.POINTER(_vp)]),
    "ms_model_destroy": (ctypes.c_int, [_vp, _vp]),
    "ms_model_weight_bytes": (ctypes.c_size_t, [_vp]),
    "ms_file_check": (ctypes.c_int, [ctypes.c_char_p, ctypes.POINTER(FileInfo), ctypes.c_char_p,
                                     ctypes.c_size_t]),
    "ms_model_load": (ctypes.c_int, [_vp, ctypes.c_char_p, ctypes.c_char_p,
                                     ctypes.POINTER(LoadOpts), ctypes.POINTER(_vp)]),
    "ms_load_stats": (ctypes.c_int, [_vp, ctypes.POINTER(ctypes.c_double),
                                     ctypes.POINTER(ctypes.c_uint64)]),
    "ms_kv_create": (ctypes.c_int, [_vp, _vp, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                    ctypes.POINTER(_vp)]),
    "ms_kv_create_typed": (ctypes.c_int, [_vp, _vp, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                          ctypes.c_int, ctypes.POINTER(_vp)]),
    "ms_kv_create_pooled": (ctypes.c_int, [_vp, _vp, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                           ctypes.c_int, ctypes.c_int, ctypes.POINTER(_vp)]),
    "ms_kv_release": (ctypes.c_int, [_vp, _vp, ctypes.c_int]),
    "ms_kv_share_prefix": (ctypes.c_int, [_vp, _vp, ctypes.c_int, ctypes.c_int, ctypes.c_int]),
    "ms_kv_pages": (ctypes.c_int, [_vp, ctypes.POINTER(ctypes.c_int),
                                   ctypes.POINTER(ctypes.c_int)]),
    "ms_kv_allow_window_overwrite": (ctypes.c_int, [_vp, _vp, ctypes.c_int]),
    "ms_kv_destroy": (ctypes.c_int, [_vp, _vp]),
    "ms_kv_reset": (ctypes.c_int, [_vp, _vp]),
    "ms_kv_bytes": (ctypes.c_size_t, [_vp]),
    "ms_kv_write": (ctypes.c_int, [_vp, _vp, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                   ctypes.c_int, _vp, _vp, _vp]),
    "ms_kv_read": (ctypes.c_int, [_vp, _vp, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                  ctypes.c_int, _vp, _vp, _vp]),
    "ms_layer_forward": (ctypes.c_int, [_vp, _vp, ctypes.c_int, _vp, _vp, _ip, _ip,
                                        ctypes.c_int, _vp]),
    "ms_forward": (ctypes.c_int, [_vp, _vp, _vp, _vp, _ip, _ip, ctypes.c_int, _vp]),
    "ms_embed": (ctypes.c_int, [_vp, _vp, _ip, ctypes.c_int, _vp, _vp]),
    "ms_lm_head": (ctypes.c_int, [_vp, _vp, _vp, ctypes.c_int, _vp, _vp, _vp]),
    "ms_decode_step": (ctypes.c_int, [_vp, _vp, _vp, _ip, _ip, _ip, ctypes.c_int, _ip]),
    "ms_generate": (ctypes.c_int, [_vp, _vp, _vp, _ip, _ip, _ip, ctypes.c_int, ctypes.c_int,
                                   _ip, _fp]),
    "ms_ctx_stream": (_vp, [_vp]),
    "ms_prefill": (ctypes.c_int, [_vp, _vp, _vp, _ip, _ip, _ip, ctypes.c_int, _ip]),
    "ms_sample": (ctypes.c_int, [_vp, _vp, ctypes.c_int, ctypes.c_int, _vp, _vp, ctypes.c_float,
                                 ctypes.c_float, _vp, _vp, _vp]),
    "ms_set_sampling": (ctypes.c_int, [_vp, _vp, ctypes.c_float, ctypes.c_float,
                                       ctypes.c_uint64]),
    "ms_tp_unique_id_bytes": (ctypes.c_size_t, []),
    "ms_tp_unique_id": (ctypes.c_int, [_vp, ctypes.c_size_t]),
    "ms_tp_init": (ctypes.c_int, [_vp, ctypes.c_int, ctypes.c_int, _vp]),
    "ms_tp_world": (ctypes.c_int, [_vp]),
}

_lib = None


class MsError(RuntimeError):
    """A non-zero ms_status, with the context's last error message."""

    def __init__(self, status, message):
        self.status = status
        self.name = STATUS_NAMES.get(status, str(status))
        super().__init__(f"{self.name}: {message}")


def lib():
    """Load the library once; raise if it is missing (no CPU fallback exists)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise ImportError(
                f"{LIB_PATH} is missing: build it with `python -m mojostream_b200.build` "
                "(nvcc, sm_100a)")
        L = ctypes.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(L, name)  # AttributeError if a declared symbol is missing
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def check(status, ctx=None):
    if status != MS_OK:
        msg = lib().ms_last_error(ctx).decode() if ctx else ""
        raise MsError(status, msg)


def int_array(values):
    arr = (ctypes.c_int * len(values))(*[int(v) for v in values])
    return arr
