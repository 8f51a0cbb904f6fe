"""ctypes binding of the native library (include/wc_t5cuda.h, include/wc_codec.h).

The library is built in-tree by `witchcraft_b200.build`; loading fails loudly
when it is missing.  There is no CPU fallback anywhere in this package.
"""
from __future__ import annotations

import ctypes
import os
import re

HERE = os.path.dirname(os.path.abspath(__file__))
# WC_T5CUDA_LIB names another build of the same library (A/B measurements)
LIB_PATH = os.environ.get("WC_T5CUDA_LIB") or os.path.join(HERE, "libwc_t5cuda.so")
INCLUDE = os.path.join(os.path.dirname(HERE), "include")
HEADER = os.path.join(INCLUDE, "wc_t5cuda.h")

WC_OK = 0
WC_W_F16_CLIPPED = 1
ERRORS = {-1: "WC_E_INVALID_ARG", -2: "WC_E_GGUF", -3: "WC_E_UNSUPPORTED", -4: "WC_E_CUDA",
          -5: "WC_E_TIMEOUT", -6: "WC_E_CONFIG"}

_lib = None

c_void_p, c_int, c_int64, c_size_t = ctypes.c_void_p, ctypes.c_int, ctypes.c_int64, ctypes.c_size_t
_P = ctypes.POINTER

_SIGNATURES = {
    "wc_t5_device_count": (c_int, []),
    "wc_t5_create": (c_int, [c_int, c_void_p, c_size_t, ctypes.c_char_p, _P(c_void_p)]),
    "wc_t5_destroy": (c_int, [c_void_p]),
    "wc_t5_last_error": (ctypes.c_char_p, [c_void_p]),
    "wc_t5_forward": (c_int, [c_void_p, c_void_p, c_void_p, c_int, c_int, c_void_p, c_void_p, c_void_p]),
    "wc_t5_forward_device": (c_int, [c_void_p, c_void_p, c_void_p, c_int, c_int, c_void_p, c_void_p, c_void_p,
                                     c_void_p]),
    "wc_t5_forward_device_noalloc": (c_int, [c_void_p, c_void_p, c_void_p, c_int, c_int, c_void_p, c_void_p,
                                             c_void_p, c_void_p]),
    "wc_t5_sync": (c_int, [c_void_p, c_void_p]),
    "wc_t5_forward_many": (c_int, [c_void_p, c_int, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p]),
    "wc_t5_forward_many_device": (c_int, [c_void_p, c_int, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p,
                                          c_void_p, c_void_p]),
    "wc_host_alloc": (c_void_p, [c_size_t]),
    "wc_host_free": (None, [c_void_p]),
    "wc_t5_dims": (c_int, [c_void_p, _P(c_int), _P(c_int), _P(c_int), _P(c_int)]),
    "wc_q4k_dequant": (c_int, [c_void_p, c_int64, c_void_p, c_void_p]),
    "wc_q4k_dequant_f16": (c_int, [c_void_p, c_int64, c_void_p, c_void_p]),
    "wc_gemm_q4k": (c_int, [c_void_p, c_int, c_int, c_void_p, c_void_p, c_int, c_int, c_void_p, c_void_p]),
    "wc_gemm_f16": (c_int, [c_void_p, c_int, c_int, c_void_p, c_void_p, c_int, c_int, c_void_p, c_void_p]),
    "wc_attention": (c_int, [c_void_p, c_int, c_int, c_int, c_void_p, c_void_p, c_int, c_int, c_void_p, c_void_p]),
    "wc_t5_relative_bucket": (c_int, [c_int, c_int, c_int, c_int]),
    "wc_selftest_wait_timeout": (c_int, [ctypes.c_uint64]),
    "wc_packed_bound": (c_int64, [c_void_p, c_int, c_int]),
    "wc_pack_embeddings_device": (c_int, [c_void_p, c_void_p, c_int, c_int, c_void_p, c_int64, c_void_p, c_void_p]),
    "wc_pack_embeddings": (c_int, [c_void_p, c_void_p, c_int, c_int, c_void_p, c_int64, c_void_p, c_int]),
    "wc_unpack_embeddings_device": (c_int, [c_void_p, c_void_p, c_void_p, c_int, c_int, c_void_p, c_int64, c_void_p,
                                            c_void_p]),
    "wc_unpack_embeddings": (c_int, [c_void_p, c_void_p, c_int, c_int, c_void_p, c_int64, c_void_p, c_int]),
    "wc_codec_last_error": (ctypes.c_char_p, []),
    "wc_assign_centers": (c_int, [c_void_p, c_int64, c_void_p, c_int64, c_int, c_void_p, c_void_p]),
    "wc_kmeans_update": (c_int, [c_void_p, c_int64, c_int, c_void_p, c_int64, c_void_p, c_void_p, c_void_p,
                                 c_void_p]),
    "wc_residual_q4": (c_int, [c_void_p, c_int64, c_int, c_void_p, c_void_p, c_void_p, c_void_p]),
    "wc_index_last_error": (ctypes.c_char_p, []),
    "wc_score_candidates": (c_int, [c_void_p, c_int, c_int, c_void_p, c_void_p, c_void_p, c_int, c_void_p, c_int64,
                                    c_void_p, c_void_p, c_void_p, c_void_p, c_int64, c_void_p, c_void_p, c_void_p]),
    "wc_q4_table": (c_int, [c_void_p]),
    "wc_similarities": (c_int, [c_void_p, c_int, c_void_p, c_int64, c_int, c_void_p, c_void_p]),
    "wc_query_last_error": (ctypes.c_char_p, []),
}


class WcError(RuntimeError):
    def __init__(self, code: int, msg: str):
        super().__init__(f"{ERRORS.get(code, code)}: {msg}")
        self.code = code


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise ImportError(f"{LIB_PATH} is not built; run `python -m witchcraft_b200.build`")
        l = ctypes.CDLL(LIB_PATH)
        for name, (res, args) in _SIGNATURES.items():
            f = getattr(l, name)
            f.restype = res
            f.argtypes = args
        _lib = l
    return _lib


def header_symbols() -> list[str]:
    """Function names declared in include/*.h."""
    names = set()
    for f in sorted(os.listdir(INCLUDE)):
        if f.endswith(".h"):
            names.update(re.findall(r"\b(wc_[a-z0-9_]+)\s*\(", open(os.path.join(INCLUDE, f)).read()))
    return sorted(names)


class F16ClipWarning(RuntimeWarning):
    """A forward clipped an f16 activation to +-65504 (WC_W_F16_CLIPPED): its
    outputs were written but may deviate from the f32 reference."""


def check(code: int, handle=None) -> None:
    if code == WC_W_F16_CLIPPED:
        import warnings
        msg = lib().wc_t5_last_error(handle)
        warnings.warn(msg.decode() if msg else "f16 activation clipped", F16ClipWarning, stacklevel=3)
        return
    if code != WC_OK:
        msg = lib().wc_t5_last_error(handle)
        raise WcError(code, msg.decode() if msg else "")
