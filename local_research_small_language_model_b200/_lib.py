"""ctypes binding of libspardab200.so (the C ABI declared in include/spardab200.h).

The library is built in-tree by ``python -m local_research_small_language_model_b200.csrc.build``
(``__graft_entry__.build()`` does it too).  There is no fallback: if the shared
library is missing, every op raises.
"""

from __future__ import annotations

import ctypes
import os
import threading

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libspardab200.so")

SD_OK = 0
SD_DTYPE_F32, SD_DTYPE_BF16, SD_DTYPE_F16 = 0, 1, 2
SD_RULE_REFERENCE, SD_RULE_ABSOLUTE = 0, 1
SD_SELECT_BEFORE_APPEND = 0x100
SD_KERR_TIMEOUT = 1

_c_void_p = ctypes.c_void_p
_i64 = ctypes.c_int64
_i32 = ctypes.c_int
_f32 = ctypes.c_float

# name -> argtypes (restype is int for all but sd_strerror)
_SIGS = {
    "sd_version": [],
    "sd_last_cuda_error": [],
    "sd_advance_len": [_c_void_p, _i32, _i32, _c_void_p],
    "sd_set_programmatic_launch": [_i32],
    "sd_decode_sparse_noalloc": [_c_void_p, _i32, _i64, _i64, _c_void_p, _i32, _i64, _i64, _c_void_p, _i64, _i64,
                                 _i64, _c_void_p, _c_void_p, _i64, _i64, _i64, _i64, _i64, _i64, _i64, _i64, _i64,
                                 _i32, _i32, _i32, _f32, _c_void_p, _i64, _i64, _c_void_p, _c_void_p],
    "sd_linear": [_c_void_p, _i32, _i64, _i64, _i64, _c_void_p, _i64, _c_void_p, _f32, _i32, _c_void_p, _i64,
                  _c_void_p, _i64, _c_void_p, _c_void_p],
    "sd_compress_blocks": [_c_void_p, _i32, _i64, _i64, _i64, _i64, _i64, _i64, _i64, _i32, _c_void_p, _c_void_p],
    "sd_select_blocks": [_c_void_p, _i32, _i64, _i64, _i64, _i64, _i64, _i64, _i64, _c_void_p, _i64, _i64, _i64,
                         _i64, _i32, _i32, _i32, _i64, _c_void_p, _c_void_p, _c_void_p],
    "sd_topk_rows": [_c_void_p, _i64, _i64, _i64, _i32, _c_void_p, _c_void_p, _c_void_p],
    "sd_gather_kv_blocks": [_c_void_p, _c_void_p, _i32, _i64, _i64, _i64, _i64, _i64, _i64, _i64, _c_void_p, _i64,
                            _i32, _c_void_p, _c_void_p, _c_void_p],
    "sd_decode_select": [_c_void_p, _i32, _i64, _i64, _c_void_p, _i64, _i64, _i64, _i64, _i64, _i64, _i64, _i32,
                         _i32, _i32, _c_void_p, _c_void_p, _i32, _c_void_p],
    "sd_decode_attention": [_c_void_p, _i32, _i64, _i64, _i64, _i64, _i64, _i64, _c_void_p, _c_void_p, _i64, _i64,
                            _i64, _i64, _c_void_p, _c_void_p, _i32, _i64, _i32, _f32, _c_void_p, _i64, _i64,
                            _c_void_p, _c_void_p],
    "sd_kv_append": [_c_void_p, _c_void_p, _i32, _i64, _i64, _i64, _i64, _i64, _i64, _i64, _i64, _i64, _i64,
                     _c_void_p, _c_void_p, _c_void_p, _i64, _i64, _i64, _i32, _c_void_p],
    "sd_decode_layer": [_c_void_p, _i32, _i64, _c_void_p, _i32, _i64, _c_void_p, _c_void_p, _i64, _c_void_p,
                        _c_void_p, _c_void_p, _c_void_p, _i64, _i64, _i64, _i64, _i64, _i64, _i32, _i32, _i32, _f32,
                        _c_void_p, _i64, _c_void_p, _c_void_p, _c_void_p, _c_void_p, _i32, _c_void_p,
                        _c_void_p, _c_void_p, _i64, _c_void_p, _c_void_p, _c_void_p],
    "sd_decode_candidates": [_c_void_p, _i32, _i64, _c_void_p, _i64, _i64, _i64, _i64, _c_void_p, _i32, _i32, _i32,
                             _f32, _c_void_p, _c_void_p, _c_void_p],
    "sd_prefill_lists": [_i32, _i32, _i64, _i64, _i64, _i32, _i32, _c_void_p, _i32, _c_void_p, _c_void_p, _i32,
                         _c_void_p],
    "sd_prefill_attention": [_c_void_p, _i32, _i64, _i64, _i64, _i64, _i64, _i64, _i64, _i64, _c_void_p, _c_void_p,
                             _i64, _i64, _i64, _c_void_p, _c_void_p, _i32, _c_void_p, _i32, _i32, _i32, _f32,
                             _c_void_p, _i64, _i64, _i64, _c_void_p],
    "sd_prefill_attention_backward": [_c_void_p, _c_void_p, _c_void_p, _c_void_p, _i32, _i64, _i64, _i64, _i64,
                                      _i64, _i64, _i64, _i64, _i64, _i64, _i64, _i64, _i64, _i64, _c_void_p,
                                      _c_void_p, _i32, _c_void_p, _i32, _i32, _i32, _f32, _c_void_p, _c_void_p,
                                      _c_void_p, _c_void_p],
    "sd_rmsnorm": [_c_void_p, _i32, _i64, _i64, _i64, _c_void_p, _f32, _c_void_p, _i64, _c_void_p],
    "sd_silu_mul": [_c_void_p, _i32, _i64, _i64, _i64, _c_void_p, _i64, _c_void_p],
    "sd_argmax_rows": [_c_void_p, _i32, _i64, _i64, _i64, _c_void_p, _i64, _c_void_p],
    "sd_rope_qk": [_c_void_p, _c_void_p, _i32, _i64, _i64, _i64, _i64, _i64, _i64, _i64, _i64, _i64, _i64, _i64,
                   _c_void_p, _c_void_p, _i64, _i64, _c_void_p, _c_void_p, _c_void_p],
    "sd_offload_prefetch": [_c_void_p, _c_void_p, _i32, _i64, _i64, _i64, _i64, _c_void_p, _c_void_p, _i32,
                            _c_void_p, _i32, _i32, _c_void_p, _c_void_p, _c_void_p, _c_void_p, _c_void_p],
    "sd_decode_layer_offload": [_c_void_p, _i32, _i64, _c_void_p, _i32, _i64, _c_void_p, _c_void_p, _i64,
                                _c_void_p, _c_void_p, _c_void_p, _i64, _c_void_p, _c_void_p, _i32, _c_void_p, _i64,
                                _i64, _i64, _i64, _i64, _i32, _i32, _i32, _f32, _c_void_p, _i64, _c_void_p,
                                _c_void_p, _c_void_p, _c_void_p, _c_void_p, _i32, _c_void_p, _c_void_p],
}

# entry points that return something other than an int status
_RESTYPES = {}

_lock = threading.Lock()
_lib = None


class SparDAError(RuntimeError):
    """Raised when a library call returns a non-zero status."""


def exported_symbols():
    """Names of every entry point declared in include/spardab200.h."""
    return ["sd_strerror"] + list(_SIGS)


def load(path: str = LIB_PATH) -> ctypes.CDLL:
    """Loads the shared library once; raises if it was not built."""
    global _lib
    with _lock:
        if _lib is not None:
            return _lib
        if not os.path.exists(path):
            raise SparDAError(
                f"{path} is missing; build it with "
                "`python -m local_research_small_language_model_b200.csrc.build` (needs nvcc)")
        lib = ctypes.CDLL(path)
        lib.sd_strerror.restype = ctypes.c_char_p
        lib.sd_strerror.argtypes = [_i32]
        for name, args in _SIGS.items():
            fn = getattr(lib, name)
            fn.restype = _RESTYPES.get(name, ctypes.c_int)
            fn.argtypes = args
        _lib = lib
        return lib


def call(name: str, *args) -> None:
    """Calls an entry point and raises SparDAError on a non-zero status."""
    lib = load()
    code = getattr(lib, name)(*args)
    if code != SD_OK:
        msg = lib.sd_strerror(code).decode()
        extra = f" (cudaError {lib.sd_last_cuda_error()})" if code == -3 else ""
        raise SparDAError(f"{name} failed: {msg}{extra}")
