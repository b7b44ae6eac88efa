"""ctypes binding of libh24.so (include/h24.h).

The library is the only implementation of the hot path: if it is missing or a
call fails, an exception is raised -- there is no CPU or PyTorch fallback.
Signatures carry plain device pointers, sizes and a CUDA stream handle.
"""
from __future__ import annotations

import ctypes
import os
import threading

_HERE = os.path.dirname(os.path.abspath(__file__))
# H24_LIBRARY selects another build of the same library (e.g. a tuning variant).
LIB_PATH = os.environ.get("H24_LIBRARY") or os.path.join(_HERE, "_lib", "libh24.so")

H24_OK = 0
H24_ERR_INVALID = 1
H24_ERR_CUDA = 2
H24_ERR_RANGE = 3
H24_ERR_TIMEOUT = 4
H24_ERR_STATE = 5
RULE_TRAIN = 0
RULE_PACK = 1
DTYPE_F32, DTYPE_F16, DTYPE_BF16 = 0, 1, 2
KERNEL_SCREEN, KERNEL_RESCORE, KERNEL_PREP = 0, 1, 2

# Every symbol include/h24.h declares, with (restype, argtypes).
_P = ctypes.c_void_p
_I64 = ctypes.c_int64
_I = ctypes.c_int
SIGNATURES = {
    "h24_last_error": (ctypes.c_char_p, []),
    "h24_version": (ctypes.c_char_p, []),
    "h24_init": (_I, [_I]),
    "h24_codebook_raw": (_I, [_P]),
    "h24_codebook_f32": (_I, [_P, _P]),
    "h24_fingerprint": (_I, [_P]),
    "h24_pack": (_I, [_P, _I64, _P, _P]),
    "h24_pack_i64": (_I, [_P, _I64, _P, _P]),
    "h24_unpack": (_I, [_P, _I64, _I64, _P, _P]),
    "h24_unpack_i64": (_I, [_P, _I64, _I64, _P, _P]),
    "h24_dequant": (_I, [_P, _P, _I64, _I64, _P, _P, _P]),
    "h24_dequant_batched": (_I, [_P, _I, _P, _P]),
    "h24_lut_gemv": (_I, [_P, _P, _I64, _I64, _P, _I64, _P, _P, _P]),
    "h24_project_layers": (_I, [_P, _I, _P]),
    "h24_int8_quantize": (_I, [_P, _I64, _I64, _P, _P, _P]),
    "h24_int8_dequant": (_I, [_P, _P, _I64, _I64, _P, _P]),
    "h24_quantize": (_I, [_P, _I64, _I, _P, _P]),
    "h24_quantize_layer": (_I, [_P, _I64, _I64, _P, _P, _P]),
    "h24_quantize_layer_host": (_I, [_P, _I64, _I64, _P, _P, _P]),
    "h24_quantize_segments": (_I, [_P, _P, _I, _I, _P, _P]),
    "h24_quantize_noalloc": (_I, [_P, _I64, _I, _P, _P]),
    "h24_quantize_layers": (_I, [_P, _I, _P]),
    "h24_quantize_typed": (_I, [_P, _I64, _I, _I, _P, _P]),
    "h24_quantize_layer_rows": (_I, [_P, _I, _I, _P]),
    "h24_quantize_layer_rows_host": (_I, [_P, _I, _I, _P]),
    "h24_row_rms": (_I, [_P, _I64, _I64, _I, _P, _P, _P]),
    "h24_launch_count": (ctypes.c_int64, []),
    "h24_gather_codewords": (_I, [_P, _I64, _I, _P, _P]),
    "h24_timing_enable": (_I, [_I]),
    "h24_timing_read": (_I, [ctypes.POINTER(ctypes.c_double), ctypes.POINTER(ctypes.c_int64)]),
    "h24_timing_read_kernel": (_I, [_I, ctypes.POINTER(ctypes.c_double), ctypes.POINTER(ctypes.c_int64)]),
    "h24_quantize_stats": (_I, [ctypes.POINTER(ctypes.c_int64)] * 3 + [_P]),
    "h24_check": (_I, [_P]),
}


class DequantLayer(ctypes.Structure):
    """Mirror of h24_dequant_layer."""
    _fields_ = [("packed", _P), ("sigma16", _P), ("out16", _P),
                ("rows", ctypes.c_int64), ("in_features", ctypes.c_int64)]


class Layer(ctypes.Structure):
    """Mirror of h24_layer."""
    _fields_ = [("w", _P), ("rows", ctypes.c_int64), ("in_features", ctypes.c_int64),
                ("sigma16_out", _P), ("packed_out", _P)]


class LayerRows(ctypes.Structure):
    """Mirror of h24_layer_rows."""
    _fields_ = [("w", _P), ("rows", ctypes.c_int64), ("in_features", ctypes.c_int64),
                ("row_begin", ctypes.c_int64), ("row_end", ctypes.c_int64),
                ("sigma16_out", _P), ("packed_out", _P)]


class ProjectLayer(ctypes.Structure):
    """Mirror of h24_project_layer."""
    _fields_ = [("latent", _P), ("out", _P), ("rows", ctypes.c_int64),
                ("in_features", ctypes.c_int64), ("sigma", _P), ("idx", _P)]


class H24Error(RuntimeError):
    """A libh24 call failed."""


_lib = None
_lock = threading.Lock()


def load() -> ctypes.CDLL:
    """Load libh24.so (raises if it has not been built)."""
    global _lib
    with _lock:
        if _lib is None:
            if not os.path.exists(LIB_PATH):
                raise H24Error(
                    f"libh24.so not found at {LIB_PATH}; build it with `python -m pollux_b200.build`")
            lib = ctypes.CDLL(LIB_PATH)
            for name, (res, args) in SIGNATURES.items():
                fn = getattr(lib, name)
                fn.restype = res
                fn.argtypes = args
            _lib = lib
    return _lib


def check(rc: int, what: str) -> None:
    """Turn a status code into the exception the reference would raise."""
    if rc == H24_OK:
        return
    msg = f"{what}: {(load().h24_last_error() or b'').decode(errors='replace')}"
    if rc == H24_ERR_INVALID:
        raise ValueError(msg)
    if rc == H24_ERR_RANGE:
        raise IndexError(msg)
    raise H24Error(msg)


def call(name: str, *args) -> None:
    check(getattr(load(), name)(*args), name)
