"""ctypes binding of ``libdiffucore_b200.so`` (declared in ``include/diffucore_b200.h``).

Loading is lazy and loud: a missing or unloadable library raises :class:`NativeLibraryError`
with the reason; nothing in this package falls back to another implementation.
Every wrapper raises ``RuntimeError`` with the library's ``dc_last_error()`` text when a call
returns a non-zero status.
"""

from __future__ import annotations

import ctypes
import threading
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "libdiffucore_b200.so"

DC_OK = 0
DTYPE_F32, DTYPE_F16, DTYPE_BF16, DTYPE_I8, DTYPE_I32 = 0, 1, 2, 3, 4
GELU_NONE, GELU_ERF, GELU_TANH = 0, 1, 2
MODE_REF, MODE_BLOCK64 = 0, 1
QDIV_IEEE, QDIV_FULL = 0, 1
ABI_VERSION = 1
NOALLOC_SCRATCH_BYTES = 32 << 20

_c_i64 = ctypes.c_int64
_c_p = ctypes.c_void_p
_c_i64p = ctypes.POINTER(ctypes.c_int64)

# name -> (restype, argtypes)
_SIGNATURES = {
    "dc_version": (ctypes.c_int, []),
    "dc_last_error": (ctypes.c_char_p, []),
    "dc_set_quant_division": (ctypes.c_int, [ctypes.c_int]),
    "dc_quant_division": (ctypes.c_int, []),
    "dc_device_error": (ctypes.c_int, [ctypes.POINTER(ctypes.c_uint), ctypes.c_int]),
    "dc_quant_rows": (ctypes.c_int, [_c_p, ctypes.c_int, _c_i64, _c_i64, _c_i64, ctypes.c_int, ctypes.c_int,
                                     _c_p, _c_p, _c_p]),
    "dc_gemm_w8a8": (ctypes.c_int, [_c_p, _c_i64, _c_p, _c_i64, _c_p, _c_p, _c_p, _c_p, _c_i64, ctypes.c_int,
                                    _c_i64, _c_i64, _c_i64, ctypes.c_int, _c_p]),
    "dc_gemm_w8a8_ex": (ctypes.c_int, [_c_p, _c_i64, _c_p, _c_i64, _c_p, _c_p, _c_p, ctypes.c_int, _c_p, _c_p,
                                       _c_i64, _c_p, _c_i64, _c_i64, _c_i64, ctypes.c_int, _c_i64, _c_i64, _c_i64,
                                       _c_p]),
    "dc_quant_rows_seg": (ctypes.c_int, [_c_p, ctypes.c_int, _c_i64, _c_i64, _c_i64, _c_i64, _c_i64, _c_i64, _c_p,
                                         _c_i64, ctypes.c_int, _c_p, _c_p, _c_p]),
    "dc_ln_mod_quant": (ctypes.c_int, [_c_p, ctypes.c_int, _c_i64, _c_i64, _c_i64, _c_p, _c_p, _c_i64, _c_i64,
                                       ctypes.c_int, _c_p, _c_p, _c_p]),
    "dc_qk_norm_rope": (ctypes.c_int, [_c_p, ctypes.c_int, _c_i64, _c_i64, _c_i64, _c_i64, _c_i64, _c_i64, _c_p,
                                       _c_p, _c_p, _c_p, _c_i64, _c_p, _c_i64, _c_p]),
    "dc_qk_norm_rope_q8": (ctypes.c_int, [_c_p, ctypes.c_int, _c_i64, _c_i64, _c_i64, _c_i64, _c_i64, _c_i64, _c_p,
                                          _c_p, _c_p, _c_p, _c_i64, _c_p, _c_i64, _c_p, _c_p, _c_i64, ctypes.c_int,
                                          _c_p]),
    "dc_rescale": (ctypes.c_int, [_c_p, _c_i64, _c_p, _c_p, _c_p, _c_p, _c_i64, ctypes.c_int, _c_i64, _c_i64,
                                  _c_p]),
    "dc_attn_workspace_size": (ctypes.c_int, [_c_i64, _c_i64, _c_i64, _c_i64, _c_i64, ctypes.c_int,
                                              ctypes.POINTER(ctypes.c_size_t)]),
    "dc_attn_workspace_layout": (ctypes.c_int, [_c_i64, _c_i64, _c_i64, _c_i64, _c_i64, ctypes.c_int, _c_i64p]),
    "dc_attn_int8_fwd": (ctypes.c_int, [_c_p, _c_p, _c_p, ctypes.c_int, _c_i64, _c_i64, _c_i64, _c_i64, _c_i64,
                                        _c_i64p, _c_i64p, _c_i64p, ctypes.c_float, ctypes.c_int, _c_p, _c_i64p,
                                        _c_p, ctypes.c_size_t, _c_p]),
    "dc_attn_int8_prep": (ctypes.c_int, [_c_p, _c_p, ctypes.c_int, _c_i64, _c_i64, _c_i64, _c_i64, _c_i64,
                                         _c_i64p, _c_i64p, ctypes.c_int, _c_p, ctypes.c_size_t, _c_p]),
    "dc_attn_int8_prep_k": (ctypes.c_int, [_c_p, ctypes.c_int, _c_i64, _c_i64, _c_i64, _c_i64, _c_i64, _c_i64p,
                                           ctypes.c_int, _c_p, ctypes.c_size_t, _c_p]),
    "dc_attn_int8_main": (ctypes.c_int, [_c_p, ctypes.c_int, _c_i64, _c_i64, _c_i64, _c_i64, _c_i64, _c_i64p,
                                         ctypes.c_float, ctypes.c_int, _c_p, _c_i64p, _c_p, ctypes.c_size_t, _c_p]),
    "dc_attn_split_partials_size": (ctypes.c_int, [_c_i64, _c_i64, _c_i64, _c_i64, _c_i64, ctypes.c_int,
                                                   ctypes.POINTER(ctypes.c_size_t)]),
    "dc_attn_int8_main_split": (ctypes.c_int, [_c_p, ctypes.c_int, _c_i64, _c_i64, _c_i64, _c_i64, _c_i64, _c_i64p,
                                               ctypes.c_float, ctypes.c_int, _c_p, _c_i64p, _c_p, ctypes.c_size_t,
                                               ctypes.c_int, _c_p, ctypes.c_size_t, _c_p]),
    "dc_attn_int8_fwd_noalloc": (ctypes.c_int, [_c_p, _c_p, _c_p, ctypes.c_int, _c_i64, _c_i64, _c_i64, _c_i64,
                                                _c_i64, _c_i64p, _c_i64p, _c_i64p, ctypes.c_float, ctypes.c_int,
                                                _c_p, _c_i64p, _c_p]),
    "dc_selftest_exp2": (ctypes.c_int, [_c_p, _c_p, _c_p, _c_i64, _c_p]),
    "dc_selftest_wait_timeout": (ctypes.c_int, [ctypes.c_longlong, _c_p, _c_p]),
}

EXPORTED = tuple(_SIGNATURES)


class NativeLibraryError(RuntimeError):
    """The sm_100a library is missing or cannot be loaded."""


_lock = threading.Lock()
_lib: ctypes.CDLL | None = None


def load() -> ctypes.CDLL:
    """The loaded library (loaded once per process)."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is not None:
            return _lib
        if not LIB_PATH.exists():
            raise NativeLibraryError(
                f"{LIB_PATH.name} is not built; run `python -m diffucore_b200.build` (needs nvcc 12.8+)")
        try:
            lib = ctypes.CDLL(str(LIB_PATH))
        except OSError as e:
            raise NativeLibraryError(f"cannot load {LIB_PATH}: {e}") from e
        for name, (res, args) in _SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        if lib.dc_version() != ABI_VERSION:
            raise NativeLibraryError(f"{LIB_PATH.name} has ABI {lib.dc_version()}, expected {ABI_VERSION}")
        _lib = lib
        return lib


def check(status: int) -> None:
    if status != DC_OK:
        msg = load().dc_last_error().decode(errors="replace")
        raise RuntimeError(f"diffucore_b200: {msg}")


def i64_array(values) -> ctypes.Array:
    vals = [int(v) for v in values]
    return (ctypes.c_int64 * len(vals))(*vals)


def device_error(clear: bool = True) -> int:
    """The device-global error word set by bounded in-kernel waits (0 = none)."""
    code = ctypes.c_uint(0)
    check(load().dc_device_error(ctypes.byref(code), 1 if clear else 0))
    return int(code.value)
