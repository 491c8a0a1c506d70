"""numpy front of ``oracle/dc_oracle.c`` (TEST INFRASTRUCTURE ONLY; see ``oracle/__init__.py``).

16-bit floats travel as ``np.uint16`` bit patterns with a dtype tag ("bf16" / "f16"); fp32 as
``np.float32``. (B, L, H, D) attention inputs may be strided views; strides pass in elements.
"""

from __future__ import annotations

import ctypes
import os
import subprocess
import threading
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
SRC = HERE / "dc_oracle.c"
LIB = HERE / "liboracle.so"
_DT = {"f32": 0, "f16": 1, "bf16": 2}
_lock = threading.Lock()
_lib = None


def build(force: bool = False) -> Path:
    """Compile the oracle with gcc (OpenMP, no FP contraction) unless up to date."""
    if not force and LIB.exists() and LIB.stat().st_mtime >= SRC.stat().st_mtime:
        return LIB
    tmp = LIB.with_suffix(".so.tmp")
    cmd = ["gcc", "-O2", "-fopenmp", "-ffp-contract=off", "-shared", "-fPIC", "-o", str(tmp), str(SRC), "-lm"]
    subprocess.run(cmd, check=True, capture_output=True, text=True)
    os.replace(tmp, LIB)
    return LIB


def _load():
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            build()
            lib = ctypes.CDLL(str(LIB))
            for name in ("or_quant_rows", "or_int_mm", "or_rescale", "or_attn_ksum", "or_attn_block_quant",
                         "or_attn_token_quant", "or_attn_from_codes", "or_attn_exact", "or_hadamard256",
                         "or_round_to", "or_to_float"):
                getattr(lib, name).restype = None
            _lib = lib
    return _lib


def _p(a: np.ndarray | None):
    return ctypes.c_void_p(0 if a is None else a.ctypes.data)


def _i64s(vals):
    vals = [int(v) for v in vals]
    return (ctypes.c_int64 * len(vals))(*vals)


def set_threads(n: int) -> None:
    """Thread count of the OpenMP regions (affects speed only, never results)."""
    os.environ["OMP_NUM_THREADS"] = str(int(n))
    try:
        gomp = ctypes.CDLL("libgomp.so.1")
        gomp.omp_set_num_threads(ctypes.c_int(int(n)))
    except OSError:
        pass


# ─── 16-bit float helpers ───────────────────────────────────────────────────────────────

def to_bits(x: np.ndarray, dtype: str) -> np.ndarray:
    """Round fp32 ``x`` to bf16 / f16 (round-half-even) and return the bit patterns."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    out = np.empty(x.shape, dtype=np.uint16)
    _load().or_round_to(_p(x), ctypes.c_int64(x.size), _DT[dtype], _p(out))
    return out


def to_float(bits: np.ndarray, dtype: str) -> np.ndarray:
    bits = np.ascontiguousarray(bits, dtype=np.uint16)
    out = np.empty(bits.shape, dtype=np.float32)
    _load().or_to_float(_p(bits), ctypes.c_int64(bits.size), _DT[dtype], _p(out))
    return out


def _elem_strides(a: np.ndarray):
    return [s // a.itemsize for s in a.strides]


# ─── quantizer / GEMM / rescale ─────────────────────────────────────────────────────────

def quant_rows(x: np.ndarray, dtype: str, group: int = 0, gelu: int = 0):
    """``(int8 [M, K], fp32 [M])``; ``x`` is [M, K] uint16 bits (bf16/f16) or float32 (f32)."""
    if x.ndim != 2 or x.strides[1] != x.itemsize:
        x = np.ascontiguousarray(x)
    M, K = x.shape
    q = np.empty((M, K), dtype=np.int8)
    s = np.empty(M, dtype=np.float32)
    _load().or_quant_rows(_p(x), _DT[dtype], ctypes.c_int64(M), ctypes.c_int64(K),
                          ctypes.c_int64(x.strides[0] // x.itemsize), group, gelu, _p(q), _p(s))
    return q, s


def hadamard256(x: np.ndarray, width: int = 3072) -> np.ndarray:
    """The library's butterfly rotation of one 256-wide fp32 group of a row ``width`` elements wide
    (the width selects the summation order of the reference's Triton butterfly)."""
    y = np.array(x, dtype=np.float32, copy=True)
    _load().or_hadamard256(_p(y), ctypes.c_int64(width))
    return y


def int_mm(q: np.ndarray, w: np.ndarray) -> np.ndarray:
    q = np.ascontiguousarray(q, dtype=np.int8)
    w = np.ascontiguousarray(w, dtype=np.int8)
    M, K = q.shape
    N = w.shape[0]
    out = np.empty((M, N), dtype=np.int32)
    _load().or_int_mm(_p(q), _p(w), ctypes.c_int64(M), ctypes.c_int64(N), ctypes.c_int64(K), _p(out))
    return out


def rescale(acc: np.ndarray, sx: np.ndarray, sw: np.ndarray, bias: np.ndarray | None, dtype: str,
            gelu: int = 0) -> np.ndarray:
    """uint16 bits of ``dtype(acc * (sx * sw))`` (+ bias, + GELU), the reference's rounding."""
    acc = np.ascontiguousarray(acc, dtype=np.int32)
    sx = np.ascontiguousarray(sx, dtype=np.float32)
    sw = np.ascontiguousarray(sw, dtype=np.float32)
    bias = None if bias is None else np.ascontiguousarray(bias, dtype=np.uint16)
    M, N = acc.shape
    out = np.empty((M, N), dtype=np.uint16)
    _load().or_rescale(_p(acc), _p(sx), _p(sw), _p(bias), _DT[dtype], ctypes.c_int64(M), ctypes.c_int64(N),
                       gelu, _p(out))
    return out


def linear(x: np.ndarray, dtype: str, wq: np.ndarray, ws: np.ndarray, bias: np.ndarray | None,
           group: int = 0) -> np.ndarray:
    """Reference ``Int8Linear.forward`` on [M, K] bits: quantize -> int_mm -> rescale."""
    q, s = quant_rows(x, dtype, group)
    return rescale(int_mm(q, wq), s, ws, bias, dtype)


# ─── attention ──────────────────────────────────────────────────────────────────────────

def attn_prep(q: np.ndarray, k: np.ndarray, dtype: str, mode: str = "ref") -> dict:
    """int8 codes and scales of q (B, Lq, H, D) and k (B, Lk, H, D), uint16 bits (views allowed):
    ``q_codes`` [B, H, Lq, D], ``q_scale`` [B, H, Lq] (per row), ``k_codes`` [B, H, Lk, D],
    ``k_scale`` [B, H, ceil(Lk/64)] and, in mode "ref", ``ksum`` [B, H, D]."""
    lib = _load()
    B, Lq, H, D = q.shape
    Lk = k.shape[1]
    nkb = (Lk + 63) // 64
    qs, ks = _i64s(_elem_strides(q)[:3]), _i64s(_elem_strides(k)[:3])
    dt = _DT[dtype]
    out = {"k_codes": np.empty((B, H, Lk, D), np.int8), "k_scale": np.empty((B, H, nkb), np.float32),
           "q_codes": np.empty((B, H, Lq, D), np.int8)}
    c = ctypes.c_int64
    if mode == "ref":
        ksum = np.empty((B, H, D), np.float32)
        lib.or_attn_ksum(_p(k), dt, c(B), c(H), c(Lk), c(D), ks, _p(ksum))
        out["ksum"] = ksum
        lib.or_attn_block_quant(_p(k), dt, c(B), c(H), c(Lk), c(D), ks, _p(ksum), _p(out["k_codes"]),
                                _p(out["k_scale"]))
        out["q_scale"] = np.empty((B, H, Lq), np.float32)
        lib.or_attn_token_quant(_p(q), dt, c(B), c(H), c(Lq), c(D), qs, _p(out["q_codes"]), _p(out["q_scale"]))
    elif mode == "block64":
        lib.or_attn_block_quant(_p(k), dt, c(B), c(H), c(Lk), c(D), ks, None, _p(out["k_codes"]),
                                _p(out["k_scale"]))
        nqb = (Lq + 63) // 64
        qblk = np.empty((B, H, nqb), np.float32)
        lib.or_attn_block_quant(_p(q), dt, c(B), c(H), c(Lq), c(D), qs, None, _p(out["q_codes"]), _p(qblk))
        out["q_scale"] = np.repeat(qblk, 64, axis=2)[:, :, :Lq].copy()
    else:
        raise ValueError(f"unknown mode {mode!r}")
    return out


def attn_int8(q: np.ndarray, k: np.ndarray, v: np.ndarray, dtype: str, sm_scale: float, mode: str = "ref",
              prep: dict | None = None) -> np.ndarray:
    """fp32 (B, Lq, H, D): exact-softmax attention over the int8 codes of ``mode``."""
    prep = prep if prep is not None else attn_prep(q, k, dtype, mode)
    B, Lq, H, D = q.shape
    Lk = k.shape[1]
    out = np.empty((B, Lq, H, D), np.float32)
    c = ctypes.c_int64
    _load().or_attn_from_codes(_p(prep["q_codes"]), _p(prep["q_scale"]), _p(prep["k_codes"]), _p(prep["k_scale"]),
                               _p(v), _DT[dtype], _i64s(_elem_strides(v)[:3]), c(B), c(H), c(Lq), c(Lk), c(D),
                               ctypes.c_double(sm_scale), _p(out))
    return out


def attn_exact(q: np.ndarray, k: np.ndarray, v: np.ndarray, dtype: str, sm_scale: float) -> np.ndarray:
    """fp32 (B, Lq, H, D): unquantized attention in double precision."""
    B, Lq, H, D = q.shape
    Lk = k.shape[1]
    out = np.empty((B, Lq, H, D), np.float32)
    c = ctypes.c_int64
    _load().or_attn_exact(_p(q), _p(k), _p(v), _DT[dtype], _i64s(_elem_strides(q)[:3]), _i64s(_elem_strides(k)[:3]),
                          _i64s(_elem_strides(v)[:3]), c(B), c(H), c(Lq), c(Lk), c(D), ctypes.c_double(sm_scale),
                          _p(out))
    return out


__all__ = ["build", "set_threads", "to_bits", "to_float", "quant_rows", "hadamard256", "int_mm", "rescale", "linear",
           "attn_prep", "attn_int8", "attn_exact"]
