"""ctypes front end of the CPU oracle (liboracle.so, built from af2_oracle.c).

TEST INFRASTRUCTURE ONLY: the parity checker and the CPU baseline. Only the
tests, ``__graft_entry__.smoke()`` and bench.py's CPU-baseline leg import this
module; the product package never does.
"""
from __future__ import annotations

import ctypes
import os
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB_PATH = HERE / "liboracle.so"

_f32p = ctypes.POINTER(ctypes.c_float)
_i8p = ctypes.POINTER(ctypes.c_int8)
_u16p = ctypes.POINTER(ctypes.c_uint16)
_f64p = ctypes.POINTER(ctypes.c_double)
_i64 = ctypes.c_int64

_lib = None


def build() -> Path:
    """Compile liboracle.so with the committed Makefile (system gcc + OpenMP)."""
    subprocess.run(["make", "-s", "-C", str(HERE)], check=True)
    return LIB_PATH


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            build()
        _lib = ctypes.CDLL(str(LIB_PATH))
        _lib.af2o_f16_bits.restype = ctypes.c_uint16
        _lib.af2o_f16_bits.argtypes = [ctypes.c_float]
        _lib.af2o_f16_value.restype = ctypes.c_double
        _lib.af2o_f16_value.argtypes = [ctypes.c_uint16]
        _lib.af2o_quantize_q8_block.argtypes = [_f32p, _i64, _i64, _i8p, _u16p]
        _lib.af2o_dequant_q8_block.argtypes = [_i8p, _u16p, _i64, _i64, _f32p]
        _lib.af2o_quantize_q8_columns.argtypes = [_f32p, _i64, _i64, _i8p, _f32p]
        _lib.af2o_dequant_q8_columns.argtypes = [_i8p, _f32p, _i64, _i64, _f32p]
        _lib.af2o_triangle_weight_count.restype = _i64
        _lib.af2o_triangle_weight_count.argtypes = [_i64, _i64]
        _lib.af2o_triangle.restype = ctypes.c_int
        _lib.af2o_triangle.argtypes = [ctypes.c_int, _i64, _i64, _i64, _f32p, _f32p, _f32p,
                                       ctypes.c_double, _f32p, ctypes.c_int]
        _lib.af2o_opm_weight_count.restype = _i64
        _lib.af2o_opm_weight_count.argtypes = [_i64, _i64, _i64]
        _lib.af2o_outer_product_mean.restype = ctypes.c_int
        _lib.af2o_outer_product_mean.argtypes = [_i64, _i64, _i64, _i64, _i64, _f32p, _f32p, _f32p,
                                                 ctypes.c_double, ctypes.c_double, _f32p, ctypes.c_int]
        _lib.af2o_transition_weight_count.restype = _i64
        _lib.af2o_transition_weight_count.argtypes = [_i64, _i64]
        _lib.af2o_transition.restype = ctypes.c_int
        _lib.af2o_transition.argtypes = [_i64, _i64, _i64, _f32p, _f32p, ctypes.c_double,
                                         ctypes.c_int, _f32p, ctypes.c_int]
        _lib.af2o_error_metrics.restype = ctypes.c_int
        _lib.af2o_error_metrics.argtypes = [_f32p, _f32p, _i64, _f64p]
    return _lib


def _ptr(a: np.ndarray, ctype):
    return a.ctypes.data_as(ctypes.POINTER(ctype))


def _f32(a) -> np.ndarray:
    return np.ascontiguousarray(a, dtype=np.float32)


def default_threads() -> int:
    return os.cpu_count() or 1


def f16_bits(values) -> np.ndarray:
    """numberToFloat16 (src/runtime/float16.ts:5-29) for every element."""
    f = lib().af2o_f16_bits
    flat = _f32(values).ravel()
    return np.array([f(float(v)) for v in flat], dtype=np.uint16).reshape(np.shape(values))


def f16_value(bits) -> np.ndarray:
    f = lib().af2o_f16_value
    flat = np.asarray(bits, dtype=np.uint16).ravel()
    return np.array([f(int(b)) for b in flat], dtype=np.float64).reshape(np.shape(bits))


def quantize_q8_block(w, block: int = 64):
    w = _f32(w).ravel()
    codes = np.zeros(w.size, np.int8)
    scales = np.zeros((w.size + block - 1) // block, np.uint16)
    lib().af2o_quantize_q8_block(_ptr(w, ctypes.c_float), w.size, block, _ptr(codes, ctypes.c_int8),
                                 _ptr(scales, ctypes.c_uint16))
    return codes, scales


def dequant_q8_block(codes, scales, block: int = 64) -> np.ndarray:
    codes = np.ascontiguousarray(codes, np.int8).ravel()
    scales = np.ascontiguousarray(scales, np.uint16).ravel()
    out = np.zeros(codes.size, np.float32)
    lib().af2o_dequant_q8_block(_ptr(codes, ctypes.c_int8), _ptr(scales, ctypes.c_uint16), codes.size,
                                block, _ptr(out, ctypes.c_float))
    return out


def quantize_q8_columns(w):
    """w is [inner, cols] ([in, out]); one f32 scale per output column."""
    w = _f32(w)
    inner, cols = w.shape
    codes = np.zeros((inner, cols), np.int8)
    scales = np.zeros(cols, np.float32)
    lib().af2o_quantize_q8_columns(_ptr(w, ctypes.c_float), inner, cols, _ptr(codes, ctypes.c_int8),
                                   _ptr(scales, ctypes.c_float))
    return codes, scales


def dequant_q8_columns(codes, scales) -> np.ndarray:
    codes = np.ascontiguousarray(codes, np.int8)
    scales = _f32(scales)
    inner, cols = codes.shape
    out = np.zeros((inner, cols), np.float32)
    lib().af2o_dequant_q8_columns(_ptr(codes, ctypes.c_int8), _ptr(scales, ctypes.c_float), inner, cols,
                                  _ptr(out, ctypes.c_float))
    return out


def triangle_weight_count(cz: int, ch: int) -> int:
    return int(lib().af2o_triangle_weight_count(cz, ch))


def triangle(direction: int, z, mask, packed, eps: float = 1e-5, threads: int | None = None) -> np.ndarray:
    """Triangle multiplication (0 outgoing, 1 incoming) without residual; z [n,n,cz]."""
    z = _f32(z)
    n, n2, cz = z.shape
    assert n == n2
    mask = _f32(mask)
    packed = _f32(packed)
    ch = _hidden_from_count(cz, packed.size)
    out = np.zeros_like(z)
    rc = lib().af2o_triangle(direction, n, cz, ch, _ptr(z, ctypes.c_float), _ptr(mask, ctypes.c_float),
                             _ptr(packed, ctypes.c_float), eps, _ptr(out, ctypes.c_float),
                             threads or default_threads())
    if rc != 0:
        raise RuntimeError(f"oracle triangle failed ({rc})")
    return out


def _hidden_from_count(cz: int, count: int) -> int:
    # count = 2cz + 4(ch cz + ch) + 2ch + (cz ch + cz) + (cz^2 + cz) is linear in ch.
    base = 2 * cz + cz + cz * cz + cz
    per = 4 * cz + 4 + 2 + cz
    ch, rem = divmod(count - base, per)
    if rem or ch <= 0:
        raise ValueError(f"{count} packed weights do not fit c_z={cz}")
    return ch


def outer_product_mean(m, mask, packed, c: int, cz: int, ln_eps: float = 1e-5, norm_eps: float = 1e-3,
                       threads: int | None = None) -> np.ndarray:
    m = _f32(m)
    s, n, cm = m.shape
    mask = _f32(mask)
    packed = _f32(packed)
    assert packed.size == lib().af2o_opm_weight_count(cm, c, cz)
    out = np.zeros((n, n, cz), np.float32)
    rc = lib().af2o_outer_product_mean(s, n, cm, c, cz, _ptr(m, ctypes.c_float), _ptr(mask, ctypes.c_float),
                                       _ptr(packed, ctypes.c_float), ln_eps, norm_eps,
                                       _ptr(out, ctypes.c_float), threads or default_threads())
    if rc != 0:
        raise RuntimeError(f"oracle OPM failed ({rc})")
    return out


def transition(x, packed, hidden: int, eps: float = 1e-5, residual: bool = False,
               threads: int | None = None) -> np.ndarray:
    x = _f32(x)
    rows, c = x.shape
    packed = _f32(packed)
    assert packed.size == lib().af2o_transition_weight_count(c, hidden)
    out = np.zeros_like(x)
    rc = lib().af2o_transition(rows, c, hidden, _ptr(x, ctypes.c_float), _ptr(packed, ctypes.c_float), eps,
                               1 if residual else 0, _ptr(out, ctypes.c_float), threads or default_threads())
    if rc != 0:
        raise RuntimeError(f"oracle transition failed ({rc})")
    return out


def error_metrics(actual, expected) -> dict:
    """errorMetrics (src/triangle/types.ts:91-110)."""
    a = _f32(actual).ravel()
    e = _f32(expected).ravel()
    if a.size != e.size or a.size == 0:
        raise ValueError("error metrics require equally sized, non-empty arrays")
    out = np.zeros(3, np.float64)
    lib().af2o_error_metrics(_ptr(a, ctypes.c_float), _ptr(e, ctypes.c_float), a.size, _ptr(out, ctypes.c_double))
    return {"meanAbsoluteError": out[0], "maxAbsoluteError": out[1], "rootMeanSquareError": out[2]}
