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
_i64p = ctypes.POINTER(ctypes.c_int64)

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
        _lib.af2o_triangle_rows.restype = ctypes.c_int
        _lib.af2o_triangle_rows.argtypes = [ctypes.c_int, _i64, _i64, _i64, _f32p, _f32p, _f32p,
                                            ctypes.c_double, _i64p, _i64, _f32p, ctypes.c_int]
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


def triangle_rows(direction: int, z, mask, packed, rows, eps: float = 1e-5, threads: int | None = None) -> np.ndarray:
    """Output rows `rows` of triangle multiplication (no residual): [len(rows), n, cz].  The
    projections cover every pair; only the listed rows are contracted and projected, each
    element computed exactly as the whole op computes it."""
    z = _f32(z)
    n, n2, cz = z.shape
    assert n == n2
    mask = _f32(mask)
    packed = _f32(packed)
    ch = _hidden_from_count(cz, packed.size)
    sel = np.ascontiguousarray(rows, np.int64)
    out = np.zeros((sel.size, n, cz), np.float32)
    rc = lib().af2o_triangle_rows(direction, n, cz, ch, _ptr(z, ctypes.c_float), _ptr(mask, ctypes.c_float),
                                  _ptr(packed, ctypes.c_float), eps, _ptr(sel, ctypes.c_int64), sel.size,
                                  _ptr(out, ctypes.c_float), threads or default_threads())
    if rc != 0:
        raise RuntimeError(f"oracle triangle rows failed ({rc})")
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


def attention(x, mask, weights: dict, batch: int, queries: int, heads: int, transpose: bool = False,
              pair_bias: dict | None = None, eps: float = 1e-5, residual=None) -> np.ndarray:
    """Gated multi-head attention as AttentionGpu.run computes it (src/evoformer/attention.ts:1334-1453),
    restated in f64 numpy; the reference has no CPU implementation of it, so this follows its kernels.

    x: [batch * queries, channels] rows (transpose=False: row b*Q+q; transpose=True: row q*B+b,
    the column / ending-node view, source_row :300-306); mask: [batch * queries] in the same
    layout (mask_index :428-433).  weights: queryNormScale/Offset [C], query/key/value/gating
    Weight [C, H*d] ([in, out], column h*d+i), gatingBias [H*d], outputWeight [H*d, C],
    outputBias [C].  pair_bias: None; {"source": "normalized-input", "projectionWeight": [C, H]}
    (bias[h, q, k] from the normalized row (q, k) of this same input, which needs batch ==
    queries: triangle attention); or {"source": "separate", "activations": [Q*Q, Cp],
    "layerNormScale", "layerNormOffset", "projectionWeight": [Cp, H]}.
    Steps: LayerNorm (:266-336); q = xn Wq / sqrt(d), k, v, gate = sigmoid(xn Wg + bg)
    (:497-566); logits = q.k + 1e9 (mask[k] - 1) + bias, clamped to +-1e8, softmax over keys,
    times the gate (ATTENTION_FLASH_SHADER :663-731); out = weighted Wo + bo, written back in the
    input's row layout, plus `residual` when given (:1261-1314)."""
    x = np.asarray(x, np.float64)
    rows, c = x.shape
    B, Q, H = batch, queries, heads
    d = c // H
    assert rows == B * Q and d * H == c
    w = {k: np.asarray(v, np.float64) for k, v in weights.items()}
    order = np.arange(rows).reshape(B, Q) if not transpose else np.arange(rows).reshape(Q, B).T
    xs = x[order.ravel()]  # rows in (b, q) order
    mk = np.asarray(mask, np.float64).ravel()[order.ravel()].reshape(B, Q)

    def layer_norm(t, scale, offset):
        mean = t.mean(-1, keepdims=True)
        var = ((t - mean) ** 2).mean(-1, keepdims=True)
        return (t - mean) / np.sqrt(var + eps) * scale + offset

    xn = layer_norm(xs, w["queryNormScale"], w["queryNormOffset"])
    q = (xn @ w["queryWeight"].reshape(c, H * d)).reshape(B, Q, H, d) / np.sqrt(d)
    k = (xn @ w["keyWeight"].reshape(c, H * d)).reshape(B, Q, H, d)
    v = (xn @ w["valueWeight"].reshape(c, H * d)).reshape(B, Q, H, d)
    g = 1 / (1 + np.exp(-(xn @ w["gatingWeight"].reshape(c, H * d) + w["gatingBias"]))).reshape(B, Q, H, d)
    logits = np.einsum("bqhd,bkhd->bhqk", q, k) + (1e9 * (mk - 1))[:, None, None, :]
    if pair_bias is not None:
        if pair_bias["source"] == "separate":
            pa = np.asarray(pair_bias["activations"], np.float64)
            pn = layer_norm(pa, np.asarray(pair_bias["layerNormScale"], np.float64),
                            np.asarray(pair_bias["layerNormOffset"], np.float64))
            bias = (pn @ np.asarray(pair_bias["projectionWeight"], np.float64).reshape(pa.shape[1], H))
            bias = bias.reshape(Q, Q, H).transpose(2, 0, 1)[None]  # [1, H, q, k]
        else:
            assert B == Q, "a bias from the normalized input needs batch == queries"
            bias = (xn @ np.asarray(pair_bias["projectionWeight"], np.float64).reshape(c, H)).reshape(B, Q, H)
            bias = bias.transpose(2, 0, 1)[None]  # row index b of the source becomes the query index
        logits = logits + bias
    logits = np.clip(logits, -1e8, 1e8)
    logits -= logits.max(-1, keepdims=True)
    p = np.exp(logits)
    p /= p.sum(-1, keepdims=True)
    weighted = np.einsum("bhqk,bkhd->bqhd", p, v) * g
    out = weighted.reshape(rows, H * d) @ w["outputWeight"].reshape(H * d, c) + w["outputBias"]
    result = np.empty_like(out)
    result[order.ravel()] = out
    if residual is not None:
        result = result + np.asarray(residual, np.float64)
    return result
