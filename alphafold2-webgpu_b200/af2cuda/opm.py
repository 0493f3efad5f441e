"""The outer-product mean and the shared dense projection (linear layer).

Host form: ``OuterProductMeanGpu(device).run(input)`` mirrors
src/evoformer/outer-product-mean.ts:538-647 -- the same
OuterProductMeanInput / OuterProductMeanWeights field names, a result with
``output``, ``elapsedMilliseconds`` and ``memory``.

Device forms: ``encode_outer_product_mean_tensors`` mirrors
encodeOuterProductMean (src/evoformer/block.ts:1115-1246) on torch CUDA
tensors; ``linear_tensors`` is createLinearShader's out (=, +=) act(A W + b)
(src/evoformer/transition.ts:91-138).
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass
from typing import Optional

import numpy as np

from . import _lib
from .device import Device
from .transition import Q8Matrix, _matrix
from .triangle import AllocationSnapshot

MAX_SAFE_INTEGER = 2**53 - 1
_DTYPES = {"f32": _lib.AF2_F32, "f16": _lib.AF2_F16, "bf16": _lib.AF2_BF16}
_NP = {_lib.AF2_F32: np.float32, _lib.AF2_F16: np.float16}
_TORCH_DTYPES = {"torch.float32": "f32", "torch.float16": "f16", "torch.bfloat16": "bf16"}
_ORDER = ("layerNormScale", "layerNormOffset", "leftWeight", "leftBias", "rightWeight", "rightBias", "outputWeight",
          "outputBias")


@dataclass(frozen=True)
class OuterProductMeanWeights:
    """OuterProductMeanWeights, outer-product-mean.ts:10-19: left/right weights
    [c_m, c] and the output weight [c*c, c_z] in [in, out] layout."""
    layerNormScale: np.ndarray
    layerNormOffset: np.ndarray
    leftWeight: np.ndarray
    leftBias: np.ndarray
    rightWeight: np.ndarray
    rightBias: np.ndarray
    outputWeight: np.ndarray
    outputBias: np.ndarray


@dataclass(frozen=True)
class OuterProductMeanInput:
    """OuterProductMeanInput, outer-product-mean.ts:21-34."""
    activations: np.ndarray
    mask: np.ndarray
    sequences: int
    length: int
    cM: int
    cOuter: int
    cZ: int
    weights: OuterProductMeanWeights
    layerNormEpsilon: Optional[float] = None
    normalizationEpsilon: Optional[float] = None
    rowBlockResidues: Optional[int] = None


@dataclass(frozen=True)
class OuterProductMeanResult:
    output: np.ndarray
    elapsedMilliseconds: float
    memory: AllocationSnapshot
    deviceMilliseconds: float = 0.0
    flops: float = 0.0


def validate_outer_product_mean_input(inp: OuterProductMeanInput) -> None:
    """validate, outer-product-mean.ts:45-65."""
    dims = (inp.sequences, inp.length, inp.cM, inp.cOuter, inp.cZ)
    if not all(isinstance(v, (int, np.integer)) and 0 < v <= MAX_SAFE_INTEGER for v in dims):
        raise _lib.RangeError("outer product mean dimensions must be positive safe integers")
    s, n, cm, c, cz = dims
    w = inp.weights
    for name, value, size in (("activations", inp.activations, s * n * cm), ("mask", inp.mask, s * n),
                              ("layerNormScale", w.layerNormScale, cm), ("layerNormOffset", w.layerNormOffset, cm),
                              ("leftWeight", w.leftWeight, cm * c), ("leftBias", w.leftBias, c),
                              ("rightWeight", w.rightWeight, cm * c), ("rightBias", w.rightBias, c),
                              ("outputWeight", w.outputWeight, c * c * cz), ("outputBias", w.outputBias, cz)):
        got = int(np.asarray(value).size)
        if got != size:
            raise _lib.RangeError(f"{name} has {got} values; expected {size}")


def pack_outer_product_mean_weights(inp: OuterProductMeanInput):
    """packOuterProductMeanWeights, outer-product-mean.ts:68-80: (data, offsets)."""
    offsets, parts, size = [], [], 0
    for name in _ORDER:
        v = np.ascontiguousarray(getattr(inp.weights, name), np.float32).ravel()
        offsets.append(size)
        parts.append(v)
        size += v.size
    return np.concatenate(parts), tuple(offsets)


def _shape(s, n, cm, c, cz):
    return _lib.OpmShape(s, n, cm, c, cz)


def opm_weight_count(s: int, n: int, cm: int, c: int, cz: int) -> int:
    shape = _shape(s, n, cm, c, cz)
    return int(_lib.lib().af2_opm_weight_count(ctypes.byref(shape)))


def opm_workspace_bytes(s: int, n: int, cm: int, c: int, cz: int, row_block: int = 0) -> int:
    shape = _shape(s, n, cm, c, cz)
    opts = _lib.OpmOptions(0.0, 0.0, row_block, 0)
    out = ctypes.c_uint64()
    _lib.check(_lib.lib().af2_opm_workspace_bytes(ctypes.byref(shape), ctypes.byref(opts), ctypes.byref(out)))
    return int(out.value)


class OuterProductMeanGpu:
    """OuterProductMeanGpu, outer-product-mean.ts:538-647."""

    def __init__(self, device: Device):
        self.device = device

    def run(self, inp: OuterProductMeanInput, host_storage: str = "f32") -> OuterProductMeanResult:
        validate_outer_product_mean_input(inp)
        io_dtype = _DTYPES[host_storage]
        if io_dtype == _lib.AF2_BF16:
            raise _lib.RangeError("the host form takes f32 or f16 arrays")
        rb = inp.rowBlockResidues
        if rb is not None and (not isinstance(rb, (int, np.integer)) or not 0 < rb <= MAX_SAFE_INTEGER):
            raise _lib.RangeError("rowBlockResidues must be a positive safe integer")
        m = np.ascontiguousarray(inp.activations, _NP[io_dtype]).ravel()
        mask = np.ascontiguousarray(inp.mask, np.float32).ravel()
        packed, _ = pack_outer_product_mean_weights(inp)
        out = np.empty(inp.length * inp.length * inp.cZ, _NP[io_dtype])
        shape = _shape(inp.sequences, inp.length, inp.cM, inp.cOuter, inp.cZ)
        opts = _lib.OpmOptions(float(inp.layerNormEpsilon or 0.0), float(inp.normalizationEpsilon or 0.0),
                               int(min(rb or 0, 2**31 - 1)), 0)
        stats = _lib.OpStats()
        status = _lib.lib().af2_outer_product_mean_host(self.device.handle, ctypes.byref(shape), m.ctypes.data,
                                                        mask.ctypes.data, packed.ctypes.data, packed.size,
                                                        ctypes.byref(opts), io_dtype, out.ctypes.data,
                                                        ctypes.byref(stats))
        _lib.check(status, self.device.handle)
        return OuterProductMeanResult(output=out.astype(np.float32) if io_dtype != _lib.AF2_F32 else out,
                                      elapsedMilliseconds=stats.host_milliseconds,
                                      memory=AllocationSnapshot(int(stats.workspace_bytes), int(stats.peak_bytes)),
                                      deviceMilliseconds=stats.device_milliseconds, flops=stats.flops)


def encode_outer_product_mean_tensors(device: Device, msa, msa_mask, packed_weights, c_outer: int, c_z: int, *,
                                      out=None, pair=None, residual: bool = True, row_block: int = 0,
                                      layer_norm_epsilon: float = 1e-5, normalization_epsilon: float = 1e-3,
                                      stream: int = 0, workspace=None):
    """Device form on torch CUDA tensors: msa [S, N, c_m] (f32/f16/bf16), msa_mask
    [S, N] f32, packed_weights f32.  With residual=True the result is added
    into `pair` [N, N, c_z] (the in-model residualTarget); otherwise it is
    written into `out`."""
    s, n, cm = msa.shape
    target = pair if residual else out
    if target is None:
        raise _lib.RangeError("a residual target (pair) or an output tensor is required")
    for t in (msa, msa_mask, packed_weights, target):
        if not t.is_cuda or not t.is_contiguous():
            raise _lib.RangeError("tensors must be contiguous CUDA tensors")
    shape = _shape(s, n, cm, c_outer, c_z)
    opts = _lib.OpmOptions(float(layer_norm_epsilon), float(normalization_epsilon), int(row_block),
                           1 if residual else 0)
    status = _lib.lib().af2_outer_product_mean(
        device.handle, ctypes.byref(shape), msa.data_ptr(), _DTYPES[_TORCH_DTYPES[str(msa.dtype)]],
        msa_mask.data_ptr(), packed_weights.data_ptr(), packed_weights.numel(), ctypes.byref(opts),
        target.data_ptr(), _DTYPES[_TORCH_DTYPES[str(target.dtype)]],
        workspace.data_ptr() if workspace is not None else None, stream or None)
    _lib.check(status, device.handle)
    return target


def linear_tensors(device: Device, a, weight, bias=None, *, out=None, relu: bool = False, residual: bool = False,
                   out_dtype=None, stream: int = 0):
    """out (=, +=) act(a W + b) on torch CUDA tensors; weight is an f32 [inner,
    columns] tensor or a Q8Matrix.  Returns out."""
    import torch
    rows, inner = a.shape
    cols = int(bias.numel()) if bias is not None else int(weight.codes.shape[1] if isinstance(weight, Q8Matrix)
                                                         else weight.shape[1])
    if out is None:
        out = torch.zeros((rows, cols), dtype=out_dtype or torch.float32, device=a.device)
    if not a.is_cuda or not a.is_contiguous() or not out.is_contiguous():
        raise _lib.RangeError("tensors must be contiguous CUDA tensors")
    shape = _lib.LinearShape(rows, inner, cols)
    m = _matrix(weight)
    status = _lib.lib().af2_linear(device.handle, ctypes.byref(shape), a.data_ptr(),
                                   _DTYPES[_TORCH_DTYPES[str(a.dtype)]], ctypes.byref(m),
                                   bias.data_ptr() if bias is not None else None, 1 if relu else 0,
                                   1 if residual else 0, out.data_ptr(), _DTYPES[_TORCH_DTYPES[str(out.dtype)]], None,
                                   stream or None)
    _lib.check(status, device.handle)
    return out
