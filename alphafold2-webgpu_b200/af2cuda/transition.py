"""The Evoformer transition (LayerNorm -> Linear -> ReLU -> Linear) and the
mixed-q8 weight formats it accepts.

Host form: ``TransitionGpu(device, {"maxChunkRows": n}).run(input)`` mirrors
src/evoformer/transition.ts:253-361 -- the same TransitionInput and
TransitionWeights field names, a result with ``output``,
``elapsedMilliseconds`` and ``memory``.

Device form: ``encode_transition_tensors`` mirrors encodeTransition
(src/evoformer/block.ts:625-740) on torch CUDA tensors, with f32 or q8
weight matrices and the residual add into the target.

``dequant_q8_tensors`` is the bit-exact decode of readTensorRange's int8
branch (src/reference/dtype.ts:86-97), run on the device.
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass
from typing import Optional, Union

import numpy as np

from . import _lib
from .device import Device
from .triangle import AllocationSnapshot

MAX_SAFE_INTEGER = 2**53 - 1
_DTYPES = {"f32": _lib.AF2_F32, "f16": _lib.AF2_F16, "bf16": _lib.AF2_BF16}
_NP = {_lib.AF2_F32: np.float32, _lib.AF2_F16: np.float16}
_TORCH_DTYPES = {"torch.float32": "f32", "torch.float16": "f16", "torch.bfloat16": "bf16"}


@dataclass(frozen=True)
class TransitionWeights:
    """TransitionWeights, transition.ts:9-16: firstWeight [channels, hidden] and
    secondWeight [hidden, channels] in [in, out] layout."""
    layerNormScale: np.ndarray
    layerNormOffset: np.ndarray
    firstWeight: np.ndarray
    firstBias: np.ndarray
    secondWeight: np.ndarray
    secondBias: np.ndarray


@dataclass(frozen=True)
class TransitionInput:
    """TransitionInput, transition.ts:18-25."""
    activations: np.ndarray
    rows: int
    channels: int
    hiddenChannels: int
    weights: TransitionWeights
    epsilon: Optional[float] = None


@dataclass(frozen=True)
class TransitionResult:
    output: np.ndarray
    elapsedMilliseconds: float
    memory: AllocationSnapshot
    deviceMilliseconds: float = 0.0
    flops: float = 0.0


_PACK_ORDER = ("layerNormScale", "layerNormOffset", "firstWeight", "firstBias", "secondWeight", "secondBias")


def validate_transition_input(inp: TransitionInput) -> None:
    """validate, transition.ts:140-156."""
    dims = (inp.rows, inp.channels, inp.hiddenChannels)
    if not all(isinstance(v, (int, np.integer)) and 0 < v <= MAX_SAFE_INTEGER for v in dims):
        raise _lib.RangeError("transition dimensions must be positive safe integers")
    c, h = inp.channels, inp.hiddenChannels
    w = inp.weights
    for name, value, expected in (("activations", inp.activations, inp.rows * c),
                                  ("layerNormScale", w.layerNormScale, c), ("layerNormOffset", w.layerNormOffset, c),
                                  ("firstWeight", w.firstWeight, c * h), ("firstBias", w.firstBias, h),
                                  ("secondWeight", w.secondWeight, h * c), ("secondBias", w.secondBias, c)):
        n = int(np.asarray(value).size)
        if n != expected:
            raise _lib.RangeError(f"{name} has {n} values; expected {expected}")


def pack_transition_weights(inp: TransitionInput):
    """packTransitionWeights, transition.ts:158-177: (data, offsets)."""
    offsets, parts, length = [], [], 0
    for name in _PACK_ORDER:
        v = np.ascontiguousarray(getattr(inp.weights, name), np.float32).ravel()
        offsets.append(length)
        parts.append(v)
        length += v.size
    return np.concatenate(parts), tuple(offsets)


def transition_weight_count(channels: int, hidden: int) -> int:
    return int(_lib.lib().af2_transition_weight_count(channels, hidden))


def transition_workspace_bytes(rows: int, channels: int, hidden: int) -> int:
    shape = _lib.TransitionShape(rows, channels, hidden)
    out = ctypes.c_uint64()
    _lib.check(_lib.lib().af2_transition_workspace_bytes(ctypes.byref(shape), ctypes.byref(out)))
    return int(out.value)


class TransitionGpu:
    """TransitionGpu, transition.ts:253-361."""

    def __init__(self, device: Device, options: Optional[dict] = None):
        self.device = device
        options = options or {}
        self.maxChunkRows = options.get("maxChunkRows")
        if self.maxChunkRows is not None and (not isinstance(self.maxChunkRows, (int, np.integer))
                                              or not 0 < self.maxChunkRows <= MAX_SAFE_INTEGER):
            raise _lib.RangeError("maxChunkRows must be a positive safe integer")

    def run(self, inp: TransitionInput, host_storage: str = "f32", residual: bool = False) -> TransitionResult:
        validate_transition_input(inp)
        io_dtype = _DTYPES[host_storage]
        if io_dtype == _lib.AF2_BF16:
            raise _lib.RangeError("the host form takes f32 or f16 arrays")
        x = np.ascontiguousarray(inp.activations, _NP[io_dtype]).ravel()
        packed, _ = pack_transition_weights(inp)
        out = np.empty(inp.rows * inp.channels, _NP[io_dtype])
        shape = _lib.TransitionShape(inp.rows, inp.channels, inp.hiddenChannels)
        opts = _lib.TransitionOptions(int(min(self.maxChunkRows or 0, 2**31 - 1)), 1 if residual else 0)
        stats = _lib.OpStats()
        eps = 1e-5 if inp.epsilon is None else float(inp.epsilon)
        status = _lib.lib().af2_transition_host(self.device.handle, ctypes.byref(shape), x.ctypes.data,
                                                packed.ctypes.data, packed.size, eps, ctypes.byref(opts), io_dtype,
                                                out.ctypes.data, ctypes.byref(stats))
        _lib.check(status, self.device.handle)
        return TransitionResult(output=out.astype(np.float32) if io_dtype != _lib.AF2_F32 else out,
                                elapsedMilliseconds=stats.host_milliseconds,
                                memory=AllocationSnapshot(int(stats.workspace_bytes), int(stats.peak_bytes)),
                                deviceMilliseconds=stats.device_milliseconds, flops=stats.flops)


@dataclass
class Q8Matrix:
    """An int8 matrix [in, out] with its scales, on the device (torch tensors).

    kind "block": scales are f16 bit patterns (uint16 stored as int16 or
    int32 tensors are accepted) for every `block` consecutive elements of the
    flattened matrix -- the reference's mixed-q8 files (block 64).
    kind "channel": f32 scales, one per output column.
    """
    codes: object
    scales: object
    kind: str = "channel"
    block: int = 64

    def c_matrix(self) -> _lib.Matrix:
        fmt = {"block": _lib.AF2_WEIGHTS_Q8_BLOCK, "channel": _lib.AF2_WEIGHTS_Q8_CHANNEL}[self.kind]
        for t in (self.codes, self.scales):
            if not t.is_cuda or not t.is_contiguous():
                raise _lib.RangeError("q8 codes and scales must be contiguous CUDA tensors")
        return _lib.Matrix(fmt, int(self.block), self.codes.data_ptr(), self.scales.data_ptr())


def _matrix(w) -> _lib.Matrix:
    if isinstance(w, Q8Matrix):
        return w.c_matrix()
    if str(w.dtype) != "torch.float32" or not w.is_cuda or not w.is_contiguous():
        raise _lib.RangeError("f32 weight matrices must be contiguous float32 CUDA tensors")
    return _lib.Matrix(_lib.AF2_WEIGHTS_F32, 0, w.data_ptr(), None)


def encode_transition_tensors(device: Device, x, weights: dict, *, out=None, residual: bool = True,
                              epsilon: float = 1e-5, stream: int = 0, workspace=None):
    """Device form on torch CUDA tensors.  x [rows, channels] f32/f16/bf16;
    weights: the TransitionWeights field names mapping to f32 CUDA tensors,
    with firstWeight / secondWeight either f32 [in, out] tensors or Q8Matrix.
    With residual=True and out=None, x is updated in place."""
    rows, channels = x.shape
    fb, sb = weights["firstBias"], weights["secondBias"]
    hidden = int(fb.numel())
    target = x if out is None else out
    for t in (x, target, fb, sb, weights["layerNormScale"], weights["layerNormOffset"]):
        if not t.is_cuda or not t.is_contiguous():
            raise _lib.RangeError("tensors must be contiguous CUDA tensors")
    cw = _lib.TransitionWeights(weights["layerNormScale"].data_ptr(), weights["layerNormOffset"].data_ptr(),
                                _matrix(weights["firstWeight"]), fb.data_ptr(), _matrix(weights["secondWeight"]),
                                sb.data_ptr())
    shape = _lib.TransitionShape(rows, channels, hidden)
    opts = _lib.TransitionOptions(0, 1 if residual else 0)
    status = _lib.lib().af2_transition(device.handle, ctypes.byref(shape), x.data_ptr(), _DTYPES[_TORCH_DTYPES[str(
        x.dtype)]], ctypes.byref(cw), float(epsilon), ctypes.byref(opts), target.data_ptr(),
        _DTYPES[_TORCH_DTYPES[str(target.dtype)]], workspace.data_ptr() if workspace is not None else None,
        stream or None)
    _lib.check(status, device.handle)
    return target


def dequant_q8_tensors(device: Device, matrix: Q8Matrix, inner: int, cols: int, *, stream: int = 0):
    """Bit-exact f32 decode of a q8 matrix on the device; returns a [inner, cols] f32 CUDA tensor."""
    import torch
    out = torch.empty((inner, cols), dtype=torch.float32, device=matrix.codes.device)
    m = matrix.c_matrix()
    status = _lib.lib().af2_dequant_q8(device.handle, ctypes.byref(m), inner, cols, out.data_ptr(), stream or None)
    _lib.check(status, device.handle)
    return out
