"""Triangle multiplication, outgoing and incoming.

Host form: ``TriangleMultiplicationOutgoingGpu(device).run(input, options)``
mirrors src/triangle/webgpu.ts:43-214 -- same input type, same option names,
a result with ``output``, ``elapsedMilliseconds`` and ``memory``.

Device form: ``encode_triangle_multiplication`` mirrors
encodeTriangleMultiplication (src/evoformer/block.ts:1497-1671) on
device-resident tensors given as raw pointers (or torch CUDA tensors through
``encode_triangle_multiplication_tensors``), with the residual add into the
pair that the in-model encoder performs.
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass, field
from typing import Optional

import numpy as np

from . import _lib
from .device import Device
from .types import (TriangleMultiplicationInput, TriangleShape, expected_weight_element_count, pack_weights,
                    validate_triangle_input)

_DTYPES = {"f32": _lib.AF2_F32, "f16": _lib.AF2_F16, "bf16": _lib.AF2_BF16}
_NP = {_lib.AF2_F32: np.float32, _lib.AF2_F16: np.float16}


@dataclass(frozen=True)
class TriangleGpuOptions:
    """TriangleGpuOptions, src/triangle/webgpu.ts:9-15.

    precision: "f32" or "f16", the weight and arithmetic precision; as in the
    reference (webgpu.ts:93-99) the pair stays f32 in and out either way.  This
    build runs both on the tensor cores with f16 operands and f32
    accumulation (the f16 bars of the reference's tests hold for both).
    blockRows: output rows per block, which bounds scratch only; results are
    bit-identical for any value.  wholeStorage: "f32" or "f16", the storage
    of the whole projection; the projected operands are always f16 in HBM
    here, so both values run the same kernels.
    hostStorage (not in the reference): "f16" passes the pair to and from the
    device as half-precision arrays instead of f32 ones.
    """
    precision: str = "f32"
    blockRows: Optional[int] = None
    wholeStorage: str = "f32"
    hostStorage: str = "f32"


@dataclass(frozen=True)
class AllocationSnapshot:
    workspaceBytes: int
    peakBytes: int


@dataclass(frozen=True)
class TriangleGpuResult:
    output: np.ndarray
    elapsedMilliseconds: float
    memory: AllocationSnapshot
    deviceMilliseconds: float = 0.0
    flops: float = 0.0


def _options(options) -> TriangleGpuOptions:
    if options is None:
        return TriangleGpuOptions()
    if isinstance(options, dict):
        return TriangleGpuOptions(**options)
    return options


class _TriangleMultiplicationGpu:
    direction: int

    def __init__(self, device: Device):
        self.device = device

    def run(self, inp: TriangleMultiplicationInput, options=None) -> TriangleGpuResult:
        validate_triangle_input(inp)
        opts = _options(options)
        if opts.precision not in ("f32", "f16"):
            raise _lib.RangeError(f"precision must be f32 or f16; received {opts.precision}")
        if opts.wholeStorage not in ("f32", "f16"):
            raise _lib.RangeError(f"wholeStorage must be f32 or f16; received {opts.wholeStorage}")
        if opts.hostStorage not in ("f32", "f16"):
            raise _lib.RangeError(f"hostStorage must be f32 or f16; received {opts.hostStorage}")
        n, cz, ch = inp.shape.length, inp.shape.cZ, inp.shape.cHidden
        block_rows = max(1, min(n, opts.blockRows if opts.blockRows is not None else n))
        io_dtype = _DTYPES[opts.hostStorage]
        z = np.ascontiguousarray(inp.z, _NP[io_dtype]).ravel()
        mask = np.ascontiguousarray(inp.mask, np.float32).ravel()
        packed, _ = pack_weights(inp.weights)
        out = np.empty(n * n * cz, _NP[io_dtype])
        shape = _lib.TriangleShape(n, cz, ch)
        copts = _lib.TriangleOptions(block_rows, 0)
        stats = _lib.OpStats()
        eps = 1e-5 if inp.epsilon is None else float(inp.epsilon)
        status = _lib.lib().af2_triangle_multiplication_host(
            self.device.handle, self.direction, ctypes.byref(shape), z.ctypes.data, mask.ctypes.data,
            packed.ctypes.data, packed.size, eps, ctypes.byref(copts), io_dtype, out.ctypes.data, ctypes.byref(stats))
        _lib.check(status, self.device.handle)
        return TriangleGpuResult(
            output=out.astype(np.float32) if io_dtype != _lib.AF2_F32 else out,
            elapsedMilliseconds=stats.host_milliseconds,
            memory=AllocationSnapshot(int(stats.workspace_bytes), int(stats.peak_bytes)),
            deviceMilliseconds=stats.device_milliseconds, flops=stats.flops)


class TriangleMultiplicationOutgoingGpu(_TriangleMultiplicationGpu):
    direction = _lib.AF2_OUTGOING


class TriangleMultiplicationIncomingGpu(_TriangleMultiplicationGpu):
    direction = _lib.AF2_INCOMING


def triangle_weight_count(c_z: int, c_hidden: int) -> int:
    return int(_lib.lib().af2_triangle_weight_count(c_z, c_hidden))


def triangle_workspace_bytes(length: int, c_z: int, c_hidden: int, block_rows: int = 0) -> int:
    shape = _lib.TriangleShape(length, c_z, c_hidden)
    opts = _lib.TriangleOptions(block_rows, 0)
    out = ctypes.c_uint64()
    _lib.check(_lib.lib().af2_triangle_workspace_bytes(ctypes.byref(shape), ctypes.byref(opts), ctypes.byref(out)))
    return int(out.value)


def encode_triangle_multiplication(device: Device, direction: str | int, shape: TriangleShape, z_ptr: int,
                                   z_dtype: str, mask_ptr: int, weights_ptr: int, weight_count: int,
                                   out_ptr: int, out_dtype: str, *, epsilon: float = 1e-5, residual: bool = False,
                                   block_rows: int = 0, workspace_ptr: int = 0, stream: int = 0) -> None:
    """Device form on raw device pointers; asynchronous on `stream` (0 = context stream)."""
    d = direction if isinstance(direction, int) else {"outgoing": 0, "incoming": 1}[direction]
    cshape = _lib.TriangleShape(shape.length, shape.cZ, shape.cHidden)
    copts = _lib.TriangleOptions(block_rows, 1 if residual else 0)
    status = _lib.lib().af2_triangle_multiplication(
        device.handle, d, ctypes.byref(cshape), z_ptr, _DTYPES[z_dtype], mask_ptr, weights_ptr, weight_count,
        float(epsilon), ctypes.byref(copts), out_ptr, _DTYPES[out_dtype], workspace_ptr or None, stream or None)
    _lib.check(status, device.handle)


_TORCH_DTYPES = {"torch.float32": "f32", "torch.float16": "f16", "torch.bfloat16": "bf16"}


def encode_triangle_multiplication_tensors(device: Device, direction: str | int, pair, mask, packed_weights, *,
                                           out=None, epsilon: float = 1e-5, residual: bool = True,
                                           block_rows: int = 0, stream: int = 0):
    """Device form on torch CUDA tensors: pair [N,N,c_z] (f32/f16/bf16), mask [N,N] f32,
    packed_weights f32.  With residual=True and out=None the pair is updated in place."""
    n, n2, cz = pair.shape
    if n != n2:
        raise _lib.RangeError("pair must be [N, N, c_z]")
    count = packed_weights.numel()
    ch = _hidden_from_count(cz, count)
    target = pair if out is None else out
    for t in (pair, mask, packed_weights, target):
        if not t.is_cuda or not t.is_contiguous():
            raise _lib.RangeError("tensors must be contiguous CUDA tensors")
    encode_triangle_multiplication(
        device, direction, TriangleShape(n, cz, ch), pair.data_ptr(), _TORCH_DTYPES[str(pair.dtype)],
        mask.data_ptr(), packed_weights.data_ptr(), count, target.data_ptr(), _TORCH_DTYPES[str(target.dtype)],
        epsilon=epsilon, residual=residual, block_rows=block_rows, stream=stream)
    return target


def _hidden_from_count(cz: int, count: int) -> int:
    base = 2 * cz + cz + cz * cz + cz
    per = 4 * cz + 4 + 2 + cz
    ch, rem = divmod(count - base, per)
    if rem or ch <= 0 or expected_weight_element_count(TriangleShape(1, cz, ch)) != count:
        raise _lib.RangeError(f"{count} packed weights do not fit c_z={cz}")
    return ch
