"""Gated multi-head attention: the Evoformer's triangle attention.

Host form: ``AttentionGpu(device).run(input)`` mirrors AttentionGpu.run
(src/evoformer/attention.ts:1321-1453) -- the same AttentionInput /
AttentionWeights field names and pair-bias objects, a result with
``output``, ``elapsedMilliseconds`` and ``memory``.

Device forms: ``encode_attention_tensors`` mirrors encodeAttention on torch
CUDA tensors, and ``encode_triangle_attention_tensors`` the two triangle
attention calls of the Evoformer block (src/evoformer/block.ts:1727-1745):
the pair attends along its rows (starting node) or, through the transposed
view, along its columns (ending node), biased by its own normalised rows, and
the result is added into the pair.
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass
from typing import Optional, Union

import numpy as np

from . import _lib
from .device import Device
from .triangle import AllocationSnapshot

_DTYPES = {"f32": _lib.AF2_F32, "f16": _lib.AF2_F16, "bf16": _lib.AF2_BF16}
_TORCH_DTYPES = {"torch.float32": "f32", "torch.float16": "f16", "torch.bfloat16": "bf16"}
_ORDER = ("queryNormScale", "queryNormOffset", "queryWeight", "keyWeight", "valueWeight", "gatingWeight",
          "gatingBias", "outputWeight", "outputBias")
AF2_PAIR_BIAS_NONE, AF2_PAIR_BIAS_NORMALIZED_INPUT = 0, 1


@dataclass(frozen=True)
class AttentionWeights:
    """AttentionWeights, attention.ts:19-29: query/key/value/gating weights [C, C] and the
    output weight [C, C], all [in, out]."""
    queryNormScale: np.ndarray
    queryNormOffset: np.ndarray
    queryWeight: np.ndarray
    keyWeight: np.ndarray
    valueWeight: np.ndarray
    gatingWeight: np.ndarray
    gatingBias: np.ndarray
    outputWeight: np.ndarray
    outputBias: np.ndarray


@dataclass(frozen=True)
class NormalizedInputPairBias:
    """NormalizedInputPairBias, attention.ts:40-43: projectionWeight [C, heads] ([in, out])."""
    projectionWeight: np.ndarray
    source: str = "normalized-input"


@dataclass(frozen=True)
class SeparatePairBias:
    """SeparatePairBias, attention.ts:31-38 (MSA row attention); accepted for signature
    parity and rejected by the kernels."""
    activations: np.ndarray
    channels: int
    layerNormScale: np.ndarray
    layerNormOffset: np.ndarray
    projectionWeight: np.ndarray
    source: str = "separate"


@dataclass(frozen=True)
class AttentionInput:
    """AttentionInput, attention.ts:47-58."""
    activations: np.ndarray
    mask: np.ndarray
    batch: int
    queryLength: int
    channels: int
    heads: int
    weights: AttentionWeights
    transpose: bool = False
    pairBias: Optional[Union[NormalizedInputPairBias, SeparatePairBias]] = None
    epsilon: Optional[float] = None


@dataclass(frozen=True)
class AttentionResult:
    output: np.ndarray
    elapsedMilliseconds: float
    memory: AllocationSnapshot
    deviceMilliseconds: float = 0.0
    flops: float = 0.0


def _bias_kind(pair_bias) -> int:
    if pair_bias is None:
        return AF2_PAIR_BIAS_NONE
    if getattr(pair_bias, "source", None) == "normalized-input":
        return AF2_PAIR_BIAS_NORMALIZED_INPUT
    raise _lib.Af2Error(_lib.AF2_ERR_UNSUPPORTED, "a separate pair-bias source (MSA row attention) is not supported")


def pack_attention_weights(inp: AttentionInput) -> tuple[np.ndarray, list[int]]:
    """packAttentionWeights, attention.ts:179-201."""
    tensors = [np.asarray(getattr(inp.weights, k), np.float32).ravel() for k in _ORDER]
    if inp.pairBias is not None and getattr(inp.pairBias, "source", None) == "separate":
        pb = inp.pairBias
        tensors += [np.asarray(t, np.float32).ravel() for t in (pb.layerNormScale, pb.layerNormOffset,
                                                                 pb.projectionWeight)]
    elif inp.pairBias is not None:
        tensors.append(np.asarray(inp.pairBias.projectionWeight, np.float32).ravel())
    offsets, size = [], 0
    for t in tensors:
        offsets.append(size)
        size += t.size
    return np.concatenate(tensors).astype(np.float32), offsets


def _shape(batch, queries, channels, heads) -> _lib.AttentionShape:
    return _lib.AttentionShape(batch, queries, channels, heads)


def attention_weight_count(batch: int, queries: int, channels: int, heads: int, pair_bias: int = 0) -> int:
    return int(_lib.lib().af2_attention_weight_count(ctypes.byref(_shape(batch, queries, channels, heads)), pair_bias))


def attention_workspace_bytes(batch: int, queries: int, channels: int, heads: int, pair_bias: int = 0) -> int:
    out = ctypes.c_uint64()
    _lib.check(_lib.lib().af2_attention_workspace_bytes(ctypes.byref(_shape(batch, queries, channels, heads)),
                                                         pair_bias, ctypes.byref(out)))
    return int(out.value)


class AttentionGpu:
    """AttentionGpu (attention.ts:1321-1453): run() uploads the input, runs the kernels,
    reads the output back and returns a fresh f32 array."""

    def __init__(self, device: Device, options=None):
        self.device = device
        self.options = options or {}

    def run(self, inp: AttentionInput, residual: bool = False) -> AttentionResult:
        kind = _bias_kind(inp.pairBias)
        packed, _ = pack_attention_weights(inp)
        shape = _shape(inp.batch, inp.queryLength, inp.channels, inp.heads)
        eps = 1e-5 if inp.epsilon is None else float(inp.epsilon)
        msg = ctypes.create_string_buffer(512)
        status = _lib.lib().af2_attention_check(ctypes.byref(shape), kind, packed.size, eps, msg, 512)
        if status != _lib.AF2_OK:
            if status == _lib.AF2_ERR_INVALID_ARGUMENT:
                raise _lib.RangeError(msg.value.decode())
            raise _lib.Af2Error(status, msg.value.decode())
        rows = inp.batch * inp.queryLength
        x = np.ascontiguousarray(inp.activations, np.float32).ravel()
        mask = np.ascontiguousarray(inp.mask, np.float32).ravel()
        if x.size != rows * inp.channels:
            raise _lib.RangeError(f"activations has {x.size} values; expected {rows * inp.channels}")
        if mask.size != rows:
            raise _lib.RangeError(f"mask has {mask.size} values; expected {rows}")
        out = np.empty(rows * inp.channels, np.float32)
        opts = _lib.AttentionOptions(1 if inp.transpose else 0, kind, 1 if residual else 0)
        stats = _lib.OpStats()
        status = _lib.lib().af2_attention_host(self.device.handle, ctypes.byref(shape), x.ctypes.data,
                                               mask.ctypes.data, packed.ctypes.data, packed.size, eps,
                                               ctypes.byref(opts), out.ctypes.data, ctypes.byref(stats))
        _lib.check(status, self.device.handle)
        return AttentionResult(out, stats.host_milliseconds,
                               AllocationSnapshot(int(stats.workspace_bytes), int(stats.peak_bytes)),
                               stats.device_milliseconds, stats.flops)


def encode_attention_tensors(device: Device, x, mask, packed_weights, *, batch: int, queries: int, heads: int,
                             transpose: bool = False, pair_bias: int = AF2_PAIR_BIAS_NONE, out=None,
                             residual: bool = True, epsilon: float = 1e-5, stream: int = 0, workspace=None):
    """Device form on torch CUDA tensors: x [batch * queries, C] (or any contiguous tensor
    with those rows), mask [batch * queries] f32, packed_weights f32 in packAttentionWeights
    order.  With residual=True and out=None, x is updated in place."""
    channels = x.shape[-1]
    target = x if out is None else out
    for t in (x, mask, packed_weights, target):
        if not t.is_cuda or not t.is_contiguous():
            raise _lib.RangeError("tensors must be contiguous CUDA tensors")
    shape = _shape(batch, queries, channels, heads)
    opts = _lib.AttentionOptions(1 if transpose else 0, pair_bias, 1 if residual else 0)
    ws = workspace.data_ptr() if workspace is not None else None
    status = _lib.lib().af2_attention(device.handle, ctypes.byref(shape), x.data_ptr(), _DTYPES[_TORCH_DTYPES[str(x.dtype)]],
                                      mask.data_ptr(), packed_weights.data_ptr(), packed_weights.numel(),
                                      float(epsilon), ctypes.byref(opts), target.data_ptr(),
                                      _DTYPES[_TORCH_DTYPES[str(target.dtype)]], ws, stream or None)
    _lib.check(status, device.handle)
    return target


def encode_triangle_attention_tensors(device: Device, direction: str, pair, pair_mask, packed_weights, heads: int,
                                      *, out=None, residual: bool = True, epsilon: float = 1e-5, stream: int = 0):
    """Triangle attention around the starting node (direction "starting": rows) or the
    ending node ("ending": the transposed view), pair [N, N, C], pair_mask [N, N] f32,
    packed_weights with the normalized-input pair projection last
    (src/evoformer/block.ts:1727-1745).  Adds into the pair by default."""
    n, n2, _ = pair.shape
    if n != n2:
        raise _lib.RangeError("pair must be [N, N, C]")
    return encode_attention_tensors(device, pair, pair_mask, packed_weights, batch=n, queries=n, heads=heads,
                                    transpose={"starting": False, "ending": True}[direction],
                                    pair_bias=AF2_PAIR_BIAS_NORMALIZED_INPUT, out=out, residual=residual,
                                    epsilon=epsilon, stream=stream)
