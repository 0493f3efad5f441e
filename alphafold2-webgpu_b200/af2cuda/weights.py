"""Per-tensor weight forms: the triangle multiplication and the outer-product mean
with each weight tensor as the reference's model files store it.

The reference decodes every stored tensor to f32 on the host
(readTensorRange, src/reference/dtype.ts:66-99) and packs the f32 values for
its shaders (src/triangle/weights.ts:4-40, outer-product-mean.ts:68-80).
Here each tensor goes to the library as it is stored -- an f32 CUDA tensor
or a block-scaled Q8Matrix (int8 codes plus f16 scale bits, block 64 in the
reference's files) -- and the codes become the kernels' f16 operands on the
device (af2_triangle_multiplication_weights, af2_outer_product_mean_weights).
The decode is exact, so the results equal the packed forms on the decoded
weights, bit for bit.

``stored_weights`` gathers one Evoformer block's tensors of an op from a
FileTensorStore (tensor_store.py) by their names.
"""
from __future__ import annotations

import ctypes

from . import _lib
from .device import Device
from .opm import _ORDER as OPM_ORDER
from .opm import _shape as _opm_shape
from .transition import Q8Matrix
from .types import ORDER as TRIANGLE_ORDER

_DTYPES = {"torch.float32": _lib.AF2_F32, "torch.float16": _lib.AF2_F16, "torch.bfloat16": _lib.AF2_BF16}


def _count(w) -> int:
    return int(w.codes.numel() if isinstance(w, Q8Matrix) else w.numel())


def _c_matrix(w, expected: int, name: str) -> _lib.Matrix:
    """One stored tensor as an af2_matrix, after checking its element count."""
    if isinstance(w, Q8Matrix):
        if w.kind != "block":
            raise _lib.RangeError(f"{name}: per-tensor weights take block-scaled q8 (the reference's format)")
        if _count(w) != expected or int(w.scales.numel()) * int(w.block) < expected:
            raise _lib.RangeError(f"{name} holds {_count(w)} codes; expected {expected}")
        if w.scales.element_size() != 2:
            raise _lib.RangeError(f"{name}: scales must be 16-bit f16 bit patterns")
        return w.c_matrix()
    if str(w.dtype) != "torch.float32" or not w.is_cuda or not w.is_contiguous():
        raise _lib.RangeError(f"{name} must be a contiguous float32 CUDA tensor or a Q8Matrix")
    if _count(w) != expected:
        raise _lib.RangeError(f"{name} holds {_count(w)} values; expected {expected}")
    return _lib.Matrix(_lib.AF2_WEIGHTS_F32, 0, w.data_ptr(), None)


def _device_tensors(*ts):
    for t in ts:
        if not t.is_cuda or not t.is_contiguous():
            raise _lib.RangeError("tensors must be contiguous CUDA tensors")


def triangle_tensor_sizes(cz: int, ch: int) -> dict:
    """Element count of each TriangleMultiplicationWeights tensor (src/triangle/types.ts:9-26)."""
    return {"layerNormInWeight": cz, "layerNormInBias": cz,
            "linearAPWeight": ch * cz, "linearAPBias": ch, "linearAGWeight": ch * cz, "linearAGBias": ch,
            "linearBPWeight": ch * cz, "linearBPBias": ch, "linearBGWeight": ch * cz, "linearBGBias": ch,
            "layerNormOutWeight": ch, "layerNormOutBias": ch,
            "linearZWeight": cz * ch, "linearZBias": cz, "linearGWeight": cz * cz, "linearGBias": cz}


def opm_tensor_sizes(cm: int, c: int, cz: int) -> dict:
    """Element count of each OuterProductMeanWeights tensor (outer-product-mean.ts:68-72)."""
    return {"layerNormScale": cm, "layerNormOffset": cm, "leftWeight": cm * c, "leftBias": c,
            "rightWeight": cm * c, "rightBias": c, "outputWeight": c * c * cz, "outputBias": cz}


def encode_triangle_multiplication_weight_tensors(device: Device, direction: str | int, pair, mask, weights: dict, *,
                                                  out=None, epsilon: float = 1e-5, residual: bool = True,
                                                  block_rows: int = 0, workspace=None, stream: int = 0):
    """Device form with per-tensor weights: pair [N,N,c_z], mask [N,N] f32, weights mapping
    every ORDER name to an f32 CUDA tensor or a block Q8Matrix.  With residual=True and
    out=None the pair is updated in place."""
    n, n2, cz = pair.shape
    if n != n2:
        raise _lib.RangeError("pair must be [N, N, c_z]")
    ch = _count(weights["linearAPBias"])
    sizes = triangle_tensor_sizes(cz, ch)
    arr = (_lib.Matrix * len(TRIANGLE_ORDER))(*[_c_matrix(weights[k], sizes[k], k) for k in TRIANGLE_ORDER])
    target = pair if out is None else out
    _device_tensors(pair, mask, target)
    d = direction if isinstance(direction, int) else {"outgoing": 0, "incoming": 1}[direction]
    shape = _lib.TriangleShape(n, cz, ch)
    opts = _lib.TriangleOptions(block_rows, 1 if residual else 0)
    status = _lib.lib().af2_triangle_multiplication_weights(
        device.handle, d, ctypes.byref(shape), pair.data_ptr(), _DTYPES[str(pair.dtype)], mask.data_ptr(), arr,
        float(epsilon), ctypes.byref(opts), target.data_ptr(), _DTYPES[str(target.dtype)],
        workspace.data_ptr() if workspace is not None else None, stream or None)
    _lib.check(status, device.handle)
    return target


def encode_outer_product_mean_weight_tensors(device: Device, msa, msa_mask, weights: dict, *, out=None, pair=None,
                                             residual: bool = True, row_block: int = 0,
                                             layer_norm_epsilon: float = 1e-5, normalization_epsilon: float = 1e-3,
                                             workspace=None, stream: int = 0):
    """Device form with per-tensor weights: msa [S,N,c_m], msa_mask [S,N] f32, weights
    mapping every OuterProductMeanWeights name to an f32 CUDA tensor or a block Q8Matrix.
    With residual=True the result is added into `pair`, else written into `out`."""
    s, n, cm = msa.shape
    c, cz = _count(weights["leftBias"]), _count(weights["outputBias"])
    sizes = opm_tensor_sizes(cm, c, cz)
    arr = (_lib.Matrix * len(OPM_ORDER))(*[_c_matrix(weights[k], sizes[k], k) for k in OPM_ORDER])
    target = pair if residual else out
    if target is None:
        raise _lib.RangeError("a residual target (pair) or an output tensor is required")
    _device_tensors(msa, msa_mask, target)
    shape = _opm_shape(s, n, cm, c, cz)
    opts = _lib.OpmOptions(float(layer_norm_epsilon), float(normalization_epsilon), int(row_block),
                           1 if residual else 0)
    status = _lib.lib().af2_outer_product_mean_weights(
        device.handle, ctypes.byref(shape), msa.data_ptr(), _DTYPES[str(msa.dtype)], msa_mask.data_ptr(), arr,
        ctypes.byref(opts), target.data_ptr(), _DTYPES[str(target.dtype)],
        workspace.data_ptr() if workspace is not None else None, stream or None)
    _lib.check(status, device.handle)
    return target


def stored_weights(store, names: dict, block=None, blocks=None, device="cuda") -> dict:
    """Weights of one op from a FileTensorStore: `names` maps each field name (ORDER or the
    OuterProductMeanWeights names) to the tensor's name in the manifest; block/blocks pick
    one Evoformer block of stacked tensors.  Each value is on the device in its stored form."""
    return {field: store.device_weight(name, block, blocks, device) for field, name in names.items()}
