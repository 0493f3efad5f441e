"""The Evoformer pair block: encodeEvoformerPairBlock (src/evoformer/block.ts:1753-1805).

``encode_evoformer_pair_block_tensors`` runs, on torch CUDA tensors and in one
library call, the outer-product mean of the MSA (optional), triangle
multiplication outgoing and incoming, triangle attention around the starting
and the ending node, and the pair transition, each added into the pair in
place -- the reference's order and residual form.
"""
from __future__ import annotations

import ctypes

from . import _lib
from .device import Device
from .transition import _matrix

_DTYPES = {"torch.float32": _lib.AF2_F32, "torch.float16": _lib.AF2_F16, "torch.bfloat16": _lib.AF2_BF16}


def encode_evoformer_pair_block_tensors(device: Device, pair, pair_mask, weights: dict, *, msa=None, msa_mask=None,
                                        c_outer: int = 32, c_hidden: int = 128, pair_heads: int = 4,
                                        include_outer_product_mean: bool = True, epsilon: float = 1e-5,
                                        stream: int = 0):
    """pair [N, N, c_z] (updated in place), pair_mask [N, N] f32, msa [S, N, c_m], msa_mask
    [S, N] f32.  weights: "outerProductMean", "triangleMultiplicationOutgoing",
    "triangleMultiplicationIncoming", "triangleAttentionStarting", "triangleAttentionEnding"
    (packed f32 CUDA tensors in each op's order, the attention ones with their pair
    projection last) and "pairTransition" (the TransitionWeights dict that
    encode_transition_tensors takes)."""
    n, n2, cz = pair.shape
    if n != n2:
        raise _lib.RangeError("pair must be [N, N, c_z]")
    s, cm = (msa.shape[0], msa.shape[2]) if msa is not None else (1, 1)
    tw = weights["pairTransition"]
    hidden = int(tw["firstBias"].numel())
    ctw = _lib.TransitionWeights(tw["layerNormScale"].data_ptr(), tw["layerNormOffset"].data_ptr(),
                                 _matrix(tw["firstWeight"]), tw["firstBias"].data_ptr(), _matrix(tw["secondWeight"]),
                                 tw["secondBias"].data_ptr())
    opm = weights.get("outerProductMean")
    cw = _lib.PairBlockWeights(opm.data_ptr() if opm is not None else None,
                               weights["triangleMultiplicationOutgoing"].data_ptr(),
                               weights["triangleMultiplicationIncoming"].data_ptr(),
                               weights["triangleAttentionStarting"].data_ptr(),
                               weights["triangleAttentionEnding"].data_ptr(), ctw)
    shape = _lib.PairBlockShape(n, s, cm, cz, c_outer, c_hidden, pair_heads, hidden)
    opts = _lib.PairBlockOptions(1 if include_outer_product_mean else 0, float(epsilon))
    status = _lib.lib().af2_evoformer_pair_block(
        device.handle, ctypes.byref(shape), ctypes.byref(cw), msa.data_ptr() if msa is not None else None,
        _DTYPES[str(msa.dtype)] if msa is not None else _lib.AF2_F32,
        msa_mask.data_ptr() if msa_mask is not None else None, pair.data_ptr(), _DTYPES[str(pair.dtype)],
        pair_mask.data_ptr(), ctypes.byref(opts), stream or None)
    _lib.check(status, device.handle)
    return pair
