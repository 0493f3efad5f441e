"""Loads libaf2cuda.so and declares its C ABI (include/af2cuda.h) for ctypes.

There is no fallback: if the library is missing or cannot be loaded the
import of an operator fails with the loader's message.
"""
from __future__ import annotations

import ctypes
import os
from pathlib import Path

PKG_DIR = Path(__file__).resolve().parent.parent
LIB_PATH = Path(os.environ.get("AF2CUDA_LIBRARY", PKG_DIR / "libaf2cuda.so"))

AF2_OK = 0
AF2_ERR_INVALID_ARGUMENT = 1
AF2_ERR_UNSUPPORTED = 2
AF2_ERR_OUT_OF_MEMORY = 3
AF2_ERR_CUDA = 4
AF2_ERR_DEVICE_TIMEOUT = 5
AF2_ERR_NCCL = 6
AF2_ERR_NO_DEVICE = 7

AF2_F32, AF2_F16, AF2_BF16 = 0, 1, 2
AF2_OUTGOING, AF2_INCOMING = 0, 1
AF2_WEIGHTS_F32, AF2_WEIGHTS_Q8_BLOCK, AF2_WEIGHTS_Q8_CHANNEL = 0, 1, 2
AF2_GEMM_MATRIX, AF2_GEMM_F32 = 0, 1

# Every symbol include/af2cuda.h declares, with (restype, argtypes).
_vp = ctypes.c_void_p
_i64 = ctypes.c_int64
_i32 = ctypes.c_int
_f64 = ctypes.c_double


class TriangleShape(ctypes.Structure):
    _fields_ = [("length", _i64), ("c_z", _i64), ("c_hidden", _i64)]


class TriangleOptions(ctypes.Structure):
    _fields_ = [("block_rows", ctypes.c_int32), ("residual", ctypes.c_int32)]


class OpStats(ctypes.Structure):
    _fields_ = [("device_milliseconds", _f64), ("host_milliseconds", _f64), ("flops", _f64),
                ("workspace_bytes", ctypes.c_uint64), ("peak_bytes", ctypes.c_uint64)]


class Matrix(ctypes.Structure):
    _fields_ = [("format", ctypes.c_int32), ("block", ctypes.c_int32), ("values", _vp), ("scales", _vp)]


class TransitionShape(ctypes.Structure):
    _fields_ = [("rows", _i64), ("channels", _i64), ("hidden_channels", _i64)]


class TransitionWeights(ctypes.Structure):
    _fields_ = [("layer_norm_scale", _vp), ("layer_norm_offset", _vp), ("first_weight", Matrix),
                ("first_bias", _vp), ("second_weight", Matrix), ("second_bias", _vp)]


class TransitionOptions(ctypes.Structure):
    _fields_ = [("max_chunk_rows", ctypes.c_int32), ("residual", ctypes.c_int32)]


class OpmShape(ctypes.Structure):
    _fields_ = [("sequences", _i64), ("length", _i64), ("c_m", _i64), ("c_outer", _i64), ("c_z", _i64)]


class OpmOptions(ctypes.Structure):
    _fields_ = [("layer_norm_epsilon", _f64), ("normalization_epsilon", _f64), ("row_block_residues", ctypes.c_int32),
                ("residual", ctypes.c_int32)]


class AttentionShape(ctypes.Structure):
    _fields_ = [("batch", _i64), ("queries", _i64), ("channels", _i64), ("heads", _i64)]


class AttentionOptions(ctypes.Structure):
    _fields_ = [("transpose", ctypes.c_int32), ("pair_bias", ctypes.c_int32), ("residual", ctypes.c_int32)]


class PairBlockShape(ctypes.Structure):
    _fields_ = [("length", _i64), ("sequences", _i64), ("c_m", _i64), ("c_z", _i64), ("c_outer", _i64),
                ("c_hidden", _i64), ("pair_heads", _i64), ("transition_hidden", _i64)]


class PairBlockWeights(ctypes.Structure):
    _fields_ = [("outer_product_mean", _vp), ("triangle_outgoing", _vp), ("triangle_incoming", _vp),
                ("attention_starting", _vp), ("attention_ending", _vp), ("pair_transition", TransitionWeights)]


class PairBlockOptions(ctypes.Structure):
    _fields_ = [("include_outer_product_mean", ctypes.c_int32), ("epsilon", _f64)]


class LinearShape(ctypes.Structure):
    _fields_ = [("rows", _i64), ("inner", _i64), ("columns", _i64)]


SIGNATURES = {
    "af2_version": (_i32, []),
    "af2_status_string": (ctypes.c_char_p, [_i32]),
    "af2_create": (_i32, [_i32, ctypes.POINTER(_vp)]),
    "af2_destroy": (None, [_vp]),
    "af2_last_error": (ctypes.c_char_p, [_vp]),
    "af2_sync": (_i32, [_vp, _vp]),
    "af2_launch_count": (ctypes.c_uint64, [_vp]),
    "af2_set_gemm_precision": (_i32, [_vp, _i32]),
    "af2_get_gemm_precision": (_i32, [_vp]),
    "af2_set_weight_cache": (_i32, [_vp, _i32]),
    "af2_clear_weight_cache": (_i32, [_vp]),
    "af2_memory_snapshot": (_i32, [_vp, ctypes.POINTER(ctypes.c_uint64), ctypes.POINTER(ctypes.c_uint64)]),
    "af2_profile_enable": (_i32, [_vp, _i32]),
    "af2_profile_reset": (_i32, [_vp]),
    "af2_profile_kernel_name": (ctypes.c_char_p, [_i32]),
    "af2_profile_read": (_i32, [_vp, ctypes.c_char_p, ctypes.POINTER(ctypes.c_uint64), ctypes.POINTER(_f64)]),
    "af2_triangle_weight_count": (_i64, [_i64, _i64]),
    "af2_triangle_check": (_i32, [_i32, ctypes.POINTER(TriangleShape), _i64, _f64, ctypes.c_char_p, ctypes.c_size_t]),
    "af2_triangle_workspace_bytes": (_i32, [ctypes.POINTER(TriangleShape), ctypes.POINTER(TriangleOptions),
                                            ctypes.POINTER(ctypes.c_uint64)]),
    "af2_triangle_multiplication_host": (_i32, [_vp, _i32, ctypes.POINTER(TriangleShape), _vp, _vp, _vp, _i64, _f64,
                                                ctypes.POINTER(TriangleOptions), _i32, _vp,
                                                ctypes.POINTER(OpStats)]),
    "af2_triangle_multiplication": (_i32, [_vp, _i32, ctypes.POINTER(TriangleShape), _vp, _i32, _vp, _vp, _i64, _f64,
                                           ctypes.POINTER(TriangleOptions), _vp, _i32, _vp, _vp]),
    "af2_triangle_multiplication_static": (_i32, [_vp, _i32, ctypes.POINTER(TriangleShape), _vp, _i32, _vp, _vp, _i64,
                                                  _f64, ctypes.POINTER(TriangleOptions), _vp, _i32, _vp]),
    "af2_dequant_q8": (_i32, [_vp, ctypes.POINTER(Matrix), _i64, _i64, _vp, _vp]),
    "af2_triangle_multiplication_weights": (_i32, [_vp, _i32, ctypes.POINTER(TriangleShape), _vp, _i32, _vp,
                                                   ctypes.POINTER(Matrix), _f64, ctypes.POINTER(TriangleOptions), _vp,
                                                   _i32, _vp, _vp]),
    "af2_outer_product_mean_weights": (_i32, [_vp, ctypes.POINTER(OpmShape), _vp, _i32, _vp, ctypes.POINTER(Matrix),
                                              ctypes.POINTER(OpmOptions), _vp, _i32, _vp, _vp]),
    "af2_transition_weight_count": (_i64, [_i64, _i64]),
    "af2_transition_check": (_i32, [ctypes.POINTER(TransitionShape), _i64, _f64, ctypes.c_char_p, ctypes.c_size_t]),
    "af2_transition_workspace_bytes": (_i32, [ctypes.POINTER(TransitionShape), ctypes.POINTER(ctypes.c_uint64)]),
    "af2_transition_host": (_i32, [_vp, ctypes.POINTER(TransitionShape), _vp, _vp, _i64, _f64,
                                   ctypes.POINTER(TransitionOptions), _i32, _vp, ctypes.POINTER(OpStats)]),
    "af2_transition": (_i32, [_vp, ctypes.POINTER(TransitionShape), _vp, _i32, ctypes.POINTER(TransitionWeights),
                              _f64, ctypes.POINTER(TransitionOptions), _vp, _i32, _vp, _vp]),
    "af2_opm_weight_count": (_i64, [ctypes.POINTER(OpmShape)]),
    "af2_opm_check": (_i32, [ctypes.POINTER(OpmShape), _i64, ctypes.c_char_p, ctypes.c_size_t]),
    "af2_opm_workspace_bytes": (_i32, [ctypes.POINTER(OpmShape), ctypes.POINTER(OpmOptions),
                                       ctypes.POINTER(ctypes.c_uint64)]),
    "af2_outer_product_mean_host": (_i32, [_vp, ctypes.POINTER(OpmShape), _vp, _vp, _vp, _i64,
                                           ctypes.POINTER(OpmOptions), _i32, _vp, ctypes.POINTER(OpStats)]),
    "af2_outer_product_mean": (_i32, [_vp, ctypes.POINTER(OpmShape), _vp, _i32, _vp, _vp, _i64,
                                      ctypes.POINTER(OpmOptions), _vp, _i32, _vp, _vp]),
    "af2_comm_unique_id": (_i32, [_vp]),
    "af2_comm_init": (_i32, [_vp, _vp, _i32, _i32]),
    "af2_comm_destroy": (_i32, [_vp]),
    "af2_comm_set_timeout": (_i32, [_vp, _f64]),
    "af2_comm_abort": (_i32, [_vp]),
    "af2_triangle_multiplication_sharded": (_i32, [_vp, _i32, ctypes.POINTER(TriangleShape), _vp, _i32, _vp, _vp, _i64,
                                                   _f64, ctypes.POINTER(TriangleOptions), _vp, _i32, _vp]),
    "af2_outer_product_mean_sharded": (_i32, [_vp, ctypes.POINTER(OpmShape), _vp, _i32, _vp, _vp, _i64,
                                              ctypes.POINTER(OpmOptions), _vp, _i32, _vp]),
    "af2_attention_weight_count": (_i64, [ctypes.POINTER(AttentionShape), _i32]),
    "af2_attention_check": (_i32, [ctypes.POINTER(AttentionShape), _i32, _i64, _f64, ctypes.c_char_p,
                                   ctypes.c_size_t]),
    "af2_attention_workspace_bytes": (_i32, [ctypes.POINTER(AttentionShape), _i32, ctypes.POINTER(ctypes.c_uint64)]),
    "af2_attention_host": (_i32, [_vp, ctypes.POINTER(AttentionShape), _vp, _vp, _vp, _i64, _f64,
                                  ctypes.POINTER(AttentionOptions), _vp, ctypes.POINTER(OpStats)]),
    "af2_attention": (_i32, [_vp, ctypes.POINTER(AttentionShape), _vp, _i32, _vp, _vp, _i64, _f64,
                             ctypes.POINTER(AttentionOptions), _vp, _i32, _vp, _vp]),
    "af2_evoformer_pair_block": (_i32, [_vp, ctypes.POINTER(PairBlockShape), ctypes.POINTER(PairBlockWeights), _vp, _i32,
                                        _vp, _vp, _i32, _vp, ctypes.POINTER(PairBlockOptions), _vp]),
    "af2_linear_workspace_bytes": (_i32, [ctypes.POINTER(LinearShape), _i32, ctypes.POINTER(ctypes.c_uint64)]),
    "af2_linear": (_i32, [_vp, ctypes.POINTER(LinearShape), _vp, _i32, ctypes.POINTER(Matrix), _vp, _i32, _i32, _vp,
                          _i32, _vp, _vp]),
}

_lib = None


def lib() -> ctypes.CDLL:
    """The loaded library; raises OSError when it is absent (no fallback)."""
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise OSError(f"libaf2cuda.so not found at {LIB_PATH}; build it with "
                          "`python alphafold2-webgpu_b200/build.py`")
        handle = ctypes.CDLL(str(LIB_PATH))
        for name, (restype, argtypes) in SIGNATURES.items():
            fn = getattr(handle, name)
            fn.restype = restype
            fn.argtypes = argtypes
        _lib = handle
    return _lib


class Af2Error(RuntimeError):
    """A non-OK af2_status, with the library's message."""

    def __init__(self, status: int, message: str):
        super().__init__(f"{message} ({lib().af2_status_string(status).decode()})")
        self.status = status


class RangeError(ValueError):
    """The reference's RangeError: a shape, length or epsilon it rejects."""


def check(status: int, ctx=None) -> None:
    if status == AF2_OK:
        return
    msg = lib().af2_last_error(ctx).decode() if ctx else lib().af2_status_string(status).decode()
    if status == AF2_ERR_INVALID_ARGUMENT:
        raise RangeError(msg)
    raise Af2Error(status, msg)
