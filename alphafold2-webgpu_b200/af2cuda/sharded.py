"""The pair representation sharded by rows across the GPUs of one box.

One process and one Device per GPU.  Rank 0 creates a unique id, the host
hands it to every rank (``torch.distributed.broadcast_object_list`` over any
process group), and every rank opens the communicator with it; the library's
NCCL exchanges then run on the given streams.  ``rows_of(length, nranks,
rank)`` is the row range a rank holds.
"""
from __future__ import annotations

import ctypes

from . import _lib
from .device import Device
from .triangle import _TORCH_DTYPES, _DTYPES, _hidden_from_count

UNIQUE_ID_BYTES = 128


def comm_unique_id() -> bytes:
    buf = ctypes.create_string_buffer(UNIQUE_ID_BYTES)
    status = _lib.lib().af2_comm_unique_id(buf)
    if status != _lib.AF2_OK:
        raise _lib.Af2Error(status, "af2_comm_unique_id failed")
    return buf.raw


def comm_init(device: Device, unique_id: bytes, nranks: int, rank: int) -> None:
    buf = ctypes.create_string_buffer(bytes(unique_id), UNIQUE_ID_BYTES)
    _lib.check(_lib.lib().af2_comm_init(device.handle, buf, nranks, rank), device.handle)


def comm_destroy(device: Device) -> None:
    _lib.check(_lib.lib().af2_comm_destroy(device.handle), device.handle)


def rows_of(length: int, nranks: int, rank: int) -> tuple[int, int]:
    """[begin, end) of the pair rows rank `rank` holds."""
    per = length // nranks
    return rank * per, (rank + 1) * per


def encode_triangle_multiplication_sharded_tensors(device: Device, direction, pair_rows, mask_rows, packed_weights,
                                                   length: int, *, out=None, residual: bool = True,
                                                   epsilon: float = 1e-5, stream: int = 0):
    """Row-sharded device form: pair_rows [L, N, c_z] and mask_rows [L, N] are this
    rank's rows (L = N / nranks, a multiple of 64; nranks divides 128).  The
    contraction is sharded by hidden channel between two all-to-alls.
    Collective: every rank calls it together."""
    rows, n, cz = pair_rows.shape
    if n != length:
        raise _lib.RangeError("pair_rows must be [rows, length, c_z]")
    d = direction if isinstance(direction, int) else {"outgoing": 0, "incoming": 1}[direction]
    count = packed_weights.numel()
    ch = _hidden_from_count(cz, count)
    target = pair_rows if out is None else out
    for t in (pair_rows, mask_rows, packed_weights, target):
        if not t.is_cuda or not t.is_contiguous():
            raise _lib.RangeError("tensors must be contiguous CUDA tensors")
    shape = _lib.TriangleShape(length, cz, ch)
    opts = _lib.TriangleOptions(0, 1 if residual else 0)
    status = _lib.lib().af2_triangle_multiplication_sharded(
        device.handle, d, ctypes.byref(shape), pair_rows.data_ptr(), _DTYPES[_TORCH_DTYPES[str(pair_rows.dtype)]],
        mask_rows.data_ptr(), packed_weights.data_ptr(), count, float(epsilon), ctypes.byref(opts),
        target.data_ptr(), _DTYPES[_TORCH_DTYPES[str(target.dtype)]], stream or None)
    _lib.check(status, device.handle)
    return target


def encode_outer_product_mean_sharded_tensors(device: Device, msa, msa_mask, packed_weights, c_outer: int, c_z: int,
                                              pair_rows, *, residual: bool = True, row_block: int = 0,
                                              layer_norm_epsilon: float = 1e-5, normalization_epsilon: float = 1e-3,
                                              stream: int = 0):
    """Row-sharded OPM: msa [S, L, c_m] this rank's residue columns of the MSA,
    msa_mask [S, N] the whole mask (the same on every rank), pair_rows [L, N, c_z]
    this rank's rows of the pair (updated when residual).  Collective: every rank
    calls it together."""
    from .opm import _TORCH_DTYPES as _T
    s, _, cm = msa.shape
    n = pair_rows.shape[1]
    if msa_mask.shape[-1] != n or n % msa.shape[1] != 0:
        raise _lib.RangeError("msa must hold this rank's residue columns and msa_mask all N of them")
    for t in (msa, msa_mask, packed_weights, pair_rows):
        if not t.is_cuda or not t.is_contiguous():
            raise _lib.RangeError("tensors must be contiguous CUDA tensors")
    shape = _lib.OpmShape(s, n, cm, c_outer, c_z)
    opts = _lib.OpmOptions(float(layer_norm_epsilon), float(normalization_epsilon), int(row_block),
                           1 if residual else 0)
    status = _lib.lib().af2_outer_product_mean_sharded(
        device.handle, ctypes.byref(shape), msa.data_ptr(), _DTYPES[_T[str(msa.dtype)]], msa_mask.data_ptr(),
        packed_weights.data_ptr(), packed_weights.numel(), ctypes.byref(opts), pair_rows.data_ptr(),
        _DTYPES[_T[str(pair_rows.dtype)]], stream or None)
    _lib.check(status, device.handle)
    return pair_rows
