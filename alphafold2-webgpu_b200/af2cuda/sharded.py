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


def comm_set_timeout(device: Device, seconds: float) -> None:
    """Deadline of the library's host waits on work with collectives (af2_comm_set_timeout):
    after it, or at the communicator's first asynchronous error, the communicator is
    aborted and the wait raises Af2Error with AF2_ERR_NCCL."""
    _lib.check(_lib.lib().af2_comm_set_timeout(device.handle, float(seconds)), device.handle)


def comm_abort(device: Device) -> None:
    """Ends this rank's communicator without a collective (af2_comm_abort): after a peer is
    lost, or when this rank leaves.  The Device stays usable."""
    _lib.check(_lib.lib().af2_comm_abort(device.handle), device.handle)


class PeerLost(RuntimeError):
    """A rank left or stopped answering between steps."""

    def __init__(self, missing, step):
        super().__init__(f"rank(s) {sorted(missing)} did not reach step {step}")
        self.missing = sorted(missing)
        self.step = step


class PeerMonitor:
    """Host-side liveness of the ranks that share a communicator, through a
    torch.distributed store (the TCPStore of the process group, for instance).

    Before each step's launches every rank calls ``step()``: it marks the rank as
    having reached the step and waits (at most ``timeout`` seconds) until every
    rank has, so a rank that left or died between steps is found on the host
    before any collective that would wait for it is queued.  A rank that leaves
    on purpose calls ``leave()``, and the others see it at once instead of at the
    deadline."""

    def __init__(self, store, rank: int, nranks: int, timeout: float = 60.0, prefix: str = "af2/peers"):
        self.store, self.rank, self.nranks = store, rank, nranks
        self.timeout, self.prefix = float(timeout), prefix
        self.count = 0

    def _key(self, what, rank, step=None):
        return f"{self.prefix}/{what}/{rank}" + ("" if step is None else f"/{step}")

    def _left(self):
        return {r for r in range(self.nranks) if r != self.rank and self.store.check([self._key("left", r)])}

    def step(self) -> int:
        """Marks this rank at the next step and waits for the others; raises PeerLost."""
        import time
        step = self.count
        self.store.set(self._key("step", self.rank, step), "1")
        waiting = set(range(self.nranks)) - {self.rank}
        deadline = time.monotonic() + self.timeout
        while waiting:
            gone = self._left() & waiting
            if gone:
                raise PeerLost(gone, step)
            for r in list(waiting):
                if self.store.check([self._key("step", r, step)]):
                    waiting.discard(r)
            if waiting and time.monotonic() > deadline:
                raise PeerLost(waiting, step)
            if waiting:
                time.sleep(0.005)
        self.count += 1
        return step

    def leave(self) -> None:
        """Tells the other ranks that this one has left (between steps)."""
        self.store.set(self._key("left", self.rank), "1")


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
