"""A CUDA device context: the af2_ctx handle behind every operator.

Plays the role the reference gives a GPUDevice from requestAlphaFoldDevice
(src/runtime/device.ts:375): operators are constructed with one.
"""
from __future__ import annotations

import ctypes

from . import _lib


class Device:
    def __init__(self, ordinal: int = 0):
        handle = ctypes.c_void_p()
        status = _lib.lib().af2_create(ordinal, ctypes.byref(handle))
        if status != _lib.AF2_OK:
            raise _lib.Af2Error(status, f"cannot open CUDA device {ordinal}")
        self.ordinal = ordinal
        self.handle = handle

    def sync(self, stream: int | None = None) -> None:
        """Waits for `stream` (default: the context's) and raises on kernel-side failures."""
        _lib.check(_lib.lib().af2_sync(self.handle, stream), self.handle)

    @property
    def launch_count(self) -> int:
        return int(_lib.lib().af2_launch_count(self.handle))

    @property
    def gemm_precision(self) -> str:
        """The installed GEMM precision: "matrix" (f16 operands, f32 accumulation) or "f32"
        (split hi/lo f16 operands for the ops that honour it), like the reference's
        gemmVariant().precision (src/runtime/gemm.ts:175,213-215)."""
        return {_lib.AF2_GEMM_MATRIX: "matrix", _lib.AF2_GEMM_F32: "f32"}[_lib.lib().af2_get_gemm_precision(self.handle)]

    def set_gemm_precision(self, precision: str) -> None:
        """Installs "matrix" or "f32" for this device's later calls (forceGemmVariant's role)."""
        code = {"matrix": _lib.AF2_GEMM_MATRIX, "f32": _lib.AF2_GEMM_F32}.get(precision)
        if code is None:
            raise _lib.RangeError(f"precision must be 'matrix' or 'f32'; received {precision}")
        _lib.check(_lib.lib().af2_set_gemm_precision(self.handle, code), self.handle)

    def set_weight_cache(self, enable: bool) -> None:
        """Keeps prepared weights per weights pointer and shape (made once; the weights must not
        change in place while cached -- see clear_weight_cache)."""
        _lib.check(_lib.lib().af2_set_weight_cache(self.handle, 1 if enable else 0), self.handle)

    def clear_weight_cache(self) -> None:
        _lib.check(_lib.lib().af2_clear_weight_cache(self.handle), self.handle)

    def memory_snapshot(self) -> dict:
        """{"currentBytes", "peakBytes"} of this context's device allocations
        (the reference allocator's snapshot(), src/runtime/allocator.ts:376-382)."""
        cur, peak = ctypes.c_uint64(), ctypes.c_uint64()
        _lib.check(_lib.lib().af2_memory_snapshot(self.handle, ctypes.byref(cur), ctypes.byref(peak)), self.handle)
        return {"currentBytes": int(cur.value), "peakBytes": int(peak.value)}

    def close(self) -> None:
        if self.handle:
            _lib.lib().af2_destroy(self.handle)
            self.handle = None

    def destroy(self) -> None:  # GPUDevice.destroy()
        self.close()

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
