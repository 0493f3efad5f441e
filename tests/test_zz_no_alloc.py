"""The allocation-free triangle entry point, af2_triangle_multiplication_static.

It exists for hosts that cannot let a library call cudaMalloc (a memory
manager that owns the device under a fixed budget, or a latency-sensitive
path where an allocation would synchronise the device): its scratch is a
fixed device array instead.  This file checks it through the C ABI against
the allocating entry point on the same inputs, for two calls in a row with
different inputs, so the second call also shows that what the first left in
the shared array does not leak into the result.  It runs last (file name) so
a failure here cannot hide an earlier one; it also passes on its own.
"""
import ctypes

import numpy as np
import pytest

from af2cuda import _lib
from helpers import pack, relative_max_error, triangle_case

pytestmark = pytest.mark.gpu

DTYPES = {"f32": _lib.AF2_F32, "bf16": _lib.AF2_BF16}


def _call(fn_name, device, direction, z, mask, w, out, residual, stream, workspace=None):
    n, _, cz = z.shape
    ch = int((w.numel() - (2 * cz + cz + cz * cz + cz)) // (4 * cz + 6 + cz))
    shape = _lib.TriangleShape(n, cz, ch)
    opts = _lib.TriangleOptions(0, 1 if residual else 0)
    zt = DTYPES["bf16" if str(z.dtype) == "torch.bfloat16" else "f32"]
    ot = DTYPES["bf16" if str(out.dtype) == "torch.bfloat16" else "f32"]
    args = [device.handle, direction, ctypes.byref(shape), z.data_ptr(), zt, mask.data_ptr(), w.data_ptr(), w.numel(),
            1e-5, ctypes.byref(opts), out.data_ptr(), ot]
    if fn_name == "af2_triangle_multiplication":
        args.append(workspace)
    args.append(stream)
    _lib.check(getattr(_lib.lib(), fn_name)(*args), device.handle)


@pytest.mark.parametrize("direction", [0, 1])
def test_static_scratch_matches_allocating_entry_point(device, direction):
    import torch
    stream = torch.cuda.Stream()
    for call, (n, seed, dtype) in enumerate([(128, 31, torch.float32), (77, 32, torch.bfloat16)]):
        z, mask, w = triangle_case(n, seed=seed + direction, mask_p=0.9, perturbed=True)
        zd = torch.from_numpy(z).to("cuda", dtype).contiguous()
        md = torch.from_numpy(mask).cuda()
        wd = torch.from_numpy(pack(w)).cuda()
        ref = torch.empty_like(zd)
        got = torch.full_like(zd, float("nan"))
        torch.cuda.synchronize()
        _call("af2_triangle_multiplication", device, direction, zd, md, wd, ref, False, stream.cuda_stream)
        device.sync(stream.cuda_stream)
        held = device.memory_snapshot()
        _call("af2_triangle_multiplication_static", device, direction, zd, md, wd, got, False, stream.cuda_stream)
        device.sync(stream.cuda_stream)
        # the static call allocated nothing through the context
        assert device.memory_snapshot() == held, f"call {call}"
        want = ref.float().cpu().numpy()
        have = got.float().cpu().numpy()
        assert np.isfinite(have).all(), f"call {call}"
        assert relative_max_error(have, want) <= 2e-3, f"call {call}"
        # same kernels, same inputs, same stream: the results agree bit for bit, so nothing a
        # previous call left in the shared array leaks into this one
        assert torch.equal(got, ref), f"call {call}"


def test_static_scratch_rejects_shapes_beyond_its_size(device):
    import torch
    z = torch.zeros(200, 200, 128, device="cuda", dtype=torch.bfloat16)
    mask = torch.ones(200, 200, device="cuda")
    w = torch.zeros(_lib.lib().af2_triangle_weight_count(128, 128), device="cuda")
    with pytest.raises(_lib.Af2Error, match="static scratch holds"):
        _call("af2_triangle_multiplication_static", device, 0, z, mask, w, z, True, 0)
