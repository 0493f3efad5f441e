"""GPU parity of triangle multiplication through the C ABI against the oracle
and the reference's golden bundles.

Tolerances: the benchmark configs' bar for f16/bf16 operands with f32
accumulation, max|d| / max|ref| <= 2e-3, and on the golden bundles also the
reference's own half-precision bar, mean < 1e-3 and max < 1e-2
(test/triangle-multiplication-outgoing.gpu.test.ts:58-92).
"""
import numpy as np
import pytest

import af2cuda
import oracle
from conftest import GOLDEN_BUNDLES, bundle_path
from helpers import bf16_round, pack, relative_max_error, triangle_case

pytestmark = pytest.mark.gpu

REL_TOL = 2e-3


def _input(z, mask, w, eps=1e-5):
    n, _, cz = z.shape
    ch = w["linearAPBias"].size
    weights = af2cuda.TriangleMultiplicationWeights(**{k: np.asarray(v, np.float32).ravel() for k, v in w.items()})
    return af2cuda.TriangleMultiplicationInput(af2cuda.TriangleShape(n, cz, ch), z.ravel(), mask.ravel(), weights, eps)


OPS = {0: af2cuda.TriangleMultiplicationOutgoingGpu, 1: af2cuda.TriangleMultiplicationIncomingGpu}


@pytest.mark.parametrize("name", GOLDEN_BUNDLES)
def test_golden_bundles(device, name):
    bundle = af2cuda.load_triangle_reference_bundle_from_files(bundle_path(name))
    result = af2cuda.TriangleMultiplicationOutgoingGpu(device).run(bundle.input)
    m = af2cuda.error_metrics(result.output, bundle.expected)
    assert m["meanAbsoluteError"] < 1e-3 and m["maxAbsoluteError"] < 1e-2, m
    assert relative_max_error(result.output, bundle.expected) <= REL_TOL
    assert result.elapsedMilliseconds > 0 and result.memory.workspaceBytes > 0


@pytest.mark.parametrize("direction", [0, 1])
@pytest.mark.parametrize("n", [5, 9, 59, 128, 130, 200])
def test_matches_oracle(device, direction, n):
    z, mask, w = triangle_case(n, seed=n, mask_p=0.85, perturbed=True)
    expected = oracle.triangle(direction, z, mask, pack(w))
    out = OPS[direction](device).run(_input(z, mask, w)).output.reshape(z.shape)
    assert np.isfinite(out).all()
    assert relative_max_error(out, expected) <= REL_TOL


@pytest.mark.parametrize("direction", [0, 1])
@pytest.mark.parametrize("cz,ch", [(64, 64), (7, 6), (128, 32)])
def test_narrow_channels(device, direction, cz, ch):
    z, mask, w = triangle_case(37, cz, ch, seed=cz + ch, mask_p=0.9, perturbed=True)
    expected = oracle.triangle(direction, z, mask, pack(w))
    out = OPS[direction](device).run(_input(z, mask, w)).output.reshape(z.shape)
    assert relative_max_error(out, expected) <= REL_TOL


@pytest.mark.parametrize("direction", [0, 1])
def test_block_rows_are_bit_identical(device, direction):
    # The reference requires blocked runs to give the same answer
    # (test/triangle-multiplication-outgoing.gpu.test.ts:48-56); here they are bit-identical.
    z, mask, w = triangle_case(130, seed=11, mask_p=0.9, perturbed=True)
    inp = _input(z, mask, w)
    op = OPS[direction](device)
    whole = op.run(inp).output
    for rows in (64, 17, 129):
        assert np.array_equal(op.run(inp, {"blockRows": rows}).output, whole), rows


def test_f16_host_storage(device):
    """hostStorage "f16" (not a reference option) moves the pair as half-precision arrays."""
    z, mask, w = triangle_case(96, seed=3, perturbed=True)
    z16 = z.astype(np.float16).astype(np.float32)
    expected = oracle.triangle(0, z16, mask, pack(w))
    out = af2cuda.TriangleMultiplicationOutgoingGpu(device).run(_input(z16, mask, w), {"hostStorage": "f16"}).output
    # f16 output rounding adds at most 2^-11 relative per element.
    assert relative_max_error(out.reshape(z.shape), expected) <= REL_TOL + 2 ** -11


@pytest.mark.parametrize("direction", [0, 1])
def test_precision_option_keeps_the_pair_f32(device, direction):
    """{precision: "f16"} selects the weight and arithmetic precision; the pair stays f32 in
    and out, as in the reference (src/triangle/webgpu.ts:56-61,93-99): the output is an f32
    array within 2e-3 of the oracle on unrounded f32 inputs, identical to the f32 option's,
    and both whole-projection storages run."""
    z, mask, w = triangle_case(80, seed=21 + direction, mask_p=0.9, perturbed=True)
    expected = oracle.triangle(direction, z, mask, pack(w))
    op = OPS[direction](device)
    out16 = op.run(_input(z, mask, w), {"precision": "f16"}).output
    assert out16.dtype == np.float32 and out16.size == z.size
    assert relative_max_error(out16.reshape(z.shape), expected) <= REL_TOL
    assert np.array_equal(out16, op.run(_input(z, mask, w), {"precision": "f32"}).output)
    assert np.array_equal(out16, op.run(_input(z, mask, w), {"precision": "f16", "wholeStorage": "f16"}).output)
    with pytest.raises(af2cuda.RangeError):
        op.run(_input(z, mask, w), {"wholeStorage": "bf16"})


def test_masked_rows_and_all_masked(device):
    z, mask, w = triangle_case(70, seed=8, perturbed=True)
    mask[:, 5:9] = 0
    mask[11, :] = 0
    for direction in (0, 1):
        expected = oracle.triangle(direction, z, mask, pack(w))
        out = OPS[direction](device).run(_input(z, mask, w)).output.reshape(z.shape)
        assert relative_max_error(out, expected) <= REL_TOL
    zero = np.zeros_like(mask)
    expected = oracle.triangle(0, z, zero, pack(w))
    out = OPS[0](device).run(_input(z, zero, w)).output.reshape(z.shape)
    assert relative_max_error(out, expected) <= REL_TOL


@pytest.mark.parametrize("direction", [0, 1])
def test_device_form_bf16_pair_in_place(device, direction):
    """The in-model form: a bf16 pair updated in place (residualTarget = pair)."""
    import torch
    n = 256
    z, mask, w = triangle_case(n, seed=21 + direction, mask_p=0.95)
    zb = bf16_round(z)
    update = oracle.triangle(direction, zb, mask, pack(w))
    pair = torch.from_numpy(zb).to("cuda", torch.bfloat16).contiguous()
    mask_d = torch.from_numpy(mask).cuda()
    w_d = torch.from_numpy(pack(w)).cuda()
    torch.cuda.synchronize()
    af2cuda.encode_triangle_multiplication_tensors(device, direction, pair, mask_d, w_d, residual=True)
    device.sync()
    got = pair.float().cpu().numpy()
    want = zb.astype(np.float64) + update
    err = np.abs(got - want)
    # The bf16 pair is updated by a TMA add of the bf16-rounded update: one
    # rounding of the update (2^-9 relative) and one of the sum (2^-9, with
    # slack), on top of the operator's own tolerance.
    bound = 2.0 ** -8 * np.abs(want) + 2.0 ** -9 * np.abs(update) + REL_TOL * np.abs(update).max()
    assert np.all(err <= bound), float((err - bound).max())


def test_device_form_f32_out_matches_host_form(device):
    import torch
    z, mask, w = triangle_case(64, seed=2, perturbed=True)
    host = af2cuda.TriangleMultiplicationIncomingGpu(device).run(_input(z, mask, w)).output
    zd = torch.from_numpy(z).cuda()
    out = torch.empty_like(zd)
    torch.cuda.synchronize()
    af2cuda.encode_triangle_multiplication_tensors(device, "incoming", zd, torch.from_numpy(mask).cuda(),
                                                   torch.from_numpy(pack(w)).cuda(), out=out, residual=False)
    device.sync()
    assert np.array_equal(out.cpu().numpy().ravel(), host)


def test_launches_are_counted(device):
    z, mask, w = triangle_case(16, seed=1)
    before = device.launch_count
    af2cuda.TriangleMultiplicationOutgoingGpu(device).run(_input(z, mask, w))
    # weight preparation, z re-layout, projection, contraction, output
    assert device.launch_count - before == 5
