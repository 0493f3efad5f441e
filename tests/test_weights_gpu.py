"""GPU parity of the per-tensor weight forms (af2_triangle_multiplication_weights,
af2_outer_product_mean_weights) with mixed-q8 tensors read from a manifest in
the reference's format (src/reference/tensor-store.ts:40-121, dtype.ts:66-99).

Bars: the device decode of each q8 tensor equals the reference's decode bit for
bit; each op's result equals, bit for bit, the packed form given the decoded
f32 weights (the decode is exact, so the q8 path may not differ at all); and
the result is within 2e-3 (max|d| / max|ref|) of the oracle on the decoded
weights."""
import numpy as np
import pytest

import af2cuda
import oracle
from helpers import pack, relative_max_error, triangle_weights

pytestmark = pytest.mark.gpu

TRI_NAMES = {k: f"triangle/{k}" for k in af2cuda.ORDER}
OPM_NAMES = {k: f"opm/{k}" for k in ("layerNormScale", "layerNormOffset", "leftWeight", "leftBias", "rightWeight",
                                     "rightBias", "outputWeight", "outputBias")}


def _triangle_store(tmp_path, rng, cz=128, ch=128, blocks=2):
    stacked = {}
    for k in af2cuda.ORDER:
        per = [triangle_weights(cz, ch, rng, perturbed=True)[k] for _ in range(blocks)]
        stacked[TRI_NAMES[k]] = np.stack(per)
    q8 = {TRI_NAMES[k] for k in af2cuda.ORDER if k.endswith("Weight") and k.startswith("linear")}
    q8 |= {TRI_NAMES["linearAGBias"]}  # a q8 vector too
    path = af2cuda.write_tensor_manifest(tmp_path / "tri", stacked, q8=q8)
    return af2cuda.FileTensorStore.open(path), q8


def _opm_store(tmp_path, rng, cm=64, c=32, cz=128, blocks=3):
    def mat(i, o):
        return (rng.standard_normal((blocks, i, o)) / np.sqrt(i)).astype(np.float32)

    def vec(k, center=0.0):
        return (center + 0.1 * rng.standard_normal((blocks, k))).astype(np.float32)

    stacked = {OPM_NAMES["layerNormScale"]: vec(cm, 1.0), OPM_NAMES["layerNormOffset"]: vec(cm),
               OPM_NAMES["leftWeight"]: mat(cm, c), OPM_NAMES["leftBias"]: vec(c),
               OPM_NAMES["rightWeight"]: mat(cm, c), OPM_NAMES["rightBias"]: vec(c),
               OPM_NAMES["outputWeight"]: mat(c * c, cz), OPM_NAMES["outputBias"]: vec(cz)}
    # every tensor q8 except the LayerNorm scale: the 32-value biases of block 1 start inside a scale block
    q8 = set(stacked) - {OPM_NAMES["layerNormScale"]}
    path = af2cuda.write_tensor_manifest(tmp_path / "opm", stacked, q8=q8)
    return af2cuda.FileTensorStore.open(path), q8


def _decoded(store, names, block, blocks):
    for name in names.values():
        store.ensure_loaded(name)
    return {k: store.read(name, block, blocks) for k, name in names.items()}


def test_device_decode_is_the_reference_decode(device, tmp_path):
    import torch
    store, q8 = _triangle_store(tmp_path, np.random.default_rng(0))
    for name in sorted(q8):
        store.ensure_loaded(name)
        for b in range(2):
            w = store.device_weight(name, b, 2)
            assert isinstance(w, af2cuda.Q8Matrix)
            got = af2cuda.dequant_q8_tensors(device, w, 1, int(w.codes.numel()))
            device.sync()
            want = torch.from_numpy(np.array(store.read(name, b, 2))).view(1, -1)
            assert torch.equal(got.cpu(), want), name


@pytest.mark.parametrize("direction", [0, 1])
@pytest.mark.parametrize("n", [40, 130])
def test_triangle_q8_tensors_equal_the_packed_form(device, tmp_path, direction, n):
    import torch
    store, _ = _triangle_store(tmp_path, np.random.default_rng(n + direction))
    rng = np.random.default_rng(1)
    z = rng.standard_normal((n, n, 128)).astype(np.float32)
    mask = (rng.random((n, n)) < 0.9).astype(np.float32)
    zd, md = torch.from_numpy(z).cuda(), torch.from_numpy(mask).cuda()
    for block in range(2):
        weights = af2cuda.stored_weights(store, TRI_NAMES, block, 2)
        decoded = _decoded(store, TRI_NAMES, block, 2)
        packed = torch.from_numpy(pack(decoded)).cuda()
        torch.cuda.synchronize()
        got = af2cuda.encode_triangle_multiplication_weight_tensors(
            device, direction, zd, md, weights, out=torch.empty_like(zd), residual=False)
        ref = af2cuda.encode_triangle_multiplication_tensors(device, direction, zd, md, packed,
                                                             out=torch.empty_like(zd), residual=False)
        device.sync()
        assert torch.equal(got, ref)
        want = oracle.triangle(direction, z, mask, pack(decoded))
        assert relative_max_error(got.cpu().numpy(), want) <= 2e-3


@pytest.mark.parametrize("n,s", [(24, 20), (70, 129)])
def test_opm_q8_tensors_equal_the_packed_form(device, tmp_path, n, s):
    import torch
    store, _ = _opm_store(tmp_path, np.random.default_rng(n))
    rng = np.random.default_rng(2)
    m = rng.standard_normal((s, n, 64)).astype(np.float32)
    mask = (rng.random((s, n)) < 0.9).astype(np.float32)
    mask[0] = 1
    md, maskd = torch.from_numpy(m).to("cuda", torch.bfloat16), torch.from_numpy(mask).cuda()
    for block in range(3):
        weights = af2cuda.stored_weights(store, OPM_NAMES, block, 3)
        if block == 1:
            assert not isinstance(weights["leftBias"], af2cuda.Q8Matrix)  # decoded: starts mid scale block
        decoded = _decoded(store, OPM_NAMES, block, 3)
        packed = np.concatenate([np.asarray(decoded[k], np.float32).ravel() for k in OPM_NAMES])
        torch.cuda.synchronize()
        got = af2cuda.encode_outer_product_mean_weight_tensors(device, md, maskd, weights,
                                                               out=torch.empty(n, n, 128, device="cuda"),
                                                               residual=False)
        ref = af2cuda.encode_outer_product_mean_tensors(device, md, maskd, torch.from_numpy(packed).cuda(), 32, 128,
                                                        out=torch.empty(n, n, 128, device="cuda"), residual=False)
        device.sync()
        assert torch.equal(got, ref)
        m_rounded = md.float().cpu().numpy()
        want = oracle.outer_product_mean(m_rounded, mask, packed, 32, 128)
        assert relative_max_error(got.cpu().numpy(), want) <= 2e-3


def test_q8_tensors_with_the_weight_cache(device, tmp_path):
    """Cached per-tensor weights give the same bits, keyed by both codes and scales."""
    import torch
    store, _ = _triangle_store(tmp_path, np.random.default_rng(5))
    weights = af2cuda.stored_weights(store, TRI_NAMES, 0, 2)
    z = torch.randn(48, 48, 128, device="cuda")
    mask = torch.ones(48, 48, device="cuda")
    torch.cuda.synchronize()

    def run():
        return af2cuda.encode_triangle_multiplication_weight_tensors(device, 0, z, mask, weights,
                                                                     out=torch.empty_like(z), residual=False)
    plain = run()
    device.set_weight_cache(True)
    try:
        a, b = run(), run()
        device.sync()
        assert torch.equal(a, plain) and torch.equal(b, plain)
        other = dict(weights)
        w = weights["linearAPWeight"]
        other["linearAPWeight"] = af2cuda.Q8Matrix(w.codes, w.scales.clone(), "block", w.block)
        other["linearAPWeight"].scales.view(torch.float16).mul_(2)
        torch.cuda.synchronize()
        c = af2cuda.encode_triangle_multiplication_weight_tensors(device, 0, z, mask, other,
                                                                  out=torch.empty_like(z), residual=False)
        device.sync()
        assert not torch.equal(c, plain)  # a new scales array is a new cache entry
    finally:
        device.set_weight_cache(False)


def test_per_channel_q8_and_bad_tensors_are_rejected(device):
    import ctypes

    import torch
    from af2cuda import _lib
    codes = torch.zeros(128 * 128, dtype=torch.int8, device="cuda")
    scales = torch.ones(128, device="cuda")
    z = torch.zeros(8, 8, 128, device="cuda")
    mask = torch.ones(8, 8, device="cuda")
    mats = (_lib.Matrix * 16)(*[_lib.Matrix(_lib.AF2_WEIGHTS_F32, 0, z.data_ptr(), None) for _ in range(16)])
    mats[2] = _lib.Matrix(_lib.AF2_WEIGHTS_Q8_CHANNEL, 0, codes.data_ptr(), scales.data_ptr())
    shape = _lib.TriangleShape(8, 128, 128)
    status = _lib.lib().af2_triangle_multiplication_weights(device.handle, 0, ctypes.byref(shape), z.data_ptr(),
                                                            _lib.AF2_F32, mask.data_ptr(), mats, 1e-5, None,
                                                            z.data_ptr(), _lib.AF2_F32, None, None)
    assert status == _lib.AF2_ERR_UNSUPPORTED
    mats[2] = _lib.Matrix(_lib.AF2_WEIGHTS_Q8_BLOCK, 64, codes.data_ptr(), None)
    status = _lib.lib().af2_triangle_multiplication_weights(device.handle, 0, ctypes.byref(shape), z.data_ptr(),
                                                            _lib.AF2_F32, mask.data_ptr(), mats, 1e-5, None,
                                                            z.data_ptr(), _lib.AF2_F32, None, None)
    assert status == _lib.AF2_ERR_INVALID_ARGUMENT
    with pytest.raises(af2cuda.RangeError):
        af2cuda.encode_triangle_multiplication_weight_tensors(
            device, 0, z, mask, {k: torch.zeros(3, device="cuda") for k in af2cuda.ORDER})
