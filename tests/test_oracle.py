"""CPU tests of the oracle: pinned against the reference's golden bundles and
known-answer tests, and cross-checked against independent numpy statements.
The oracle is the checker the GPU parity tests trust, so it is pinned first."""
import numpy as np
import pytest

import oracle
from conftest import GOLDEN_BUNDLES, bundle_path
from helpers import (opm_reference_test_case, opm_reference_test_expected, pack, triangle_case,
                     triangle_weights)

import af2cuda


@pytest.mark.parametrize("name", GOLDEN_BUNDLES)
def test_oracle_matches_golden_bundle(name):
    bundle = af2cuda.load_triangle_reference_bundle_from_files(bundle_path(name))
    inp = bundle.input
    n, cz = inp.shape.length, inp.shape.cZ
    packed, _ = af2cuda.pack_weights(inp.weights)
    out = oracle.triangle(0, inp.z.reshape(n, n, cz), inp.mask.reshape(n, n), packed, inp.epsilon)
    m = oracle.error_metrics(out, bundle.expected)
    if bundle.source.startswith("OpenFold"):
        # The reference's own CPU bar against the OpenFold oracle (test/cpu-reference.test.ts:18-28).
        assert m["meanAbsoluteError"] < 1e-7 and m["maxAbsoluteError"] < 1e-6, m
    else:
        # The reference's f32 bar against official AlphaFold activations
        # (test/triangle-multiplication-outgoing.gpu.test.ts:40-46).
        assert m["meanAbsoluteError"] < 1e-5 and m["maxAbsoluteError"] < 1e-4, m


def test_golden_bundles_are_intact():
    import hashlib
    import json
    from conftest import GOLDEN
    sums = json.loads((GOLDEN / "SHA256SUMS.json").read_text())
    for rel, digest in sums.items():
        assert hashlib.sha256((GOLDEN / rel).read_bytes()).hexdigest() == digest, rel


def test_error_metrics_known_answer():
    # test/cpu-reference.test.ts:35-41.
    m = oracle.error_metrics(np.array([1, 3], np.float32), np.array([2, 1], np.float32))
    assert m["meanAbsoluteError"] == 1.5 and m["maxAbsoluteError"] == 2
    assert m["rootMeanSquareError"] == pytest.approx(np.sqrt(2.5), rel=1e-15)
    assert af2cuda.error_metrics([1, 3], [2, 1]) == pytest.approx(
        {"meanAbsoluteError": 1.5, "maxAbsoluteError": 2.0, "rootMeanSquareError": np.sqrt(2.5)})


def test_oracle_is_deterministic_across_thread_counts():
    z, mask, w = triangle_case(7, 8, 5, seed=3, mask_p=0.8, perturbed=True)
    one = oracle.triangle(0, z, mask, pack(w), threads=1)
    many = oracle.triangle(0, z, mask, pack(w), threads=4)
    assert np.array_equal(one, many)


def _numpy_triangle(direction, z, mask, w, eps=1e-5):
    """An independent float64 numpy statement of the triangle update."""
    def ln(x, g, b):
        m = x.mean(-1, keepdims=True)
        v = ((x - m) ** 2).mean(-1, keepdims=True)
        return (x - m) / np.sqrt(v + eps) * g + b
    sig = lambda v: 1 / (1 + np.exp(-v))
    f = {k: np.asarray(v, np.float64) for k, v in w.items()}
    zn = ln(z.astype(np.float64), f["layerNormInWeight"], f["layerNormInBias"])
    m = mask[..., None].astype(np.float64)
    a = (zn @ f["linearAPWeight"].T + f["linearAPBias"]) * sig(zn @ f["linearAGWeight"].T + f["linearAGBias"]) * m
    b = (zn @ f["linearBPWeight"].T + f["linearBPBias"]) * sig(zn @ f["linearBGWeight"].T + f["linearBGBias"]) * m
    x = np.einsum("ikc,jkc->ijc", a, b) if direction == 0 else np.einsum("kjc,kic->ijc", a, b)
    xn = ln(x, f["layerNormOutWeight"], f["layerNormOutBias"])
    return (xn @ f["linearZWeight"].T + f["linearZBias"]) * sig(zn @ f["linearGWeight"].T + f["linearGBias"])


@pytest.mark.parametrize("direction", [0, 1])
def test_oracle_matches_independent_numpy(direction):
    z, mask, w = triangle_case(11, 16, 12, seed=5, mask_p=0.7, perturbed=True)
    out = oracle.triangle(direction, z, mask, pack(w))
    ref = _numpy_triangle(direction, z, mask, w)
    assert np.abs(out - ref).max() < 1e-5 * np.abs(ref).max()


def test_incoming_is_outgoing_of_the_transposed_pair():
    """incoming(z) = transpose(outgoing(transpose(z))) with the mask transposed:
    pins the incoming restatement, which has no golden bundle in the reference."""
    z, mask, w = triangle_case(9, 8, 6, seed=7, mask_p=0.8, perturbed=True)
    incoming = oracle.triangle(1, z, mask, pack(w))
    outgoing_t = oracle.triangle(0, np.ascontiguousarray(z.transpose(1, 0, 2)), np.ascontiguousarray(mask.T), pack(w))
    np.testing.assert_allclose(incoming, outgoing_t.transpose(1, 0, 2), rtol=0, atol=2e-6)


def test_f16_packing_known_answers():
    # numberToFloat16 (src/runtime/float16.ts:5-29) on exact and rounding cases.
    cases = {1.0: 0x3C00, -2.0: 0xC000, 65504.0: 0x7BFF, 65520.0: 0x7C00, 1e-8: 0x0000, 0.0: 0x0000,
             float("inf"): 0x7C00, 2.0 ** -14: 0x0400, 2.0 ** -24: 0x0001, 1.0 + 2.0 ** -11: 0x3C00,
             1.0 + 3 * 2.0 ** -11: 0x3C02}
    for value, bits in cases.items():
        assert int(oracle.f16_bits(np.float32(value))) == bits, value
    assert np.isnan(oracle.f16_value(0x7E00))
    # Normal values agree with IEEE round-to-nearest-even (numpy).
    rng = np.random.default_rng(0)
    x = (rng.standard_normal(4096) * 100).astype(np.float32)
    assert np.array_equal(oracle.f16_bits(x), x.astype(np.float16).view(np.uint16))
    assert np.array_equal(oracle.f16_value(oracle.f16_bits(x)), x.astype(np.float16).astype(np.float64))


def test_reference_f16_and_int8_known_answers():
    """The reference's own KATs: numberToFloat16 (test/float16.test.ts:5-30) and the
    int8 block decode with stored f16 scales (test/dtype.test.ts:6-23)."""
    cases = [(0.0, 0x0000), (-0.0, 0x8000), (1.0, 0x3C00), (-2.0, 0xC000), (float("inf"), 0x7C00),
             (float("-inf"), 0xFC00), (0.5, 0x3800), (-4.0, 0xC400),
             # round to nearest even
             (-0.748291015625, 0xB9FC), (16.1171875, 0x4C08), (52.859375, 0x529C), (-78.96875, 0xD4F0),
             (0.000061005353927612305, 0x0400)]
    for value, bits in cases:
        assert int(oracle.f16_bits(np.float32(value))) == bits, value
    assert int(oracle.f16_bits(np.float32("nan"))) & 0x7C00 == 0x7C00
    assert oracle.f16_value(0x3C00) == 1 and oracle.f16_value(0xC000) == -2
    assert oracle.f16_value(0x0001) == 2.0 ** -24 and oracle.f16_value(0x7C00) == float("inf")
    codes = np.array([1, -2, 3, -4, 5], np.int8)
    scales = np.array([0x3800, 0x4000], np.uint16)  # 0.5, 2.0
    assert oracle.dequant_q8_block(codes, scales, 4).tolist() == [0.5, -1, 1.5, -2, 10]


def test_q8_block_round_trip():
    rng = np.random.default_rng(1)
    w = (rng.standard_normal(1000) / 8).astype(np.float32)
    w[64:128] = 0  # an all-zero block keeps a zero scale and decodes to zeros
    codes, scales = oracle.quantize_q8_block(w, 64)
    assert codes.min() >= -127 and codes.max() <= 127
    assert scales[1] == 0
    decoded = oracle.dequant_q8_block(codes, scales, 64)
    blocks = np.repeat(oracle.f16_value(scales), 64)[: w.size]
    # decode is code * scale exactly (dtype.ts:86-97): a 7-bit by 11-bit product, exact in f32.
    assert np.array_equal(decoded, (codes.astype(np.float64) * blocks).astype(np.float32))
    assert np.abs(decoded - w).max() <= blocks.max() / 2 + 1e-7


def test_q8_column_round_trip():
    rng = np.random.default_rng(2)
    w = (rng.standard_normal((128, 512)) / np.sqrt(128)).astype(np.float32)
    codes, scales = oracle.quantize_q8_columns(w)
    decoded = oracle.dequant_q8_columns(codes, scales)
    assert np.array_equal(decoded, codes.astype(np.float32) * scales[None, :])
    assert np.all(np.abs(decoded - w) <= scales[None, :] / 2 + 1e-7)
    assert np.all(np.abs(codes).max(0) == 127)


def test_outer_product_mean_matches_numpy():
    rng = np.random.default_rng(4)
    s, n, cm, c, cz = 9, 8, 12, 32, 16
    m = rng.standard_normal((s, n, cm)).astype(np.float32)
    mask = (rng.random((s, n)) < 0.8).astype(np.float32)
    parts = [1 + 0.1 * rng.standard_normal(cm), 0.1 * rng.standard_normal(cm),
             rng.standard_normal((cm, c)) / np.sqrt(cm), 0.1 * rng.standard_normal(c),
             rng.standard_normal((cm, c)) / np.sqrt(cm), 0.1 * rng.standard_normal(c),
             rng.standard_normal((c * c, cz)) / c, 0.1 * rng.standard_normal(cz)]
    packed = np.concatenate([np.asarray(p, np.float32).ravel() for p in parts])
    out = oracle.outer_product_mean(m, mask, packed, c, cz)
    f = [np.asarray(p, np.float64) for p in parts]
    x = m.astype(np.float64)
    xn = (x - x.mean(-1, keepdims=True)) / np.sqrt(x.var(-1, keepdims=True) + 1e-5) * f[0] + f[1]
    left = (xn @ f[2] + f[3]) * mask[..., None]
    right = (xn @ f[4] + f[5]) * mask[..., None]
    outer = np.einsum("sia,sjb->ijab", left, right).reshape(n, n, c * c)
    cnt = np.einsum("si,sj->ij", mask, mask)
    ref = (outer @ f[6] + f[7]) / (1e-3 + cnt)[..., None]
    assert np.abs(out - ref).max() < 1e-5 * np.abs(ref).max()


def test_outer_product_mean_on_the_reference_tests_own_case():
    """The reference's OPM test case (spread inputs, every third mask entry zero):
    the oracle reproduces that test's CPU `reference()` with its f32 stores exactly
    (the reference holds its GPU path to mean < 2e-5, max < 2e-4 against it)."""
    m, mask, w, _ = opm_reference_test_case()
    packed = np.concatenate([np.asarray(w[k], np.float32).ravel() for k in
                             ("layerNormScale", "layerNormOffset", "leftWeight", "leftBias", "rightWeight",
                              "rightBias", "outputWeight", "outputBias")])
    expected = opm_reference_test_expected(m, mask, w)
    got = oracle.outer_product_mean(m, mask, packed, 32, 16)
    assert np.array_equal(got, expected)
    assert np.abs(expected).max() > 0.1  # not a degenerate case


def test_opm_rounding_stages_on_the_reference_tests_own_case():
    """Which f16 rounding points carry the f16 path's 1.45e-2 distance (max|d| / max|ref|) from
    the reference test's own OPM case: rounded alone, the outer products give 8e-3 and W_o 8e-3
    (1.4e-2 together); with both exact, the input side (LN(m), W_left/W_right, left/right)
    still gives 2.5e-3.  So no single split stage meets 2e-3 on this case: every GEMM operand
    has to be split, which is the AF2_GEMM_F32 precision (GPU test in test_opm_gpu.py)."""
    m, mask, w, _ = opm_reference_test_case()
    expected = opm_reference_test_expected(m, mask, w)
    s, n, cm = m.shape
    c, cz = 32, w["outputBias"].size

    def model(xn16, w16, lr16, outer16, wo16):
        def f16(a, on):
            a = np.asarray(a, np.float64)
            return a.astype(np.float16).astype(np.float64) if on else a
        x = m.astype(np.float64)
        xn = f16((x - x.mean(-1, keepdims=True)) / np.sqrt(x.var(-1, keepdims=True) + 1e-5) * w["layerNormScale"]
                 + w["layerNormOffset"], xn16)
        msk = mask.astype(np.float64)[..., None]
        left = f16((xn @ f16(w["leftWeight"].reshape(cm, c), w16) + w["leftBias"]) * msk, lr16)
        right = f16((xn @ f16(w["rightWeight"].reshape(cm, c), w16) + w["rightBias"]) * msk, lr16)
        outer = f16(np.einsum("sia,sjb->ijab", left, right).reshape(n, n, c * c), outer16)
        cnt = np.einsum("si,sj->ij", mask.astype(np.float64), mask.astype(np.float64))
        out = (outer @ f16(w["outputWeight"].reshape(c * c, cz), wo16) + w["outputBias"]) / (1e-3 + cnt)[..., None]
        return np.abs(out - expected).max() / np.abs(expected).max()

    assert model(0, 0, 0, 0, 0) < 1e-5
    assert 1.3e-2 < model(1, 1, 1, 1, 1) < 1.6e-2
    assert 7e-3 < model(0, 0, 0, 1, 0) < 9e-3
    assert 7e-3 < model(0, 0, 0, 0, 1) < 9e-3
    assert 1.3e-2 < model(0, 0, 0, 1, 1) < 1.5e-2
    assert 2e-3 < model(1, 1, 1, 0, 0) < 3e-3


def test_projection_first_ordering_matches_the_oracle():
    """The reference's legacy projection-first OPM (OUTER_PRODUCT_MEAN_INTERMEDIATE_SHADER /
    OUTPUT_SHADER, src/evoformer/outer-product-mean.ts:260-311): per sequence and residue i,
    t[s,i,b,z] = sum_a left[s,i,a] W_o[a*c+b, z], then out[i,j,z] = (b_o[z] + sum_{s,b}
    t[s,i,b,z] right[s,j,b]) / (eps + count).  It is the same sum in another order, so it
    must agree with the contract-first oracle to rounding."""
    rng = np.random.default_rng(11)
    s, n, cm, c, cz = 7, 6, 10, 32, 12
    m = rng.standard_normal((s, n, cm)).astype(np.float32)
    mask = (rng.random((s, n)) < 0.8).astype(np.float32)
    parts = [1 + 0.1 * rng.standard_normal(cm), 0.1 * rng.standard_normal(cm),
             rng.standard_normal((cm, c)) / np.sqrt(cm), 0.1 * rng.standard_normal(c),
             rng.standard_normal((cm, c)) / np.sqrt(cm), 0.1 * rng.standard_normal(c),
             rng.standard_normal((c * c, cz)) / c, 0.1 * rng.standard_normal(cz)]
    packed = np.concatenate([np.asarray(p, np.float32).ravel() for p in parts])
    f = [np.asarray(p, np.float32).astype(np.float64) for p in parts]
    x = m.astype(np.float64)
    xn = (x - x.mean(-1, keepdims=True)) / np.sqrt(x.var(-1, keepdims=True) + 1e-5) * f[0] + f[1]
    left = (xn @ f[2] + f[3]) * mask[..., None]
    right = (xn @ f[4] + f[5]) * mask[..., None]
    t = np.einsum("sia,abz->sibz", left, f[6].reshape(c, c, cz))
    cnt = np.einsum("si,sj->ij", mask, mask)
    projection_first = (f[7] + np.einsum("sibz,sjb->ijz", t, right)) / (1e-3 + cnt)[..., None]
    got = oracle.outer_product_mean(m, mask, packed, c, cz)
    assert np.abs(got - projection_first).max() < 1e-5 * np.abs(projection_first).max()


@pytest.mark.parametrize("residual", [False, True])
def test_transition_matches_numpy(residual):
    rng = np.random.default_rng(6)
    rows, c, h = 50, 16, 64
    x = rng.standard_normal((rows, c)).astype(np.float32)
    parts = [1 + 0.1 * rng.standard_normal(c), 0.1 * rng.standard_normal(c), rng.standard_normal((c, h)) / 4,
             0.1 * rng.standard_normal(h), rng.standard_normal((h, c)) / 8, 0.1 * rng.standard_normal(c)]
    packed = np.concatenate([np.asarray(p, np.float32).ravel() for p in parts])
    out = oracle.transition(x, packed, h, residual=residual)
    f = [np.asarray(p, np.float64) for p in parts]
    xd = x.astype(np.float64)
    xn = (xd - xd.mean(-1, keepdims=True)) / np.sqrt(xd.var(-1, keepdims=True) + 1e-5) * f[0] + f[1]
    ref = np.maximum(xn @ f[2] + f[3], 0) @ f[4] + f[5] + (xd if residual else 0)
    assert np.abs(out - ref).max() < 1e-5 * np.abs(ref).max()


def test_triangle_weights_helper_matches_reference_count():
    for cz, ch in [(7, 6), (128, 128), (64, 32)]:
        w = triangle_weights(cz, ch, np.random.default_rng(0))
        assert pack(w).size == oracle.triangle_weight_count(cz, ch) == \
            af2cuda.expected_weight_element_count(af2cuda.TriangleShape(1, cz, ch))
