"""GPU parity of the outer-product mean and the shared linear layer.

The reference checks OuterProductMeanGpu against its own CPU formulation at
2e-5 / 2e-4 in f32 (test/outer-product-mean-reference.gpu.test.ts:128-129)
and requires blocked runs to be bit-identical
(test/evoformer-outer-product-mean.gpu.test.ts:78-81).  This build multiplies
f16 operands with f32 accumulation, so the parity bar is the benchmark
configs' max|d| / max|ref| <= 2e-3 against the oracle's restatement of that
CPU formulation; blocked runs are bit-identical here too.
"""
import numpy as np
import pytest

import af2cuda
import oracle
from helpers import (bf16_round, opm_f16_operand_model, opm_reference_test_case, opm_reference_test_expected,
                     relative_max_error)

pytestmark = pytest.mark.gpu

REL_TOL = 2e-3


def opm_case(s, n, cm, c=32, cz=128, seed=0, mask_p=0.9):
    rng = np.random.default_rng(seed)
    m = rng.standard_normal((s, n, cm)).astype(np.float32)
    mask = (rng.random((s, n)) < mask_p).astype(np.float32)
    mask[0] = 1  # row 0 all ones, as in the benchmark config
    w = dict(
        layerNormScale=(1 + 0.1 * rng.standard_normal(cm)).astype(np.float32),
        layerNormOffset=(0.1 * rng.standard_normal(cm)).astype(np.float32),
        leftWeight=(rng.standard_normal((cm, c)) / np.sqrt(cm)).astype(np.float32),
        leftBias=(0.1 * rng.standard_normal(c)).astype(np.float32),
        rightWeight=(rng.standard_normal((cm, c)) / np.sqrt(cm)).astype(np.float32),
        rightBias=(0.1 * rng.standard_normal(c)).astype(np.float32),
        outputWeight=(rng.standard_normal((c * c, cz)) / np.sqrt(c * c)).astype(np.float32),
        outputBias=(0.1 * rng.standard_normal(cz)).astype(np.float32),
    )
    return m, mask, w


def opm_packed(w):
    return np.concatenate([np.asarray(w[k], np.float32).ravel() for k in
                           ("layerNormScale", "layerNormOffset", "leftWeight", "leftBias", "rightWeight", "rightBias",
                            "outputWeight", "outputBias")])


def opm_input(m, mask, w, c=32, **kw):
    s, n, cm = m.shape
    cz = w["outputBias"].size
    return af2cuda.OuterProductMeanInput(m.ravel(), mask.ravel(), s, n, cm, c, cz,
                                         af2cuda.OuterProductMeanWeights(**w), **kw)


# S <= 640: three residues j per fused tile; 700 sequences: two (the resident right operand is larger)
@pytest.mark.parametrize("s,n,cm,cz", [(5, 9, 16, 8), (37, 30, 64, 128), (64, 64, 256, 128), (3, 13, 7, 5),
                                       (130, 21, 256, 64), (700, 20, 16, 32)])
def test_opm_matches_oracle(device, s, n, cm, cz):
    m, mask, w = opm_case(s, n, cm, cz=cz, seed=s + n + cm)
    expected = oracle.outer_product_mean(m, mask, opm_packed(w), 32, cz)
    result = af2cuda.OuterProductMeanGpu(device).run(opm_input(m, mask, w))
    out = result.output.reshape(n, n, cz)
    assert np.isfinite(out).all()
    assert relative_max_error(out, expected) <= REL_TOL
    assert result.elapsedMilliseconds > 0


@pytest.mark.parametrize("dtype", ["bfloat16", "float16"])
@pytest.mark.parametrize("s,n,cm,cz", [(5, 9, 16, 8), (130, 21, 256, 64), (300, 17, 200, 128), (3, 13, 8, 5),
                                       (256, 33, 128, 128), (700, 20, 48, 32)])
def test_opm_16bit_msa_matches_oracle(device, dtype, s, n, cm, cz):
    """A 16-bit MSA is normalised and projected by one kernel (LayerNorm in
    shared memory, no normalised copy in HBM): ragged c_m (zero-filled past
    c_m), sequence counts that do not fill the last 128-sequence tile, and the
    two- and three-residue outer tiles behind it."""
    import torch
    m, mask, w = opm_case(s, n, cm, cz=cz, seed=2 * s + n + cm)
    mt = torch.from_numpy(m).to("cuda", getattr(torch, dtype))
    expected = oracle.outer_product_mean(mt.float().cpu().numpy(), mask, opm_packed(w), 32, cz)
    out = torch.zeros((n, n, cz), dtype=torch.float32, device="cuda")
    af2cuda.encode_outer_product_mean_tensors(device, mt, torch.from_numpy(mask).cuda(),
                                              torch.from_numpy(opm_packed(w)).cuda(), 32, cz, out=out,
                                              residual=False)
    device.sync()
    got = out.cpu().numpy()
    assert np.isfinite(got).all()
    assert relative_max_error(got, expected) <= REL_TOL


@pytest.mark.parametrize("s,n,cm,cz", [(1030, 12, 16, 24), (40, 20, 32, 160)])
def test_opm_two_kernel_path_matches_oracle(device, s, n, cm, cz):
    """More than 1024 sequences, or c_z above 128: the outer products go through
    the HBM scratch and the shared output GEMM instead of the fused kernel."""
    m, mask, w = opm_case(s, n, cm, cz=cz, seed=s + n)
    expected = oracle.outer_product_mean(m, mask, opm_packed(w), 32, cz)
    out = af2cuda.OuterProductMeanGpu(device).run(opm_input(m, mask, w)).output.reshape(n, n, cz)
    assert np.isfinite(out).all()
    assert relative_max_error(out, expected) <= REL_TOL


def test_opm_blocks_are_bit_identical(device):
    m, mask, w = opm_case(33, 46, 64, cz=32, seed=5)
    whole = af2cuda.OuterProductMeanGpu(device).run(opm_input(m, mask, w)).output
    for rb in (4, 12, 45):
        blocked = af2cuda.OuterProductMeanGpu(device).run(opm_input(m, mask, w, rowBlockResidues=rb)).output
        assert np.array_equal(blocked, whole), rb


def test_opm_on_the_reference_tests_own_case(device):
    """test/outer-product-mean-reference.gpu.test.ts:104-130 on this build: its spread
    inputs, masked entries and rowBlockResidues 3 against that test's CPU reference.
    The case cancels heavily (outputs below 0.4 from products whose magnitudes sum to
    about 5000 per output), which magnifies f16 operand rounding: the result meets the
    reference's half-precision max bar (max |d| < 1e-2,
    test/triangle-multiplication-outgoing.gpu.test.ts:58-92) but not its mean bar (1e-3;
    measured 1.6e-3) nor 2e-3 of max|ref|, which hold on the benchmark configs' inputs.
    That this distance is the f16 rounding and nothing else is pinned by a model of the
    kernels' rounding points, which the GPU result matches far inside the distance.
    The residue blocks of the reference's blocked-run test
    (test/evoformer-outer-product-mean.gpu.test.ts:75-81) give the same bits."""
    m, mask, w, row_block = opm_reference_test_case()
    expected = opm_reference_test_expected(m, mask, w)
    out = af2cuda.OuterProductMeanGpu(device).run(opm_input(m, mask, w, rowBlockResidues=row_block)).output
    out = out.reshape(expected.shape)
    assert np.isfinite(out).all()
    err = oracle.error_metrics(out, expected)
    assert err["maxAbsoluteError"] < 1e-2, err
    model = opm_f16_operand_model(m, mask, w)
    # the model's own distance from the reference is about 5.5e-3 at most
    assert np.abs(out - model).max() <= 5e-4, float(np.abs(out - model).max())
    for rb in (None, 1, 7, 32):
        again = af2cuda.OuterProductMeanGpu(device).run(opm_input(m, mask, w, rowBlockResidues=rb)).output
        assert np.array_equal(again.reshape(expected.shape), out), rb


def test_opm_f32_precision_meets_the_reference_tests_f32_bar(device):
    """The same case with the f32 GEMM precision installed (the reference's own f32 path,
    which its test holds to mean |d| < 2e-5 and max |d| < 2e-4,
    test/outer-product-mean-reference.gpu.test.ts:128-129): every operand of the three GEMMs
    carried as an f16 hi / lo pair on the tensor cores.  It also meets 2e-3 of max|ref|, and
    its residue blocks give the same bits."""
    m, mask, w, row_block = opm_reference_test_case()
    expected = opm_reference_test_expected(m, mask, w)
    device.set_gemm_precision("f32")
    try:
        out = af2cuda.OuterProductMeanGpu(device).run(opm_input(m, mask, w, rowBlockResidues=row_block)).output
        out = out.reshape(expected.shape)
        err = oracle.error_metrics(out, expected)
        assert err["meanAbsoluteError"] < 2e-5 and err["maxAbsoluteError"] < 2e-4, err
        assert relative_max_error(out, expected) <= REL_TOL
        for rb in (None, 1, 7):
            again = af2cuda.OuterProductMeanGpu(device).run(opm_input(m, mask, w, rowBlockResidues=rb)).output
            assert np.array_equal(again.reshape(expected.shape), out), rb
    finally:
        device.set_gemm_precision("matrix")
    assert device.gemm_precision == "matrix"


@pytest.mark.parametrize("s,n,cm,cz", [(37, 30, 64, 128), (130, 21, 256, 64), (700, 20, 16, 32)])
def test_opm_f32_precision_matches_oracle_tightly(device, s, n, cm, cz):
    """f32 GEMM precision on the benchmark law's inputs: within 2e-5 of max|ref| (f32 level),
    where the default f16-operand path is held to 2e-3."""
    m, mask, w = opm_case(s, n, cm, cz=cz, seed=s + n + cm)
    expected = oracle.outer_product_mean(m, mask, opm_packed(w), 32, cz)
    device.set_gemm_precision("f32")
    try:
        out = af2cuda.OuterProductMeanGpu(device).run(opm_input(m, mask, w)).output.reshape(n, n, cz)
    finally:
        device.set_gemm_precision("matrix")
    assert relative_max_error(out, expected) <= 2e-5, relative_max_error(out, expected)


def test_opm_fully_masked_residues(device):
    m, mask, w = opm_case(20, 17, 32, cz=16, seed=9)
    mask[:, 3] = 0  # residue 3 never observed: count 0, output = b_o / eps
    expected = oracle.outer_product_mean(m, mask, opm_packed(w), 32, 16)
    out = af2cuda.OuterProductMeanGpu(device).run(opm_input(m, mask, w)).output.reshape(17, 17, 16)
    assert relative_max_error(out, expected) <= REL_TOL


def test_opm_device_form_into_bf16_pair(device):
    """encodeOuterProductMean with residualTarget = pair: bf16 MSA in, bf16 pair updated."""
    import torch
    s, n, cm, cz = 48, 40, 256, 128
    m, mask, w = opm_case(s, n, cm, cz=cz, seed=3)
    mb = bf16_round(m)
    update = oracle.outer_product_mean(mb, mask, opm_packed(w), 32, cz)
    rng = np.random.default_rng(1)
    pair0 = bf16_round(rng.standard_normal((n, n, cz)).astype(np.float32))
    pair = torch.from_numpy(pair0).to("cuda", torch.bfloat16)
    torch.cuda.synchronize()
    af2cuda.encode_outer_product_mean_tensors(device, torch.from_numpy(mb).to("cuda", torch.bfloat16),
                                              torch.from_numpy(mask).cuda(), torch.from_numpy(opm_packed(w)).cuda(),
                                              32, cz, pair=pair, residual=True)
    device.sync()
    got = pair.float().cpu().numpy()
    want = pair0.astype(np.float64) + update
    bound = 2.0 ** -8 * np.abs(want) + REL_TOL * np.abs(update).max()
    assert np.all(np.abs(got - want) <= bound), float((np.abs(got - want) - bound).max())


def _linear_reference(a, w, b, relu):
    y = a.astype(np.float64) @ w.astype(np.float64)
    if b is not None:
        y = y + b
    return np.maximum(y, 0) if relu else y


@pytest.mark.parametrize("rows,inner,cols,relu", [(300, 100, 70, True), (1, 7, 3, False), (257, 256, 384, False),
                                                  (4096, 128, 512, True)])
def test_linear_matches_numpy(device, rows, inner, cols, relu):
    import torch
    rng = np.random.default_rng(rows + inner + cols)
    a = rng.standard_normal((rows, inner)).astype(np.float32)
    w = (rng.standard_normal((inner, cols)) / np.sqrt(inner)).astype(np.float32)
    b = (0.1 * rng.standard_normal(cols)).astype(np.float32)
    out = af2cuda.linear_tensors(device, torch.from_numpy(a).cuda(), torch.from_numpy(w).cuda(),
                                 torch.from_numpy(b).cuda(), relu=relu)
    device.sync()
    assert relative_max_error(out.cpu().numpy(), _linear_reference(a, w, b, relu)) <= REL_TOL


def test_linear_q8_residual_f16(device):
    import torch
    rng = np.random.default_rng(4)
    rows, inner, cols = 513, 128, 512
    a = rng.standard_normal((rows, inner)).astype(np.float16)
    w = (rng.standard_normal((inner, cols)) / np.sqrt(inner)).astype(np.float32)
    codes, scales = oracle.quantize_q8_columns(w)
    dense = oracle.dequant_q8_columns(codes, scales)
    base = rng.standard_normal((rows, cols)).astype(np.float32)
    out = torch.from_numpy(base).cuda()
    q8 = af2cuda.Q8Matrix(torch.from_numpy(codes).cuda(), torch.from_numpy(scales).cuda(), "channel")
    af2cuda.linear_tensors(device, torch.from_numpy(a).cuda(), q8, None, out=out, residual=True)
    device.sync()
    want = base + _linear_reference(a.astype(np.float32), dense, None, False)
    assert relative_max_error(out.cpu().numpy(), want) <= REL_TOL


def test_linear_bf16_input(device):
    import torch
    rng = np.random.default_rng(8)
    a = bf16_round(rng.standard_normal((200, 64)).astype(np.float32))
    w = (rng.standard_normal((64, 96)) / 8).astype(np.float32)
    out = af2cuda.linear_tensors(device, torch.from_numpy(a).to("cuda", torch.bfloat16), torch.from_numpy(w).cuda())
    device.sync()
    assert relative_max_error(out.cpu().numpy(), _linear_reference(a, w, None, False)) <= REL_TOL


def _gemm_test_values(count, seed):
    """values() of test/gemm-half-precision.gpu.test.ts:44-51: a 32-bit linear congruential
    generator (multiplier 1664525, increment 1013904223), each value state / 2^32 - 0.5, as f32."""
    out = np.empty(count, np.float64)
    state = seed & 0xFFFFFFFF
    for i in range(count):
        state = (state * 1664525 + 1013904223) & 0xFFFFFFFF
        out[i] = state / 2.0 ** 32 - 0.5
    return out.astype(np.float32)


@pytest.mark.parametrize("inner", [256, 1024])
@pytest.mark.parametrize("seeds", [(0x1234567, 0x89ABCDEF, 0x2468ACE), (0x13579BD, 0x2468ACE, 0x1234567)])
def test_linear_on_the_reference_gemm_test_cases(device, inner, seeds):
    """The shared projection (createLinearShader) on the cases of
    test/gemm-half-precision.gpu.test.ts:200-236: GEMM_TILE_ROWS + 17 = 81 rows, 132
    columns, both contraction depths the model runs, deterministic inputs, against A W + b
    summed in double precision; the reference's bar for f16 operands with f32 sums is a
    worst error below 2e-3 of the largest output (tolerance(), :35-41)."""
    import torch
    rows, cols = 64 + 17, 132
    a = _gemm_test_values(rows * inner, seeds[0]).reshape(rows, inner)
    w = _gemm_test_values(inner * cols, seeds[1]).reshape(inner, cols)
    b = _gemm_test_values(cols, seeds[2])
    expected = a.astype(np.float64) @ w.astype(np.float64) + b
    out = af2cuda.linear_tensors(device, torch.from_numpy(a).cuda(), torch.from_numpy(w).cuda(),
                                 torch.from_numpy(b).cuda())
    device.sync()
    got = out.cpu().numpy()
    assert np.abs(got - expected).max() / np.abs(expected).max() < 2e-3
