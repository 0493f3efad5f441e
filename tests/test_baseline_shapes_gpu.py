"""GPU parity at the benchmark configs' own shapes, against the oracle.

The other GPU tests stop at sizes the oracle finishes in a second; these run
the configs the benchmark measures:

- the metric's triangle multiplication at N = 1024 (bf16 pair ~N(0,1), mask
  ones, weights ~N(0, 1/fan_in)), both directions, checked on a sample of
  output rows (the oracle projects every pair, then contracts and projects
  only the sampled rows exactly as the whole op would); the incoming
  direction also with the multimer config's chain-block mask (1 only inside
  the diagonal chain blocks);
- config 3's outer-product mean in full (S = 512, N = 256, c_m = 256, c = 32,
  c_z = 128, f32 MSA, Bernoulli(0.9) mask with row 0 ones);
- config 2's mixed-q8 pair transition in full (65,536 f16 rows, 128 -> 512
  -> 128, int8 weights with f32 per-output-channel scales), against the
  oracle on the exactly decoded weights.

Bar: max|d| / max|ref| <= 2e-3 (f16 tensor-core operands, f32 accumulation),
plus the f16 output rounding where the output is f16.
"""
import numpy as np
import pytest

import af2cuda
import oracle
from helpers import bf16_round, pack, relative_max_error, triangle_weights

pytestmark = pytest.mark.gpu

REL_TOL = 2e-3


@pytest.mark.parametrize("direction,chains", [(0, 1), (1, 1), (1, 4)])
def test_triangle_at_the_metric_shape_on_sampled_rows(device, direction, chains):
    import torch
    n, cz = 1024, 128
    rng = np.random.default_rng(100 + direction + chains)
    z = bf16_round(rng.standard_normal((n, n, cz)).astype(np.float32))
    chain = np.arange(n) // (n // chains)
    mask = (chain[:, None] == chain[None, :]).astype(np.float32)
    w = pack(triangle_weights(cz, cz, rng))
    zd = torch.from_numpy(z).to("cuda", torch.bfloat16)
    md = torch.from_numpy(mask).cuda()
    wd = torch.from_numpy(w).cuda()
    out = torch.empty(n, n, cz, device="cuda", dtype=torch.float32)
    torch.cuda.synchronize()
    af2cuda.encode_triangle_multiplication_tensors(device, direction, zd, md, wd, out=out, residual=False)
    device.sync()
    # the first and last rows of each 256-row pair tile and of each chain, plus random ones
    rows = sorted({0, 1, 255, 256, 511, 767, 1022, 1023, *rng.integers(0, n, 4).tolist()})
    expected = oracle.triangle_rows(direction, z, mask, w, rows)
    got = out[rows].cpu().numpy()
    assert np.isfinite(got).all()
    assert relative_max_error(got, expected) <= REL_TOL, relative_max_error(got, expected)


def test_opm_config3_in_full(device):
    s, n, cm, c, cz = 512, 256, 256, 32, 128
    rng = np.random.default_rng(3)
    m = rng.standard_normal((s, n, cm)).astype(np.float32)
    mask = (rng.random((s, n)) < 0.9).astype(np.float32)
    mask[0] = 1
    w = dict(layerNormScale=np.ones(cm, np.float32), layerNormOffset=np.zeros(cm, np.float32),
             leftWeight=(rng.standard_normal((cm, c)) / np.sqrt(cm)).astype(np.float32),
             leftBias=np.zeros(c, np.float32),
             rightWeight=(rng.standard_normal((cm, c)) / np.sqrt(cm)).astype(np.float32),
             rightBias=np.zeros(c, np.float32),
             outputWeight=(rng.standard_normal((c * c, cz)) / np.sqrt(c * c)).astype(np.float32),
             outputBias=np.zeros(cz, np.float32))
    packed = np.concatenate([w[k].ravel() for k in ("layerNormScale", "layerNormOffset", "leftWeight", "leftBias",
                                                    "rightWeight", "rightBias", "outputWeight", "outputBias")])
    expected = oracle.outer_product_mean(m, mask, packed, c, cz)
    inp = af2cuda.OuterProductMeanInput(m.ravel(), mask.ravel(), s, n, cm, c, cz, af2cuda.OuterProductMeanWeights(**w))
    out = af2cuda.OuterProductMeanGpu(device).run(inp).output.reshape(n, n, cz)
    assert np.isfinite(out).all()
    assert relative_max_error(out, expected) <= REL_TOL, relative_max_error(out, expected)


def test_transition_config2_in_full(device):
    import torch
    rows, c, h = 65536, 128, 512
    rng = np.random.default_rng(2)
    x = rng.standard_normal((rows, c)).astype(np.float16)
    w1 = (rng.standard_normal((c, h)) / np.sqrt(c)).astype(np.float32)
    w2 = (rng.standard_normal((h, c)) / np.sqrt(h)).astype(np.float32)
    (c1, s1), (c2, s2) = oracle.quantize_q8_columns(w1), oracle.quantize_q8_columns(w2)
    ln_s, ln_o = np.ones(c, np.float32), np.zeros(c, np.float32)
    b1, b2 = np.zeros(h, np.float32), np.zeros(c, np.float32)
    dense = np.concatenate([ln_s, ln_o, oracle.dequant_q8_columns(c1, s1).ravel(), b1,
                            oracle.dequant_q8_columns(c2, s2).ravel(), b2])
    expected = oracle.transition(x.astype(np.float32), dense, h)
    cuda = {k: torch.from_numpy(v).cuda() for k, v in dict(ln_s=ln_s, ln_o=ln_o, b1=b1, b2=b2).items()}
    weights = {"layerNormScale": cuda["ln_s"], "layerNormOffset": cuda["ln_o"],
               "firstWeight": af2cuda.Q8Matrix(torch.from_numpy(c1).cuda(), torch.from_numpy(s1).cuda(), "channel"),
               "firstBias": cuda["b1"],
               "secondWeight": af2cuda.Q8Matrix(torch.from_numpy(c2).cuda(), torch.from_numpy(s2).cuda(), "channel"),
               "secondBias": cuda["b2"]}
    xd = torch.from_numpy(x).cuda()
    out = torch.empty_like(xd)
    torch.cuda.synchronize()
    af2cuda.encode_transition_tensors(device, xd, weights, out=out, residual=False)
    device.sync()
    got = out.float().cpu().numpy()
    assert np.isfinite(got).all()
    assert relative_max_error(got, expected) <= REL_TOL + 2 ** -11, relative_max_error(got, expected)
