"""The shape rules that choose between two kernels, and their environment overrides
(AF2_OPM_TILE_RESIDUES, AF2_TRANSITION_WIDE): the alternative gives the same result
(bit-identical for the fused outer-product mean with two or three residues per tile;
within the 2e-3 bar of the oracle for the two transition paths), so the choice is a
matter of speed only, measured in bench.py."""
import os

import numpy as np
import pytest

import af2cuda
import oracle
from helpers import relative_max_error

pytestmark = pytest.mark.gpu


@pytest.fixture()
def env():
    saved = {k: os.environ.get(k) for k in ("AF2_OPM_TILE_RESIDUES", "AF2_TRANSITION_WIDE")}
    yield os.environ
    for k, v in saved.items():
        if v is None:
            os.environ.pop(k, None)
        else:
            os.environ[k] = v


def test_opm_two_or_three_residues_per_tile_are_bit_identical(device, env):
    import torch
    from test_opm_gpu import opm_case, opm_packed
    for n, s in ((70, 40), (130, 300)):
        m, mask, w = opm_case(s, n, 64, cz=128, seed=n)
        md = torch.from_numpy(m).to("cuda", torch.bfloat16)
        maskd = torch.from_numpy(mask).cuda()
        pw = torch.from_numpy(opm_packed(w)).cuda()
        outs = []
        for j in ("3", "2"):
            env["AF2_OPM_TILE_RESIDUES"] = j
            torch.cuda.synchronize()
            outs.append(af2cuda.encode_outer_product_mean_tensors(device, md, maskd, pw, 32, 128,
                                                                   out=torch.empty(n, n, 128, device="cuda"),
                                                                   residual=False))
            device.sync()
        assert torch.equal(outs[0], outs[1]), n


def test_transition_wide_path_matches_the_fused_kernel(device, env):
    import torch
    rng = np.random.default_rng(3)
    rows, c, h = 3000, 128, 512
    x = rng.standard_normal((rows, c)).astype(np.float32)
    w = {"layerNormScale": (1 + 0.1 * rng.standard_normal(c)).astype(np.float32),
         "layerNormOffset": (0.1 * rng.standard_normal(c)).astype(np.float32),
         "firstWeight": (rng.standard_normal((c, h)) / np.sqrt(c)).astype(np.float32),
         "firstBias": (0.1 * rng.standard_normal(h)).astype(np.float32),
         "secondWeight": (rng.standard_normal((h, c)) / np.sqrt(h)).astype(np.float32),
         "secondBias": (0.1 * rng.standard_normal(c)).astype(np.float32)}
    packed = np.concatenate([w[k].ravel() for k in ("layerNormScale", "layerNormOffset", "firstWeight", "firstBias",
                                                      "secondWeight", "secondBias")])
    ref = oracle.transition(x, packed, h, residual=True)
    wd = {k: torch.from_numpy(v).cuda() for k, v in w.items()}
    outs = []
    for wide in ("0", "1"):
        env["AF2_TRANSITION_WIDE"] = wide
        xd = torch.from_numpy(x).cuda()
        torch.cuda.synchronize()
        af2cuda.encode_transition_tensors(device, xd, wd)
        device.sync()
        outs.append(xd.cpu().numpy())
        assert relative_max_error(outs[-1], ref) <= 2e-3, wide
    assert not np.array_equal(outs[0], np.zeros_like(outs[0]))
