"""GPU parity of the wide transition path: channels above 128 or hidden above
1024, the MSA transition (c_m 256 -> 1024 -> 256) among them.  The fused
kernel holds C <= 128 and H <= 1024, so these run the reference's own kernel
sequence (src/evoformer/transition.ts:264-361): LayerNorm into an f16 copy,
then the shared tcgen05 linear kernel twice, the hidden activations in a
chunked HBM scratch.  Same bar as the fused transition: max|d| / max|ref| <=
2e-3 against the oracle; row chunks bit-identical."""
import numpy as np
import pytest

import af2cuda
import oracle
from helpers import bf16_round, relative_max_error
from test_transition_gpu import REL_TOL, _device_weights, _q8_case, make_input, packed, transition_case

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("rows,c,h", [(300, 256, 1024), (77, 200, 600), (129, 64, 2048), (9, 130, 8)])
def test_wide_host_form_matches_oracle(device, rows, c, h):
    """LayerNorm, then the shared linear kernel twice with the hidden activations in HBM."""
    x, w = transition_case(rows, c, h, seed=rows + c + h)
    expected = oracle.transition(x, packed(w), h)
    out = af2cuda.TransitionGpu(device).run(make_input(x, w)).output.reshape(rows, c)
    assert np.isfinite(out).all()
    assert relative_max_error(out, expected) <= REL_TOL


@pytest.mark.parametrize("kind", ["channel", "block"])
def test_msa_transition_q8_in_place(device, kind):
    """encodeTransition on bf16 MSA rows [S*N, 256] with mixed-q8 weights, residual in place."""
    import torch
    x16, dense, wd = _q8_case(kind, torch, seed=21, rows=1000, c=256, h=1024)
    xb = bf16_round(x16)
    update = oracle.transition(xb, packed(dense), 1024)
    xd = torch.from_numpy(xb).to("cuda", torch.bfloat16)
    torch.cuda.synchronize()
    af2cuda.encode_transition_tensors(device, xd, wd, residual=True)
    device.sync()
    got = xd.float().cpu().numpy()
    want = xb.astype(np.float64) + update
    bound = 2.0 ** -8 * np.abs(want) + (REL_TOL + 2 ** -11) * np.abs(update).max()
    assert np.all(np.abs(got - want) <= bound), float((np.abs(got - want) - bound).max())


def test_wide_row_chunks_are_result_neutral(device):
    """At hidden 16384 one chunk of the wide path holds 8192 rows: 9000 rows run as two
    chunks give the bits of the same rows run in two separate calls."""
    import torch
    c, h = 64, 16384
    x, w = transition_case(9000, c, h, seed=8)
    wd = _device_weights(w, torch)
    xd = torch.from_numpy(x).cuda()
    whole = torch.empty_like(xd)
    parts = torch.empty_like(xd)
    torch.cuda.synchronize()
    af2cuda.encode_transition_tensors(device, xd, wd, out=whole, residual=False)
    for r0, r1 in ((0, 4000), (4000, 9000)):
        af2cuda.encode_transition_tensors(device, xd[r0:r1], wd, out=parts[r0:r1], residual=False)
    device.sync()
    assert torch.equal(whole, parts)
    expected = oracle.transition(x[:40], packed(w), h)
    assert relative_max_error(whole[:40].cpu().numpy(), expected) <= REL_TOL
