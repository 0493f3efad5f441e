"""GPU parity of the Evoformer pair block (encodeEvoformerPairBlock,
src/evoformer/block.ts:1753-1805) against the oracle's composition of the six
ops, and against the library's own op entry points called one by one.

The block adds into an f32 pair, in the reference's order: outer-product mean,
triangle multiplication outgoing and incoming, triangle attention starting and
ending, pair transition.  Bar: max|d| / max|ref| <= 2e-3 against the oracle
composition (each op's f16-operand error is bounded by that; six of them
compound to well inside it on these inputs), and bit-identical to the ops
called in the same order through their own device forms.
"""
import math

import numpy as np
import pytest

import af2cuda
import oracle
from helpers import pack, relative_max_error, triangle_weights

pytestmark = pytest.mark.gpu

REL_TOL = 2e-3
ATT_ORDER = ("queryNormScale", "queryNormOffset", "queryWeight", "keyWeight", "valueWeight", "gatingWeight",
             "gatingBias", "outputWeight", "outputBias")


def _block_case(n, s, cm, cz=128, heads=4, seed=0):
    rng = np.random.default_rng(seed)

    def mat(i, o):
        return (rng.standard_normal((i, o)) / math.sqrt(i)).astype(np.float32)

    def vec(k, center=0.0, scale=0.1):
        return (center + scale * rng.standard_normal(k)).astype(np.float32)

    pair = rng.standard_normal((n, n, cz)).astype(np.float32)
    pair_mask = (rng.random((n, n)) < 0.95).astype(np.float32)
    msa = rng.standard_normal((s, n, cm)).astype(np.float32)
    msa_mask = (rng.random((s, n)) < 0.9).astype(np.float32)
    msa_mask[0] = 1
    opm = np.concatenate([vec(cm, 1.0), vec(cm), mat(cm, 32).ravel(), vec(32), mat(cm, 32).ravel(), vec(32),
                          mat(32 * 32, cz).ravel(), vec(cz)])
    tri = [pack(triangle_weights(cz, cz, rng, perturbed=True)) for _ in range(2)]
    att = []
    for _ in range(2):
        w = dict(queryNormScale=vec(cz, 1.0), queryNormOffset=vec(cz), queryWeight=mat(cz, cz), keyWeight=mat(cz, cz),
                 valueWeight=mat(cz, cz), gatingWeight=mat(cz, cz), gatingBias=vec(cz, 0, 0.5),
                 outputWeight=mat(cz, cz), outputBias=vec(cz))
        att.append((w, mat(cz, heads)))
    tr = dict(layerNormScale=vec(cz, 1.0), layerNormOffset=vec(cz), firstWeight=mat(cz, 4 * cz),
              firstBias=vec(4 * cz), secondWeight=mat(4 * cz, cz), secondBias=vec(cz))
    return pair, pair_mask, msa, msa_mask, opm, tri, att, tr


def _att_packed(w, wb):
    return np.concatenate([np.asarray(w[k], np.float32).ravel() for k in ATT_ORDER] + [wb.ravel()])


def _device_weights(opm, tri, att, tr, torch):
    cuda = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda()  # noqa: E731
    return {"outerProductMean": cuda(opm), "triangleMultiplicationOutgoing": cuda(tri[0]),
            "triangleMultiplicationIncoming": cuda(tri[1]),
            "triangleAttentionStarting": cuda(_att_packed(*att[0])), "triangleAttentionEnding": cuda(_att_packed(*att[1])),
            "pairTransition": {k: cuda(v) for k, v in tr.items()}}


@pytest.mark.parametrize("n,s,cm", [(48, 20, 64), (130, 33, 256)])
def test_pair_block_matches_the_oracle_composition(device, n, s, cm):
    import torch
    pair, pair_mask, msa, msa_mask, opm, tri, att, tr = _block_case(n, s, cm, seed=n)
    z = pair.astype(np.float32)
    z = z + oracle.outer_product_mean(msa, msa_mask, opm, 32, 128)
    z = z + oracle.triangle(0, z, pair_mask, tri[0])
    z = z + oracle.triangle(1, z, pair_mask, tri[1])
    for transpose, (w, wb) in ((False, att[0]), (True, att[1])):
        upd = oracle.attention(z.reshape(n * n, 128), pair_mask.ravel(), w, n, n, 4, transpose=transpose,
                               pair_bias={"source": "normalized-input", "projectionWeight": wb})
        z = (z + upd.reshape(n, n, 128)).astype(np.float32)
    tr_packed = np.concatenate([tr[k].ravel() for k in ("layerNormScale", "layerNormOffset", "firstWeight",
                                                         "firstBias", "secondWeight", "secondBias")])
    z = oracle.transition(z.reshape(n * n, 128), tr_packed, 512, residual=True).reshape(n, n, 128)

    wd = _device_weights(opm, tri, att, tr, torch)
    pd = torch.from_numpy(pair).cuda()
    torch.cuda.synchronize()
    af2cuda.encode_evoformer_pair_block_tensors(device, pd, torch.from_numpy(pair_mask).cuda(), wd,
                                                msa=torch.from_numpy(msa).cuda(),
                                                msa_mask=torch.from_numpy(msa_mask).cuda())
    device.sync()
    got = pd.cpu().numpy()
    assert np.isfinite(got).all()
    assert relative_max_error(got, z) <= REL_TOL, relative_max_error(got, z)


def test_pair_block_is_the_ops_in_order(device):
    """The block call equals the six device-form calls in the reference's order, bit for bit,
    on a bf16 pair; and without the outer-product mean it skips exactly that op."""
    import torch
    n, s, cm = 64, 16, 64
    pair, pair_mask, msa, msa_mask, opm, tri, att, tr = _block_case(n, s, cm, seed=3)
    wd = _device_weights(opm, tri, att, tr, torch)
    m = torch.from_numpy(pair_mask).cuda()
    msa_d, msa_m = torch.from_numpy(msa).to("cuda", torch.bfloat16), torch.from_numpy(msa_mask).cuda()
    for with_opm in (True, False):
        a = torch.from_numpy(pair).to("cuda", torch.bfloat16)
        b = a.clone()
        torch.cuda.synchronize()
        af2cuda.encode_evoformer_pair_block_tensors(device, a, m, wd, msa=msa_d, msa_mask=msa_m,
                                                    include_outer_product_mean=with_opm)
        if with_opm:
            af2cuda.encode_outer_product_mean_tensors(device, msa_d, msa_m, wd["outerProductMean"], 32, 128, pair=b,
                                                      residual=True)
        af2cuda.encode_triangle_multiplication_tensors(device, 0, b, m, wd["triangleMultiplicationOutgoing"])
        af2cuda.encode_triangle_multiplication_tensors(device, 1, b, m, wd["triangleMultiplicationIncoming"])
        af2cuda.encode_triangle_attention_tensors(device, "starting", b, m, wd["triangleAttentionStarting"], 4)
        af2cuda.encode_triangle_attention_tensors(device, "ending", b, m, wd["triangleAttentionEnding"], 4)
        af2cuda.encode_transition_tensors(device, b.view(n * n, 128), wd["pairTransition"])
        device.sync()
        assert torch.equal(a, b), with_opm
