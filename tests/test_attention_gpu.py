"""GPU parity of the gated multi-head attention (triangle attention) against the oracle.

The reference has no CPU implementation of attention and its attention fixture
(test/fixtures/evoformer/model1-query-59-block0/) is not in its checkout, so
parity is against the oracle's restatement of AttentionGpu.run
(src/evoformer/attention.ts:1334-1453), which the CPU tests check against a
loop statement of the reference's kernels: parity unpinned by golden vectors.
Bar: max|d| / max|ref| <= 2e-3 (f16 tensor-core operands, f32 accumulation and
softmax statistics).  The ending-node view is checked bit for bit against the
starting node on the transposed pair, and fully masked rows against the
uniform average the reference's logit clamp gives them.
"""
import math

import numpy as np
import pytest

import af2cuda
import oracle
from helpers import bf16_round, relative_max_error

pytestmark = pytest.mark.gpu

REL_TOL = 2e-3


def attention_weights(rng, c, heads, bias=True, perturbed=True):
    def mat(i, o):
        return (rng.standard_normal((i, o)) / math.sqrt(i)).astype(np.float32)

    w = dict(queryNormScale=(1 + (0.1 if perturbed else 0) * rng.standard_normal(c)).astype(np.float32),
             queryNormOffset=((0.1 if perturbed else 0) * rng.standard_normal(c)).astype(np.float32),
             queryWeight=mat(c, c), keyWeight=mat(c, c), valueWeight=mat(c, c), gatingWeight=mat(c, c),
             gatingBias=((0.5 if perturbed else 0) * rng.standard_normal(c)).astype(np.float32),
             outputWeight=mat(c, c), outputBias=((0.1 if perturbed else 0) * rng.standard_normal(c)).astype(np.float32))
    return w, (mat(c, heads) if bias else None)


def run_host(device, x, mask, w, wb, batch, queries, heads, transpose):
    c = x.shape[-1]
    inp = af2cuda.AttentionInput(x.ravel(), mask.ravel(), batch, queries, c, heads, af2cuda.AttentionWeights(**w),
                                 transpose=transpose,
                                 pairBias=None if wb is None else af2cuda.NormalizedInputPairBias(wb))
    return af2cuda.AttentionGpu(device).run(inp).output.reshape(batch * queries, c)


def expected(x, mask, w, wb, batch, queries, heads, transpose):
    pb = None if wb is None else {"source": "normalized-input", "projectionWeight": wb}
    return oracle.attention(x.reshape(batch * queries, -1), mask.ravel(), w, batch, queries, heads,
                            transpose=transpose, pair_bias=pb)


@pytest.mark.parametrize("transpose", [False, True])
@pytest.mark.parametrize("n", [5, 37, 128, 130, 200])
def test_triangle_attention_matches_oracle(device, n, transpose):
    rng = np.random.default_rng(n + transpose)
    c, heads = 128, 4
    x = rng.standard_normal((n, n, c)).astype(np.float32)
    mask = (rng.random((n, n)) < 0.9).astype(np.float32)
    w, wb = attention_weights(rng, c, heads)
    out = run_host(device, x, mask, w, wb, n, n, heads, transpose)
    ref = expected(x, mask, w, wb, n, n, heads, transpose)
    assert np.isfinite(out).all()
    assert relative_max_error(out, ref) <= REL_TOL, relative_max_error(out, ref)


def test_attention_without_bias_and_batch_unlike_queries(device):
    """The plain gated attention (no pair bias): batch 3 rows of 70 positions, two heads."""
    rng = np.random.default_rng(7)
    b, q, c, heads = 3, 70, 64, 2
    x = rng.standard_normal((b * q, c)).astype(np.float32)
    mask = (rng.random(b * q) < 0.8).astype(np.float32)
    w, _ = attention_weights(rng, c, heads, bias=False)
    for transpose in (False, True):
        out = run_host(device, x, mask, w, None, b, q, heads, transpose)
        ref = expected(x, mask, w, None, b, q, heads, transpose)
        assert relative_max_error(out, ref) <= REL_TOL, (transpose, relative_max_error(out, ref))


def test_fully_masked_rows_average_uniformly(device):
    """A batch row with every key masked: 1e9 (mask - 1) swamps the scores and the bias and
    the clamp at -1e8 makes every logit equal, so each query averages all values uniformly."""
    rng = np.random.default_rng(11)
    n, c, heads = 40, 128, 4
    x = rng.standard_normal((n, n, c)).astype(np.float32)
    mask = np.ones((n, n), np.float32)
    mask[6, :] = 0
    mask[:, 9] = 0
    w, wb = attention_weights(rng, c, heads)
    out = run_host(device, x, mask, w, wb, n, n, heads, False)
    ref = expected(x, mask, w, wb, n, n, heads, False)
    assert relative_max_error(out, ref) <= REL_TOL
    assert relative_max_error(out.reshape(n, n, c)[6], ref.reshape(n, n, c)[6]) <= REL_TOL


def test_ending_node_is_the_starting_node_of_the_transposed_pair(device):
    import torch
    rng = np.random.default_rng(12)
    n, c, heads = 96, 128, 4
    x = rng.standard_normal((n, n, c)).astype(np.float32)
    mask = (rng.random((n, n)) < 0.9).astype(np.float32)
    w, wb = attention_weights(rng, c, heads)
    packed = np.concatenate([np.asarray(w[k], np.float32).ravel() for k in
                             ("queryNormScale", "queryNormOffset", "queryWeight", "keyWeight", "valueWeight",
                              "gatingWeight", "gatingBias", "outputWeight", "outputBias")] + [wb.ravel()])
    pd = torch.from_numpy(packed).cuda()
    z = torch.from_numpy(x).cuda()
    zt = z.transpose(0, 1).contiguous()
    m = torch.from_numpy(mask).cuda()
    mt = m.t().contiguous()
    ending = torch.empty_like(z)
    starting_t = torch.empty_like(z)
    torch.cuda.synchronize()
    af2cuda.encode_triangle_attention_tensors(device, "ending", z, m, pd, heads, out=ending, residual=False)
    af2cuda.encode_triangle_attention_tensors(device, "starting", zt, mt, pd, heads, out=starting_t, residual=False)
    device.sync()
    assert torch.equal(ending, starting_t.transpose(0, 1))


@pytest.mark.parametrize("direction", ["starting", "ending"])
def test_device_form_bf16_pair_in_place(device, direction):
    """encodeAttention with residualTarget = pair on a bf16 pair: pair += attention(pair)."""
    import torch
    rng = np.random.default_rng(13)
    n, c, heads = 150, 128, 4
    x = bf16_round(rng.standard_normal((n, n, c)).astype(np.float32))
    mask = (rng.random((n, n)) < 0.9).astype(np.float32)
    w, wb = attention_weights(rng, c, heads)
    packed = np.concatenate([np.asarray(w[k], np.float32).ravel() for k in
                             ("queryNormScale", "queryNormOffset", "queryWeight", "keyWeight", "valueWeight",
                              "gatingWeight", "gatingBias", "outputWeight", "outputBias")] + [wb.ravel()])
    update = expected(x, mask, w, wb, n, n, heads, direction == "ending").reshape(n, n, c)
    pair = torch.from_numpy(x).to("cuda", torch.bfloat16)
    torch.cuda.synchronize()
    af2cuda.encode_triangle_attention_tensors(device, direction, pair, torch.from_numpy(mask).cuda(),
                                              torch.from_numpy(packed).cuda(), heads)
    device.sync()
    got = pair.float().cpu().numpy()
    want = x.astype(np.float64) + update
    ulp = 2.0 ** -8
    bound = ulp * np.abs(want) + REL_TOL * np.abs(update).max()
    assert np.all(np.abs(got - want) <= bound), float((np.abs(got - want) - bound).max())


def test_attention_rejects_what_the_reference_rejects(device):
    rng = np.random.default_rng(1)
    w, wb = attention_weights(rng, 96, 2)
    x = np.zeros((4 * 4, 96), np.float32)
    with pytest.raises(af2cuda.RangeError, match="head dimension no larger than 32"):
        run_host(device, x, np.ones(16, np.float32), w, None, 4, 4, 2, False)
