"""CPU tests of the oracle's attention restatement (groundwork for triangle attention,
the next pair-stack operator): the reference has no CPU implementation of it, so the
restatement is checked against an independent loop statement of the reference's
kernels (online softmax, as ATTENTION_FLASH_SHADER computes it,
src/evoformer/attention.ts:663-731), the starting/ending-node transpose identity of
triangle attention, and the fully masked row the logit clamp makes uniform."""
import math

import numpy as np

import oracle


def _weights(rng, c, h):
    return dict(queryNormScale=1 + 0.1 * rng.standard_normal(c), queryNormOffset=0.1 * rng.standard_normal(c),
                queryWeight=rng.standard_normal((c, c)) / math.sqrt(c),
                keyWeight=rng.standard_normal((c, c)) / math.sqrt(c),
                valueWeight=rng.standard_normal((c, c)) / math.sqrt(c),
                gatingWeight=rng.standard_normal((c, c)) / math.sqrt(c), gatingBias=0.1 * rng.standard_normal(c),
                outputWeight=rng.standard_normal((c, c)) / math.sqrt(c), outputBias=0.1 * rng.standard_normal(c))


def _loops(x, mask, w, B, Q, H, transpose, bias_w, bias_fn=None):
    """Kernel by kernel with scalar loops: LayerNorm per row, the four projections, the
    online-softmax flash loop with the 1e9 mask bias, the +-1e8 clamp and the gate, then
    the output projection written back to the source row."""
    rows, c = x.shape
    d = c // H

    def src(b, q):
        return b * Q + q if not transpose else q * B + b

    xn = {}
    for b in range(B):
        for q in range(Q):
            r = x[src(b, q)]
            mean = sum(r) / c
            var = sum((t - mean) ** 2 for t in r) / c
            inv = 1 / math.sqrt(var + 1e-5)
            xn[b, q] = [(r[i] - mean) * inv * w["queryNormScale"][i] + w["queryNormOffset"][i] for i in range(c)]

    def proj(vec, mat, col):
        return sum(vec[i] * mat[i][col] for i in range(c))

    out = np.zeros((rows, c))
    for b in range(B):
        for q in range(Q):
            weighted = [0.0] * c
            for h in range(H):
                qv = [proj(xn[b, q], w["queryWeight"], h * d + i) / math.sqrt(d) for i in range(d)]
                gate = [1 / (1 + math.exp(-(proj(xn[b, q], w["gatingWeight"], h * d + i) + w["gatingBias"][h * d + i])))
                        for i in range(d)]
                acc = [0.0] * d
                run_max, run_sum = -1e30, 0.0
                for k in range(Q):
                    kv = [proj(xn[b, k], w["keyWeight"], h * d + i) for i in range(d)]
                    vv = [proj(xn[b, k], w["valueWeight"], h * d + i) for i in range(d)]
                    logit = sum(qv[i] * kv[i] for i in range(d)) + 1e9 * (mask[src(b, k)] - 1)
                    if bias_w is not None:
                        logit += sum(xn[q, k][i] * bias_w[i][h] for i in range(c))
                    if bias_fn is not None:
                        logit += bias_fn(h, q, k)
                    logit = min(max(logit, -1e8), 1e8)
                    new_max = max(run_max, logit)
                    scale, e = math.exp(run_max - new_max), math.exp(logit - new_max)
                    run_sum = run_sum * scale + e
                    run_max = new_max
                    acc = [acc[i] * scale + e * vv[i] for i in range(d)]
                for i in range(d):
                    weighted[h * d + i] = acc[i] / run_sum * gate[i]
            for col in range(c):
                out[src(b, q), col] = sum(weighted[i] * w["outputWeight"][i][col] for i in range(c)) + \
                    w["outputBias"][col]
    return out


def test_attention_restatement_matches_the_kernel_loops():
    rng = np.random.default_rng(3)
    B = Q = 4
    c, H = 8, 2
    w = _weights(rng, c, H)
    bias_w = rng.standard_normal((c, H)) / math.sqrt(c)
    for transpose in (False, True):
        x = rng.standard_normal((B * Q, c))
        mask = (rng.random(B * Q) < 0.75).astype(np.float64)
        got = oracle.attention(x, mask, w, B, Q, H, transpose=transpose,
                               pair_bias={"source": "normalized-input", "projectionWeight": bias_w})
        want = _loops(x, mask, w, B, Q, H, transpose, bias_w)
        np.testing.assert_allclose(got, want, rtol=1e-9, atol=1e-9)


def test_ending_node_is_the_starting_node_of_the_transposed_pair():
    """Triangle attention around the ending node (transpose=True) on z equals the starting-node
    form on z transposed, transposed back (AF2's ending node, attention.ts transpose flag)."""
    rng = np.random.default_rng(5)
    n, c, H = 5, 8, 2
    w = _weights(rng, c, H)
    bias = {"source": "normalized-input", "projectionWeight": rng.standard_normal((c, H))}
    z = rng.standard_normal((n, n, c))
    mask = (rng.random((n, n)) < 0.8).astype(np.float64)
    ending = oracle.attention(z.reshape(n * n, c), mask.ravel(), w, n, n, H, transpose=True, pair_bias=bias)
    zt = np.ascontiguousarray(z.transpose(1, 0, 2))
    starting = oracle.attention(zt.reshape(n * n, c), np.ascontiguousarray(mask.T).ravel(), w, n, n, H,
                                transpose=False, pair_bias=bias)
    np.testing.assert_allclose(ending.reshape(n, n, c), starting.reshape(n, n, c).transpose(1, 0, 2),
                               rtol=1e-12, atol=1e-12)


def test_fully_masked_row_attends_uniformly():
    """Every key masked: all logits clamp to -1e8, so the softmax is uniform over the keys."""
    rng = np.random.default_rng(7)
    B, Q, c, H = 2, 6, 8, 2
    w = _weights(rng, c, H)
    x = rng.standard_normal((B * Q, c))
    mask = np.ones(B * Q)
    mask[:Q] = 0  # batch entry 0: no key survives
    got = oracle.attention(x, mask, w, B, Q, H)
    xn = x[:Q]
    xn = (xn - xn.mean(-1, keepdims=True)) / np.sqrt(xn.var(-1, keepdims=True) + 1e-5) * w["queryNormScale"] + \
        w["queryNormOffset"]
    v = xn @ w["valueWeight"]
    g = 1 / (1 + np.exp(-(xn @ w["gatingWeight"] + w["gatingBias"])))
    want = (v.mean(0, keepdims=True) * g) @ w["outputWeight"] + w["outputBias"]
    np.testing.assert_allclose(got[:Q], want, rtol=1e-10, atol=1e-10)


def test_separate_pair_bias_matches_the_kernel_loops():
    """MSA row attention's bias: the pair [Q*Q, Cp] normalised with its own LayerNorm and
    projected to one value per head (createAttentionPairBiasShader, attention.ts:631-661),
    read at (query, key)."""
    rng = np.random.default_rng(9)
    B, Q, c, H, cp = 3, 4, 8, 2, 6
    w = _weights(rng, c, H)
    pair = rng.standard_normal((Q * Q, cp))
    ln_s, ln_o = 1 + 0.1 * rng.standard_normal(cp), 0.1 * rng.standard_normal(cp)
    pw = rng.standard_normal((cp, H)) / math.sqrt(cp)
    x = rng.standard_normal((B * Q, c))
    mask = (rng.random(B * Q) < 0.8).astype(np.float64)
    got = oracle.attention(x, mask, w, B, Q, H, pair_bias={"source": "separate", "activations": pair,
                                                              "layerNormScale": ln_s, "layerNormOffset": ln_o,
                                                              "projectionWeight": pw})

    def bias(h, q, k):
        r = pair[q * Q + k]
        mean = r.mean()
        inv = 1 / math.sqrt(((r - mean) ** 2).mean() + 1e-5)
        return float((((r - mean) * inv * ln_s + ln_o) * pw[:, h]).sum())

    want = _loops(x, mask, w, B, Q, H, False, None, bias)
    np.testing.assert_allclose(got, want, rtol=1e-9, atol=1e-9)
