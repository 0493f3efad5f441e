"""Seeded synthetic inputs shared by the tests and the benchmark.

Inputs follow the benchmark configs' laws: activations ~N(0,1), projection
weights ~N(0, 1/fan_in) in the reference's layouts, LayerNorm gamma = 1 and
beta = 0 unless `perturbed` asks for non-trivial LayerNorm and bias values
(which the reference's own deterministic inputs also use,
src/testing/deterministic-input.ts:18-51).
"""
from __future__ import annotations

import numpy as np

ORDER = (
    "layerNormInWeight", "layerNormInBias",
    "linearAPWeight", "linearAPBias", "linearAGWeight", "linearAGBias",
    "linearBPWeight", "linearBPBias", "linearBGWeight", "linearBGBias",
    "layerNormOutWeight", "layerNormOutBias",
    "linearZWeight", "linearZBias", "linearGWeight", "linearGBias",
)


def triangle_weights(cz: int, ch: int, rng: np.random.Generator, perturbed: bool = False) -> dict:
    def normal(shape, fan_in):
        return (rng.standard_normal(shape) / np.sqrt(fan_in)).astype(np.float32)

    def vec(n, center=0.0, scale=0.0):
        if not perturbed:
            return np.full(n, center, np.float32)
        return (center + scale * (rng.random(n) * 2 - 1)).astype(np.float32)

    return {
        "layerNormInWeight": vec(cz, 1.0, 0.1), "layerNormInBias": vec(cz, 0.0, 0.05),
        "linearAPWeight": normal((ch, cz), cz), "linearAPBias": vec(ch, 0.0, 0.03),
        "linearAGWeight": normal((ch, cz), cz), "linearAGBias": vec(ch, 0.0, 0.5),
        "linearBPWeight": normal((ch, cz), cz), "linearBPBias": vec(ch, 0.0, 0.03),
        "linearBGWeight": normal((ch, cz), cz), "linearBGBias": vec(ch, 0.0, 0.5),
        "layerNormOutWeight": vec(ch, 1.0, 0.1), "layerNormOutBias": vec(ch, 0.0, 0.05),
        "linearZWeight": normal((cz, ch), ch), "linearZBias": vec(cz, 0.0, 0.03),
        "linearGWeight": normal((cz, cz), cz), "linearGBias": vec(cz, 0.0, 0.5),
    }


def pack(weights: dict) -> np.ndarray:
    return np.concatenate([np.asarray(weights[k], np.float32).ravel() for k in ORDER])


def triangle_case(n: int, cz: int = 128, ch: int = 128, seed: int = 0, mask_p: float = 1.0,
                  perturbed: bool = False):
    rng = np.random.default_rng(seed)
    z = rng.standard_normal((n, n, cz)).astype(np.float32)
    mask = np.ones((n, n), np.float32) if mask_p >= 1 else (rng.random((n, n)) < mask_p).astype(np.float32)
    w = triangle_weights(cz, ch, rng, perturbed)
    return z, mask, w


def relative_max_error(actual, expected) -> float:
    """max|actual - expected| / max|expected| (the benchmark configs' tolerance measure)."""
    a = np.asarray(actual, np.float64)
    e = np.asarray(expected, np.float64)
    return float(np.abs(a - e).max() / max(np.abs(e).max(), 1e-30))


def bf16_round(x: np.ndarray) -> np.ndarray:
    """f32 -> bf16 (round to nearest even) -> f32, bit manipulation only."""
    a = np.ascontiguousarray(x, np.float32).copy()
    u = a.view(np.uint32)
    u[:] = ((u.astype(np.uint64) + 0x7FFF + ((u >> 16) & 1)) >> 16 << 16).astype(np.uint32)
    return a


def spread(count: int, seed: float) -> np.ndarray:
    """The reference OPM test's inputs, sin((index + 1) * seed) * 0.7 stored as f32
    (test/outer-product-mean-reference.gpu.test.ts:81-88)."""
    return (np.sin(np.arange(1, count + 1, dtype=np.float64) * seed) * 0.7).astype(np.float32)


def opm_reference_test_case():
    """The case of test/outer-product-mean-reference.gpu.test.ts:104-124: 9 sequences,
    8 residues, c_m 12, 32 outer channels, c_z 16, every third mask entry (flat
    [S, N] index) zero, spread-valued weights, rowBlockResidues 3.
    Returns (m [S, N, c_m], mask [S, N], weights dict, row_block)."""
    s, n, cm, c, cz = 9, 8, 12, 32, 16
    mask = np.ones(s * n, np.float32)
    mask[::3] = 0
    w = dict(layerNormScale=spread(cm, 0.31), layerNormOffset=spread(cm, 0.17),
             leftWeight=spread(cm * c, 0.11), leftBias=spread(c, 0.23),
             rightWeight=spread(cm * c, 0.13), rightBias=spread(c, 0.29),
             outputWeight=spread(c * c * cz, 0.07), outputBias=spread(cz, 0.37))
    return spread(s * n * cm, 0.19).reshape(s, n, cm), mask.reshape(s, n), w, 3


def opm_reference_test_expected(m, mask, w, c: int = 32) -> np.ndarray:
    """The reference test's own `reference()` (test/outer-product-mean-reference.gpu.test.ts:22-79)
    restated with its storage: sums in f64 (JS numbers), every Float32Array store
    rounded to f32, the per-pair outer accumulator a Float32Array updated per sequence."""
    s, n, cm = m.shape
    cz = w["outputBias"].size
    x = m.astype(np.float64).reshape(s * n, cm)
    mean = x.sum(1, keepdims=True) / cm
    inv = 1 / np.sqrt(((x - mean) ** 2).sum(1, keepdims=True) / cm + 1e-5)
    xn = ((x - mean) * inv * w["layerNormScale"].astype(np.float64)
          + w["layerNormOffset"].astype(np.float64)).astype(np.float32).astype(np.float64)
    flat_mask = mask.reshape(-1).astype(np.float64)

    def project(weight, bias):
        total = bias.astype(np.float64) + xn @ weight.reshape(cm, c).astype(np.float64)
        return (flat_mask[:, None] * total).astype(np.float32).reshape(s, n, c)

    left, right = project(w["leftWeight"], w["leftBias"]), project(w["rightWeight"], w["rightBias"])
    wo = w["outputWeight"].reshape(c * c, cz).astype(np.float64)
    out = np.zeros((n, n, cz), np.float32)
    for i in range(n):
        for j in range(n):
            pair = np.zeros(c * c, np.float32)
            count = 0.0
            for q in range(s):
                count += float(mask[q, i]) * float(mask[q, j])
                prod = np.outer(left[q, i].astype(np.float64), right[q, j].astype(np.float64)).ravel()
                pair = (pair.astype(np.float64) + prod).astype(np.float32)
            total = w["outputBias"].astype(np.float64) + pair.astype(np.float64) @ wo
            out[i, j] = (total * (1 / (1e-3 + count))).astype(np.float32)
    return out


def opm_f16_operand_model(m, mask, w, c: int = 32) -> np.ndarray:
    """The OPM with this build's rounding points for an f32 MSA, in f64 otherwise:
    LN(m)*gamma + beta, the projection weights, left/right (masked, biased), the outer
    products and W_o are rounded to f16 (the kernels' power-of-two scalings are exact
    and left out); sums are exact.  Used to show that a GPU result's distance from the
    reference is the f16 operand rounding and nothing else."""
    s, n, cm = m.shape
    cz = w["outputBias"].size

    def f16(a):
        return np.asarray(a, np.float64).astype(np.float16).astype(np.float64)

    x = m.astype(np.float64)
    xn = f16((x - x.mean(-1, keepdims=True)) / np.sqrt(x.var(-1, keepdims=True) + 1e-5) * w["layerNormScale"]
             + w["layerNormOffset"])
    msk = mask.astype(np.float64)[..., None]
    left = f16((xn @ f16(w["leftWeight"].reshape(cm, c)) + w["leftBias"]) * msk)
    right = f16((xn @ f16(w["rightWeight"].reshape(cm, c)) + w["rightBias"]) * msk)
    outer = f16(np.einsum("sia,sjb->ijab", left, right).reshape(n, n, c * c))
    cnt = np.einsum("si,sj->ij", mask.astype(np.float64), mask.astype(np.float64))
    return (outer @ f16(w["outputWeight"].reshape(c * c, cz)) + w["outputBias"]) / (1e-3 + cnt)[..., None]
