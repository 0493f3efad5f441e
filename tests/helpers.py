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
