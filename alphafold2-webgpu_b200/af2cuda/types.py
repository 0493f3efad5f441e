"""The triangle operator's data contract, mirroring src/triangle/types.ts and
src/triangle/weights.ts of the reference."""
from __future__ import annotations

import math
from dataclasses import dataclass
from typing import Optional

import numpy as np

from ._lib import RangeError

MAX_SAFE_INTEGER = 2**53 - 1

# src/triangle/weights.ts:4-10.
ORDER = (
    "layerNormInWeight", "layerNormInBias",
    "linearAPWeight", "linearAPBias", "linearAGWeight", "linearAGBias",
    "linearBPWeight", "linearBPBias", "linearBGWeight", "linearBGBias",
    "layerNormOutWeight", "layerNormOutBias",
    "linearZWeight", "linearZBias", "linearGWeight", "linearGBias",
)


@dataclass(frozen=True)
class TriangleShape:
    """TriangleShape, types.ts:3-7."""
    length: int
    cZ: int
    cHidden: int


@dataclass(frozen=True)
class TriangleMultiplicationWeights:
    """TriangleMultiplicationWeights, types.ts:9-26: projection weights are [out, in]."""
    layerNormInWeight: np.ndarray
    layerNormInBias: np.ndarray
    linearAPWeight: np.ndarray
    linearAPBias: np.ndarray
    linearAGWeight: np.ndarray
    linearAGBias: np.ndarray
    linearBPWeight: np.ndarray
    linearBPBias: np.ndarray
    linearBGWeight: np.ndarray
    linearBGBias: np.ndarray
    layerNormOutWeight: np.ndarray
    layerNormOutBias: np.ndarray
    linearZWeight: np.ndarray
    linearZBias: np.ndarray
    linearGWeight: np.ndarray
    linearGBias: np.ndarray


@dataclass(frozen=True)
class TriangleMultiplicationInput:
    """TriangleMultiplicationInput, types.ts:28-33."""
    shape: TriangleShape
    z: np.ndarray
    mask: np.ndarray
    weights: TriangleMultiplicationWeights
    epsilon: Optional[float] = None


def _positive_integer(name: str, value) -> None:
    if not isinstance(value, (int, np.integer)) or isinstance(value, bool) or value <= 0 or value > MAX_SAFE_INTEGER:
        raise RangeError(f"{name} must be a positive safe integer; received {value}")


def _expect_length(name: str, value: np.ndarray, length: int) -> None:
    if np.asarray(value).size != length:
        raise RangeError(f"{name} has {np.asarray(value).size} values; expected {length}")


def validate_triangle_input(inp: TriangleMultiplicationInput) -> None:
    """validateTriangleInput, types.ts:54-89 (RangeError on any mismatch)."""
    length, cz, ch = inp.shape.length, inp.shape.cZ, inp.shape.cHidden
    _positive_integer("length", length)
    _positive_integer("cZ", cz)
    _positive_integer("cHidden", ch)
    pair_count = length * length
    if pair_count * max(cz, ch) > MAX_SAFE_INTEGER:
        raise RangeError("tensor dimensions exceed JavaScript's safe integer range")
    _expect_length("z", inp.z, pair_count * cz)
    _expect_length("mask", inp.mask, pair_count)
    w = inp.weights
    expected = {
        "layerNormInWeight": cz, "layerNormInBias": cz,
        "linearAPWeight": ch * cz, "linearAPBias": ch, "linearAGWeight": ch * cz, "linearAGBias": ch,
        "linearBPWeight": ch * cz, "linearBPBias": ch, "linearBGWeight": ch * cz, "linearBGBias": ch,
        "layerNormOutWeight": ch, "layerNormOutBias": ch,
        "linearZWeight": cz * ch, "linearZBias": cz, "linearGWeight": cz * cz, "linearGBias": cz,
    }
    for name in ORDER:
        _expect_length(name, getattr(w, name), expected[name])
    if inp.epsilon is not None and (not inp.epsilon > 0 or not math.isfinite(inp.epsilon)):
        raise RangeError(f"epsilon must be finite and positive; received {inp.epsilon}")


def error_metrics(actual, expected) -> dict:
    """errorMetrics, types.ts:91-110: mean, max and RMS of the absolute error (f64)."""
    a = np.asarray(actual, np.float32).ravel().astype(np.float64)
    e = np.asarray(expected, np.float32).ravel().astype(np.float64)
    if a.size != e.size or a.size == 0:
        raise RangeError("error metrics require equally sized, non-empty arrays")
    d = np.abs(a - e)
    return {"meanAbsoluteError": float(d.mean()), "maxAbsoluteError": float(d.max()),
            "rootMeanSquareError": float(math.sqrt((d * d).mean()))}


def expected_weight_element_count(shape: TriangleShape) -> int:
    """expectedWeightElementCount, weights.ts:36-40."""
    cz, ch = shape.cZ, shape.cHidden
    return 2 * cz + 4 * (ch * cz + ch) + 2 * ch + (cz * ch + cz) + (cz * cz + cz)


def pack_weights(weights: TriangleMultiplicationWeights) -> tuple[np.ndarray, dict]:
    """packWeights, weights.ts:20-34 (f32): one array in ORDER plus offsets."""
    offsets, parts, count = {}, [], 0
    for name in ORDER:
        arr = np.ascontiguousarray(getattr(weights, name), np.float32).ravel()
        offsets[name] = count
        count += arr.size
        parts.append(arr)
    return np.concatenate(parts), offsets
