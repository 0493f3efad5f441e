"""Reader for the reference's frozen operator bundles: a manifest.json plus raw
little-endian float32 tensors (src/reference/bundle.ts:1-20, loader
src/reference/node.ts:13-42)."""
from __future__ import annotations

import json
from dataclasses import dataclass
from pathlib import Path

import numpy as np

from .types import (ORDER, TriangleMultiplicationInput, TriangleMultiplicationWeights, TriangleShape)


@dataclass(frozen=True)
class TriangleReferenceBundle:
    input: TriangleMultiplicationInput
    expected: np.ndarray
    source: str


def load_triangle_reference_bundle_from_files(manifest_path) -> TriangleReferenceBundle:
    path = Path(manifest_path)
    manifest = json.loads(path.read_text())
    if manifest.get("formatVersion") != 1 or manifest.get("operator") != "TriangleMultiplicationOutgoing":
        raise ValueError("unsupported triangle reference manifest")

    def tensor(name: str) -> np.ndarray:
        record = manifest["tensors"].get(name)
        if record is None or record["dtype"] != "float32":
            raise ValueError(f"missing float32 tensor {name}")
        data = np.fromfile(path.parent / record["file"], dtype="<f4")
        if data.size != int(np.prod(record["shape"])):
            raise ValueError(f"{name} has {data.size} values; expected {int(np.prod(record['shape']))}")
        return data

    shape = TriangleShape(**{k: int(v) for k, v in manifest["shape"].items()})
    weights = TriangleMultiplicationWeights(**{name: tensor(name) for name in ORDER})
    inp = TriangleMultiplicationInput(shape=shape, z=tensor("z"), mask=tensor("mask"), weights=weights,
                                      epsilon=float(manifest["epsilon"]))
    return TriangleReferenceBundle(input=inp, expected=tensor("expected"), source=manifest["source"])
