"""Binary tensor manifests: the reference's model-weight files, read straight into
device memory in their stored form.

A manifest.json holds a `tensors` table mapping each name to a record
{file, shape, dtype, byteOffset, block, scaleOffset} in little-endian shard
files (BinaryTensorRecord, src/reference/tensor-store.ts:4-13).  dtype is
"float32", "float16" or "int8"; an int8 tensor keeps one f16 scale (its 16
bits) per `block` consecutive elements of the flattened tensor at
scaleOffset, and element i decodes to code[i] * f16(scale[i // block])
(readTensorRange, src/reference/dtype.ts:66-99).  Model tensors stack the 48
Evoformer blocks along their first axis; `block`/`blocks` select one
(blockRange, dtype.ts:101-110).

FileTensorStore mirrors the reference's FileTensorStore (tensor-store.ts:40-121):
`tensor`, `shape`, `ensure_loaded` and `read` decode to f32 on the host exactly
as the reference does.  `device_weight` is this library's addition: it puts a
tensor on the GPU as it is stored -- int8 codes and f16 scale bits for q8
records, which the per-tensor weight forms (af2_triangle_multiplication_weights,
af2_outer_product_mean_weights, af2_transition) turn into f16 operands on the
device -- so the weights cross PCIe and sit in HBM at a quarter of their f32
size.

`write_tensor_manifest` writes such files, with the reference quantizer's
format and arithmetic (tools/quantize-web-model.ts:74-121): shards aligned to
4 bytes per tensor, the scales aligned to 2, a scale of f16(max|w|/127) per
block (0 -> 1) and codes clamp(round(w / scale), +-127) with JavaScript's
Math.round (ties toward +infinity).
"""
from __future__ import annotations

import json
import math
from pathlib import Path

import numpy as np

from ._lib import RangeError

_WIDTHS = {"float32": 4, "float16": 2, "int8": 1}
MAX_SAFE_INTEGER = 2**53 - 1


def _safe_int(v) -> bool:
    return isinstance(v, (int, np.integer)) and not isinstance(v, bool) and abs(int(v)) <= MAX_SAFE_INTEGER


def tensor_elements(record: dict) -> int:
    """tensorElements (dtype.ts:5-9)."""
    elements = 1
    for d in record["shape"]:
        elements *= int(d)
    if not _safe_int(elements) or elements <= 0:
        raise ValueError("tensor has an invalid element count")
    return elements


def tensor_byte_length(record: dict) -> int:
    """tensorByteLength (dtype.ts:12-26): stored bytes from byteOffset through the final scale."""
    elements = tensor_elements(record)
    if record["dtype"] not in _WIDTHS:
        raise ValueError(f"unsupported tensor dtype {record['dtype']!r}")
    if record["dtype"] != "int8":
        return elements * _WIDTHS[record["dtype"]]
    byte_offset = record.get("byteOffset", 0)
    block, scale_offset = record.get("block"), record.get("scaleOffset")
    if block is None or not _safe_int(block) or block <= 0:
        raise ValueError("int8 tensor has an invalid block size")
    if (scale_offset is None or not _safe_int(scale_offset) or scale_offset < byte_offset + elements
            or scale_offset % 2 != 0):
        raise ValueError("int8 tensor has an invalid scale offset")
    return scale_offset - byte_offset + math.ceil(elements / block) * 2


def float16_to_number(bits) -> np.ndarray:
    """float16ToNumber (dtype.ts:28-35) for an array of f16 bit patterns: the exact value
    (subnormals, signed zeros, infinities and NaN included), as f32."""
    return np.asarray(bits, dtype=np.uint16).view(np.float16).astype(np.float32)


def block_range(elements: int, block=None, blocks=None) -> tuple[int, int]:
    """blockRange (dtype.ts:101-110): element range of one block of a tensor stacked along its
    first axis, or the whole tensor."""
    if block is None:
        return 0, elements
    if (blocks is None or not _safe_int(blocks) or blocks <= 0 or elements % blocks != 0 or not _safe_int(block)
            or block < 0 or block >= blocks):
        raise RangeError("stacked parameter block is out of range")
    size = elements // blocks
    return block * size, size


def _check_range(record: dict, buffer, byte_offset: int, start: int, count: int) -> int:
    elements = tensor_elements(record)
    byte_length = tensor_byte_length(record)
    if not _safe_int(byte_offset) or byte_offset < 0 or byte_offset + byte_length > len(buffer):
        raise ValueError("tensor points outside its shard")
    if not (_safe_int(start) and _safe_int(count)) or start < 0 or count < 0 or start + count > elements:
        raise RangeError("tensor range is out of bounds")
    return elements


def read_tensor_range(record: dict, buffer, byte_offset: int, start: int, count: int) -> np.ndarray:
    """readTensorRange (dtype.ts:66-99): `count` f32 values from value `start` of a stored
    tensor whose record begins at `byte_offset` of `buffer`.  Block scales are indexed by
    absolute position, so a range that starts inside a block decodes as the whole tensor
    would."""
    elements = _check_range(record, buffer, byte_offset, start, count)
    dtype = record["dtype"]
    if dtype == "float32":
        if byte_offset % 4 != 0:
            raise ValueError("float32 tensor has an unaligned byte offset")
        return np.frombuffer(buffer, dtype="<f4", count=count, offset=byte_offset + start * 4)
    if dtype == "float16":
        stored = np.frombuffer(buffer, dtype="<u2", count=count, offset=byte_offset + start * 2)
        return float16_to_number(stored)
    block = int(record["block"])
    codes = np.frombuffer(buffer, dtype=np.int8, count=count, offset=byte_offset + start)
    scale_at = byte_offset + int(record["scaleOffset"]) - int(record.get("byteOffset", 0))
    scales = float16_to_number(np.frombuffer(buffer, dtype="<u2", count=math.ceil(elements / block),
                                             offset=scale_at))
    index = np.arange(start, start + count, dtype=np.int64) // block
    # a 7-bit code times an 11-bit scale is exact in f32, as in the reference's f64 product
    return (codes.astype(np.float32) * scales[index]).astype(np.float32)


class FileTensorStore:
    """FileTensorStore (tensor-store.ts:40-121) over a manifest on disk."""

    def __init__(self, manifest_path, manifest: dict):
        self.manifest_path = Path(manifest_path)
        self.manifest = manifest
        self._directory = self.manifest_path.parent
        self._files: dict[str, bytes] = {}
        self._loaded: dict[str, bytes] = {}

    @classmethod
    def open(cls, manifest_path) -> "FileTensorStore":
        path = Path(manifest_path).resolve()
        manifest = json.loads(path.read_text())
        if manifest.get("tensors") is None:
            raise ValueError(f"{path} has no tensor table")
        return cls(path, manifest)

    def _record(self, name: str) -> dict:
        record = self.manifest["tensors"].get(name)
        if record is None:
            raise KeyError(f"manifest contains no tensor named {name}")
        return record

    def _file(self, file: str) -> bytes:
        data = self._files.get(file)
        if data is None:
            path = (self._directory / file).resolve()
            if self._directory.resolve() not in path.parents:
                raise ValueError(f"{file} escapes the manifest directory")
            data = path.read_bytes()
            self._files[file] = data
        return data

    def names(self) -> list[str]:
        return list(self.manifest["tensors"])

    def shape(self, name: str) -> tuple[int, ...]:
        return tuple(int(d) for d in self._record(name)["shape"])

    def record(self, name: str) -> dict:
        return dict(self._record(name))

    def tensor(self, name: str) -> np.ndarray:
        """The whole tensor decoded to f32 (FileTensorStore.tensor / #load)."""
        record = self._record(name)
        data = self._file(record["file"])
        offset = int(record.get("byteOffset", 0))
        if not _safe_int(offset) or offset < 0 or offset + tensor_byte_length(record) > len(data):
            raise ValueError(f"{name} points outside {record['file']}")
        return read_tensor_range(record, data, offset, 0, tensor_elements(record))

    def ensure_loaded(self, name: str) -> None:
        record = self._record(name)
        self._loaded.setdefault(record["file"], self._file(record["file"]))

    def read(self, name: str, block=None, blocks=None) -> np.ndarray:
        """One stacked block (or the whole tensor) decoded to f32 from a retained shard
        (FileTensorStore.read)."""
        record = self._record(name)
        data = self._loaded.get(record["file"])
        if data is None:
            raise RuntimeError(f"{name} has not been loaded; call ensure_loaded first")
        start, count = block_range(tensor_elements(record), block, blocks)
        return read_tensor_range(record, data, int(record.get("byteOffset", 0)), start, count)

    def device_weight(self, name: str, block=None, blocks=None, device="cuda"):
        """One stacked block (or the whole tensor) on the GPU in its stored form.

        int8 records come back as a Q8Matrix (kind "block") holding the range's codes and the
        scales of the blocks it spans; float32 as an f32 tensor; float16 as the exact f32
        values.  A q8 range that starts inside a scale block (a stacked tensor whose per-block
        size is not a multiple of the scale block: the outer-product-mean biases of 32
        values) cannot be indexed from its own first element, so it comes back as its exact
        f32 decode."""
        import torch

        from .transition import Q8Matrix
        record = self._record(name)
        data = self._file(record["file"])
        elements = tensor_elements(record)
        start, count = block_range(elements, block, blocks)
        offset = int(record.get("byteOffset", 0))
        _check_range(record, data, offset, start, count)
        if record["dtype"] == "int8" and start % int(record["block"]) == 0:
            qb = int(record["block"])
            codes = np.frombuffer(data, dtype=np.int8, count=count, offset=offset + start)
            first, last = start // qb, (start + count + qb - 1) // qb
            scales = np.frombuffer(data, dtype="<u2", count=last - first,
                                   offset=int(record["scaleOffset"]) + 2 * first).view(np.int16)
            return Q8Matrix(torch.from_numpy(codes.copy()).to(device), torch.from_numpy(scales.copy()).to(device),
                            "block", qb)
        values = read_tensor_range(record, data, offset, start, count)
        return torch.from_numpy(np.array(values, dtype=np.float32)).to(device)


def _js_round(q: np.ndarray) -> np.ndarray:
    """Math.round: the nearest integer, ties toward +infinity (exact for |q| < 2^52)."""
    r = np.floor(q)
    return r + (q - r >= 0.5)


def quantize_q8_block(values, block: int = 64) -> tuple[np.ndarray, np.ndarray]:
    """The reference quantizer's int8 branch (tools/quantize-web-model.ts:102-116) over the
    flattened tensor: returns (int8 codes, uint16 f16 scale bits)."""
    v = np.asarray(values, dtype=np.float32).ravel()
    if not np.isfinite(v).all():
        raise ValueError("tensor contains a non-finite value")
    nblocks = math.ceil(v.size / block)
    padded = np.zeros(nblocks * block, np.float64)
    padded[:v.size] = np.abs(v)
    maximum = padded.reshape(nblocks, block).max(axis=1)
    scale_bits = (maximum / 127).astype(np.float16).view(np.uint16)
    scale = scale_bits.view(np.float16).astype(np.float64)
    scale[scale == 0] = 1.0
    q = v.astype(np.float64) / np.repeat(scale, block)[:v.size]
    codes = np.clip(_js_round(q), -127, 127).astype(np.int8)
    return codes, scale_bits


def write_tensor_manifest(directory, tensors: dict, *, q8=(), float16=(), file: str = "weights.v1.q8.bin",
                          block: int = 64) -> Path:
    """Writes `tensors` (name -> array) into one shard and a manifest.json beside it, in the
    reference quantizer's layout; names in `q8` become int8 records, names in `float16`
    float16 records, the rest stay float32.  Returns the manifest path."""
    directory = Path(directory)
    directory.mkdir(parents=True, exist_ok=True)
    q8, float16 = set(q8), set(float16)
    shard = bytearray()
    records = {}

    def align(width: int) -> None:
        shard.extend(b"\0" * ((width - len(shard) % width) % width))

    for name, value in tensors.items():
        arr = np.asarray(value, dtype=np.float32)
        align(4)
        base = {"file": file, "shape": [int(d) for d in arr.shape] or [1], "byteOffset": len(shard)}
        if name in q8:
            codes, scales = quantize_q8_block(arr, block)
            shard.extend(codes.tobytes())
            align(2)
            records[name] = {**base, "dtype": "int8", "block": block, "scaleOffset": len(shard)}
            shard.extend(scales.astype("<u2").tobytes())
        elif name in float16:
            shard.extend(arr.astype("<f2").tobytes())
            records[name] = {**base, "dtype": "float16"}
        else:
            shard.extend(arr.astype("<f4").tobytes())
            records[name] = {**base, "dtype": "float32"}
    (directory / file).write_bytes(bytes(shard))
    manifest = {"bundle": {"version": 1, "encoding": "mixed-q8-f16-scale-le" if q8 else "f32-le",
                           "tensors": len(records), "bytes": len(shard),
                           "files": [{"file": file, "bytes": len(shard)}]},
                "tensors": records}
    path = directory / "manifest.json"
    path.write_text(json.dumps(manifest, indent=1))
    return path
