"""CPU tests of the C ABI: the library loads, exports every symbol the header
declares, and its host-side logic (validation, sizing) behaves like the
reference's.  No kernel runs here."""
import ctypes
import re
import subprocess
from pathlib import Path

import numpy as np
import pytest

import af2cuda
from af2cuda import _lib
from conftest import ROOT, bundle_path

HEADER = ROOT / "include" / "af2cuda.h"


def declared_symbols() -> list[str]:
    text = re.sub(r"/\*.*?\*/", "", HEADER.read_text(), flags=re.S)
    return sorted(set(re.findall(r"\b(af2_[a-z0-9_]+)\s*\(", text)))


def test_library_exports_every_declared_symbol():
    lib = _lib.lib()
    names = declared_symbols()
    assert len(names) >= 10
    for name in names:
        assert hasattr(lib, name), name
    # ...and the ctypes table covers exactly the header.
    assert sorted(_lib.SIGNATURES) == names
    exported = subprocess.run(["nm", "-D", "--defined-only", str(_lib.LIB_PATH)], capture_output=True, text=True).stdout
    public = sorted(set(re.findall(r"\bT (af2_[a-z0-9_]+)$", exported, flags=re.M)))
    assert public == names


def test_build_targets_sm100a_only():
    import importlib.util
    spec = importlib.util.spec_from_file_location("af2_build", ROOT / "alphafold2-webgpu_b200" / "build.py")
    build = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(build)
    assert build.ARCH == ["-gencode", "arch=compute_100a,code=sm_100a"]


def test_version_and_status_strings():
    lib = _lib.lib()
    assert lib.af2_version() == 1
    assert lib.af2_status_string(_lib.AF2_ERR_INVALID_ARGUMENT) == b"invalid argument"
    assert lib.af2_status_string(99) == b"unknown status"


def test_weight_count_matches_reference_formula():
    for cz, ch in [(7, 6), (128, 128), (64, 64), (1, 1)]:
        expected = af2cuda.expected_weight_element_count(af2cuda.TriangleShape(1, cz, ch))
        assert af2cuda.triangle_weight_count(cz, ch) == expected
    assert af2cuda.triangle_weight_count(128, 128) == 99_584  # packWeights at c = 128


def _check(direction, n, cz, ch, count=None, eps=1e-5):
    shape = _lib.TriangleShape(n, cz, ch)
    msg = ctypes.create_string_buffer(256)
    if count is None:
        count = af2cuda.triangle_weight_count(max(cz, 1), max(ch, 1))
    st = _lib.lib().af2_triangle_check(direction, ctypes.byref(shape), count, eps, msg, 256)
    return st, msg.value.decode()


def test_c_validation_mirrors_validate_triangle_input():
    assert _check(0, 5, 7, 6) == (0, "")
    assert _check(1, 1024, 128, 128)[0] == 0
    st, msg = _check(0, 0, 7, 6)
    assert st == _lib.AF2_ERR_INVALID_ARGUMENT and msg == "length must be a positive safe integer; received 0"
    st, msg = _check(0, 5, -1, 6)
    assert st == _lib.AF2_ERR_INVALID_ARGUMENT and "cZ must be a positive safe integer" in msg
    st, msg = _check(0, 5, 7, 6, count=10)
    assert st == _lib.AF2_ERR_INVALID_ARGUMENT and msg == "packed weights have 10 values; expected 323"
    for eps in (0.0, -1.0, float("inf"), float("nan")):
        assert _check(0, 5, 7, 6, eps=eps)[0] == _lib.AF2_ERR_INVALID_ARGUMENT
    assert _check(2, 5, 7, 6)[0] == _lib.AF2_ERR_INVALID_ARGUMENT
    assert _check(0, 2**27, 128, 128)[1] == "tensor dimensions exceed JavaScript's safe integer range"
    # valid for the reference, beyond the kernels
    assert _check(0, 5, 256, 128)[0] == _lib.AF2_ERR_UNSUPPORTED


def test_python_validation_mirrors_reference():
    bundle = af2cuda.load_triangle_reference_bundle_from_files(bundle_path("openfold-triangle-small"))
    inp = bundle.input
    af2cuda.validate_triangle_input(inp)
    bad = af2cuda.TriangleMultiplicationInput(inp.shape, inp.z[1:], inp.mask, inp.weights)
    with pytest.raises(af2cuda.RangeError, match="z has"):
        af2cuda.validate_triangle_input(bad)
    with pytest.raises(af2cuda.RangeError, match="epsilon must be finite and positive"):
        af2cuda.validate_triangle_input(af2cuda.TriangleMultiplicationInput(inp.shape, inp.z, inp.mask,
                                                                            inp.weights, epsilon=0.0))
    with pytest.raises(af2cuda.RangeError, match="length must be a positive safe integer"):
        af2cuda.validate_triangle_input(af2cuda.TriangleMultiplicationInput(
            af2cuda.TriangleShape(0, 7, 6), inp.z, inp.mask, inp.weights))


def test_workspace_bytes_scale_with_block_rows():
    whole = af2cuda.triangle_workspace_bytes(1024, 128, 128)
    blocked = af2cuda.triangle_workspace_bytes(1024, 128, 128, block_rows=128)
    # a, b and the z re-layout stay; the contracted block shrinks 8x.
    assert whole - blocked == 128 * (1024 - 128) * 1024 * 2
    assert whole < 1.2e9


def test_no_device_is_reported_not_faked():
    import torch
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    handle = ctypes.c_void_p()
    assert _lib.lib().af2_create(0, ctypes.byref(handle)) == _lib.AF2_ERR_NO_DEVICE
    with pytest.raises(af2cuda.Af2Error):
        af2cuda.Device(0)


def test_loader_fails_loudly_without_the_library(tmp_path, monkeypatch):
    monkeypatch.setattr(_lib, "LIB_PATH", tmp_path / "missing.so")
    monkeypatch.setattr(_lib, "_lib", None)
    with pytest.raises(OSError, match="libaf2cuda.so not found"):
        _lib.lib()


def _tcheck(rows, c, h, count=None, eps=1e-5):
    shape = _lib.TransitionShape(rows, c, h)
    msg = ctypes.create_string_buffer(256)
    if count is None:
        count = af2cuda.transition_weight_count(max(c, 1), max(h, 1))
    st = _lib.lib().af2_transition_check(ctypes.byref(shape), count, eps, msg, 256)
    return st, msg.value.decode()


def test_transition_weight_count_and_validation():
    # packTransitionWeights: LN scale + offset, W1, b1, W2, b2 (transition.ts:158-177)
    assert af2cuda.transition_weight_count(128, 512) == 2 * 128 + 128 * 512 + 512 + 512 * 128 + 128
    assert _tcheck(65536, 128, 512) == (0, "")
    assert _tcheck(0, 128, 512) == (_lib.AF2_ERR_INVALID_ARGUMENT,
                                    "transition dimensions must be positive safe integers")
    assert _tcheck(5, 7, 6, count=3) == (_lib.AF2_ERR_INVALID_ARGUMENT, "packed weights have 3 values; expected 111")
    for eps in (0.0, -1.0, float("inf"), float("nan")):
        assert _tcheck(5, 7, 6, eps=eps)[0] == _lib.AF2_ERR_INVALID_ARGUMENT
    # the MSA transition (c_m 256 -> 1024) takes the two-GEMM path; the limits lie beyond it
    assert _tcheck(5, 256, 1024) == (0, "")
    st, msg = _tcheck(5, 8192, 1024)
    assert st == _lib.AF2_ERR_UNSUPPORTED and "above 4096" in msg
    st, msg = _tcheck(5, 64, 32768)
    assert st == _lib.AF2_ERR_UNSUPPORTED and "above 16384" in msg


def test_transition_python_validation_and_packing():
    rng = np.random.default_rng(0)
    c, h = 4, 6
    w = af2cuda.TransitionWeights(*(rng.standard_normal(n).astype(np.float32) for n in (c, c, c * h, h, h * c, c)))
    inp = af2cuda.TransitionInput(rng.standard_normal(3 * c).astype(np.float32), 3, c, h, w)
    af2cuda.validate_transition_input(inp)
    data, offsets = af2cuda.pack_transition_weights(inp)
    assert offsets == (0, c, 2 * c, 2 * c + c * h, 2 * c + c * h + h, 2 * c + 2 * c * h + h)
    assert data.size == af2cuda.transition_weight_count(c, h)
    assert np.array_equal(data[offsets[4]:offsets[5]], w.secondWeight)
    bad = af2cuda.TransitionInput(inp.activations[:-1], 3, c, h, w)
    with pytest.raises(af2cuda.RangeError, match="activations has 11 values; expected 12"):
        af2cuda.validate_transition_input(bad)
    with pytest.raises(af2cuda.RangeError):
        af2cuda.TransitionGpu.__new__(af2cuda.TransitionGpu).__init__(None, {"maxChunkRows": 0})


def test_transition_workspace_is_small():
    # the hidden activations never reach HBM: scratch is prepared weights plus
    # a bounded normalised copy, independent of rows beyond 65536
    small = af2cuda.transition_workspace_bytes(65536, 128, 512)
    big = af2cuda.transition_workspace_bytes(4 * 65536, 128, 512)
    assert small == big and small < 32 << 20


def test_wide_transition_workspace_is_bounded_per_chunk():
    # channels above 128: the hidden activations go through HBM one row chunk at a time,
    # so the scratch stops growing once the rows exceed one chunk (about 256 MiB of hidden)
    one = af2cuda.transition_workspace_bytes(4096, 256, 1024)
    many = af2cuda.transition_workspace_bytes(512 * 1024, 256, 1024)
    more = af2cuda.transition_workspace_bytes(4 * 512 * 1024, 256, 1024)
    assert one < many == more < 400 << 20


def test_opm_weight_count_and_validation():
    shape = _lib.OpmShape(512, 256, 256, 32, 128)
    count = af2cuda.opm_weight_count(512, 256, 256, 32, 128)
    assert count == 2 * 256 + 2 * (256 * 32 + 32) + 32 * 32 * 128 + 128
    msg = ctypes.create_string_buffer(256)
    assert _lib.lib().af2_opm_check(ctypes.byref(shape), count, msg, 256) == 0
    assert _lib.lib().af2_opm_check(ctypes.byref(shape), count - 1, msg, 256) == _lib.AF2_ERR_INVALID_ARGUMENT
    assert msg.value.decode() == f"packed weights have {count - 1} values; expected {count}"
    bad = _lib.OpmShape(0, 256, 256, 32, 128)
    assert _lib.lib().af2_opm_check(ctypes.byref(bad), count, msg, 256) == _lib.AF2_ERR_INVALID_ARGUMENT
    c16 = _lib.OpmShape(512, 256, 256, 16, 128)
    n16 = af2cuda.opm_weight_count(512, 256, 256, 16, 128)
    assert _lib.lib().af2_opm_check(ctypes.byref(c16), n16, msg, 256) == _lib.AF2_ERR_UNSUPPORTED


def test_opm_python_validation_and_packing():
    rng = np.random.default_rng(0)
    s, n, cm, c, cz = 2, 3, 4, 32, 5
    w = af2cuda.OuterProductMeanWeights(*(rng.standard_normal(k).astype(np.float32)
                                          for k in (cm, cm, cm * c, c, cm * c, c, c * c * cz, cz)))
    inp = af2cuda.OuterProductMeanInput(rng.standard_normal(s * n * cm).astype(np.float32),
                                        np.ones(s * n, np.float32), s, n, cm, c, cz, w)
    af2cuda.validate_outer_product_mean_input(inp)
    data, offsets = af2cuda.pack_outer_product_mean_weights(inp)
    assert data.size == af2cuda.opm_weight_count(s, n, cm, c, cz)
    assert offsets[6] == 2 * cm + 2 * (cm * c + c) and np.array_equal(data[offsets[6]:offsets[7]], w.outputWeight)
    with pytest.raises(af2cuda.RangeError, match="mask has 5 values; expected 6"):
        af2cuda.validate_outer_product_mean_input(
            af2cuda.OuterProductMeanInput(inp.activations, np.ones(5, np.float32), s, n, cm, c, cz, w))


def test_opm_workspace_blocks_bound_the_outer_scratch():
    # c_z above 128: the two-kernel path, whose outer-product scratch the residue blocks bound
    whole = af2cuda.opm_workspace_bytes(512, 768, 256, 32, 160)
    b4 = af2cuda.opm_workspace_bytes(512, 768, 256, 32, 160, row_block=4)
    b8 = af2cuda.opm_workspace_bytes(512, 768, 256, 32, 160, row_block=8)
    assert b4 < b8 <= whole
    assert b8 - b4 == 4 * 768 * 32 * 32 * 2  # four more residue rows of f16 outer products


def test_opm_fused_workspace_has_no_outer_scratch():
    # S <= 1024 and c_z <= 128: the outer products stay on chip, whatever the residue block
    fused = af2cuda.opm_workspace_bytes(512, 768, 256, 32, 128)
    assert fused == af2cuda.opm_workspace_bytes(512, 768, 256, 32, 128, row_block=4)
    assert fused < 768 * 768 * 32 * 32 * 2 // 4


def _attention_check(b, q, c, h, bias=1, count=None, eps=1e-5):
    shape = _lib.AttentionShape(b, q, c, h)
    if count is None:
        count = _lib.lib().af2_attention_weight_count(ctypes.byref(shape), bias)
    msg = ctypes.create_string_buffer(256)
    st = _lib.lib().af2_attention_check(ctypes.byref(shape), bias, count, eps, msg, 256)
    return st, msg.value.decode()


def test_attention_weight_count_is_pack_attention_weights_length():
    c, h = 128, 4
    rng = np.random.default_rng(0)
    w = af2cuda.AttentionWeights(*(rng.standard_normal(n).astype(np.float32) for n in
                                   (c, c, c * c, c * c, c * c, c * c, c, c * c, c)))
    for bias in (None, af2cuda.NormalizedInputPairBias(np.zeros(c * h, np.float32))):
        inp = af2cuda.AttentionInput(np.zeros(0), np.zeros(0), 8, 8, c, h, w, pairBias=bias)
        packed, offsets = af2cuda.pack_attention_weights(inp)
        assert packed.size == af2cuda.attention_weight_count(8, 8, c, h, 0 if bias is None else 1)
        assert offsets[:3] == [0, c, 2 * c]


def test_attention_validation_mirrors_the_reference():
    assert _attention_check(64, 64, 128, 4) == (_lib.AF2_OK, "")
    st, msg = _attention_check(64, 64, 96, 2)
    assert st == _lib.AF2_ERR_INVALID_ARGUMENT and "head dimension no larger than 32" in msg
    st, msg = _attention_check(0, 64, 128, 4, count=1)
    assert st == _lib.AF2_ERR_INVALID_ARGUMENT and "positive safe integers" in msg
    st, msg = _attention_check(64, 64, 128, 4, count=5)
    assert st == _lib.AF2_ERR_INVALID_ARGUMENT and "expected" in msg
    st, msg = _attention_check(64, 64, 128, 4, eps=0)
    assert st == _lib.AF2_ERR_INVALID_ARGUMENT and "epsilon" in msg
    # valid for the reference, outside the kernels: head dimension 16, or a bias with batch != queries
    assert _attention_check(64, 64, 64, 4)[0] == _lib.AF2_ERR_UNSUPPORTED
    assert _attention_check(3, 64, 128, 4)[0] == _lib.AF2_ERR_UNSUPPORTED
    assert _attention_check(3, 64, 128, 4, bias=0)[0] == _lib.AF2_OK
