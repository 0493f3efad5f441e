"""The binary tensor manifest reader and writer (af2cuda.tensor_store) against the
oracle's restatement of the reference's q8 format: readTensorRange
(src/reference/dtype.ts:66-99) and the quantizer (tools/quantize-web-model.ts:98-119).
CPU only: decode and quantize bit for bit, stacked-block ranges, and the
reference's error cases."""
import json

import numpy as np
import pytest

import af2cuda
import oracle
from af2cuda import tensor_store as ts


def _tensors(rng):
    return {
        "stack/left_projection/weights": (rng.standard_normal((3, 64, 32)) / 8).astype(np.float32),
        "stack/left_projection/bias": (0.1 * rng.standard_normal((3, 32))).astype(np.float32),
        "stack/layer_norm/scale": (1 + 0.1 * rng.standard_normal((3, 64))).astype(np.float32),
        "single/odd": rng.standard_normal(77).astype(np.float32),
        "single/half": rng.standard_normal((5, 7)).astype(np.float32),
        "single/zeros": np.zeros(130, np.float32),
    }


@pytest.fixture()
def store(tmp_path):
    rng = np.random.default_rng(7)
    tensors = _tensors(rng)
    q8 = {"stack/left_projection/weights", "stack/left_projection/bias", "single/odd", "single/zeros"}
    path = af2cuda.write_tensor_manifest(tmp_path, tensors, q8=q8, float16={"single/half"})
    return af2cuda.FileTensorStore.open(path), tensors, q8


def test_quantizer_matches_the_oracle_bit_for_bit():
    rng = np.random.default_rng(0)
    for w in (rng.standard_normal(4096).astype(np.float32) * 3, rng.standard_normal(100).astype(np.float32) * 1e-6,
              np.zeros(64, np.float32), (rng.standard_normal(513) * 1e4).astype(np.float32)):
        codes, scales = af2cuda.quantize_q8_block(w)
        ocodes, oscales = oracle.quantize_q8_block(w)
        assert np.array_equal(codes, ocodes)
        assert np.array_equal(scales, oscales)


def test_quantizer_rounds_ties_toward_positive_infinity():
    # block max 127 gives scale f16(1.0) = 1: the codes are Math.round of the values
    w = np.array([127, 2.5, -2.5, 0.5, -0.5, 1.5, -1.5] + [0] * 57, np.float32)
    codes, scales = af2cuda.quantize_q8_block(w)
    assert scales[0] == 0x3C00
    assert codes[:7].tolist() == [127, 3, -2, 1, 0, 2, -1]


def test_whole_tensors_decode_as_the_oracle(store):
    st, tensors, q8 = store
    for name, value in tensors.items():
        got = st.tensor(name)
        assert got.dtype == np.float32 and got.size == value.size
        if name in q8:
            codes, scales = oracle.quantize_q8_block(value)
            assert np.array_equal(got, oracle.dequant_q8_block(codes, scales)), name
            assert np.abs(got - value.ravel()).max() <= np.abs(value).max() / 127 * 0.5 + 1e-12
        elif name == "single/half":
            assert np.array_equal(got, value.ravel().astype(np.float16).astype(np.float32))
        else:
            assert np.array_equal(got, value.ravel())
        assert st.shape(name) == value.shape


def test_stacked_blocks_decode_as_slices_of_the_whole(store):
    st, tensors, _ = store
    for name in ("stack/left_projection/weights", "stack/left_projection/bias", "stack/layer_norm/scale"):
        st.ensure_loaded(name)
        whole = st.tensor(name)
        per = whole.size // 3
        for b in range(3):
            # the bias blocks of 32 values start inside a 64-value scale block for b = 1
            assert np.array_equal(st.read(name, b, 3), whole[b * per:(b + 1) * per]), (name, b)


def test_read_needs_ensure_loaded_and_ranges_are_checked(store):
    st, _, _ = store
    with pytest.raises(RuntimeError):
        st.read("single/odd")
    st.ensure_loaded("single/odd")
    with pytest.raises(af2cuda.RangeError):
        st.read("single/odd", 0, 2)  # 77 values do not split into 2 blocks
    with pytest.raises(af2cuda.RangeError):
        st.read("stack/left_projection/bias", 3, 3)
    with pytest.raises(KeyError):
        st.shape("missing")


def test_manifest_layout_follows_the_quantizer(store):
    st, tensors, q8 = store
    for name in tensors:
        r = st.record(name)
        assert r["byteOffset"] % 4 == 0
        if name in q8:
            assert r["dtype"] == "int8" and r["block"] == 64
            assert r["scaleOffset"] % 2 == 0 and r["scaleOffset"] >= r["byteOffset"] + tensors[name].size
            n = tensors[name].size
            assert af2cuda.tensor_byte_length(r) == r["scaleOffset"] - r["byteOffset"] + 2 * ((n + 63) // 64)


def test_invalid_records_are_rejected():
    good = {"file": "x", "shape": [10], "dtype": "int8", "byteOffset": 0, "block": 64, "scaleOffset": 10}
    assert af2cuda.tensor_byte_length(good) == 12
    for bad in ({**good, "block": 0}, {**good, "scaleOffset": 9}, {**good, "scaleOffset": 11},
                {**good, "block": None}):
        with pytest.raises(ValueError):
            af2cuda.tensor_byte_length(bad)
    with pytest.raises(ValueError):
        af2cuda.tensor_elements({"shape": [0, 3]})
    buf = bytes(11)
    with pytest.raises(ValueError):
        af2cuda.read_tensor_range(good, buf, 0, 0, 10)  # the scales run past the shard
    f32 = {"file": "x", "shape": [2], "dtype": "float32"}
    with pytest.raises(ValueError):
        af2cuda.read_tensor_range(f32, bytes(12), 2, 0, 2)  # unaligned f32


def test_manifest_without_a_tensor_table_is_rejected(tmp_path):
    p = tmp_path / "manifest.json"
    p.write_text(json.dumps({"bundle": {}}))
    with pytest.raises(ValueError):
        af2cuda.FileTensorStore.open(p)


def test_float16_decode_covers_subnormals_and_specials():
    bits = np.array([0x0001, 0x03FF, 0x8000, 0x7C00, 0xFC00, 0x3C00, 0x7BFF], np.uint16)
    got = ts.float16_to_number(bits)
    assert np.array_equal(got[[0, 1, 2, 5, 6]], oracle.f16_value(bits[[0, 1, 2, 5, 6]]).astype(np.float32))
    assert np.signbit(got[2]) and np.isinf(got[3]) and np.isinf(got[4]) and got[4] < 0
