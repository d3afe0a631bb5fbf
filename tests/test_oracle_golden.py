"""The CPU oracle against fixtures produced by the reference's own code
(tests/golden/make_golden.py) and the reference's literal known answers."""

import struct
from pathlib import Path

import numpy as np
import pytest

from oracle import bf16 as ob
from oracle import codec as oc
from oracle import quant as oq

GOLDEN = Path(__file__).resolve().parent / "golden"


@pytest.fixture(scope="module")
def codec():
    return np.load(GOLDEN / "reference_codec.npz")


@pytest.fixture(scope="module")
def quant():
    return np.load(GOLDEN / "reference_quant.npz")


CODEC_CASES = ("all_patterns", "mixed_tail", "normal_ragged", "coded_only", "raw_only")


@pytest.mark.parametrize("name", CODEC_CASES)
def test_pack_bits_matches_reference(codec, name):
    bits = codec[f"{name}__bits"]
    packed = oc.pack_bits(bits)
    np.testing.assert_array_equal(packed.metadata, codec[f"{name}__metadata"])
    import hashlib
    assert hashlib.sha256(packed.payload.tobytes()).hexdigest() == str(codec[f"{name}__payload_sha256"])
    assert packed.storage_bytes == int(codec[f"{name}__storage_bytes"])
    assert packed.source_sha256 == str(codec[f"{name}__source_sha256"])
    np.testing.assert_array_equal(oc.unpack_bits(packed), bits)
    np.testing.assert_array_equal(oc.decode_bf16(packed.payload.tobytes(), packed.metadata, packed.n, packed.k), bits)


def test_exact_storage_and_raw_metadata(codec):
    # tests/test_compressed_bf16.py:29-34: a coded block is 100 bytes, a raw one 132.
    assert int(codec["coded_only__storage_bytes"]) == 100
    assert int(codec["raw_only__storage_bytes"]) == 132
    assert int(codec["raw_only__metadata"][0]) == 0x80000000


def test_literal_pair_and_raw_block_known_answers():
    # tests/test_bf16_reference.py:15-28 (literal bytes read from the reference test).
    payload = bytes([0x80, 0x00, 0x20]) + bytes(93)
    got = oc.decode_bf16(payload, np.array([127 << 23], dtype=np.uint32), 1, 2)
    np.testing.assert_array_equal(got, np.array([[0xBF80, 0x4080]], dtype=np.uint16))
    original = [0x0000, 0x8000, 0x0001, 0x7FC1, 0xFF80, 0xFFFF, 0x3F80, 0x4000] * 8
    payload = bytes(96) + struct.pack("<64H", *original)
    got = oc.decode_bf16(payload, np.array([127 << 23, 0x80000003], dtype=np.uint32), 1, 128)
    np.testing.assert_array_equal(got[0, :64], np.full(64, 0x3F80, dtype=np.uint16))
    np.testing.assert_array_equal(got[0, 64:], np.array(original, dtype=np.uint16))


@pytest.mark.parametrize("payload,metadata", [
    (bytes(95), [127 << 23]),                       # truncated payload
    (bytes(96), [(127 << 23) | 1]),                  # non-canonical offset
    (bytes([0, 1, 0]) + bytes(93), [255 << 23]),     # exponent overflow
])
def test_corruption_is_rejected(payload, metadata):
    with pytest.raises(ValueError):
        oc.decode_bf16(payload, np.array(metadata, dtype=np.uint32), 1, 64)


def test_corrupted_metadata_and_bad_inputs_fail():
    packed = oc.pack_bits(np.full((1, 64), 0x3F80, dtype=np.uint16))
    bad = oc.Packed(packed.payload, packed.metadata | np.uint32(1), 1, 64, packed.source_sha256)
    with pytest.raises(ValueError):
        oc.unpack_bits(bad)
    for value in (np.ones((1, 64), dtype=np.float32), np.empty((0, 64), dtype=np.uint16), np.ones(64, dtype=np.uint16)):
        with pytest.raises(ValueError):
            oc.pack_bits(value)


def test_round_bf16_bits_matches_reference(codec):
    np.testing.assert_array_equal(ob.round_bf16_bits(codec["round__values"]), codec["round__bits"])


def test_rounding_known_answers():
    # tests/test_projection_accuracy.py:24-37.
    mid = 1.00390625
    np.testing.assert_array_equal(ob.round_bf16_bits(np.array([mid - 1e-12, mid, mid + 1e-12])), [0x3F80, 0x3F80, 0x3F81])
    np.testing.assert_array_equal(ob.round_bf16_bits(np.array([0.0, -0.0, 2.0 ** -133, -(2.0 ** -133), 2.0 ** 128])),
                                  [0, 0x8000, 1, 0x8001, 0x7F80])
    np.testing.assert_array_equal(ob.round_bf16_bits(np.array([-(2.0 ** -135), -(2.0 ** -134), 2.0 ** -135])),
                                  [0x8000, 0x8000, 0])


def test_check_outputs_matches_reference(codec):
    ref = codec["check__ref"]
    expected = codec["check__results"]
    for (dtype, delta), (passed, violations) in zip((("fp32", 0.0), ("fp32", 2e-4), ("bf16", 0.0)), expected):
        actual = ref + delta
        if dtype == "bf16":
            actual = ob.bf16_values(ob.round_bf16_bits(actual))
        report = ob.check_outputs(ref, actual, output_dtype=dtype)
        assert (report["passed"], report["violations"]) == (bool(passed), int(violations))


def test_check_outputs_known_answers():
    # tests/test_projection_accuracy.py:39-57.
    assert ob.check_outputs(np.array([1.0]), np.array([1.00001], np.float32), output_dtype="fp32")["passed"]
    assert not ob.check_outputs(np.array([1.0]), np.array([1.01], np.float32), output_dtype="fp32")["passed"]
    report = ob.check_outputs(np.array([1.00390625, 1.00390625]), np.array([1.0, 1.0078125]), output_dtype="bf16")
    assert report["passed"] and report["exact_rounding_fraction"] == 0.5 and report["within_one_ulp_fraction"] == 1.0
    assert not ob.check_outputs(np.array([1.0]), np.array([1.0078125]), output_dtype="bf16")["passed"]
    report = ob.check_outputs(np.array([0.0]), np.array([2.0 ** -20]), output_dtype="bf16")
    assert report["passed"] and report["within_one_ulp_fraction"] == 0.0
    assert not ob.check_outputs(np.array([1.0]), np.array([float("nan")]), output_dtype="fp32")["passed"]
    assert not ob.check_outputs(np.array([float("inf")]), np.array([float("inf")]), output_dtype="bf16")["passed"]
    with pytest.raises(ValueError):
        ob.check_outputs(np.array([1.0]), np.array([1.0001]), output_dtype="bf16")


def test_int8_quantizer_matches_reference(quant):
    codes, scales = oq.int8_quantize_g64(quant["w"], semantics="cpu")
    np.testing.assert_array_equal(codes, quant["int8__codes"])
    np.testing.assert_array_equal(scales.view(np.uint32), quant["int8__scales"].view(np.uint32))
    deq = oq.int8_dequantize(codes, scales)
    np.testing.assert_array_equal(deq.view(np.uint32), quant["int8__dequant"].view(np.uint32))
    np.testing.assert_array_equal(quant["zero__int8_scales"], np.ones((5, 1), dtype=np.float32))


@pytest.mark.parametrize("case", ["fp4", "ties"])
def test_fp4_quantizer_matches_reference(quant, case):
    w = quant["w"] if case == "fp4" else quant["ties"]
    packed, scales, glob = oq.fp4_quantize_e4m3(w, semantics="cpu")
    np.testing.assert_array_equal(packed, quant[f"{case}__packed"])
    np.testing.assert_array_equal(scales, quant[f"{case}__scales"])
    assert np.float32(glob).view(np.uint32) == np.float32(quant[f"{case}__global"]).view(np.uint32)
    if case == "fp4":
        deq = oq.fp4_dequantize_e4m3(packed, scales, glob)
        np.testing.assert_array_equal(deq.view(np.uint32), quant["fp4__dequant"].view(np.uint32))


def test_fp4_zero_tensor(quant):
    packed, scales, glob = oq.fp4_quantize_e4m3(np.zeros((5, 16), dtype=np.float32), semantics="cpu")
    np.testing.assert_array_equal(packed, quant["zero__fp4_packed"])
    assert float(glob) == float(quant["zero__fp4_global"]) == 1.0
    assert not oq.fp4_dequantize_e4m3(packed, scales, glob).any()


def test_e2m1_table_known_answer():
    # bench_fp4.py:21-31: codes 0..15 decode to the E2M1 table; E4M3 byte 56 is 1.0.
    table = [0, .5, 1, 1.5, 2, 3, 4, 6, -0., -.5, -1, -1.5, -2, -3, -4, -6]
    np.testing.assert_array_equal(oq.e2m1_to_f32(np.arange(16, dtype=np.uint8)), np.array(table, np.float32))
    assert oq.e4m3_to_f32(np.array([56], np.uint8))[0] == 1.0
    codes = np.arange(16, dtype=np.uint8).reshape(1, 16)
    packed = oq.pack_nibbles(codes)
    deq = oq.fp4_dequantize_e4m3(packed, np.array([[56]], np.uint8), np.float32(1.0))
    np.testing.assert_array_equal(deq[0], np.array(table, np.float32))
    assert np.signbit(deq[0, 8])


def test_e4m3_round_trip_and_rounding():
    codes = np.arange(256, dtype=np.uint8)
    values = oq.e4m3_to_f32(codes)
    finite = ~np.isnan(values)
    np.testing.assert_array_equal(oq.f32_to_e4m3(values[finite]), codes[finite])
    # Ties to even and the NaN boundary of torch's float8_e4m3fn conversion.
    np.testing.assert_array_equal(oq.f32_to_e4m3(np.array([448, 464, 465, 480, 1.0625, 1.1875], np.float32)),
                                  [0x7E, 0x7E, 0x7F, 0x7F, 0x38, 0x3A])


def test_baseline_variants_round_trip():
    from oracle.gemv import normal_f32
    w = normal_f32(3, (16, 128), 0.02)
    codes, scales = oq.int8_quantize_row(w)
    assert codes.dtype == np.int8 and scales.shape == (16,)
    np.testing.assert_allclose(oq.int8_dequantize(codes, scales), w, atol=float(scales.max()) / 2 + 1e-9)
    packed, s16 = oq.fp4_quantize_f16(w)
    assert packed.shape == (16, 64) and s16.dtype == np.float16
    deq = oq.fp4_dequantize_f16(packed, s16)
    assert np.abs(deq - w).max() <= np.abs(w).max() / 6 * 1.01


def test_cuda_scalar_division_semantics():
    """torch on CUDA divides by a Python number as a multiply by the FP32
    reciprocal; the oracle's "cuda" semantics differ from "cpu" by one ulp at most."""
    a = np.float32(np.random.default_rng(0).random(10000) * 3).astype(np.float32)
    cuda, cpu = oq.scalar_divide(a, 127, "cuda"), oq.scalar_divide(a, 127, "cpu")
    diff = np.abs(cuda.view(np.int32).astype(np.int64) - cpu.view(np.int32).astype(np.int64))
    assert diff.max() == 1 and 0 < np.count_nonzero(diff) < 0.2 * a.size
    w = np.random.default_rng(1).standard_normal((64, 256)).astype(np.float32)
    c1, s1 = oq.int8_quantize_g64(w, "cuda")
    c2, s2 = oq.int8_quantize_g64(w, "cpu")
    assert np.abs(s1.view(np.int32).astype(np.int64) - s2.view(np.int32)).max() <= 1


LOSSLESS_CASES = ("mixed", "normal", "wide")


@pytest.fixture(scope="module")
def lossless():
    return np.load(GOLDEN / "reference_lossless.npz")


@pytest.mark.parametrize("name", LOSSLESS_CASES)
def test_lossless_f32_v1_pack_matches_reference(lossless, name):
    """oracle.lossless.lf32_pack produces the reference packer's bytes
    (lossless_weights.pack_weights), and unpacking restores every FP32 bit."""
    from oracle import lossless as ol

    w = lossless[f"{name}__w"]
    mantissa, exponents, metadata = ol.lf32_pack(w)
    np.testing.assert_array_equal(mantissa, lossless[f"{name}__lf32_mantissa"])
    np.testing.assert_array_equal(exponents, lossless[f"{name}__lf32_exponents"])
    np.testing.assert_array_equal(metadata, lossless[f"{name}__lf32_metadata"])
    back = ol.lf32_unpack(mantissa, exponents, metadata)
    np.testing.assert_array_equal(back.view(np.uint32), w.view(np.uint32))


@pytest.mark.parametrize("name", LOSSLESS_CASES)
def test_fp28_pack_matches_reference(lossless, name):
    """oracle.lossless.fp28_pack produces packed_fp32.pack_weights' words, and
    unpacking restores every FP32 bit (NaN payloads, -0, infinities, subnormals)."""
    from oracle import lossless as ol

    w = lossless[f"{name}__w"]
    payload, metadata = ol.fp28_pack(w)
    np.testing.assert_array_equal(payload, lossless[f"{name}__fp28_payload"])
    np.testing.assert_array_equal(metadata, lossless[f"{name}__fp28_metadata"])
    back = ol.fp28_unpack(payload, metadata)
    np.testing.assert_array_equal(back.view(np.uint32), w.view(np.uint32))


def test_lossless_block_kinds_present(lossless):
    """The fixtures hold both narrow (delta) and wide blocks of both formats."""
    for name in LOSSLESS_CASES:
        for fmt in ("lf32", "fp28"):
            wide = lossless[f"{name}__{fmt}_metadata"].view(np.uint32) & 1
            if name == "mixed":
                assert wide.any() and not wide.all()
