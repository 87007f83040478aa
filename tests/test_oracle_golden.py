"""Pin the CPU oracle against the reference's own golden vectors and known answers.

The vectors come from tinygrad-dx12's ``test/backend/test_packed.py`` and
``test/backend/test_linalg.py`` (transcribed into ``tests/golden/packed_golden.json``).
"""

import math

import numpy as np
import pytest

from oracle import packed_ref as ref


def _payload_bytes(codes, bits):
    """test_packed.py:81-84, an independent big-integer encoder."""
    number = sum(int(code) << (i * bits) for i, code in enumerate(codes))
    return np.frombuffer(number.to_bytes((len(codes) * bits + 7) // 8, "little"), np.uint8)


@pytest.mark.parametrize("fmt", ["fp4_e2m1", "fp6_e2m3", "fp6_e3m2"])
def test_complete_ocp_payloads(golden, fmt):
    """test_packed.py:87-101: every finite payload and both signed zeros."""
    positive = golden["golden_payload_tables"][fmt]
    bits = 4 if fmt.startswith("fp4") else 6
    expected = [*positive, *[-x for x in positive]]
    data = _payload_bytes(list(range(1 << bits)), bits)
    actual = ref.dequant(data, fmt, (1 << bits,)).tolist()
    assert actual == expected
    assert math.copysign(1, actual[len(positive)]) == -1
    # the vectorised encoder agrees with the big-integer encoder
    assert np.array_equal(ref.pack_codes(np.arange(1 << bits), bits), data)


@pytest.mark.parametrize("fmt", ["int4", "uint4"])
def test_integer_nibbles(golden, fmt):
    kat = golden["known_answers"]["integer_nibbles"]
    data = _payload_bytes(kat["codes"], 4)
    assert ref.dequant(data, fmt, (16,)).tolist() == kat[fmt]
    assert ref.dequant(data, fmt, (16,)).dtype == np.int32


def test_scales_stay_with_k_blocks(golden):
    kat = golden["known_answers"]["scales_stay_with_k_blocks"]
    spec = ref.PackedSpec(np.array(kat["data"], np.uint8), kat["format"], tuple(kat["shape"]),
                          np.array(kat["scales"], np.float32), kat["block_size"])
    out = ref.matmul_ref(spec, np.array(kat["rhs"], np.float32))
    assert out.tolist() == kat["expected"]


def test_matrix_intermediate_preserves_activations(golden):
    kat = golden["known_answers"]["matrix_intermediate"]
    w = ref.PackedSpec(np.array([0], np.uint8), "fp6_e2m3", (1, 1))
    assert ref.matrix_intermediate(np.array([[1.125]], np.float32), w) == kat["fp6_e2m3_unscaled_with_float32"]
    assert ref.matrix_intermediate(w, w) == kat["fp6_e2m3_unscaled_pair"]
    enc = ref.dequant(w.data, "fp6_e2m3", (1, 1), dtype="fp8e5m2")
    assert enc.view(ref.FP8E5M2).astype(np.float32).tolist() == kat["unpack_fp8e5m2_code0"]


def test_double_block_scales(golden):
    kat = golden["known_answers"]["double_block_scales"]
    spec = ref.PackedSpec(np.array(kat["data"], np.uint8), kat["format"], tuple(kat["shape"]),
                          np.array(kat["scales"], np.float64), kat["block_size"])
    dec = ref.dequant(spec.data, spec.format, spec.shape, spec.scales, spec.block_size)
    assert dec.dtype == np.float64 and dec.tolist() == kat["unpack"]
    assert ref.matrix_intermediate(spec, spec) == kat["intermediate"]
    assert ref.matmul_ref(spec, np.array(kat["rhs"], np.float32)).tolist() == kat["matmul"]


def _large_expected(kat, fmt, kind, scaled, golden):
    bits = 4 if fmt == "uint4" else 6
    boundary = 2**31 // bits if kind == "bit" else 2**31
    pattern = kat["pattern"]
    lo, hi = kat["window"]
    expected = []
    for index in range(boundary + lo, boundary + hi):
        byte, shift = divmod(index * bits, 8)
        payload = ((pattern[byte % 17] | pattern[(byte + 1) % 17] << 8) >> shift) & ((1 << bits) - 1)
        value = payload if fmt == "uint4" else golden["golden_payload_tables"][fmt][payload & 31] * (-1 if payload & 32 else 1)
        expected.append(value * (kat["scale_cycle"][index // 32 % 3] if scaled else 1))
    return boundary, expected


@pytest.mark.parametrize("case", range(7))
def test_large_packed_bit_positions(golden, case):
    """test_packed.py:147-174: windows straddling 2^31 bits / elements (oracle decodes a window)."""
    kat = golden["known_answers"]["large_bit_positions"]
    fmt, kind, scaled = kat["cases"][case]
    boundary, expected = _large_expected(kat, fmt, kind, scaled, golden)
    bits = 4 if fmt == "uint4" else 6
    lo, hi = kat["window"]
    start, stop = boundary + lo, boundary + hi
    # only the bytes around the window are materialised; they follow the 17-byte pattern
    first_byte = (start * bits // 8) // 12 * 12  # whole words for both 4- and 6-bit formats
    last_byte = (stop * bits + 7) // 8 + 12
    local = np.array([kat["pattern"][b % 17] for b in range(first_byte, last_byte)], np.uint8)
    elem0 = first_byte * 8 // bits
    p = ref.payloads(local, fmt, start - elem0, stop - elem0)
    vals = ref.decode_values(p, fmt).astype(np.float64)
    if scaled:
        vals = vals * np.array([kat["scale_cycle"][i // 32 % 3] for i in range(start, stop)])
    assert vals.tolist() == expected


@pytest.mark.parametrize("i", range(3))
def test_packed_integer_matmul_precision(golden, i):
    kat = golden["known_answers"]["packed_integer_matmul_precision"][i]
    spec = ref.PackedSpec(np.array([kat["byte"]], np.uint8), kat["format"], (1, 2))
    x = np.array([[v] for v in kat["values"]], ref.np_dtype(kat["dtype"]))
    out = ref.matmul_ref(spec, x)
    assert out.dtype == ref.np_dtype(kat["dtype"]) and out.tolist() == [[kat["expected"]]]


@pytest.mark.parametrize("i", range(2))
def test_accumulator_width(golden, i):
    kat = golden["known_answers"]["accumulator_width"][i]
    a = np.array([kat["values"]], ref.np_dtype(kat["dtype"]))
    out = ref.matmul_ref(a, a.T.copy())
    assert ref.dtype_name(out.dtype) == kat["acc"] and out.tolist() == [[kat["expected"]]]


def test_readme_uint4(golden):
    kat = golden["known_answers"]["readme_uint4"]
    spec = ref.PackedSpec(np.array(kat["data"], np.uint8), kat["format"], tuple(kat["shape"]))
    assert ref.dequant(spec.data, spec.format, spec.shape).tolist() == kat["unpack"]
    assert ref.matmul_ref(spec, np.array(kat["column"], np.float32)).tolist() == kat["matmul"]


def test_benchmark_code_maps(golden):
    """scripts/benchmark_dtypes.py:70-74: the {-1,0,1} payload maps decode to -1, 0, 1."""
    for fmt, mapping in golden["known_answers"]["benchmark_code_maps"].items():
        bits = ref.FORMATS[fmt][0]
        codes = [mapping[k] for k in ("-1", "0", "1")]
        data = ref.pack_codes(np.array(codes), bits)
        assert ref.dequant(data, fmt, (3,)).tolist() == [-1, 0, 1]


def test_fp8_shortcut_matches_ml_dtypes():
    """dx12.py:78-92: the exact FP8 encodings equal a numeric round trip of every payload."""
    for fmt, targets in ref.FP8_CANDIDATES.items():
        bits = ref.FORMATS[fmt][0]
        data = ref.pack_codes(np.arange(1 << bits), bits)
        vals = ref.dequant(data, fmt, (1 << bits,))
        for t in targets:
            enc = ref.dequant(data, fmt, (1 << bits,), dtype=t)
            dec = enc.view(ref.np_dtype(t)).astype(np.float32)
            assert np.array_equal(dec, vals) and np.array_equal(np.signbit(dec), np.signbit(vals))


def test_dtype_lattice():
    assert ref.least_upper_dtype("float16", "bfloat16") == "float32"
    assert ref.least_upper_dtype("int64", "float16") == "float16"
    assert ref.least_upper_dtype("float32", "float64") == "float64"
    assert ref.accumulator("float16", "float16") == "float32"
    assert ref.accumulator("uint8", "uint8") == "uint32"
    assert ref.accumulator("int8", "int8") == "int32"
    assert ref.accumulator("int64", "int64") == "int64"


def test_pack_roundtrip_random():
    rng = np.random.default_rng(0)
    for fmt in ref.FORMATS:
        bits = ref.FORMATS[fmt][0]
        codes = ref.random_codes(rng, fmt, 1001)
        data = ref.pack_codes(codes, bits)
        assert data.size == (1001 * bits + 7) // 8
        assert np.array_equal(ref.payloads(data, fmt, 0, 1001), codes)
        assert np.array_equal(ref.payloads(data, fmt, 17, 530), codes[17:530])
