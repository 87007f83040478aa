"""The oracle's C restatement (timed CPU baseline) agrees with the numpy restatement:
bit-exact decode and float32 matmul within the parity tolerances."""

import ctypes

import numpy as np
import pytest

from oracle import build as obuild
from oracle import packed_ref as ref
from tests.helpers import errors

FMT = {"int4": 0, "uint4": 1, "fp4_e2m1": 2, "fp6_e2m3": 3, "fp6_e3m2": 4}


@pytest.fixture(scope="module")
def clib():
    return obuild.load()


def _ptr(a):
    return a.ctypes.data_as(ctypes.c_void_p) if a is not None else None


@pytest.mark.parametrize("fmt", list(FMT))
@pytest.mark.parametrize("kind", [None, "f16u", "e8m0"])
def test_c_dequant_bit_exact(clib, fmt, kind):
    spec = ref.make_packed(np.random.default_rng(1), fmt, 37, 96, 32, kind)
    out = np.empty((37, 96), np.float32)
    sdt, sc = 0, None
    if kind == "f16u":
        sdt, sc = 12, spec.scales
    elif kind == "e8m0":
        sdt, sc = 16, ref.e8m0_bytes(spec.scales)
    clib.oref_dequant_f32(_ptr(spec.data), spec.data.size, FMT[fmt], 37, 96, _ptr(sc), sdt, 32, _ptr(out))
    exp = ref.dequant(spec.data, fmt, (37, 96), spec.scales, 32, "float32", spec.scale_dtype)
    assert np.array_equal(out.view(np.uint32), exp.view(np.uint32))


def test_c_golden_tables(clib, golden):
    for fmt in ("fp4_e2m1", "fp6_e2m3", "fp6_e3m2"):
        bits = ref.FORMATS[fmt][0]
        data = ref.pack_codes(np.arange(1 << bits), bits)
        out = np.empty(1 << bits, np.float32)
        clib.oref_dequant_f32(_ptr(data), data.size, FMT[fmt], 1, 1 << bits, None, 0, 32, _ptr(out))
        pos = golden["golden_payload_tables"][fmt]
        assert out.tolist() == [*pos, *[-x for x in pos]]
        assert np.signbit(out[len(pos)])


@pytest.mark.parametrize("fmt,kind,xdt", [("int4", "f16u", 12), ("fp4_e2m1", "e8m0", 13), ("fp6_e3m2", "f16row", 12)])
def test_c_linear_matches_numpy(clib, fmt, kind, xdt):
    rng = np.random.default_rng(2)
    spec = ref.make_packed(rng, fmt, 64, 256, 32, kind)
    m = 3
    x = rng.standard_normal((m, 256)).astype(np.float32)
    xs = x.astype(np.float16) if xdt == 12 else x.astype(ref.BF16)
    sc = ref.e8m0_bytes(spec.scales) if kind == "e8m0" else spec.scales
    sdt = 16 if kind == "e8m0" else 12
    y = np.empty((m, 64), np.float32)
    assert clib.oref_linear(_ptr(spec.data), spec.data.size, FMT[fmt], 64, 256, _ptr(sc), sdt, spec.block_size,
                            _ptr(np.ascontiguousarray(xs)), xdt, m, _ptr(y), 2) == 0
    r = ref.packed_linear_ref(spec, xs.astype(np.float32))
    elem, fro = errors(y, r)
    assert elem <= 1e-4 and fro <= 1e-6
