"""Device decode (b200_dequant) against the oracle and the reference's golden vectors."""

import ctypes
import math

import numpy as np
import pytest
import torch

from oracle import packed_ref as ref
from tests.helpers import bits_equal, to_device, to_numpy, TORCH_OF

pytestmark = pytest.mark.gpu
DEV = "cuda:0"


def _payload_bytes(codes, bits):
    number = sum(int(c) << (i * bits) for i, c in enumerate(codes))
    return list(number.to_bytes((len(codes) * bits + 7) // 8, "little"))


@pytest.mark.parametrize("fmt", ["fp4_e2m1", "fp6_e2m3", "fp6_e3m2"])
def test_complete_ocp_payloads_gpu(golden, fmt):
    import tinygrad_dx12_b200 as tg

    positive = golden["golden_payload_tables"][fmt]
    bits = 4 if fmt.startswith("fp4") else 6
    data = torch.tensor(_payload_bytes(list(range(1 << bits)), bits), dtype=torch.uint8, device=DEV)
    actual = tg.PackedTensor(data, fmt, (1 << bits,)).unpack().cpu().tolist()
    assert actual == [*positive, *[-x for x in positive]]
    assert math.copysign(1, actual[len(positive)]) == -1


@pytest.mark.parametrize("fmt", ["int4", "uint4"])
def test_integer_nibbles_gpu(golden, fmt):
    import tinygrad_dx12_b200 as tg

    kat = golden["known_answers"]["integer_nibbles"]
    data = torch.tensor(_payload_bytes(kat["codes"], 4), dtype=torch.uint8, device=DEV)
    out = tg.PackedTensor(data, fmt, (16,)).unpack()
    assert out.dtype == torch.int32 and out.cpu().tolist() == kat[fmt]


@pytest.mark.parametrize("fmt", list(ref.FORMATS))
@pytest.mark.parametrize("scale", [None, "float16", "bfloat16", "float32", "float64", "e8m0"])
@pytest.mark.parametrize("shape,bs", [((64, 96), 32), ((7, 33), 5), ((3, 130), 128), ((1, 1), 1)])
def test_dequant_bit_exact(fmt, scale, shape, bs):
    rng = np.random.default_rng(hash((fmt, scale, shape)) & 0xFFFF)
    rows, cols = shape
    spec = ref.make_packed(rng, fmt, rows, cols, bs, "e8m0" if scale == "e8m0" else ("f16u" if scale else None))
    if scale not in (None, "e8m0"):
        spec = ref.PackedSpec(spec.data, fmt, shape, spec.scales.astype(ref.np_dtype(scale)), bs)
    w = to_device(spec, DEV, scale)
    got = to_numpy(w.unpack())
    exp = ref.dequant(spec.data, fmt, shape, spec.scales, bs, None, spec.scale_dtype)
    assert got.dtype == exp.dtype
    assert bits_equal(got, exp)


@pytest.mark.parametrize("fmt", list(ref.FORMATS))
@pytest.mark.parametrize("dtype", ["float16", "bfloat16", "float32", "float64", "int32"])
def test_dequant_explicit_dtype(fmt, dtype):
    rng = np.random.default_rng(3)
    spec = ref.make_packed(rng, fmt, 16, 64, 32, "f16u")
    w = to_device(spec, DEV)
    tdt = {"int32": torch.int32, **TORCH_OF}[dtype]
    got = to_numpy(w.unpack(tdt))
    exp = ref.dequant(spec.data, fmt, (16, 64), spec.scales, 32, dtype)
    assert bits_equal(got, exp)
    # unscaled too
    w0 = to_device(ref.PackedSpec(spec.data, fmt, (16, 64)), DEV)
    assert bits_equal(to_numpy(w0.unpack(tdt)), ref.dequant(spec.data, fmt, (16, 64), dtype=dtype))


@pytest.mark.parametrize("fmt,target", [(f, t) for f, ts in ref.FP8_CANDIDATES.items() for t in ts])
def test_fp8_exact_encoding(fmt, target):
    import tinygrad_dx12_b200 as tg

    bits = ref.FORMATS[fmt][0]
    data_np = ref.pack_codes(np.arange(1 << bits), bits)
    w = tg.PackedTensor(torch.from_numpy(data_np).to(DEV), fmt, (1 << bits,))
    tdt = torch.float8_e4m3fn if target == "fp8e4m3" else torch.float8_e5m2
    got = w.unpack(tdt)
    assert got.dtype == tdt
    assert np.array_equal(got.view(torch.uint8).cpu().numpy(), ref.dequant(data_np, fmt, (1 << bits,), dtype=target))


def test_scales_stay_with_k_blocks_gpu(golden):
    import tinygrad_dx12_b200 as tg

    kat = golden["known_answers"]["scales_stay_with_k_blocks"]
    w = tg.PackedTensor(torch.tensor(kat["data"], dtype=torch.uint8, device=DEV), kat["format"], tuple(kat["shape"]),
                        torch.tensor(kat["scales"], device=DEV), kat["block_size"])
    assert tg.matmul(w, torch.tensor(kat["rhs"], device=DEV)).cpu().tolist() == kat["expected"]
    from tinygrad_dx12_b200.packed import matmul as decomp_matmul

    assert decomp_matmul(w, torch.tensor(kat["rhs"], device=DEV)).cpu().tolist() == kat["expected"]


def test_double_block_scales_gpu(golden):
    import tinygrad_dx12_b200 as tg

    kat = golden["known_answers"]["double_block_scales"]
    w = tg.PackedTensor(torch.tensor(kat["data"], dtype=torch.uint8, device=DEV), kat["format"], tuple(kat["shape"]),
                        torch.tensor(kat["scales"], dtype=torch.float64, device=DEV), kat["block_size"])
    dec = w.unpack()
    assert dec.dtype == torch.float64 and dec.cpu().tolist() == kat["unpack"]
    assert tg.matrix_intermediate(w, w) == torch.float64
    assert tg.matmul(w, torch.tensor(kat["rhs"], device=DEV)).cpu().tolist() == kat["matmul"]


def test_readme_uint4_gpu(golden):
    import tinygrad_dx12_b200 as tg

    kat = golden["known_answers"]["readme_uint4"]
    w = tg.PackedTensor(torch.tensor(kat["data"], dtype=torch.uint8, device=DEV), "uint4", (2, 2))
    assert w.unpack().cpu().tolist() == kat["unpack"]
    assert tg.matmul(w, torch.tensor(kat["column"], device=DEV)).cpu().tolist() == kat["matmul"]
    assert tg.matvec(w, torch.tensor(kat["vector"], device=DEV)).cpu().tolist() == kat["matvec"]


@pytest.mark.parametrize("i", range(3))
def test_packed_integer_matmul_precision_gpu(golden, i):
    import tinygrad_dx12_b200 as tg

    kat = golden["known_answers"]["packed_integer_matmul_precision"][i]
    dt = {"int32": torch.int32, "int64": torch.int64, "uint64": torch.uint64}[kat["dtype"]]
    w = tg.PackedTensor(torch.tensor([kat["byte"]], dtype=torch.uint8, device=DEV), kat["format"], (1, 2))
    x = torch.tensor([[v] for v in kat["values"]], dtype=dt, device=DEV)
    out = w.matmul(x)
    assert out.dtype == dt
    assert int(out.cpu().to(torch.int64 if dt != torch.uint64 else torch.uint64)[0, 0]) == kat["expected"]


@pytest.mark.parametrize("i", range(2))
@pytest.mark.parametrize("scope", ["auto", "tiled"])
def test_accumulator_width_gpu(golden, i, scope):
    import tinygrad_dx12_b200 as tg

    kat = golden["known_answers"]["accumulator_width"][i]
    dt = {"int8": torch.int8, "uint8": torch.uint8}[kat["dtype"]]
    a = torch.tensor([kat["values"]], dtype=dt, device=DEV)
    out = tg.matmul(a, a.t().contiguous(), scope=scope)
    assert out.dtype == {"int32": torch.int32, "uint32": torch.uint32}[kat["acc"]]
    assert int(out.cpu().to(torch.int64)[0, 0]) == kat["expected"]


@pytest.mark.parametrize("case", range(7))
def test_large_packed_bit_positions_gpu(golden, case):
    """test_packed.py:147-174: decode windows across 2^31 bits / elements from a >2^31-element
    stream (1.6 GB of storage on the device), through the element-window C-ABI call."""
    from tinygrad_dx12_b200 import _lib
    import tinygrad_dx12_b200 as tg

    kat = golden["known_answers"]["large_bit_positions"]
    fmt, kind, scaled = kat["cases"][case]
    bits = 4 if fmt == "uint4" else 6
    boundary = 2**31 // bits if kind == "bit" else 2**31
    count = boundary + 32
    nbytes = (count * bits + 7) // 8
    pattern = torch.tensor(kat["pattern"], dtype=torch.uint8, device=DEV)
    storage = pattern.repeat((nbytes + 16) // 17)[:nbytes].contiguous()
    scales = None
    if scaled:
        nsc = (count + 31) // 32
        scales = torch.tensor(kat["scale_cycle"], dtype=torch.float32, device=DEV).repeat((nsc + 2) // 3)[:nsc].contiguous()
    w = tg.PackedTensor(storage, fmt, (count,), scales)
    lo, hi = kat["window"]
    out = torch.empty(hi - lo, dtype=torch.float32 if (scaled or fmt != "uint4") else torch.int32, device=DEV)
    d = w.desc()
    odt = _lib.DT["float32" if out.dtype == torch.float32 else "int32"]
    _lib.call("b200_dequant", ctypes.byref(d), boundary + lo, hi - lo, out.data_ptr(), odt,
              torch.cuda.current_stream().cuda_stream)
    expected = []
    for index in range(boundary + lo, boundary + hi):
        byte, shift = divmod(index * bits, 8)
        p = ((kat["pattern"][byte % 17] | kat["pattern"][(byte + 1) % 17] << 8) >> shift) & ((1 << bits) - 1)
        value = p if fmt == "uint4" else golden["golden_payload_tables"][fmt][p & 31] * (-1 if p & 32 else 1)
        expected.append(value * (kat["scale_cycle"][index // 32 % 3] if scaled else 1))
    assert out.cpu().tolist() == expected
    del storage, scales
    torch.cuda.empty_cache()
