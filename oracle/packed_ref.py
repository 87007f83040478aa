"""CPU restatement (numpy) of tinygrad-dx12's packed low-bit decode and matmul.

TEST INFRASTRUCTURE ONLY. This module is the checker: only ``tests/``,
``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline / reference legs may
import it. The product package ``tinygrad_dx12_b200`` never imports it and has no
CPU fallback.

Reference files restated here (paths inside the tinygrad-dx12 project):

* ``src/tinygrad_dx12/codegen/decomp/dx12.py:10-11``  FORMATS / FP8_CANDIDATES
* ``src/tinygrad_dx12/codegen/decomp/dx12.py:32-47``  PackedTensor validation
* ``src/tinygrad_dx12/codegen/decomp/dx12.py:49-106`` unpack: word build, payload,
  INT4/UINT4 value, FP4/FP6 value, exact-FP8 shortcut, block scales
* ``src/tinygrad_dx12/codegen/decomp/dx12.py:115-138`` matrix_intermediate
* ``src/tinygrad_dx12/renderer/linalg.py:33-35``      accumulator dtype
* ``src/tinygrad_dx12/codegen/linalg.py:169-174``     the CPU-device matmul branch

The reference's arithmetic runs inside tinygrad (git e4570fcb46b3725d3eb9243507a507b4ae19131b,
v0.14.0), which is not vendored. Its dtype promotion lattice (``least_upper_dtype``,
``sum_acc_dtype``) is restated below from tinygrad's published ``dtype.py``.

Parity pin: the decode is checked against every golden table and known-answer test in
the reference's ``test/backend/test_packed.py:8-174`` and ``test/backend/test_linalg.py``
(integer precision, accumulator width), transcribed into ``tests/golden/packed_golden.json``
by ``tests/golden/make_golden.py``. Large-shape matmul summation order is not pinned by
the reference (tinygrad's CPU reduction order); those cases use the tolerances stated in
the tests.
"""

from __future__ import annotations

import math
from dataclasses import dataclass

import numpy as np

try:  # bf16 / fp8 host types; present in this image (ml_dtypes 0.5)
    import ml_dtypes

    BF16 = np.dtype(ml_dtypes.bfloat16)
    FP8E4M3 = np.dtype(ml_dtypes.float8_e4m3fn)
    FP8E5M2 = np.dtype(ml_dtypes.float8_e5m2)
except ImportError:  # pragma: no cover - the image always has ml_dtypes
    ml_dtypes = None
    BF16 = FP8E4M3 = FP8E5M2 = None

# (total bits, exponent bits, mantissa bits, exponent bias) -- dx12.py:10
FORMATS = {
    "int4": (4, 0, 0, 0),
    "uint4": (4, 0, 0, 0),
    "fp4_e2m1": (4, 2, 1, 1),
    "fp6_e2m3": (6, 2, 3, 1),
    "fp6_e3m2": (6, 3, 2, 3),
}
# exact unscaled FP8 destinations per format -- dx12.py:11
FP8_CANDIDATES = {"fp4_e2m1": ("fp8e4m3", "fp8e5m2"), "fp6_e2m3": ("fp8e4m3",), "fp6_e3m2": ("fp8e4m3", "fp8e5m2")}

# ----------------------------------------------------------------------------------
# dtype names and tinygrad's promotion lattice (tinygrad dtype.py, restated)
# ----------------------------------------------------------------------------------
DTYPES = (
    "bool", "int8", "uint8", "int16", "uint16", "int32", "uint32", "int64", "uint64",
    "fp8e4m3", "fp8e5m2", "float16", "bfloat16", "float32", "float64",
)
_PRIORITY = {name: i for i, name in enumerate(DTYPES)}
_LATTICE = {
    "bool": ("int8", "uint8"),
    "int8": ("int16",),
    "int16": ("int32",),
    "int32": ("int64",),
    "int64": ("fp8e4m3", "fp8e5m2"),
    "uint8": ("int16", "uint16"),
    "uint16": ("int32", "uint32"),
    "uint32": ("int64", "uint64"),
    "uint64": ("fp8e4m3", "fp8e5m2"),
    "fp8e5m2": ("float16", "bfloat16"),
    "fp8e4m3": ("float16", "bfloat16"),
    "float16": ("float32",),
    "bfloat16": ("float32",),
    "float32": ("float64",),
    "float64": (),
}


def _upper(name: str) -> set[str]:
    out = {name}
    for nxt in _LATTICE[name]:
        out |= _upper(nxt)
    return out


def least_upper_dtype(*names: str) -> str:
    """Smallest common upper bound in tinygrad's lattice (ties broken by lattice priority)."""
    common = set.intersection(*(_upper(n) for n in names))
    return min(common, key=lambda n: _PRIORITY[n])


def is_float(name: str) -> bool:
    return name in ("fp8e4m3", "fp8e5m2", "float16", "bfloat16", "float32", "float64")


def is_unsigned(name: str) -> bool:
    return name in ("uint8", "uint16", "uint32", "uint64")


def sum_acc_dtype(name: str) -> str:
    """tinygrad's default reduction dtype: uint32/int32/float32 floors."""
    if is_unsigned(name):
        return least_upper_dtype(name, "uint32")
    if not is_float(name):  # ints and bool
        return least_upper_dtype(name, "int32")
    return least_upper_dtype(name, "float32")


def accumulator(a: str, b: str) -> str:
    """renderer/linalg.py:33-35 -- sum_acc_dtype(least_upper(a, b))."""
    return sum_acc_dtype(least_upper_dtype(a, b))


def np_dtype(name: str) -> np.dtype:
    return {
        "bool": np.dtype(np.bool_), "int8": np.dtype(np.int8), "uint8": np.dtype(np.uint8),
        "int16": np.dtype(np.int16), "uint16": np.dtype(np.uint16), "int32": np.dtype(np.int32),
        "uint32": np.dtype(np.uint32), "int64": np.dtype(np.int64), "uint64": np.dtype(np.uint64),
        "float16": np.dtype(np.float16), "float32": np.dtype(np.float32), "float64": np.dtype(np.float64),
        "bfloat16": BF16, "fp8e4m3": FP8E4M3, "fp8e5m2": FP8E5M2,
    }[name]


def dtype_name(dt: np.dtype) -> str:
    dt = np.dtype(dt)
    for name in DTYPES:
        if np_dtype(name) == dt:
            return name
    raise ValueError(f"unsupported dtype {dt}")


# ----------------------------------------------------------------------------------
# packing (test-side encoder, test_packed.py:81-84 and benchmark_dtypes.py:129-152)
# ----------------------------------------------------------------------------------
def pack_codes(codes: np.ndarray, bits: int) -> np.ndarray:
    """Pack payload codes least-significant bit first into a flat uint8 stream.

    Same rule as the reference test encoder ``payload_bytes`` (test_packed.py:81-84):
    code i occupies bits [i*bits, (i+1)*bits) of a little-endian integer.
    """
    flat = np.asarray(codes, dtype=np.uint8).reshape(-1)
    if bits == 4:
        n = flat.size
        if n % 2:
            flat = np.concatenate([flat, np.zeros(1, np.uint8)])
        pairs = flat.reshape(-1, 2)
        return (pairs[:, 0] & 0xF) | ((pairs[:, 1] & 0xF) << 4)
    shifts = np.arange(bits, dtype=np.uint8)
    return np.packbits(((flat[:, None] >> shifts) & 1).reshape(-1), bitorder="little")


# ----------------------------------------------------------------------------------
# decode (dx12.py:69-106)
# ----------------------------------------------------------------------------------
def payloads(data: np.ndarray, fmt: str, start: int = 0, stop: int | None = None) -> np.ndarray:
    """Payload codes of elements [start, stop): dx12.py:69-77.

    Words of ``bits//2`` bytes hold four elements LSB first; the stream is padded to a
    whole word. ``start``/``stop`` select a window without decoding the whole stream
    (the reference's large-offset test slices the same way, test_packed.py:164).
    """
    bits = FORMATS[fmt][0]
    group = bits // 2
    data = np.asarray(data, dtype=np.uint8).reshape(-1)
    total_words = -(-data.size // group)
    if stop is None:
        stop = total_words * 4
    w0, w1 = start // 4, -(-stop // 4)
    raw = data[w0 * group: w1 * group]
    raw = np.concatenate([raw, np.zeros((w1 - w0) * group - raw.size, np.uint8)]).reshape(-1, group).astype(np.uint32)
    word = raw[:, 0].copy()
    for i in range(1, group):
        word |= raw[:, i] << np.uint32(8 * i)
    shifts = np.arange(4, dtype=np.uint32) * np.uint32(bits)
    flat = ((word[:, None] >> shifts) & np.uint32((1 << bits) - 1)).reshape(-1)
    return flat[start - w0 * 4: stop - w0 * 4]


def decode_values(payload: np.ndarray, fmt: str) -> np.ndarray:
    """Payload -> numeric value: int32 for INT4/UINT4 (dx12.py:93-94), float32 otherwise (:95-100)."""
    bits, _, mantissa, bias = FORMATS[fmt]
    p = payload.astype(np.uint32)
    if fmt == "int4":
        return ((p.astype(np.int32) ^ 8) - 8).astype(np.int32)
    if fmt == "uint4":
        return p.astype(np.int32)
    fraction = (p & ((1 << mantissa) - 1)).astype(np.float32)
    exponent = ((p >> mantissa) & ((1 << (bits - mantissa - 1)) - 1)).astype(np.int32)
    significand = np.where(exponent == 0, fraction, fraction + np.float32(1 << mantissa)).astype(np.float32)
    power = np.exp2((np.where(exponent == 0, 1, exponent) - bias - mantissa).astype(np.float32)).astype(np.float32)
    value = (significand * power).astype(np.float32)
    return np.where((p & (1 << (bits - 1))) != 0, -value, value).astype(np.float32)


def fp8_encode(payload: np.ndarray, fmt: str, target: str) -> np.ndarray:
    """Exact FP4/FP6 -> FP8 bit encoding for unscaled payloads (dx12.py:78-92)."""
    bits, _, mantissa, bias = FORMATS[fmt]
    tm, tb = (3, 7) if target == "fp8e4m3" else (2, 15)
    p = payload.astype(np.uint32)
    fraction = p & ((1 << mantissa) - 1)
    exponent = (p >> mantissa) & ((1 << (bits - mantissa - 1)) - 1)
    subnormal = np.zeros_like(p)
    for high in range(mantissa):
        encoded = ((tb + 1 - bias - mantissa + high) << tm) | ((fraction << (tm - high)) & ((1 << tm) - 1))
        subnormal = np.where(fraction >= (1 << high), encoded, subnormal)
    normal = ((exponent + tb - bias) << tm) | (fraction << (tm - mantissa))
    encoded = ((p >> (bits - 1)) << 7) | np.where(exponent == 0, subnormal, normal)
    return encoded.astype(np.uint8)


def default_unpack_dtype(fmt: str, scale_dtype: str | None) -> str:
    """dx12.py:57-64."""
    if scale_dtype is not None:
        return least_upper_dtype("float32", scale_dtype)
    return "int32" if fmt in ("int4", "uint4") else "float32"


def cast(values: np.ndarray, name: str) -> np.ndarray:
    """Numeric conversion to ``name`` (round-to-nearest-even for floats, truncation to ints)."""
    return values.astype(np_dtype(name))


def dequant(data, fmt: str, shape, scales=None, block_size: int = 32, dtype: str | None = None,
            scale_dtype: str | None = None) -> np.ndarray:
    """PackedTensor.unpack restated (dx12.py:49-106).

    ``scales`` is a numpy array of shape ``shape[:-1] + (ceil(K/block_size),)``; its dtype
    is taken from the array unless ``scale_dtype`` names it (for bf16/e8m0 inputs passed as
    float32 values). Returns a numpy array of ``dtype`` (FP8 results as uint8 bit patterns).
    """
    shape = tuple(int(s) for s in shape)
    sdt = None if scales is None else (scale_dtype or dtype_name(np.asarray(scales).dtype))
    dtype = dtype or default_unpack_dtype(fmt, sdt)
    count = math.prod(shape)
    if count == 0:
        return np.zeros(shape, np.uint8 if dtype.startswith("fp8") else np_dtype(dtype))
    p = payloads(data, fmt, 0, count)
    if scales is None and dtype in FP8_CANDIDATES.get(fmt, ()):
        return fp8_encode(p, fmt, dtype).reshape(shape)
    value = decode_values(p, fmt).reshape(shape)
    if scales is not None:
        sdt_name = least_upper_dtype("float32", sdt, dtype)
        s = np.asarray(scales)
        if s.shape != shape[:-1] + (-(-shape[-1] // block_size),):
            raise ValueError("packed scales have incompatible shape")
        expanded = np.repeat(s.astype(np_dtype(sdt_name)), block_size, axis=-1)[..., : shape[-1]]
        value = value.astype(np_dtype(sdt_name)) * expanded
    if dtype.startswith("fp8"):
        return cast(value.astype(np.float32), dtype).view(np.uint8)
    return cast(value, dtype)


# ----------------------------------------------------------------------------------
# matrix_intermediate and the CPU matmul branch (dx12.py:115-138, linalg.py:169-174)
# ----------------------------------------------------------------------------------
@dataclass(frozen=True)
class PackedSpec:
    """Host-side description of a packed operand for the oracle (mirrors PackedTensor's fields)."""

    data: np.ndarray
    format: str
    shape: tuple
    scales: np.ndarray | None = None
    block_size: int = 32
    scale_dtype: str | None = None

    @property
    def sdt(self) -> str | None:
        if self.scales is None:
            return None
        return self.scale_dtype or dtype_name(self.scales.dtype)


def matrix_intermediate(a, b) -> str:
    """dx12.py:115-138 on dtype names; plain operands are numpy arrays (or dtype-name strings)."""
    def cands(op):
        if isinstance(op, PackedSpec):
            return set(FP8_CANDIDATES.get(op.format, ())) if op.scales is None else set()
        return {op if isinstance(op, str) else dtype_name(op.dtype)}

    common = cands(a) & cands(b)
    for dt in ("fp8e4m3", "fp8e5m2"):
        if dt in common:
            return dt

    def declared(op):
        if isinstance(op, PackedSpec):
            if op.scales is not None:
                return least_upper_dtype("float32", op.sdt)
            return {"int4": "int8", "uint4": "uint8"}.get(op.format, "float16")
        return op if isinstance(op, str) else dtype_name(op.dtype)

    return least_upper_dtype(declared(a), declared(b))


def matmul_ref(a, b, dtype: str | None = None) -> np.ndarray:
    """linalg.py:169-174: unpack packed operands to the intermediate, matmul with an
    accumulator of ``dtype or accumulator(lhs, rhs)``; output in that dtype.

    Float accumulation is done in float32 (float64 when the accumulator is float64) through
    numpy/BLAS; integer accumulation in int64/uint64 then cast, matching a wide reduction.
    """
    inter = matrix_intermediate(a, b)
    inter = accumulator(inter, inter)

    def operand(op):
        if isinstance(op, PackedSpec):
            v = dequant(op.data, op.format, op.shape, op.scales, op.block_size, inter, op.scale_dtype)
            return v, inter
        return op, dtype_name(op.dtype)

    (lhs, ld), (rhs, rd) = operand(a), operand(b)
    out = dtype or accumulator(ld, rd)
    if is_float(out):
        work = np.float64 if out == "float64" else np.float32
        res = lhs.astype(np.float32 if ld != "float64" else np.float64).astype(work) @ rhs.astype(work)
        return cast(res, out)
    work = np.uint64 if is_unsigned(out) else np.int64
    res = lhs.astype(work) @ rhs.astype(work)
    return res.astype(np_dtype(out))


def packed_linear_ref(spec: PackedSpec, x: np.ndarray, out_dtype: str | None = None) -> np.ndarray:
    """y[M,N] = x[M,K] @ dequant(W)[N,K]^T in float32 (the reference call ``matmul(W, x.T).T``,
    linalg.py:169-174), then cast to ``out_dtype`` (e.g. the ``.cast(float16)`` of config 1).

    Dequant happens once to float32 (materialised, as ``.contiguous()`` at linalg.py:172).
    """
    w = dequant(spec.data, spec.format, spec.shape, spec.scales, spec.block_size, "float32", spec.scale_dtype)
    y = x.astype(np.float32) @ w.T
    return cast(y, out_dtype) if out_dtype else y


# ----------------------------------------------------------------------------------
# seeded synthetic inputs for the benchmark configs c1..c5 (test infrastructure)
# ----------------------------------------------------------------------------------
E2M1_CODES = np.arange(16, dtype=np.uint8)
E3M2_CODES = np.arange(64, dtype=np.uint8)  # all 64 are finite (-0 is code 32)


def random_codes(rng: np.random.Generator, fmt: str, n: int) -> np.ndarray:
    bits = FORMATS[fmt][0]
    return rng.integers(0, 1 << bits, size=n, dtype=np.uint8)


def make_packed(rng: np.random.Generator, fmt: str, rows: int, cols: int, block_size: int,
                scale_kind: str | None) -> PackedSpec:
    """Random codes + scales. scale_kind: None | 'f16u' (fp16 ~U(0.005,0.02)) |
    'f16row' (fp16 ~U(0.01,0.05), one scale per row) | 'e8m0' (2^e, e in {-8..-2})."""
    codes = random_codes(rng, fmt, rows * cols)
    data = pack_codes(codes, FORMATS[fmt][0])
    scales, sdt = None, None
    if scale_kind == "f16u":
        scales = rng.uniform(0.005, 0.02, size=(rows, -(-cols // block_size))).astype(np.float16)
    elif scale_kind == "f16row":
        block_size = cols
        scales = rng.uniform(0.01, 0.05, size=(rows, 1)).astype(np.float16)
    elif scale_kind == "e8m0":
        e = rng.integers(-8, -1, size=(rows, -(-cols // block_size)))
        scales = np.exp2(e).astype(np.float32)
        sdt = "e8m0"
    elif scale_kind is not None:
        raise ValueError(scale_kind)
    return PackedSpec(data, fmt, (rows, cols), scales, block_size, None if sdt is None else "float32")


def e8m0_bytes(scales_pow2: np.ndarray) -> np.ndarray:
    """Encode exact powers of two as E8M0 bytes (biased exponent, bias 127)."""
    m, e = np.frexp(np.asarray(scales_pow2, np.float64))
    if not np.all(m == 0.5):
        raise ValueError("E8M0 scales must be powers of two")
    return (e - 1 + 127).astype(np.uint8)
