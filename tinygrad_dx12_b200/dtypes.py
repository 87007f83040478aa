"""dtype mapping and promotion for the B200 packed path.

The matrix API follows tinygrad's promotion rules, which tinygrad-dx12 uses for every dtype
decision (``src/tinygrad_dx12/codegen/decomp/dx12.py:58-64,103,129-138``,
``src/tinygrad_dx12/renderer/linalg.py:33-35``): the ``least_upper_dtype`` lattice and the
``sum_acc_dtype`` reduction floor of tinygrad's ``dtype.py`` (tinygrad e4570fcb, v0.14.0),
restated here over torch dtypes. A decoded E8M0 scale tensor (``torch.float8_e8m0fnu``) is
promoted like float32: every E8M0 value is exactly a float32 power of two.
"""

from __future__ import annotations

import functools

import torch

NAMES = {
    torch.bool: "bool", torch.int8: "int8", torch.uint8: "uint8", torch.int16: "int16", torch.uint16: "uint16",
    torch.int32: "int32", torch.uint32: "uint32", torch.int64: "int64", torch.uint64: "uint64",
    torch.float8_e4m3fn: "fp8e4m3", torch.float8_e5m2: "fp8e5m2", torch.float16: "float16",
    torch.bfloat16: "bfloat16", torch.float32: "float32", torch.float64: "float64",
}
E8M0 = getattr(torch, "float8_e8m0fnu", None)
TORCH = {v: k for k, v in NAMES.items()}

ORDER = ("bool", "int8", "uint8", "int16", "uint16", "int32", "uint32", "int64", "uint64",
         "fp8e4m3", "fp8e5m2", "float16", "bfloat16", "float32", "float64")
_PRIORITY = {n: i for i, n in enumerate(ORDER)}
_LATTICE = {
    "bool": ("int8", "uint8"), "int8": ("int16",), "int16": ("int32",), "int32": ("int64",),
    "int64": ("fp8e4m3", "fp8e5m2"), "uint8": ("int16", "uint16"), "uint16": ("int32", "uint32"),
    "uint32": ("int64", "uint64"), "uint64": ("fp8e4m3", "fp8e5m2"), "fp8e5m2": ("float16", "bfloat16"),
    "fp8e4m3": ("float16", "bfloat16"), "float16": ("float32",), "bfloat16": ("float32",),
    "float32": ("float64",), "float64": (),
}


def name(dtype: torch.dtype) -> str:
    """tinygrad-style name of a torch dtype (E8M0 scales promote as float32)."""
    if E8M0 is not None and dtype == E8M0:
        return "float32"
    try:
        return NAMES[dtype]
    except KeyError:
        raise ValueError(f"unsupported dtype {dtype}") from None


def code_name(dtype: torch.dtype) -> str:
    """Name used for the C-ABI dtype code (E8M0 keeps its own code)."""
    if E8M0 is not None and dtype == E8M0:
        return "e8m0"
    return name(dtype)


def _upper(n: str) -> set[str]:
    out = {n}
    for p in _LATTICE[n]:
        out |= _upper(p)
    return out


@functools.lru_cache(maxsize=1024)
def least_upper_dtype(*dts: torch.dtype) -> torch.dtype:
    common = set.intersection(*(_upper(name(d)) for d in dts))
    return TORCH[min(common, key=_PRIORITY.__getitem__)]


def is_float(dt: torch.dtype) -> bool:
    return name(dt) in ("fp8e4m3", "fp8e5m2", "float16", "bfloat16", "float32", "float64")


def is_unsigned(dt: torch.dtype) -> bool:
    return name(dt) in ("uint8", "uint16", "uint32", "uint64")


@functools.lru_cache(maxsize=256)
def sum_acc_dtype(dt: torch.dtype) -> torch.dtype:
    if is_unsigned(dt):
        return least_upper_dtype(dt, torch.uint32)
    if not is_float(dt):
        return least_upper_dtype(dt, torch.int32)
    return least_upper_dtype(dt, torch.float32)


@functools.lru_cache(maxsize=256)
def accumulator(a: torch.dtype, b: torch.dtype) -> torch.dtype:
    """renderer/linalg.py:33-35."""
    return sum_acc_dtype(least_upper_dtype(a, b))
