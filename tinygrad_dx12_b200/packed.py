"""Packed low-bit tensors on the B200 device.

Drop-in for tinygrad-dx12 ``src/tinygrad_dx12/codegen/decomp/dx12.py``: the same
``FORMATS`` / ``FP8_CANDIDATES`` tables (:10-11), the same ``PackedTensor`` fields,
validation and byte layout (:14-47), the same ``unpack`` dtype rules (:49-106), the same
``matrix_intermediate`` selection (:115-138) and the decomp ``matmul`` helper (:141-149).
Tensors are torch CUDA tensors; decoding runs in the library's ``b200_dequant`` kernel.
There is no CPU path: a packed operand on any other device is rejected.
"""

from __future__ import annotations

import functools
import math
from dataclasses import dataclass

import torch

from . import _lib
from . import dtypes as D

# (total bits, exponent bits, mantissa bits, exponent bias); integers have no exponent.
FORMATS = {"int4": (4, 0, 0, 0), "uint4": (4, 0, 0, 0), "fp4_e2m1": (4, 2, 1, 1), "fp6_e2m3": (6, 2, 3, 1),
           "fp6_e3m2": (6, 3, 2, 3)}
FP8_CANDIDATES = {"fp4_e2m1": (torch.float8_e4m3fn, torch.float8_e5m2), "fp6_e2m3": (torch.float8_e4m3fn,),
                  "fp6_e3m2": (torch.float8_e4m3fn, torch.float8_e5m2)}


def _require_cuda(t: torch.Tensor, what: str) -> None:
    if t.device.type != "cuda":
        raise ValueError(f"{what} must be a CUDA tensor on the B200 device, not {t.device}")


_RAW_STREAM = getattr(torch._C, "_cuda_getCurrentRawStream", None)  # torch's fast accessor


def stream_ptr(device: torch.device) -> int:
    """Handle of ``device``'s current CUDA stream (the same value as
    ``torch.cuda.current_stream(device).cuda_stream``, about 2 us cheaper per call)."""
    if _RAW_STREAM is not None:
        return _RAW_STREAM(device.index if device.index is not None else torch.cuda.current_device())
    return torch.cuda.current_stream(device).cuda_stream


@dataclass(frozen=True)
class PackedTensor:
    """Packed low-bit weights on a CUDA device, in the byte layout of tinygrad-dx12.

    ``data`` is a 1-D uint8 tensor holding the codes of a tensor of logical shape ``shape``
    back to back, lowest bits first (a 6-bit code can span two bytes). ``format`` names the
    code type (``FORMATS``: int4, uint4, and the OCP FP4 E2M1 / FP6 E2M3 / FP6 E3M2 codes,
    all finite). ``scales``, when given, holds one multiplier per run of ``block_size`` codes
    along the last axis, shape ``shape[:-1] + (ceil(K / block_size),)``, on the same device;
    a ``torch.float8_e8m0fnu`` tensor counts as the powers of two its bytes encode.
    """

    data: torch.Tensor
    format: str
    shape: tuple
    scales: torch.Tensor | None = None
    block_size: int = 32

    def __post_init__(self) -> None:
        """Reject missing format metadata, insufficient storage, and incompatible scales (dx12.py:32-47)."""
        object.__setattr__(self, "shape", tuple(int(s) for s in self.shape))
        if self.format not in FORMATS:
            raise ValueError(f"unknown packed format {self.format!r}")
        if not self.shape or any(x < 0 for x in self.shape):
            raise ValueError("packed shape must contain nonnegative dimensions")
        if not isinstance(self.data, torch.Tensor) or self.data.dtype is not torch.uint8 or self.data.dim() != 1:
            raise ValueError("packed data must be a flat uint8 Tensor")
        if self.data.numel() < (math.prod(self.shape) * FORMATS[self.format][0] + 7) // 8:
            raise ValueError("packed storage is smaller than the declared shape")
        if self.block_size < 1:
            raise ValueError("packed block size must be positive")
        if self.scales is not None:
            expected = self.shape[:-1] + ((self.shape[-1] + self.block_size - 1) // self.block_size,)
            if tuple(self.scales.shape) != expected or self.scales.device != self.data.device:
                raise ValueError("packed scales have incompatible shape or device")

    # ---- helpers -----------------------------------------------------------------------
    @property
    def device(self) -> torch.device:
        return self.data.device

    @property
    def dtype(self) -> torch.dtype:
        """Declared numeric type used by matrix_intermediate (dx12.py:131-136)."""
        if self.scales is not None:
            return D.least_upper_dtype(torch.float32, self.scales.dtype)
        return {"int4": torch.int8, "uint4": torch.uint8}.get(self.format, torch.float16)

    @property
    def rows(self) -> int:
        return math.prod(self.shape[:-1])

    @property
    def cols(self) -> int:
        return self.shape[-1]

    def scale_flags(self) -> int:
        """``B200_FLAG_SCALES_ORDINARY`` when the scales are E8M0 and none is byte 0x00 (2^-127) or
        0xFF (NaN), else 0. Checked once per tensor (one reduction on the device, one read back)
        and cached: after writing such a byte into ``scales`` in place, call
        ``refresh_scale_flags()``."""
        cached = self.__dict__.get("_sflags")
        if cached is not None:
            return cached
        f = 0
        s = self.scales
        if s is not None and s.dtype == torch.float8_e8m0fnu and s.device.type == "cuda":
            b = s.view(torch.uint8)
            if b.numel() == 0 or not bool(((b == 0) | (b == 255)).any()):
                f = _lib.FLAG_SCALES_ORDINARY
        object.__setattr__(self, "_sflags", f)
        return f

    def refresh_scale_flags(self) -> None:
        """Forget the cached scale check (see ``scale_flags``)."""
        self.__dict__.pop("_sflags", None)

    def desc(self) -> _lib.PackedDesc:
        """The C-ABI descriptor (rows = prod(shape[:-1]), cols = shape[-1]).

        Cached while ``data`` and ``scales`` are contiguous (the descriptor then holds only their
        device addresses, which in-place updates keep)."""
        cached = self.__dict__.get("_desc")
        if cached is not None:
            return cached
        _require_cuda(self.data, "packed data")
        contiguous = self.data.is_contiguous() and (self.scales is None or self.scales.is_contiguous())
        data = self.data if self.data.is_contiguous() else self.data.contiguous()
        scales = None
        if self.scales is not None:
            scales = self.scales if self.scales.is_contiguous() else self.scales.contiguous()
        d = _lib.PackedDesc()
        d.data = data.data_ptr() if data.numel() else None
        d.data_bytes = data.numel()
        d.format = _lib.FMT[self.format]
        d.scale_dtype = _lib.DT[D.code_name(scales.dtype)] if scales is not None else 0
        d.rows, d.cols, d.block_size = self.rows, self.cols, self.block_size
        d.scales = scales.data_ptr() if scales is not None and scales.numel() else None
        d._keep = (data, scales)  # keep contiguous copies alive for the call
        if contiguous:
            object.__setattr__(self, "_desc", d)
        return d

    def default_dtype(self) -> torch.dtype:
        """dx12.py:57-64."""
        integer = self.format in ("int4", "uint4")
        if self.scales is not None:
            return D.least_upper_dtype(torch.float32, self.scales.dtype)
        return torch.int32 if integer else torch.float32

    def unpack(self, dtype: torch.dtype | None = None) -> torch.Tensor:
        """The decoded tensor (codes times their block's scale) as ``dtype``, via ``b200_dequant``.

        Without ``dtype``: float32 for FP codes and for scaled integers (float64 when the scales
        are float64), int32 for unscaled integers. FP codes without scales requested as an FP8
        type that holds them exactly are re-encoded bit for bit (dx12.py:78-92).
        """
        dtype = dtype or self.default_dtype()
        _require_cuda(self.data, "packed data")
        count = math.prod(self.shape)
        fp8 = dtype in (torch.float8_e4m3fn, torch.float8_e5m2)
        out = torch.empty(self.shape, device=self.device, dtype=torch.uint8 if fp8 else dtype)
        if count:
            d = self.desc()
            _lib.call("b200_dequant", ctypes_ref(d), 0, count, out.data_ptr(), _lib.DT[D.name(dtype)],
                      stream_ptr(self.device))
        return out.view(dtype) if fp8 else out

    def matmul(self, other: torch.Tensor | "PackedTensor") -> torch.Tensor:
        """The explicit matrix API (dx12.py:108-112 -> codegen/linalg.py:136)."""
        from .linalg import matmul

        return matmul(self, other)


def ctypes_ref(d: _lib.PackedDesc):
    import ctypes

    return ctypes.byref(d)


def _operand_key(op):
    """What matrix_intermediate depends on: a dtype, or a packed format and its scale dtype."""
    if isinstance(op, PackedTensor):
        return ("packed", op.format, None if op.scales is None else op.scales.dtype)
    return ("tensor", op.dtype)


@functools.lru_cache(maxsize=512)
def _intermediate_for(ka, kb) -> torch.dtype:
    cands, declared = [], []
    for k in (ka, kb):
        if k[0] == "tensor":
            cands.append({k[1]})
            declared.append(k[1])
        else:
            _, fmt, sdt = k
            cands.append(set(FP8_CANDIDATES.get(fmt, ())) if sdt is None else set())
            declared.append(D.least_upper_dtype(torch.float32, sdt) if sdt is not None else
                            {"int4": torch.int8, "uint4": torch.uint8}.get(fmt, torch.float16))
    both = set.intersection(*cands)
    for dt in (torch.float8_e4m3fn, torch.float8_e5m2):
        if dt in both:
            return dt
    return D.least_upper_dtype(*declared)


def matrix_intermediate(a: torch.Tensor | PackedTensor, b: torch.Tensor | PackedTensor, native16: bool = False) -> torch.dtype:
    """The dtype both operands of a matmul are brought to (dx12.py:115-138).

    An FP8 type is chosen when it holds both operands exactly (unscaled FP4/FP6 codes or FP8
    tensors); otherwise the declared types are promoted, a scaled packed operand counting as
    at least float32. ``native16`` exists so reference call sites keep working; it is ignored.
    """
    return _intermediate_for(_operand_key(a), _operand_key(b))


def matmul(a: torch.Tensor | PackedTensor, b: torch.Tensor | PackedTensor) -> torch.Tensor:
    """Decomp helper (dx12.py:141-149): unpack with default dtypes, then an ordinary matmul.

    The ordinary matmul is the library's generic kernel (no fused decode), accumulating in
    tinygrad's default reduction dtype of the two operand types.
    """
    from .linalg import _generic_matmul

    lhs, rhs = [op.unpack() if isinstance(op, PackedTensor) else op for op in (a, b)]
    out_dtype = D.least_upper_dtype(lhs.dtype, rhs.dtype)
    return _generic_matmul(lhs, rhs, out_dtype, D.sum_acc_dtype(out_dtype))
