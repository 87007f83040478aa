"""Shared test helpers: build torch operands from oracle specs and compare outputs.

Parity bar (stated once, used by every linear test):
* dequantised values: bitwise equality of the float32 (or other output dtype) patterns,
  including -0.0;
* fused matmul outputs: with r the float32 oracle result cast to the output dtype,
  ``max |y - r| / max(|r|, floor) <= 1e-2`` with ``floor = 1e-3 * rms(r)`` and
  ``||y - r||_F / ||r||_F <= 1e-3``, all accumulation in float32.
"""

from __future__ import annotations

import numpy as np
import torch

from oracle import packed_ref as ref

ELEM_TOL, FRO_TOL, FLOOR = 1e-2, 1e-3, 1e-3

TORCH_OF = {"float16": torch.float16, "bfloat16": torch.bfloat16, "float32": torch.float32, "float64": torch.float64}


def to_device(spec: ref.PackedSpec, device, scale_dtype: str | None = None):
    """PackedTensor on ``device`` from an oracle spec; ``scale_dtype`` converts the scales
    (e.g. 'bfloat16', 'float32', 'e8m0')."""
    import tinygrad_dx12_b200 as tg

    data = torch.from_numpy(np.ascontiguousarray(spec.data)).to(device)
    scales = None
    if spec.scales is not None:
        sd = scale_dtype or (spec.scale_dtype or ref.dtype_name(spec.scales.dtype))
        if sd == "e8m0":
            scales = torch.from_numpy(ref.e8m0_bytes(spec.scales)).to(device).view(torch.float8_e8m0fnu)
        else:
            scales = torch.from_numpy(spec.scales.astype(np.float32)).to(device).to(TORCH_OF[sd])
    return tg.PackedTensor(data, spec.format, spec.shape, scales, spec.block_size)


def oracle_scales(spec: ref.PackedSpec, scale_dtype: str | None):
    """The scale values the device sees, as a float array plus the oracle dtype name."""
    if spec.scales is None:
        return None, None
    if scale_dtype in (None, "e8m0"):
        return spec.scales, spec.scale_dtype
    cast = spec.scales.astype(ref.np_dtype(scale_dtype))
    return cast, scale_dtype


def to_numpy(t: torch.Tensor) -> np.ndarray:
    """Host copy of a device tensor, including bf16 / fp8 (returned as ml_dtypes arrays)."""
    t = t.detach().cpu()
    if t.dtype == torch.bfloat16:
        return t.view(torch.int16).numpy().view(ref.BF16)
    if t.dtype in (torch.float8_e4m3fn, torch.float8_e5m2):
        return t.view(torch.uint8).numpy().view(ref.FP8E4M3 if t.dtype == torch.float8_e4m3fn else ref.FP8E5M2)
    return t.numpy()


def errors(y: np.ndarray, r: np.ndarray) -> tuple[float, float]:
    y = y.astype(np.float64)
    r = r.astype(np.float64)
    rms = np.sqrt(np.mean(r * r)) if r.size else 0.0
    floor = max(FLOOR * rms, 1e-30)
    elem = float(np.max(np.abs(y - r) / np.maximum(np.abs(r), floor))) if r.size else 0.0
    fro = float(np.linalg.norm(y - r) / max(np.linalg.norm(r), 1e-30))
    return elem, fro


def assert_close(y: np.ndarray, r32: np.ndarray, out_dtype: str) -> tuple[float, float]:
    r = r32.astype(ref.np_dtype(out_dtype)).astype(np.float64) if out_dtype != "float32" else r32
    elem, fro = errors(y, r)
    assert elem <= ELEM_TOL and fro <= FRO_TOL, f"elementwise {elem:.3e} (<= {ELEM_TOL}), frobenius {fro:.3e} (<= {FRO_TOL})"
    return elem, fro


def bits_equal(a: np.ndarray, b: np.ndarray) -> bool:
    a, b = np.ascontiguousarray(a), np.ascontiguousarray(b)
    return a.dtype.itemsize == b.dtype.itemsize and a.shape == b.shape and np.array_equal(
        a.view(np.uint8), b.view(np.uint8))
