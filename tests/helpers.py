"""Shared test helpers: build torch operands from oracle specs and compare outputs.

Parity bar (stated once, used by every linear test):
* dequantised values: bitwise equality of the float32 (or other output dtype) patterns,
  including -0.0;
* fused matmul outputs: with r the float32 oracle result cast to the output dtype,
  ``max |y - r| / max(|r|, floor) <= 1e-2`` with ``floor = 1e-2 * rms(r)`` and
  ``||y - r||_F / ||r||_F <= 1e-3``, all accumulation in float32.

The floor: an elementwise relative error is ill-posed for outputs near zero, so outputs
smaller than 1 % of the RMS output are held to an absolute bound of 1e-4 * rms(r), the scale
of float32 accumulation error over thousands of terms on the tensor cores (their adds into the
fp32 accumulator are not round-to-nearest). Failures report the worst element's |r| and
|y - r| in units of rms(r).
"""

from __future__ import annotations

import numpy as np
import torch

from oracle import packed_ref as ref

ELEM_TOL, FRO_TOL, FLOOR = 1e-2, 1e-3, 1e-2

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


def worst(y: np.ndarray, r: np.ndarray) -> str:
    """The element with the largest floored relative error, in units of rms(r)."""
    y = y.astype(np.float64)
    r = r.astype(np.float64)
    rms = max(np.sqrt(np.mean(r * r)), 1e-30)
    rel = np.abs(y - r) / np.maximum(np.abs(r), max(FLOOR * rms, 1e-30))
    i = np.unravel_index(int(np.argmax(rel)), rel.shape)
    return (f"worst at {tuple(int(v) for v in i)}: |r| = {abs(r[i]) / rms:.3e} rms, |y - r| = "
            f"{abs(y[i] - r[i]) / rms:.3e} rms, {int(np.sum(rel > ELEM_TOL))} elements over {ELEM_TOL}")


def assert_close(y: np.ndarray, r32: np.ndarray, out_dtype: str) -> tuple[float, float]:
    r = r32.astype(ref.np_dtype(out_dtype)).astype(np.float64) if out_dtype != "float32" else r32
    elem, fro = errors(y, r)
    assert elem <= ELEM_TOL and fro <= FRO_TOL, (
        f"elementwise {elem:.3e} (<= {ELEM_TOL}), frobenius {fro:.3e} (<= {FRO_TOL}); {worst(y, r)}")
    return elem, fro


def bits_equal(a: np.ndarray, b: np.ndarray) -> bool:
    a, b = np.ascontiguousarray(a), np.ascontiguousarray(b)
    return a.dtype.itemsize == b.dtype.itemsize and a.shape == b.shape and np.array_equal(
        a.view(np.uint8), b.view(np.uint8))


_CLIB = None
_C_FMT = {"int4": 0, "uint4": 1, "fp4_e2m1": 2, "fp6_e2m3": 3, "fp6_e3m2": 4}


def fast_dequant(spec: ref.PackedSpec, scale_dtype: str | None = None, rows: np.ndarray | None = None) -> np.ndarray:
    """float32 dequant of ``spec`` (or of the listed ``rows``) through the oracle's C restatement
    (OpenMP, bit-exact with ``ref.dequant`` -- tests/test_oracle_c.py): the checker for
    full-size matrices, where the numpy restatement would take minutes. ``scale_dtype`` is the
    dtype the device sees ('e8m0', 'float16', 'bfloat16', 'float32' or None for the spec's own)."""
    import ctypes

    from oracle import build as obuild

    global _CLIB
    if _CLIB is None:
        _CLIB = obuild.load()
    n, k = spec.shape
    sdt, sc = 0, None
    if spec.scales is not None:
        name = scale_dtype or spec.scale_dtype or ref.dtype_name(spec.scales.dtype)
        if name == "e8m0":  # E8M0 bytes decode to exactly these float32 powers of two
            name = "float32"
        if name == "float16":
            sdt, sc = 12, np.ascontiguousarray(spec.scales.astype(np.float16))
        elif name == "bfloat16":
            sdt, sc = 13, np.ascontiguousarray(spec.scales.astype(ref.BF16)).view(np.uint16)
        else:
            sdt, sc = 14, np.ascontiguousarray(spec.scales.astype(np.float32))
    ptr = lambda a: a.ctypes.data_as(ctypes.c_void_p)  # noqa: E731
    data = np.ascontiguousarray(spec.data)
    bits = ref.FORMATS[spec.format][0]
    if rows is None:
        out = np.empty((n, k), np.float32)
        rc = _CLIB.oref_dequant_f32(ptr(data), data.size, _C_FMT[spec.format], n, k,
                                    None if sc is None else ptr(sc), sdt, spec.block_size, ptr(out))
        assert rc == 0
        return out
    # selected rows: each row is byte-aligned when k * bits % 8 == 0 (all benchmark shapes)
    assert (k * bits) % 8 == 0
    rb, nblk = k * bits // 8, sc.shape[1] if sc is not None else 0
    out = np.empty((len(rows), k), np.float32)
    for i, r in enumerate(np.asarray(rows)):
        d = np.ascontiguousarray(data[r * rb:(r + 1) * rb])
        s = None if sc is None else np.ascontiguousarray(sc[r:r + 1])
        o = out[i:i + 1]
        rc = _CLIB.oref_dequant_f32(ptr(d), d.size, _C_FMT[spec.format], 1, k, None if s is None else ptr(s), sdt,
                                    spec.block_size, ptr(o))
        assert rc == 0 and nblk >= 0
    return out
