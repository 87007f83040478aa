"""Public matrix API on the B200 device: ``matmul`` and ``matvec``.

Drop-in for tinygrad-dx12 ``src/tinygrad_dx12/codegen/linalg.py`` with the same signatures,
argument checks and dtype rules:

* ``matmul(a, b, scope="auto", tile=None, dtype=None)`` (linalg.py:136-223). ``dtype`` sets
  the output precision; every fused kernel accumulates in float32 (the reference leaves
  internal arithmetic to the device, linalg.py:152-155).
* ``matvec(matrix, vector, output_dtype=None, thread=None)`` (linalg.py:226-298).
* ``choose_matrix`` (linalg.py:90-133) reports the kernel the library selects.

Scopes. ``auto`` selects a fused kernel when one supports the operands and otherwise the
ordinary path (decode kernel + the library's generic matmul kernel), like the reference's
fallback to ordinary compute. ``Wave`` requests the warp-scope fused decode GEMV,
``ThreadGroup`` the CTA-scope tcgen05 GEMM; when the library rejects an explicit scope a
``RuntimeError`` is raised. ``tiled`` is ordinary compute. Unknown scopes raise ``ValueError``.

The fused call form is ``matmul(W, x.T)`` with ``W`` a ``PackedTensor`` of shape (N, K) and
``x`` (M, K): the result is (N, M) (a transposed view of a row-major (M, N) buffer), so
``matmul(W, x.T).T`` is ``x @ W^T``. No path runs on the CPU.
"""

from __future__ import annotations

from typing import NamedTuple

import torch

from . import _lib
from . import dtypes as D
from .packed import FORMATS, PackedTensor, matrix_intermediate, stream_ptr, ctypes_ref

SCOPES = ("auto", "Wave", "ThreadGroup", "tiled")
FUSED_IO = (torch.float16, torch.bfloat16, torch.float32)
_SCOPE_PATHS = {"auto": ("auto",), "Wave": ("mx", "gemv", "simt"), "ThreadGroup": ("gemm",)}


def _device_of(op) -> torch.device:
    return op.data.device if isinstance(op, PackedTensor) else op.device


def _check_cuda(device: torch.device) -> None:
    if device.type != "cuda":
        raise ValueError(f"the B200 matrix API requires CUDA tensors (got device {device})")


DENSE_IO = (torch.float16, torch.bfloat16)


def _tensor_core_layout(lhs: torch.Tensor, rhs: torch.Tensor, out_dtype: torch.dtype):
    """16-bit operands for the tcgen05 dense GEMM: lhs row-major, rhs K-major (columns with k
    contiguous), both 16-byte aligned; copies an operand only when its layout does not fit."""
    if lhs.dtype != rhs.dtype or lhs.dtype not in DENSE_IO or out_dtype not in FUSED_IO:
        return lhs, rhs
    m, k = lhs.shape
    if k % 8 or k < 16 or m * rhs.shape[1] * k < (1 << 18):
        return lhs, rhs  # tiny or unaligned: the tiled kernel
    if lhs.stride(1) != 1 or lhs.stride(0) % 8 or lhs.data_ptr() % 16:
        lhs = lhs.contiguous()
    if rhs.stride(0) != 1 or rhs.stride(1) % 8 or rhs.data_ptr() % 16:
        rhs = rhs.t().contiguous().t()
    return lhs, rhs


def _generic_matmul(lhs: torch.Tensor, rhs: torch.Tensor, out_dtype: torch.dtype, acc_dtype: torch.dtype) -> torch.Tensor:
    """Ordinary matmul through ``b200_matmul_generic`` (linalg.py:188-189, the 'tiled' scope);
    16-bit operands run on the tcgen05 dense GEMM."""
    lhs, rhs = _tensor_core_layout(lhs, rhs, out_dtype)
    m, k = lhs.shape
    n = rhs.shape[1]
    fp8_out = out_dtype in (torch.float8_e4m3fn, torch.float8_e5m2)
    out = torch.empty((m, n), device=lhs.device, dtype=torch.uint8 if fp8_out else out_dtype)
    if m and n:
        def arg(t):
            return t.view(torch.uint8) if t.dtype in (torch.float8_e4m3fn, torch.float8_e5m2) else t
        a, b = arg(lhs), arg(rhs)
        _lib.call("b200_matmul_generic", a.data_ptr(), _lib.DT[D.name(lhs.dtype)], lhs.stride(0), lhs.stride(1),
                  b.data_ptr(), _lib.DT[D.name(rhs.dtype)], rhs.stride(0), rhs.stride(1), out.data_ptr(),
                  _lib.DT[D.name(out_dtype)], out.stride(0), out.stride(1), m, n, k, _lib.DT[D.name(acc_dtype)],
                  stream_ptr(lhs.device))
    return out.view(out_dtype) if fp8_out else out


_EXACT_IN_BF16 = ("fp4_e2m1", "fp6_e2m3", "fp6_e3m2")


def _fused_operands(a, b, out_dtype):
    """The (W, x) pair for a fused call, or None when the fused kernels cannot take it.

    A packed right operand (the packed x packed products, dx12.py:115-138) is decoded to bf16
    first when that is exact: FP4 / FP6 codes, unscaled or with E8M0 scales (at most 4
    significant bits times a power of two inside bf16's range). The left operand then runs
    through the fused kernels as the weights (its codes read by the tensor cores)."""
    if not isinstance(a, PackedTensor) or len(a.shape) != 2:
        return None
    if isinstance(b, PackedTensor):
        exact = b.format in _EXACT_IN_BF16 and (b.scales is None or b.scales.dtype == torch.float8_e8m0fnu)
        if not exact or len(b.shape) != 2 or out_dtype not in FUSED_IO:
            return None
        if a.scales is not None and D.name(a.scales.dtype) == "float64":
            return None
        return a, b.unpack(torch.bfloat16).t()  # x[m, k] = b[k, m], exact
    if b.dtype not in FUSED_IO or out_dtype not in FUSED_IO:
        return None
    if a.scales is not None and D.name(a.scales.dtype) == "float64":
        return None
    return a, b.t()  # x[m, k] = b[k, m]


def _aligned_x(x: torch.Tensor) -> torch.Tensor:
    """Fused kernels read x rows with 16-byte vector loads: stage (copy) a strided or
    misaligned view, as the reference stages unaligned matrix inputs (linalg.py:61-87)."""
    es = x.element_size()

    def ok(t: torch.Tensor) -> bool:
        return t.stride(1) == 1 and t.data_ptr() % 16 == 0 and (t.shape[0] == 1 or (t.stride(0) * es) % 16 == 0)

    if ok(x):
        return x
    y = x.contiguous()
    if ok(y):
        return y
    k = x.shape[1]
    kp = -(-k * es // 16) * 16 // es
    buf = torch.zeros((x.shape[0], kp), dtype=x.dtype, device=x.device)
    buf[:, :k] = x
    return buf[:, :k]


def _packed_linear(w: PackedTensor, x: torch.Tensor, out_dtype: torch.dtype, path: str, flags: int = 0,
                   y: torch.Tensor | None = None) -> torch.Tensor:
    """y[M, N] = x[M, K] @ dequant(W)[N, K]^T through ``b200_packed_linear`` (``flags``: B200_FLAG_*);
    ``y``, when given, is the destination (unit column stride)."""
    x = _aligned_x(x)
    m = x.shape[0]
    ldx = x.stride(0) if m > 1 else -(-x.shape[1] // 8) * 8
    if y is None:
        y = torch.empty((m, w.rows), device=x.device, dtype=out_dtype)
    d = w.desc()
    _lib.call("b200_packed_linear", ctypes_ref(d), x.data_ptr(), _lib.DT[D.name(x.dtype)], m, ldx, 1,
              y.data_ptr(), _lib.DT[D.name(out_dtype)], y.stride(0) if m > 1 else w.rows, 1,
              _lib.PATH[path] | flags | w.scale_flags(), stream_ptr(x.device))
    return y


def _packed_linear_multi(w: PackedTensor, x: torch.Tensor, y_ptrs, out_dtype: torch.dtype, ldy: int,
                         flags: int = 0) -> None:
    """``b200_packed_linear_multi``: the same y written to every address of ``y_ptrs`` (a ctypes
    array of device pointers in this process, e.g. peer-mapped buffers), row pitch ``ldy``."""
    x = _aligned_x(x)
    m = x.shape[0]
    ldx = x.stride(0) if m > 1 else -(-x.shape[1] // 8) * 8
    d = w.desc()
    _lib.call("b200_packed_linear_multi", ctypes_ref(d), x.data_ptr(), _lib.DT[D.name(x.dtype)], m, ldx, y_ptrs,
              len(y_ptrs), _lib.DT[D.name(out_dtype)], ldy, flags | w.scale_flags(), stream_ptr(x.device))


def linear_plan(w: PackedTensor, x_dtype: torch.dtype, m: int, out_dtype: torch.dtype, path: str = "auto") -> str | None:
    """Name of the fused kernel the library would run ('mx', 'gemv', 'gemm', 'simt') or None."""
    d = w.desc()
    rc = _lib.lib().b200_packed_linear_plan(ctypes_ref(d), _lib.DT[D.name(x_dtype)], m, _lib.DT[D.name(out_dtype)],
                                            _lib.PATH[path])
    return _lib.PATH_NAME.get(rc) if rc > 0 else None


def choose_matrix(w: PackedTensor, x_dtype: torch.dtype, m: int, out_dtype: torch.dtype, scope: str = "auto"):
    """Selected (scope, kernel) for these operands (linalg.py:90-133); 'tiled' means ordinary compute."""
    if scope not in SCOPES:
        raise ValueError(f"unknown matrix scope {scope!r}")
    if scope == "tiled":
        return ("tiled", None)
    for path in _SCOPE_PATHS[scope]:
        plan = linear_plan(w, x_dtype, m, out_dtype, path)
        if plan is not None:
            return ({"mx": "Wave", "gemv": "Wave", "gemm": "ThreadGroup", "simt": "Wave"}[plan], plan)
    return ("tiled", None)


class Estimates(NamedTuple):
    """Cost of one matrix product, for profilers (the reference attaches
    ``Estimates(2*m*n*k, bytes)`` to its LinAlg program, codegen/linalg.py:50-56).

    ``ops`` and ``mem`` follow the reference: 2·m·n·k, and the output plus both operands at
    the dtypes its matrix program sees them (a packed operand as the decoded intermediate).
    ``packed_mem`` is what the fused kernels move instead: packed codes, scales, the other
    operand and the output, each read or written once."""

    ops: int
    mem: int
    packed_mem: int


def estimates(a: torch.Tensor | PackedTensor, b: torch.Tensor | PackedTensor,
              dtype: torch.dtype | None = None) -> Estimates:
    """Estimates of ``matmul(a, b, dtype=dtype)`` (shapes and dtypes only; no device work)."""
    if len(a.shape) != 2 or len(b.shape) != 2 or a.shape[1] != b.shape[0]:
        raise ValueError("matrix operands must have compatible rank-two shapes")
    intermediate = matrix_intermediate(a, b)
    m, k, n = a.shape[0], a.shape[1], b.shape[1]
    lhs_dt = intermediate if isinstance(a, PackedTensor) else a.dtype
    rhs_dt = intermediate if isinstance(b, PackedTensor) else b.dtype
    out_dt = dtype or D.accumulator(lhs_dt, rhs_dt)
    size = lambda dt: torch.empty((), dtype=dt).element_size()  # noqa: E731
    mem = m * n * size(out_dt) + m * k * size(lhs_dt) + k * n * size(rhs_dt)

    def moved(op, rows, cols, dt):
        if isinstance(op, PackedTensor):
            scales = 0 if op.scales is None else op.scales.numel() * op.scales.element_size()
            return -(-op.shape[0] * op.shape[1] * FORMATS[op.format][0] // 8) + scales
        return rows * cols * size(dt)

    packed = m * n * size(out_dt) + moved(a, m, k, lhs_dt) + moved(b, k, n, rhs_dt)
    return Estimates(2 * m * n * k, mem, packed)


_profile_hook = None


def set_profile_hook(hook) -> None:
    """Install ``hook(kernel, estimates)`` (or None): called after every ``matmul`` launch with
    the kernel that ran ('mx', 'gemv', 'gemm', 'simt' or 'generic') and its Estimates."""
    global _profile_hook
    _profile_hook = hook


def _report(kernel: str, a, b, dtype) -> None:
    if _profile_hook is not None:
        _profile_hook(kernel, estimates(a, b, dtype))


# decode kernels that store y with plain stores (the GEMMs write it with TMA stores), so y may be
# a pinned host buffer
_HOST_Y_PLANS = ("gemv", "mx", "simt")


_STAGING: dict = {}  # (device, stream, dtype) -> device buffer reused by every staged call on that stream


def _stage_host(t: torch.Tensor, device: torch.device) -> torch.Tensor:
    """A pinned host tensor on ``device``: for 16/32-bit floats laid out row- or column-major, the
    library's copy kernel reads it over the host link (for a decode step's few KB this costs a
    few microseconds, well under a DMA copy's setup) into a buffer kept per stream (calls on one
    stream run in order, so the next call's copy starts after this call's kernel has read it);
    anything else goes through ``to``."""
    if not t.is_pinned():
        raise ValueError("a host matrix operand must be in pinned memory (torch.Tensor.pin_memory())")
    tt = t.t()
    src = t if t.is_contiguous() else tt if tt.is_contiguous() else None
    if src is None or t.dtype not in FUSED_IO:
        return t.to(device, non_blocking=True)
    stream = stream_ptr(device)
    key = (device.index, stream, src.dtype)
    buf = _STAGING.get(key)
    n = src.numel()
    if buf is None or buf.numel() < n:
        buf = torch.empty(max(n, 1 << 14), device=device, dtype=src.dtype)
        _STAGING[key] = buf
    dst = buf[:n].view(src.shape)
    code = _lib.DT[D.name(src.dtype)]
    _lib.call("b200_cast", src.data_ptr(), code, dst.data_ptr(), code, n, stream)
    return dst if src is t else dst.t()


def _host_decode_step(a: PackedTensor, b: torch.Tensor, dtype, out):
    """The lean form of the host-I/O call for a decode step, or None when it does not apply:
    b = x.T with x (M, K) pinned and row-major, ``dtype`` given, out = y.T with y (M, N) pinned
    and row-major (or None), and a decode kernel (plain stores) as the plan. Two library calls:
    the staging copy of x and the fused kernel storing into y."""
    if dtype not in FUSED_IO or b.dtype not in FUSED_IO or b.dim() != 2 or len(a.shape) != 2:
        return None
    kdim, m = b.shape
    if a.shape[1] != kdim or kdim % 8 or b.stride(0) != 1 or (m > 1 and b.stride(1) != kdim) or b.storage_offset():
        return None
    n = a.shape[0]
    if out is not None and (out.device.type != "cpu" or out.dtype != dtype or tuple(out.shape) != (n, m)
                            or out.stride(0) != 1 or (m > 1 and out.stride(1) != n)):
        return None
    if a.scales is not None and a.scales.dtype == torch.float64:
        return None
    plans = a.__dict__.setdefault("_plans", {})
    pkey = (b.dtype, m, dtype)
    if pkey not in plans:
        plans[pkey] = linear_plan(a, b.dtype, m, dtype)
    path = plans[pkey]
    if path not in _HOST_Y_PLANS:
        return None
    if not b.is_pinned() or (out is not None and not out.is_pinned()):
        raise ValueError("host matrix operands must be in pinned memory (torch.Tensor.pin_memory())")
    device = a.data.device
    stream = stream_ptr(device)
    key = (device.index, stream, b.dtype)
    buf = _STAGING.get(key)
    if buf is None or buf.numel() < m * kdim:
        buf = torch.empty(max(m * kdim, 1 << 14), device=device, dtype=b.dtype)
        _STAGING[key] = buf
    xcode, ycode = _lib.DT[D.name(b.dtype)], _lib.DT[D.name(dtype)]
    _lib.call("b200_cast", b.data_ptr(), xcode, buf.data_ptr(), xcode, m * kdim, stream)
    y = torch.empty((m, n), device=device, dtype=dtype) if out is None else out
    # B200_FLAG_PDL: the decode kernel streams its weights while the staging copy runs, and waits
    # for the copy before reading x
    _lib.call("b200_packed_linear", ctypes_ref(a.desc()), buf.data_ptr(), xcode, m, kdim, 1, y.data_ptr(), ycode, n,
              1, _lib.PATH[path] | a.scale_flags() | _lib.FLAG_PDL, stream)
    if _profile_hook is not None:
        _report(path, a, b, dtype)
    return out if out is not None else y.t()


def matmul(a: torch.Tensor | PackedTensor, b: torch.Tensor | PackedTensor, scope: str = "auto",
           tile: tuple[int, int, int] | None = None, dtype: torch.dtype | None = None,
           out: torch.Tensor | None = None) -> torch.Tensor:
    """Multiply two matrices on the B200 device (linalg.py:136-223).

    Packed operands decode inside the fused kernels; other combinations decode with
    ``b200_dequant`` to the common intermediate and multiply with the generic kernel.
    ``dtype`` declares the output precision (accumulation is float32 in the fused kernels,
    the output dtype's reduction type in the generic one). No gradients are defined.

    Host I/O for decode steps whose tokens arrive from and return to the host (no counterpart
    in the reference): ``b`` may be a pinned host tensor, staged onto ``a``'s device by a small
    library kernel, and ``out`` a tensor of the result's shape and dtype (pinned host or on the
    device) that receives the result -- the decode kernels store into a pinned ``out`` directly
    when its transpose is contiguous, other paths go through a device buffer and a copy. Both
    are asynchronous on the current stream: synchronize before reading ``out``, and keep the
    host tensors alive until then.
    """
    if scope not in SCOPES:
        raise ValueError(f"unknown matrix scope {scope!r}")
    automatic = scope == "auto"
    if isinstance(b, torch.Tensor) and b.device.type == "cpu" and _device_of(a).type == "cuda":
        if automatic and tile is None and isinstance(a, PackedTensor):
            y = _host_decode_step(a, b, dtype, out)
            if y is not None:
                return y
        b = _stage_host(b, _device_of(a))
    device, other_device = _device_of(a), _device_of(b)
    if device != other_device:
        raise ValueError("matrix operands must belong to one device")
    if len(a.shape) != 2 or len(b.shape) != 2 or a.shape[1] != b.shape[0]:
        raise ValueError("matrix operands must have compatible rank-two shapes")
    _check_cuda(device)
    if tile is not None and any(x < 1 for x in tile):
        raise ValueError("matrix tile dimensions must be positive")
    intermediate = matrix_intermediate(a, b)
    m, k, n = a.shape[0], a.shape[1], b.shape[1]
    lhs_dt = intermediate if isinstance(a, PackedTensor) else a.dtype
    rhs_dt = intermediate if isinstance(b, PackedTensor) else b.dtype
    out_dtype = dtype or D.accumulator(lhs_dt, rhs_dt)
    if out is not None and (tuple(out.shape) != (m, n) or out.dtype != out_dtype):
        raise ValueError(f"out must be a {out_dtype} tensor of shape {(m, n)}")
    if out is not None and out.device.type == "cpu" and not out.is_pinned():
        raise ValueError("a host out tensor must be in pinned memory (torch.Tensor.pin_memory())")
    if 0 in (m, k, n):
        return _deliver(torch.zeros((m, n), device=device, dtype=out_dtype), out)
    if scope != "tiled":
        fused = _fused_operands(a, b, out_dtype)
        if fused is not None:
            w, x = fused
            if automatic and out is not None and (out.device.type == "cpu" or out.device == device) \
                    and out.t().is_contiguous():
                plans = w.__dict__.setdefault("_plans", {})  # the plan depends on shapes and dtypes only
                pkey = (x.dtype, x.shape[0], out_dtype)
                path = plans.get(pkey, "") if pkey in plans else plans.setdefault(
                    pkey, linear_plan(w, x.dtype, x.shape[0], out_dtype))
                if path is not None and (out.device == device or path in _HOST_Y_PLANS):
                    _packed_linear(w, x, out_dtype, path, y=out.t())  # the kernel stores into out itself
                    _report(path, a, b, dtype)
                    return out
            if automatic:  # one library call: it picks the kernel or reports that none fits
                try:
                    y = _deliver(_packed_linear(w, x, out_dtype, "auto").t(), out)
                    if _profile_hook is not None:
                        _report(linear_plan(w, x.dtype, x.shape[0], out_dtype) or "auto", a, b, dtype)
                    return y
                except _lib.B200Error as error:
                    if error.code != _lib.ERR_UNSUPPORTED:
                        raise
            else:
                for path in _SCOPE_PATHS[scope]:
                    if linear_plan(w, x.dtype, x.shape[0], out_dtype, path) is not None:
                        y = _deliver(_packed_linear(w, x, out_dtype, path).t(), out)
                        _report(path, a, b, dtype)
                        return y
        if not automatic:
            raise RuntimeError(f"B200 {scope} {tile} rejected: no fused kernel for these operands")
    # ordinary compute: decode to the intermediate, then the generic matmul
    wide = D.accumulator(intermediate, intermediate) if scope == "tiled" else intermediate
    lhs = a.unpack(wide) if isinstance(a, PackedTensor) else a
    rhs = b.unpack(wide) if isinstance(b, PackedTensor) else b
    acc = D.sum_acc_dtype(out_dtype) if D.is_float(out_dtype) else out_dtype
    y = _deliver(_generic_matmul(lhs, rhs, out_dtype, acc), out)
    _report("generic", a, b, dtype)
    return y


def _deliver(y: torch.Tensor, out: torch.Tensor | None) -> torch.Tensor:
    if out is None:
        return y
    out.copy_(y, non_blocking=True)
    return out


def matvec(matrix: torch.Tensor | PackedTensor, vector: torch.Tensor, output_dtype: torch.dtype | None = None,
           thread: bool | None = None) -> torch.Tensor:
    """Matrix-vector product (linalg.py:226-298).

    ``thread=None`` is a one-column ``matmul``. ``thread=True`` requests the warp-scope
    decode GEMV (the B200 counterpart of the reference's thread-scope matrix API) and falls
    back to ordinary compute when it cannot run; ``thread=False`` selects ordinary compute.
    """
    device = _device_of(matrix)
    if len(matrix.shape) != 2 or vector.dim() != 1 or matrix.shape[1] != vector.shape[0] or device != vector.device:
        raise ValueError("matvec expects a matrix and matching vector on one device")
    intermediate = matrix_intermediate(matrix, vector)
    output_dtype = output_dtype or D.accumulator(intermediate, intermediate)
    if thread is None:
        return matmul(matrix, vector.reshape(-1, 1), dtype=output_dtype).reshape(matrix.shape[0])
    if thread:
        try:
            return matmul(matrix, vector.reshape(-1, 1), scope="Wave", dtype=output_dtype).reshape(matrix.shape[0])
        except RuntimeError as error:
            if "rejected" not in str(error):
                raise
    return matmul(matrix, vector.reshape(-1, 1), scope="tiled", dtype=output_dtype).reshape(matrix.shape[0])
