"""ctypes binding of the C-ABI library ``libb200packed.so`` (declared in ``include/b200_packed.h``).

The reference crosses into native code through COM vtables via ctypes
(tinygrad-dx12 ``src/tinygrad_dx12/runtime/support/dx12.py:21-59``) and raises
``RuntimeError("<operation> failed: HRESULT 0x...")`` on failure (``dx12.py:11-15``).
This module does the same for the B200 library: every call's int32 status is checked and
turned into ``RuntimeError("<operation> failed: <code> <message>")``.

There is no fallback: if the library is missing, every entry point raises.
"""

from __future__ import annotations

import ctypes
import os
import pathlib
import threading

LIB_PATH = pathlib.Path(__file__).resolve().parent / "libb200packed.so"

OK, ERR_INVALID, ERR_UNSUPPORTED, ERR_CUDA, ERR_TIMEOUT, ERR_INJECTED = 0, -1, -2, -3, -4, -5
FMT = {"int4": 0, "uint4": 1, "fp4_e2m1": 2, "fp6_e2m3": 3, "fp6_e3m2": 4}
DT = {
    None: 0, "bool": 1, "int8": 2, "uint8": 3, "int16": 4, "uint16": 5, "int32": 6, "uint32": 7, "int64": 8,
    "uint64": 9, "fp8e4m3": 10, "fp8e5m2": 11, "float16": 12, "bfloat16": 13, "float32": 14, "float64": 15,
    "e8m0": 16,
}
PATH = {"auto": 0, "gemv": 1, "gemm": 2, "simt": 3, "mx": 4}
PATH_NAME = {v: k for k, v in PATH.items()}
FLAG_PDL = 0x100               # B200_FLAG_PDL
FLAG_SCALES_ORDINARY = 0x200   # B200_FLAG_SCALES_ORDINARY


class PackedDesc(ctypes.Structure):
    """``b200_packed_desc``."""

    _fields_ = [
        ("data", ctypes.c_void_p),
        ("data_bytes", ctypes.c_int64),
        ("format", ctypes.c_int32),
        ("scale_dtype", ctypes.c_int32),
        ("rows", ctypes.c_int64),
        ("cols", ctypes.c_int64),
        ("block_size", ctypes.c_int64),
        ("scales", ctypes.c_void_p),
    ]


_P, _I32, _I64, _SZ = ctypes.c_void_p, ctypes.c_int32, ctypes.c_int64, ctypes.c_size_t
_DESC = ctypes.POINTER(PackedDesc)
SIGNATURES = {
    "b200_version": ([], _I32),
    "b200_last_error": ([ctypes.c_char_p, _SZ], _I32),
    "b200_inject_failure": ([_I32, _I32], _I32),
    "b200_validate": ([_DESC], _I32),
    "b200_dequant": ([_DESC, _I64, _I64, _P, _I32, _P], _I32),
    "b200_packed_linear": ([_DESC, _P, _I32, _I64, _I64, _I64, _P, _I32, _I64, _I64, _I32, _P], _I32),
    "b200_packed_linear_plan": ([_DESC, _I32, _I64, _I32, _I32], _I32),
    "b200_matmul_generic": ([_P, _I32, _I64, _I64, _P, _I32, _I64, _I64, _P, _I32, _I64, _I64, _I64, _I64, _I64, _I32, _P], _I32),
    "b200_cast": ([_P, _I32, _P, _I32, _I64, _P], _I32),
    "b200_device_count": ([ctypes.POINTER(_I32)], _I32),
    "b200_malloc": ([_I32, _SZ, ctypes.POINTER(_P)], _I32),
    "b200_free": ([_I32, _P], _I32),
    "b200_memcpy": ([_P, _P, _SZ, _I32, _P], _I32),
    "b200_stream_create": ([_I32, ctypes.POINTER(_P)], _I32),
    "b200_stream_destroy": ([_P], _I32),
    "b200_stream_wait": ([_P, _I64], _I32),
    "b200_event_create": ([ctypes.POINTER(_P)], _I32),
    "b200_event_record": ([_P, _P], _I32),
    "b200_event_elapsed_ms": ([_P, _P, ctypes.POINTER(ctypes.c_float)], _I32),
    "b200_event_destroy": ([_P], _I32),
    "b200_device_wait_flag": ([_P, _I32, _I64, _P, _P], _I32),
    "b200_packed_linear_multi": ([_DESC, _P, _I32, _I64, _I64, _P, _I32, _I32, _I64, _I32, _P], _I32),
    "b200_packed_linear_noalloc": ([_DESC, _P, _I32, _I64, _I64, _P, _I32, _I64, _P], _I32),
    "b200_peer_allreduce_add_rmsnorm": ([_P, _P, _P, _I32, _I32, _I64, _I64, _P, _I32, _P, _I32, _I64, _I64,
                                         ctypes.c_float, _P], _I32),
    "b200_ipc_get_handle": ([_P, _P], _I32),
    "b200_ipc_open": ([_P, ctypes.POINTER(_P)], _I32),
    "b200_ipc_close": ([_P], _I32),
    "b200_add_rmsnorm": ([_P, _I32, _P, _P, _I32, _I64, _I64, ctypes.c_float, _P], _I32),
    "b200_gate_mul": ([_P, _I32, _P, _I32, _I64, _I64, _P], _I32),
    "b200_device_status": ([_I32, ctypes.POINTER(ctypes.c_uint32), _I32], _I32),
}

_lock = threading.Lock()
_lib: ctypes.CDLL | None = None


class B200Error(RuntimeError):
    """A failed C-ABI call; ``code`` is the library status."""

    def __init__(self, op: str, code: int, message: str):
        super().__init__(f"{op} failed: {code} {message}")
        self.code = code


def lib() -> ctypes.CDLL:
    """Load the library once (raises if it has not been built)."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            path = os.environ.get("B200_LIB", str(LIB_PATH))
            if not pathlib.Path(path).exists():
                raise RuntimeError(f"B200 C-ABI library not built: {path} (run __graft_entry__.build())")
            handle = ctypes.CDLL(path)
            for name, (args, res) in SIGNATURES.items():
                fn = getattr(handle, name)
                fn.argtypes, fn.restype = args, res
            _lib = handle
    return _lib


def last_error() -> str:
    buf = ctypes.create_string_buffer(1024)
    lib().b200_last_error(buf, len(buf))
    return buf.value.decode(errors="replace")


def check(status: int, op: str) -> int:
    if status < 0:
        raise B200Error(op, status, last_error())
    return status


def call(name: str, *args) -> int:
    return check(getattr(lib(), name)(*args), name)
