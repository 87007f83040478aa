"""The C-ABI library without a GPU: it loads, exports every symbol of include/b200_packed.h,
validates descriptors like PackedTensor.__post_init__, reports errors, and honours the
failure injector. No call here launches a kernel."""

import ctypes
import pathlib
import re

import pytest

from tinygrad_dx12_b200 import _lib

ROOT = pathlib.Path(__file__).resolve().parent.parent


def _declared():
    text = (ROOT / "include" / "b200_packed.h").read_text()
    return sorted(set(re.findall(r"^\s*int32_t\s+(b200_\w+)\s*\(", text, re.M)))


def test_header_declares_entry_points():
    names = _declared()
    assert "b200_packed_linear" in names and "b200_dequant" in names and len(names) >= 20


def test_library_exports_every_declared_symbol():
    lib = _lib.lib()
    missing = [n for n in _declared() if not hasattr(lib, n)]
    assert not missing, missing


def test_bindings_cover_header():
    assert set(_declared()) <= set(_lib.SIGNATURES)


def test_version_and_device_count():
    assert _lib.lib().b200_version() >= 100
    n = ctypes.c_int32(-1)
    assert _lib.lib().b200_device_count(ctypes.byref(n)) == 0 and n.value >= 0


def _desc(**kw):
    d = _lib.PackedDesc()
    d.data = 4096
    d.data_bytes = 8
    d.format = 0
    d.scale_dtype = 0
    d.rows, d.cols, d.block_size = 4, 4, 32
    d.scales = None
    for k, v in kw.items():
        setattr(d, k, v)
    return d


@pytest.mark.parametrize("kw,msg", [
    ({"format": 9}, "unknown packed format"),
    ({"rows": -1}, "nonnegative"),
    ({"data_bytes": 7}, "smaller than the declared shape"),
    ({"block_size": 0}, "block size must be positive"),
    ({"scales": 4096, "scale_dtype": 99}, "unsupported scale dtype"),
])
def test_validate_rejects(kw, msg):
    rc = _lib.lib().b200_validate(ctypes.byref(_desc(**kw)))
    assert rc == _lib.ERR_INVALID
    assert msg in _lib.last_error()


def test_validate_accepts_and_six_bit_storage():
    assert _lib.lib().b200_validate(ctypes.byref(_desc())) == 0
    # 6-bit: 4x4 elements need 12 bytes
    assert _lib.lib().b200_validate(ctypes.byref(_desc(format=4, data_bytes=11))) == _lib.ERR_INVALID
    assert _lib.lib().b200_validate(ctypes.byref(_desc(format=4, data_bytes=12))) == 0


def test_error_raises_runtime_error():
    with pytest.raises(RuntimeError, match="b200_validate failed: -1"):
        _lib.call("b200_validate", ctypes.byref(_desc(format=9)))


def test_injected_failure_is_reported_without_running():
    lib = _lib.lib()
    lib.b200_inject_failure(1, _lib.ERR_INJECTED)
    rc = lib.b200_dequant(ctypes.byref(_desc()), 0, 16, None, 14, None)
    assert rc == _lib.ERR_INJECTED and "injected" in _lib.last_error()
    # one-shot: the next call is validated normally (window check fails before any launch)
    assert lib.b200_dequant(ctypes.byref(_desc()), 0, 17, None, 14, None) == _lib.ERR_INVALID
    lib.b200_inject_failure(0, 0)


def test_dequant_window_and_dtype_checks():
    lib = _lib.lib()
    assert lib.b200_dequant(ctypes.byref(_desc()), -1, 2, None, 14, None) == _lib.ERR_INVALID
    assert lib.b200_dequant(ctypes.byref(_desc()), 0, 4, None, 0, None) == _lib.ERR_INVALID
    assert lib.b200_dequant(ctypes.byref(_desc()), 0, 0, None, 14, None) == 0  # empty window: no launch


def test_plan_selection_without_gpu():
    lib = _lib.lib()
    d = _desc(rows=4096, cols=4096, data_bytes=4096 * 2048, scales=4096, scale_dtype=12, block_size=32)
    f16, f32 = _lib.DT["float16"], _lib.DT["float32"]
    assert lib.b200_packed_linear_plan(ctypes.byref(d), f16, 1, f16, _lib.PATH["simt"]) == _lib.PATH["simt"]
    assert lib.b200_packed_linear_plan(ctypes.byref(d), f32, 1, f32, _lib.PATH["auto"]) > 0
    # block sizes that are not multiples of 32 have no fused kernel
    d2 = _desc(rows=4, cols=64, data_bytes=128, scales=4096, scale_dtype=12, block_size=5)
    assert lib.b200_packed_linear_plan(ctypes.byref(d2), f16, 1, f16, _lib.PATH["auto"]) == _lib.ERR_UNSUPPORTED


def test_bounded_host_wait_rejects_unbounded_device_wait():
    lib = _lib.lib()
    assert lib.b200_device_wait_flag(4096, 1, -1, 4096, None) == _lib.ERR_INVALID
