"""The runtime entry points and device-side failure detection, on a B200, through the C-ABI.

* b200_malloc / b200_free / b200_memcpy (all three kinds) / b200_stream_create /
  b200_stream_wait / b200_stream_destroy / b200_event_* -- the allocator, queue and fence
  plumbing that replaces tinygrad-dx12's DX12 runtime (runtime/ops_dx12.py: DX12Allocator
  _alloc/_free/_copyin/_copyout, submit, and the bounded fence wait of DX12Device.wait at
  :206-228).
* failure detection without a GPU fault: a device wait on a flag nothing sets gives up after
  its bound and reports B200_ERR_TIMEOUT; the fused peer reduction run as rank 0 of two ranks
  in one process, where rank 1's signal never comes (a local buffer stands in for the peer),
  gives up after its short timeout, sets the sticky device error bit, returns, and leaves the
  context usable (a later kernel runs and the bit clears).
Nothing here traps, faults or waits without a bound.
"""

from __future__ import annotations

import ctypes
import time

import numpy as np
import pytest
import torch

from tinygrad_dx12_b200 import _lib

pytestmark = pytest.mark.gpu
DEV = "cuda:0"


def _status(clear=True) -> int:
    v = ctypes.c_uint32(0)
    _lib.call("b200_device_status", 0, ctypes.byref(v), 1 if clear else 0)
    return v.value


def test_allocator_copies_stream_and_events():
    lib = _lib.lib()
    n = 1 << 20
    host = np.arange(n, dtype=np.uint32)
    back = np.zeros_like(host)
    a, b, s = ctypes.c_void_p(), ctypes.c_void_p(), ctypes.c_void_p()
    e0, e1 = ctypes.c_void_p(), ctypes.c_void_p()
    _lib.call("b200_malloc", 0, host.nbytes, ctypes.byref(a))
    _lib.call("b200_malloc", 0, host.nbytes, ctypes.byref(b))
    _lib.call("b200_stream_create", 0, ctypes.byref(s))
    _lib.call("b200_event_create", ctypes.byref(e0))
    _lib.call("b200_event_create", ctypes.byref(e1))
    try:
        _lib.call("b200_event_record", e0, s)
        _lib.call("b200_memcpy", a, host.ctypes.data_as(ctypes.c_void_p), host.nbytes, 0, s)  # host -> device
        _lib.call("b200_memcpy", b, a, host.nbytes, 2, s)                                     # device -> device
        _lib.call("b200_memcpy", back.ctypes.data_as(ctypes.c_void_p), b, host.nbytes, 1, s)  # device -> host
        _lib.call("b200_event_record", e1, s)
        assert lib.b200_stream_wait(s, 10_000) == 0
        ms = ctypes.c_float(-1.0)
        _lib.call("b200_event_elapsed_ms", e0, e1, ctypes.byref(ms))
        assert ms.value >= 0.0
        assert np.array_equal(back, host)
        assert lib.b200_memcpy(a, b, 16, 7, s) == _lib.ERR_INVALID  # unknown copy kind
    finally:
        _lib.call("b200_event_destroy", e0)
        _lib.call("b200_event_destroy", e1)
        _lib.call("b200_stream_destroy", s)
        _lib.call("b200_free", 0, a)
        _lib.call("b200_free", 0, b)


def test_stream_wait_times_out_on_a_busy_stream_then_completes():
    """b200_stream_wait with a 0 ms budget on a stream still running a bounded device wait
    reports TIMEOUT instead of blocking; the same wait with a real budget then succeeds."""
    lib = _lib.lib()
    s = ctypes.c_void_p()
    _lib.call("b200_stream_create", 0, ctypes.byref(s))
    flag = torch.zeros(1, dtype=torch.int32, device=DEV)
    status = torch.full((1,), 7, dtype=torch.int32, device=DEV)
    try:
        # 10^6 polls of a flag nothing sets, each after a 256 ns sleep: under a second or two,
        # after which the kernel gives up by itself
        _lib.call("b200_device_wait_flag", flag.data_ptr(), 1, 1_000_000, status.data_ptr(), s)
        assert lib.b200_stream_wait(s, 0) == _lib.ERR_TIMEOUT
        assert "timed out" in _lib.last_error()
        assert lib.b200_stream_wait(s, 60_000) == 0
        assert status.item() == _lib.ERR_TIMEOUT
    finally:
        _lib.call("b200_stream_destroy", s)


def test_device_wait_flag_times_out_and_sees_a_set_flag():
    flag = torch.zeros(1, dtype=torch.int32, device=DEV)
    status = torch.full((1,), 7, dtype=torch.int32, device=DEV)
    t0 = time.monotonic()
    _lib.call("b200_device_wait_flag", flag.data_ptr(), 1, 100_000, status.data_ptr(), None)
    torch.cuda.synchronize()
    assert status.item() == _lib.ERR_TIMEOUT
    assert time.monotonic() - t0 < 30.0
    flag.fill_(1)
    _lib.call("b200_device_wait_flag", flag.data_ptr(), 1, 100_000, status.data_ptr(), None)
    torch.cuda.synchronize()
    assert status.item() == 0


def test_peer_reduce_gives_up_on_a_silent_peer():
    """Rank 0 of a two-rank reduction whose peer never signals: the kernel waits its 2 ms
    budget, sets the device error bit and returns; h still receives the sum of the partial
    slots (rank 1's slot is zero here) and the context keeps working."""
    from tinygrad_dx12_b200 import dtypes as D
    from tinygrad_dx12_b200 import stack as S
    from tinygrad_dx12_b200.packed import stream_ptr

    assert _status() in (0, 1)  # clear anything left by earlier tests
    rows_max, hidden = 2, 4096
    part = torch.zeros((2, rows_max, hidden), dtype=torch.float32, device=DEV)  # [rank][row][:]
    flags = torch.zeros((2, 2 * rows_max), dtype=torch.int32, device=DEV)      # one array per "rank"
    epoch = torch.zeros(rows_max, dtype=torch.int32, device=DEV)
    g = torch.Generator(device=DEV).manual_seed(4)
    part[0, :1] = torch.randn((1, hidden), device=DEV, generator=g)
    h = torch.randn((1, hidden), device=DEV, generator=g).to(torch.bfloat16)
    h_expect = (h.float() + part[0, :1]).to(torch.bfloat16)
    x = torch.empty_like(h)
    P = ctypes.c_void_p * 8
    partials = P(part[0].data_ptr(), part[1].data_ptr())
    flag_ptrs = P(flags[0].data_ptr(), flags[1].data_ptr())
    t0 = time.monotonic()
    _lib.call("b200_peer_allreduce_add_rmsnorm", partials, flag_ptrs, epoch.data_ptr(), 0, 2, rows_max,
              2_000_000, h.data_ptr(), _lib.DT[D.name(h.dtype)], x.data_ptr(), _lib.DT[D.name(x.dtype)], 1, hidden,
              S.EPS, stream_ptr(h.device))
    torch.cuda.synchronize()
    assert time.monotonic() - t0 < 30.0
    assert _status() & 1, "the give-up must set the sticky device error bit"
    assert _status() == 0, "clearing the status resets it"
    assert torch.equal(h, h_expect)
    # this rank signalled both flag arrays: its own slot in rank 0's array and in rank 1's
    assert flags[0, 0].item() == 1 and flags[1, 0].item() == 1 and epoch[0].item() == 1
    # the context is still usable
    y = torch.ones(1024, device=DEV) * 3
    assert float(y.sum().item()) == 3072.0
