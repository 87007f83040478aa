"""b200_packed_linear_noalloc: the few-token packed matmul for callers that cannot allocate
device memory once they run (a serving process whose pool already owns all free HBM, a decode
loop that must never take a first-call cudaMalloc). Its split-K scratch is a fixed device array
of the library, so these tests check it against b200_packed_linear on the same operands: the
first call made on a non-blocking side stream, two calls in a row bitwise equal, and the
refusal of a shape whose partials exceed the fixed scratch. Collected last on purpose: it must
also pass after every other test has used the library's own workspaces."""

import ctypes

import numpy as np
import pytest
import torch

from oracle import packed_ref as ref
from tests.helpers import to_device

pytestmark = pytest.mark.gpu
DEV = "cuda:0"
SCRATCH_BYTES, TICKET_BYTES = 2 << 20, 4096 * 4


def _noalloc(w, x, y, stream=None):
    from tinygrad_dx12_b200 import _lib
    from tinygrad_dx12_b200 import dtypes as D
    from tinygrad_dx12_b200.packed import stream_ptr

    d = w.desc()
    s = stream.cuda_stream if stream is not None else stream_ptr(x.device)
    return _lib.lib().b200_packed_linear_noalloc(ctypes.byref(d), x.data_ptr(), _lib.DT[D.name(x.dtype)], x.shape[0],
                                                  x.stride(0), y.data_ptr(), _lib.DT[D.name(y.dtype)], y.stride(0), s)


def test_first_call_on_side_stream():
    """The first call of the process runs on a torch side stream (created non-blocking): the
    set-up must not race the kernel on that stream, and the result equals packed_linear's."""
    from tinygrad_dx12_b200.linalg import _packed_linear

    spec = ref.make_packed(np.random.default_rng(10), "fp4_e2m1", 4096, 4096, 32, "e8m0")
    w = to_device(spec, DEV, "e8m0")
    x = torch.randn((6, 4096), device=DEV).to(torch.bfloat16)
    expect = _packed_linear(w, x, torch.bfloat16, "gemv")
    torch.cuda.synchronize()
    side = torch.cuda.Stream(device=DEV)
    for _ in range(2):
        y = torch.full((6, 4096), float("nan"), device=DEV, dtype=torch.bfloat16)
        torch.cuda.synchronize()
        assert _noalloc(w, x, y, side) == 0
        side.synchronize()
        assert torch.equal(y, expect)


@pytest.mark.parametrize("fmt,kind,sdt,rows,cols,m,xdt", [
    ("fp4_e2m1", "e8m0", "e8m0", 8192, 8192, 8, torch.bfloat16),
    ("int4", "f16u", "float16", 4096, 4096, 12, torch.float16),
    ("uint4", "f16row", "float16", 1000, 1024, 5, torch.float16),
])
def test_matches_packed_linear_twice(fmt, kind, sdt, rows, cols, m, xdt):
    from tinygrad_dx12_b200.linalg import _packed_linear

    spec = ref.make_packed(np.random.default_rng(11), fmt, rows, cols, 32 if kind != "f16row" else cols, kind)
    w = to_device(spec, DEV, sdt)
    x = torch.randn((m, cols), device=DEV).to(xdt)
    expect = _packed_linear(w, x, xdt, "gemv")
    for _ in range(2):
        y = torch.full((m, rows), float("nan"), device=DEV, dtype=xdt)
        assert _noalloc(w, x, y) == 0
        torch.cuda.synchronize()
        assert torch.equal(y, expect)


def test_rejects_scratch_beyond_limit():
    """A shape sized from this device's SM count so that the kernel splits K at least twice
    (rows = 128 x SMs/2 with 32 tokens) and its fp32 partials exceed the fixed scratch."""
    from tinygrad_dx12_b200 import _lib

    sms = torch.cuda.get_device_properties(DEV).multi_processor_count
    rows, m, cols = 128 * max(sms // 2, 1), 32, 8192
    splits = min(16, cols // 512, max(sms // (rows // 128), 1))
    if splits < 2 or splits * m * rows * 4 <= SCRATCH_BYTES - TICKET_BYTES:
        pytest.skip(f"{sms} SMs: no shape of this family exceeds the scratch")
    spec = ref.make_packed(np.random.default_rng(12), "fp4_e2m1", rows, cols, 32, "e8m0")
    w = to_device(spec, DEV, "e8m0")
    x = torch.randn((m, cols), device=DEV).to(torch.bfloat16)
    y = torch.empty((m, rows), device=DEV, dtype=torch.bfloat16)
    assert _noalloc(w, x, y) == _lib.ERR_UNSUPPORTED
    assert "scratch" in _lib.last_error()
