"""b200_packed_linear_noalloc (split-K decode GEMM with its scratch in a fixed device array)
against b200_packed_linear on the same operands: two calls in a row, bitwise equal, and the
rejection of a shape whose partials exceed the fixed scratch. Collected last on purpose: it
must also pass after every other test has used the library's own workspaces."""

import ctypes

import numpy as np
import pytest
import torch

from oracle import packed_ref as ref
from tests.helpers import to_device

pytestmark = pytest.mark.gpu
DEV = "cuda:0"


def _noalloc(w, x, y):
    from tinygrad_dx12_b200 import _lib
    from tinygrad_dx12_b200 import dtypes as D
    from tinygrad_dx12_b200.packed import stream_ptr

    d = w.desc()
    return _lib.lib().b200_packed_linear_noalloc(ctypes.byref(d), x.data_ptr(), _lib.DT[D.name(x.dtype)], x.shape[0],
                                                  x.stride(0), y.data_ptr(), _lib.DT[D.name(y.dtype)], y.stride(0),
                                                  stream_ptr(x.device))


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
    from tinygrad_dx12_b200 import _lib

    spec = ref.make_packed(np.random.default_rng(12), "fp4_e2m1", 8192, 8192, 32, "e8m0")
    w = to_device(spec, DEV, "e8m0")
    x = torch.randn((32, 8192), device=DEV).to(torch.bfloat16)  # 2 x 32 x 8192 fp32 partials > 2 MiB - 16 KiB
    y = torch.empty((32, 8192), device=DEV, dtype=torch.bfloat16)
    assert _noalloc(w, x, y) == _lib.ERR_UNSUPPORTED
    assert "scratch" in _lib.last_error()
