"""Projection stacks on the GPU: the glue kernels (b200_add_rmsnorm, b200_gate_mul) against
torch fp32 references of the same ops, and TPStack through the CUDA library against the
unsharded oracle chain (oracle/stack_ref.py) at reduced sizes (hidden 256, 2 layers).

Tolerance: relative Frobenius error of the final h <= 1e-3 (fp16 activations) or 4e-3
(bf16, one bf16 ulp is 2^-8 of a value and a rounding flip carries through the layers)."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from tests.stack_helpers import CONFIGS, initial_h, oracle_forward, to_numpy
from tinygrad_dx12_b200 import stack as S

pytestmark = pytest.mark.gpu
DEV = "cuda:0"


@pytest.mark.parametrize("dt", [torch.float16, torch.bfloat16, torch.float32])
@pytest.mark.parametrize("with_partial", [False, True])
@pytest.mark.parametrize("shape", [(1, 8192), (3, 4096), (64, 257)])
def test_add_rmsnorm(dt, with_partial, shape):
    g = torch.Generator(device=DEV).manual_seed(1)
    h = torch.randn(shape, device=DEV, generator=g).to(dt)
    p = torch.randn(shape, device=DEV, generator=g) * 3 if with_partial else None
    x = torch.empty_like(h)
    h_ref = (h.float() + p).to(dt) if with_partial else h.clone()
    hr = h_ref.float()
    x_ref = (hr * torch.rsqrt(hr.pow(2).mean(-1, keepdim=True) + S.EPS)).to(dt)
    S.CudaOps().add_rmsnorm(h, p, x)
    torch.cuda.synchronize()
    assert torch.equal(h, h_ref)
    err = (x.float() - x_ref.float()).abs().max().item()
    ulp = {torch.float16: 2**-10, torch.bfloat16: 2**-7, torch.float32: 2**-20}[dt]
    assert err <= 4 * ulp * x_ref.float().abs().max().item()


@pytest.mark.parametrize("dt", [torch.float16, torch.bfloat16])
def test_gate_mul(dt):
    g = torch.Generator(device=DEV).manual_seed(2)
    gu = torch.randn((5, 2 * 3584), device=DEV, generator=g).to(dt)
    out = torch.empty((5, 3584), device=DEV, dtype=dt)
    S.CudaOps().gate_mul(gu, out)
    ref = (gu[:, :3584].float() * gu[:, 3584:].float()).to(dt)
    assert torch.equal(out, ref)


@pytest.mark.parametrize("name", sorted(CONFIGS))
@pytest.mark.parametrize("m", [1, 3, 40])
def test_stack_matches_oracle(name, m):
    cfg = CONFIGS[name]
    st = S.TPStack(cfg, 0, 1, device=DEV, matrix_fn=lambda layer, proj: _cuda(S.make_matrix(cfg, layer, proj, "cpu")))
    h = st.forward(initial_h(cfg, m).to(DEV))
    torch.cuda.synchronize()
    y, r = to_numpy(h), oracle_forward(cfg, initial_h(cfg, m))
    tol = 4e-3 if cfg.act == torch.bfloat16 else 1e-3
    assert np.all(np.isfinite(y))
    assert np.linalg.norm(y - r) / np.linalg.norm(r) <= tol


def _cuda(w):
    from tinygrad_dx12_b200.packed import PackedTensor

    return PackedTensor(w.data.to(DEV), w.format, w.shape, None if w.scales is None else w.scales.to(DEV), w.block_size)


def test_peer_reduce_single_rank_matches_add_rmsnorm():
    """b200_peer_allreduce_add_rmsnorm with one rank (it waits only on its own flag) equals
    b200_add_rmsnorm of the same partial over several epochs and both buffers."""
    import ctypes

    from tinygrad_dx12_b200 import _lib
    from tinygrad_dx12_b200 import dtypes as D
    from tinygrad_dx12_b200.packed import stream_ptr

    rows_max, hidden = 4, 4096
    part = torch.zeros((2, rows_max, hidden), dtype=torch.float32, device=DEV)
    flags = torch.zeros(rows_max, dtype=torch.int32, device=DEV)
    epoch = torch.zeros(rows_max, dtype=torch.int32, device=DEV)
    P = ctypes.c_void_p * 8
    g = torch.Generator(device=DEV).manual_seed(3)
    h = torch.randn((3, hidden), device=DEV, generator=g).to(torch.bfloat16)
    h_ref = h.clone()
    x = torch.empty_like(h)
    x_ref = torch.empty_like(h)
    for step in range(5):
        slot = step % 2
        part[slot, :3] = torch.randn((3, hidden), device=DEV, generator=g)
        _lib.call("b200_peer_allreduce_add_rmsnorm", P(part[slot].data_ptr()), P(flags.data_ptr()), epoch.data_ptr(),
                  0, 1, rows_max, int(1e9), h.data_ptr(), _lib.DT[D.name(h.dtype)], x.data_ptr(),
                  _lib.DT[D.name(x.dtype)], 3, hidden, S.EPS, stream_ptr(h.device))
        S.CudaOps().add_rmsnorm(h_ref, part[slot, :3].contiguous(), x_ref)
        torch.cuda.synchronize()
        assert torch.equal(h, h_ref)  # the residual sum is elementwise: bitwise equal
        # x: the sum of squares is reduced in a different thread order -> within 2 bf16 ulps
        assert (x.float() - x_ref.float()).abs().max().item() <= 2 * 2**-7 * x_ref.float().abs().max().item()
    assert epoch[:3].tolist() == [5, 5, 5] and flags[:3].tolist() == [5, 5, 5]
    v = ctypes.c_uint32(0)
    _lib.call("b200_device_status", 0, ctypes.byref(v), 1)
    assert v.value == 0
