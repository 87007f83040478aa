"""Parity at the shapes the benchmark times, through the persistent loops those shapes take.

* c3 at full size (M=4096, N=14336, K=4096, FP6 E3M2, per-row fp16 scales): the tcgen05 GEMM
  runs 16 x 112 = 1792 tiles over one CTA per SM, so every CTA carries its shared-memory ring,
  tensor-memory accumulators and their phases across about 12 tiles. All of y is compared.
* the GEMM with E8M0 per-32 scales and bf16 x at the c5 gate shape (28672 x 8192, M=2048):
  1792 tiles again; every 7th weight row is compared for all tokens (4096 rows).
* the streamed decode GEMV with far more 32-row blocks than resident CTAs: the c5 gate|up
  projection (57344 x 8192 FP4 E8M0, 1792 row blocks) and the c4 gate|up projection
  (28672 x 4096 INT4, fp16 group-128 scales, 896 row blocks), M = 1 and 2, all rows.
* one full-size c4 layer and one full-size c5 layer through TPStack: every projection against
  the oracle on the input the chain fed it, and the chain's output against the oracle chain.

The checker is the oracle: weights decoded by its C restatement (bit-exact with the numpy one,
tests/test_oracle_c.py), products in float32 on the host. Tolerances are the parity bar of
tests/helpers.py: max |y - r| / max(|r|, 1e-2 rms(r)) <= 1e-2 and relative Frobenius <= 1e-3.
"""

from __future__ import annotations

import functools

import numpy as np
import pytest
import torch

from oracle import packed_ref as ref
from oracle import stack_ref
from tests.helpers import TORCH_OF, assert_close, errors, fast_dequant, to_device

pytestmark = pytest.mark.gpu
DEV = "cuda:0"


@functools.lru_cache(maxsize=2)
def _spec(fmt, rows, cols, bs, kind, seed):
    return ref.make_packed(np.random.default_rng(seed), fmt, rows, cols, bs, kind)


def _x(m, k, dt, seed, scale=1.0):
    rng = np.random.default_rng(seed)
    return torch.from_numpy((rng.standard_normal((m, k)) * scale).astype(np.float32)).to(DEV).to(TORCH_OF[dt])


def _linear(spec, scale_dtype, x, ydt, path):
    from tinygrad_dx12_b200.linalg import _packed_linear, linear_plan

    w = to_device(spec, DEV, scale_dtype)
    plan = linear_plan(w, x.dtype, x.shape[0], TORCH_OF[ydt], path)
    assert plan is not None, f"no {path} kernel for this shape"
    y = _packed_linear(w, x, TORCH_OF[ydt], path)
    torch.cuda.synchronize()
    del w
    return plan, y.float().cpu().numpy()


def test_c3_full_size_gemm():
    spec = _spec("fp6_e3m2", 14336, 4096, 4096, "f16row", 3)
    x = _x(4096, 4096, "float16", 0, 0.125)
    plan, y = _linear(spec, None, x, "float16", "auto")
    assert plan == "gemm"
    r = x.float().cpu().numpy() @ fast_dequant(spec).T
    assert_close(y, r, "float16")


def test_gemm_e8m0_many_tiles_sampled_rows():
    spec = _spec("fp4_e2m1", 28672, 8192, 32, "e8m0", 5)
    x = _x(2048, 8192, "bfloat16", 1)
    plan, y = _linear(spec, "e8m0", x, "bfloat16", "gemm")
    rows = np.arange(0, 28672, 7)
    r = x.float().cpu().numpy() @ fast_dequant(spec, "e8m0", rows=rows).T
    assert_close(y[:, rows], r, "bfloat16")


@pytest.mark.parametrize("m", [1, 2])
@pytest.mark.parametrize("case", ["c5_gate_up", "c4_gate_up"])
def test_decode_gemv_many_row_blocks(case, m):
    if case == "c5_gate_up":
        spec, sdt, xdt = _spec("fp4_e2m1", 57344, 8192, 32, "e8m0", 6), "e8m0", "bfloat16"
    else:
        spec, sdt, xdt = _spec("int4", 28672, 4096, 128, "f16u", 7), None, "float16"
    x = _x(m, spec.shape[1], xdt, 2)
    plan, y = _linear(spec, sdt, x, xdt, "gemv")
    assert plan == "gemv"
    r = x.float().cpu().numpy() @ fast_dequant(spec, sdt).T
    assert_close(y, r, xdt)


class _LazyLayers:
    """Full-size oracle layers built one at a time (a c5 layer decodes to 3.4 GB of float32)."""

    def __init__(self, cfg, n):
        self.cfg, self.n = cfg, n

    def __len__(self):
        return self.n

    def __getitem__(self, layer):
        from tests.stack_helpers import spec_of
        from tinygrad_dx12_b200 import stack as S

        return {p: spec_of(S.make_matrix(self.cfg, layer, p, "cpu")) for p in self.cfg.proj_shapes()}


def _c_linear(spec, x):
    return x.astype(np.float32) @ fast_dequant(spec).T


@pytest.mark.parametrize("name,m", [("c4", 1), ("c4", 16), ("c5", 1)])
def test_full_size_layer(name, m):
    """One full-size layer of the c4 (8B-shaped INT4) or c5 (70B-shaped FP4) stack through the
    CUDA library (fused projections, glue kernels).

    Every projection is checked against the oracle on the activation the GPU chain fed it, with
    the parity bar of tests/helpers.py. The chain's final h is then compared with the oracle
    chain run from the same h0: the chain rounds to the activation dtype after every step, so a
    one-ulp difference in an early rounding (fp32 sums in another order) moves later steps'
    inputs; with bf16 activations (2^-8 relative per ulp) that spread reaches about 1e-3 of h
    after one layer, so the end-to-end bound is 4e-3 (bf16) / 1e-3 (fp16) in relative
    Frobenius norm."""
    from tests.helpers import assert_close
    from tests.stack_helpers import ACT, initial_h, spec_of
    from tinygrad_dx12_b200 import stack as S

    cfg = {"c4": S.C4, "c5": S.C5}[name]

    def on_device(layer, proj):
        from tinygrad_dx12_b200.packed import PackedTensor

        w = S.make_matrix(cfg, layer, proj, "cpu")
        return PackedTensor(w.data.to(DEV), w.format, w.shape, w.scales.to(DEV), w.block_size)

    class Recording(S.CudaOps):
        def __init__(self):
            super().__init__()
            self.calls = []

        def linear(self, w, x, out_dtype):
            y = super().linear(w, x, out_dtype)
            self.calls.append((w, x.clone(), y.clone()))
            return y

    ops = Recording()
    st = S.TPStack(cfg, 0, 1, device=DEV, layers=1, matrix_fn=on_device, ops=ops)
    h = st.forward(initial_h(cfg, m).to(DEV))
    torch.cuda.synchronize()
    assert len(ops.calls) == 4  # qkv, o, gate|up, down
    act = ACT[cfg.act]
    for w, x, y in ops.calls:
        r = x.float().cpu().numpy() @ fast_dequant(spec_of(w)).T
        assert_close(y.float().cpu().numpy(), r, act if y.dtype == cfg.act else "float32")
    y = h.float().cpu().numpy()
    del st, ops
    r = stack_ref.stack_forward(_LazyLayers(cfg, 1), initial_h(cfg, m).float().numpy(), act, _c_linear)
    elem, fro = errors(y, r)
    assert np.all(np.isfinite(y))
    assert fro <= (4e-3 if cfg.act == torch.bfloat16 else 1e-3), f"frobenius {fro:.3e} (elementwise {elem:.3e})"
