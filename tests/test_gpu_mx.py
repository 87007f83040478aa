"""The block-scaled tcgen05 decode kernel (B200_PATH_MX, csrc/gemv_mx.cu) against the float32
oracle: FP4 E2M1 / FP6 E2M3 / FP6 E3M2 weights read natively by the tensor cores (kind::mxf4
with x in eight FP4 pieces for FP4 weights at 1-2 tokens; kind::mxf8f6f4 with x in E4M3 pieces
otherwise), E8M0 per-32 weight scales applied by the tensor cores, per-row or no scales, bf16
and fp16 x, 1..64 tokens, and the stream-K work split: tiles finished by one CTA, tiles shared
by two or three, and tiles shared by dozens (fewer units than SMs). Tolerances:
tests/helpers.py."""

from __future__ import annotations

import functools

import numpy as np
import pytest
import torch

from oracle import packed_ref as ref
from tests.helpers import TORCH_OF, assert_close, fast_dequant, oracle_scales, to_device

pytestmark = pytest.mark.gpu
DEV = "cuda:0"


@functools.lru_cache(maxsize=4)
def _spec(fmt, rows, cols, bs, kind, seed):
    return ref.make_packed(np.random.default_rng(seed), fmt, rows, cols, bs, kind)


def _wref(spec, sdt):
    if spec.shape[0] * spec.shape[1] >= 1 << 22:
        return fast_dequant(spec, sdt)
    sc, sd = oracle_scales(spec, sdt)
    return ref.dequant(spec.data, spec.format, spec.shape, sc, spec.block_size, "float32", sd)


def _run(spec, sdt, m, xdt, ydt, seed=0, xscale=1.0, flags=0):
    from tinygrad_dx12_b200.linalg import _packed_linear, linear_plan

    rng = np.random.default_rng(seed)
    w = to_device(spec, DEV, sdt)
    x = torch.from_numpy((rng.standard_normal((m, spec.shape[1])) * xscale).astype(np.float32)).to(DEV).to(TORCH_OF[xdt])
    assert linear_plan(w, x.dtype, m, TORCH_OF[ydt], "mx") == "mx"
    y = _packed_linear(w, x, TORCH_OF[ydt], "mx", flags)
    torch.cuda.synchronize()
    r = x.float().cpu().numpy() @ _wref(spec, sdt).T
    assert_close(y.float().cpu().numpy(), r, ydt)
    return w, x, y


@pytest.mark.parametrize("m", [1, 2, 3, 8, 16, 32, 33, 64])
def test_c2_fp4_e8m0(m):
    """Config c2 (FP4 E2M1 8192 x 8192, per-32 E8M0, bf16 x / y): 64 tiles x 32 stages; at 1..4
    tokens two CTAs of a cluster take a tile's K halves, above that 148 CTAs share the tiles
    (stream-K)."""
    _run(_spec("fp4_e2m1", 8192, 8192, 32, "e8m0", 2), "e8m0", m, "bfloat16", "bfloat16")


@pytest.mark.parametrize("fmt", ["fp4_e2m1", "fp6_e2m3", "fp6_e3m2"])
@pytest.mark.parametrize("kind,sdt", [("e8m0", "e8m0"), ("f16row", None), (None, None)])
@pytest.mark.parametrize("xdt,m", [("bfloat16", 1), ("bfloat16", 7), ("float16", 1), ("float16", 5), ("float16", 42)])
def test_formats_scales_x_dtypes(fmt, kind, sdt, xdt, m):
    bs = 32 if kind != "f16row" else 2048
    spec = _spec(fmt, 1000, 2048, bs, kind, 3)  # 8 stages of 256
    _run(spec, sdt, m, xdt, "float32", xscale=0.25)


@pytest.mark.parametrize("rows,cols", [(128, 512), (129, 512), (300, 1536), (256, 8192), (4768, 1024),
                                       (57344, 8192), (9600, 1024), (9472, 2048)])
@pytest.mark.parametrize("m", [1, 4])
def test_stream_k_splits(rows, cols, m):
    """Both work splits of the 1..4-token FP4 kernel. Pair split (two CTAs per 128-row tile, the
    second pushing its partials to the first through distributed shared memory; matrices of at
    most 74 tiles with an even stage count): ragged rows, one to 38 tiles, 2 to 32 stages, and
    9472 x 2048 with its 148 CTAs filling every SM. Stream-K with tickets: 9600 x 1024 (75 tiles,
    300 units over 148 CTAs) and the c5 gate|up shape (448 tiles x 32 stages); odd stage counts
    (unscaled K = 256) in test_single_stage_unscaled. Per-32 E8M0 scales need K % 512 == 0 here (a 16-byte row of scale bytes
    per TMA box)."""
    _run(_spec("fp4_e2m1", rows, cols, 32, "e8m0", 4), "e8m0", m, "bfloat16", "bfloat16")


@pytest.mark.parametrize("m", [1, 3])
def test_single_stage_unscaled(m):
    """K = 256: one stage per tile (unscaled codes); K = 128 is below one stage and goes to the
    other kernels."""
    from tinygrad_dx12_b200.linalg import linear_plan

    _run(_spec("fp4_e2m1", 300, 256, 32, None, 5), None, m, "bfloat16", "float32")
    short = to_device(_spec("fp4_e2m1", 300, 128, 32, None, 5), DEV)
    assert linear_plan(short, torch.bfloat16, m, torch.float32, "mx") is None
    assert linear_plan(short, torch.bfloat16, m, torch.float32, "auto") is not None


def test_repeated_calls_and_pdl_flag():
    """Back-to-back calls on one stream (tile tickets reset every call), with and without the
    programmatic-dependent-launch flag, give bitwise identical results (fixed reduction order)."""
    spec = _spec("fp4_e2m1", 8192, 8192, 32, "e8m0", 2)
    w, x, y0 = _run(spec, "e8m0", 3, "bfloat16", "float32")
    from tinygrad_dx12_b200.linalg import _packed_linear

    outs = [_packed_linear(w, x, torch.float32, "mx", 0x100 if i % 2 else 0) for i in range(6)]
    torch.cuda.synchronize()
    for o in outs:
        assert torch.equal(o, y0)


@pytest.mark.parametrize("m", [1, 2])
def test_x_blocks_with_zeros_and_wide_range(m):
    """Blocks of x that are all zero, values spanning 2^-20..2^20 inside one block: the error
    of the per-block piece scales stays below 2^-17 of the block maximum, at one token and at
    two."""
    from tinygrad_dx12_b200.linalg import _packed_linear

    spec = _spec("fp4_e2m1", 512, 4096, 32, "e8m0", 7)
    w = to_device(spec, DEV, "e8m0")
    rng = np.random.default_rng(8)
    xv = rng.standard_normal((m, 4096)) * np.exp2(rng.integers(-20, 21, size=(m, 4096)))
    xv[:, 64:128] = 0.0
    x = torch.from_numpy(xv.astype(np.float32)).to(DEV).to(torch.bfloat16)
    y = _packed_linear(w, x, torch.float32, "mx").cpu().numpy()
    r = x.float().cpu().numpy() @ _wref(spec, "e8m0").T
    assert_close(y, r, "float32")


def test_multi_destination_epilogue():
    """b200_packed_linear_multi on this kernel writes the same y to every destination."""
    from tinygrad_dx12_b200.linalg import _packed_linear, _packed_linear_multi
    import ctypes

    spec = _spec("fp4_e2m1", 1024, 4096, 32, "e8m0", 9)
    w = to_device(spec, DEV, "e8m0")
    x = torch.randn((1, 4096), device=DEV).to(torch.bfloat16)
    outs = [torch.full((1, 1024), float("nan"), device=DEV) for _ in range(3)]
    ptrs = (ctypes.c_void_p * 3)(*[o.data_ptr() for o in outs])
    _packed_linear_multi(w, x, ptrs, torch.float32, 1024, flags=4)  # B200_PATH_MX
    expect = _packed_linear(w, x, torch.float32, "mx")
    torch.cuda.synchronize()
    for o in outs:
        assert torch.equal(o, expect)
