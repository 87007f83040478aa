"""Split-K decode GEMM for a few tokens (3 <= M <= 32, and 33..64 for the scale layouts the
tcgen05 GEMM declines; 4-bit formats) against the float32 oracle: every 4-bit format x scale layout (none, per-row, per-32 E8M0 / fp16 / bf16 / fp32,
group 64 / 128 / 512), fp16 and bf16 x, f16 / bf16 / f32 y, token counts on both sides of
the 8-token tile edges, shapes with one and many K slices and a ragged last row block, and
bf16 activations beyond the fp16 range or far below it (the per-token prescale).
Tolerances: tests/helpers.py."""

import functools

import numpy as np
import pytest
import torch

from oracle import packed_ref as ref
from tests.helpers import TORCH_OF, assert_close, oracle_scales, to_device

pytestmark = pytest.mark.gpu
DEV = "cuda:0"


@functools.lru_cache(maxsize=16)
def _case(fmt, rows, cols, bs, kind, seed=0):
    spec = ref.make_packed(np.random.default_rng(seed), fmt, rows, cols, bs, kind)
    return spec


def _check(spec, scale_dtype, m, xdt, ydt, x=None, seed=1):
    from tinygrad_dx12_b200.linalg import _packed_linear, linear_plan

    w = to_device(spec, DEV, scale_dtype)
    if x is None:
        rng = np.random.default_rng(seed)
        x = torch.from_numpy(rng.standard_normal((m, spec.shape[1])).astype(np.float32)).to(DEV).to(TORCH_OF[xdt])
    assert linear_plan(w, x.dtype, m, TORCH_OF[ydt], "gemv") == "gemv"
    y = _packed_linear(w, x, TORCH_OF[ydt], "gemv").float().cpu().numpy()
    sc, sdt = oracle_scales(spec, scale_dtype)
    wf = ref.dequant(spec.data, spec.format, spec.shape, sc, spec.block_size, "float32", sdt)
    assert_close(y, x.float().cpu().numpy() @ wf.T, ydt)


SCALES = [(None, 32, None), ("f16row", 0, None), ("e8m0", 32, "e8m0"), ("e8m0", 32, "bfloat16"),
          ("f16u", 32, "float16"), ("f16u", 32, "float32"), ("f16u", 64, "float16"), ("f16u", 128, "float16"),
          ("f16u", 512, "bfloat16"), ("f16u", 128, "float32"), ("f16u", 64, "float32"), ("e8m0", 128, "e8m0")]


@pytest.mark.parametrize("fmt", ["int4", "uint4", "fp4_e2m1"])
@pytest.mark.parametrize("kind,bs,sdt", SCALES)
@pytest.mark.parametrize("xdt", ["float16", "bfloat16"])
def test_formats_scales(fmt, kind, bs, sdt, xdt):
    spec = _case(fmt, 384, 2048, bs or 2048, kind)
    _check(spec, sdt, 11, xdt, xdt)


@pytest.mark.parametrize("m", [3, 7, 8, 9, 16, 17, 24, 31, 32])
@pytest.mark.parametrize("rows,cols", [(256, 1024), (4096, 4096), (1000, 512)])
def test_token_counts_and_splits(m, rows, cols):
    spec = _case("fp4_e2m1", rows, cols, 32, "e8m0")
    _check(spec, "e8m0", m, "bfloat16", "bfloat16")


@pytest.mark.parametrize("ydt", ["float16", "bfloat16", "float32"])
def test_output_dtypes(ydt):
    spec = _case("int4", 640, 4096, 128, "f16u")
    _check(spec, "float16", 16, "float16", ydt)


@pytest.mark.parametrize("mag", [1e6, 3e-8])
def test_bf16_prescale(mag):
    spec = _case("fp4_e2m1", 256, 2048, 32, "e8m0")
    rng = np.random.default_rng(3)
    x = rng.standard_normal((8, 2048)).astype(np.float32) * mag
    x[2] *= 1e-3  # tokens of different magnitude in one chunk
    xt = torch.from_numpy(x).to(DEV).to(torch.bfloat16)
    _check(spec, "e8m0", 8, "bfloat16", "float32", x=xt)


@pytest.mark.parametrize("exps", [(-20, -15), (10, 20), (-3, 3)])
def test_e8m0_exponent_ranges(exps):
    """E8M0 scales of small, large and mixed exponents (each block's fp32 sum is scaled)."""
    rng = np.random.default_rng(5)
    spec = ref.make_packed(rng, "fp4_e2m1", 256, 2048, 32, None)
    e = rng.integers(exps[0], exps[1] + 1, size=(256, 64))
    spec = ref.PackedSpec(spec.data, spec.format, spec.shape, np.exp2(e).astype(np.float32), 32, "float32")
    _check(spec, "e8m0", 8, "bfloat16", "float32")
    _check(spec, "e8m0", 20, "float16", "float32")


def test_c2_full_size_m8_m32():
    spec = _case("fp4_e2m1", 8192, 8192, 32, "e8m0")
    for m in (8, 32):
        _check(spec, "e8m0", m, "bfloat16", "bfloat16", seed=m)


def test_repeated_calls_reuse_workspace():
    """Split-K tickets reset after each call: many back-to-back calls stay correct."""
    from tinygrad_dx12_b200.linalg import _packed_linear

    spec = _case("int4", 512, 4096, 32, "f16u")
    w = to_device(spec, DEV, "float16")
    x = torch.randn((12, 4096), device=DEV).to(torch.float16)
    ys = [_packed_linear(w, x, torch.float32, "gemv") for _ in range(20)]
    for y in ys[1:]:
        assert torch.equal(y, ys[0])


def test_first_call_on_side_stream():
    """The first split-K call on a new (non-blocking) torch stream creates that stream's
    workspace and clears its tickets on the same stream, so it is ordered before the kernel."""
    from tinygrad_dx12_b200.linalg import _packed_linear

    spec = _case("fp4_e2m1", 1024, 4096, 32, "e8m0", seed=4)
    w = to_device(spec, DEV, "e8m0")
    x = torch.randn((8, 4096), device=DEV).to(torch.bfloat16)
    want = _packed_linear(w, x, torch.float32, "gemv")
    torch.cuda.synchronize()
    for _ in range(3):
        side = torch.cuda.Stream(DEV)
        side.wait_stream(torch.cuda.current_stream(DEV))
        with torch.cuda.stream(side):
            got = _packed_linear(w, x, torch.float32, "gemv")
        side.synchronize()
        assert torch.equal(got, want)


WIDE_SCALES = [("f16u", 32, "float16"), ("f16u", 32, "bfloat16"), ("f16u", 32, "float32"), ("f16u", 128, "float16"),
               ("f16u", 512, "bfloat16")]


@pytest.mark.parametrize("m", [33, 48, 64])
@pytest.mark.parametrize("fmt", ["int4", "fp4_e2m1"])
@pytest.mark.parametrize("kind,bs,sdt", WIDE_SCALES)
@pytest.mark.parametrize("xdt", ["float16", "bfloat16"])
def test_64_token_tile(m, fmt, kind, bs, sdt, xdt):
    """33..64 tokens with the scale layouts the tcgen05 GEMM declines (per-32 non-E8M0, wider
    groups): the 64-token tile, several K slices, ragged rows."""
    spec = _case(fmt, 1000, 2048, bs, kind)
    _check(spec, sdt, m, xdt, xdt)


def test_64_token_tile_auto_plan():
    """The automatic plan takes the decode kernel for c4-like operands at 33..64 tokens and the
    tcgen05 GEMM where it applies (E8M0 per-32 scales)."""
    from tinygrad_dx12_b200.linalg import linear_plan

    c4 = to_device(_case("int4", 512, 4096, 128, "f16u"), DEV, "float16")
    c2 = to_device(_case("fp4_e2m1", 512, 4096, 32, "e8m0"), DEV, "e8m0")
    for m in (33, 64):
        assert linear_plan(c4, torch.float16, m, torch.float16, "auto") == "gemv"
        assert linear_plan(c2, torch.bfloat16, m, torch.bfloat16, "auto") == "gemm"
    assert linear_plan(c4, torch.float16, 65, torch.float16, "auto") == "simt"
