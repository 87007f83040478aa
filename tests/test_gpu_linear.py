"""Fused packed linear (GEMV / tcgen05 GEMM / SIMT) against the float32 oracle.

Shapes cover the headline configs (c1 and c2 at full size; c3 at full K with fewer rows --
the full-size c3 GEMM and the other shapes the benchmark times are in test_gpu_fullsize.py),
odd tails, every format and scale dtype, and the three x / y dtypes. Tolerances:
tests/helpers.py.
"""

import functools

import numpy as np
import pytest
import torch

from oracle import packed_ref as ref
from tests.helpers import TORCH_OF, assert_close, oracle_scales, to_device

pytestmark = pytest.mark.gpu
DEV = "cuda:0"


@functools.lru_cache(maxsize=8)
def _spec(fmt, rows, cols, bs, kind, seed):
    return ref.make_packed(np.random.default_rng(seed), fmt, rows, cols, bs, kind)


_WCACHE: dict = {}


def _wref(spec, scale_dtype):
    """float32 oracle weights; cached per live spec object (the entry holds the spec so its
    id cannot be reused by another object while cached)."""
    key = (id(spec), scale_dtype)
    hit = _WCACHE.get(key)
    if hit is None or hit[0] is not spec:
        if len(_WCACHE) > 4:
            _WCACHE.clear()
        sc, sdt = oracle_scales(spec, scale_dtype)
        hit = (spec, ref.dequant(spec.data, spec.format, spec.shape, sc, spec.block_size, "float32", sdt))
        _WCACHE[key] = hit
    return hit[1]


def _run(spec, scale_dtype, m, xdt, ydt, path="auto", seed=0, xscale=1.0):
    import tinygrad_dx12_b200 as tg
    from tinygrad_dx12_b200.linalg import _packed_linear, linear_plan

    rng = np.random.default_rng(seed)
    w = to_device(spec, DEV, scale_dtype)
    x = torch.from_numpy((rng.standard_normal((m, spec.shape[1])) * xscale).astype(np.float32)).to(DEV).to(TORCH_OF[xdt])
    plan = linear_plan(w, x.dtype, m, TORCH_OF[ydt], path)
    if plan is None:
        pytest.skip(f"path {path} does not take fmt={spec.format} scale={scale_dtype} m={m} x={xdt}")
    y = _packed_linear(w, x, TORCH_OF[ydt], path).float().cpu().numpy()
    r = x.float().cpu().numpy() @ _wref(spec, scale_dtype).T
    assert_close(y, r, ydt)
    return plan, x, w, y


PATHS = ["auto", "gemv", "simt", "gemm"]


@pytest.mark.parametrize("path", PATHS)
@pytest.mark.parametrize("m", [1, 2, 3, 8, 17, 32])
def test_c1_int4_gemv(path, m):
    """Config c1 shape: INT4 4096x4096, per-32 fp16 scales, fp16 x and y."""
    spec = _spec("int4", 4096, 4096, 32, "f16u", 1)
    _run(spec, None, m, "float16", "float16", path)


@pytest.mark.parametrize("path", PATHS)
@pytest.mark.parametrize("m", [1, 8, 32])
@pytest.mark.parametrize("scale", ["e8m0", "bfloat16"])
def test_c2_fp4_gemv(path, m, scale):
    """Config c2: FP4 E2M1 8192x8192, per-32 2^e scales (E8M0 bytes or decoded bf16), bf16 x/y."""
    spec = _spec("fp4_e2m1", 8192, 8192, 32, "e8m0", 2)
    _run(spec, scale, m, "bfloat16", "bfloat16", path)


@pytest.mark.parametrize("path", PATHS)
@pytest.mark.parametrize("m", [64, 256, 300])
def test_c3_fp6_gemm_reduced(path, m):
    """Config c3 at full K=4096 with 1024 rows: FP6 E3M2, per-row fp16 scales, fp16 x (N(0,1)/8)."""
    spec = _spec("fp6_e3m2", 1024, 4096, 4096, "f16row", 3)
    _run(spec, None, m, "float16", "float16", path, xscale=0.125)


@pytest.mark.parametrize("fmt", list(ref.FORMATS))
@pytest.mark.parametrize("scale", [None, "float16", "bfloat16", "float32", "e8m0"])
@pytest.mark.parametrize("xdt", ["float16", "bfloat16", "float32"])
@pytest.mark.parametrize("m", [1, 5, 33, 130])
def test_formats_scales_dtypes(fmt, scale, xdt, m):
    rng = np.random.default_rng(7)
    kind = None if scale is None else ("e8m0" if scale == "e8m0" else "f16u")
    spec = ref.make_packed(rng, fmt, 384, 512, 64, kind)
    if scale not in (None, "e8m0"):
        spec = ref.PackedSpec(spec.data, fmt, spec.shape, spec.scales.astype(ref.np_dtype(scale)), 64)
    _run(spec, scale, m, xdt, "float32", "auto")


@pytest.mark.parametrize("rows,cols,m", [(1, 32, 1), (3, 64, 2), (129, 96, 7), (1000, 160, 33), (17, 4096, 1)])
@pytest.mark.parametrize("fmt", ["int4", "fp6_e2m3"])
def test_odd_shapes(rows, cols, m, fmt):
    spec = ref.make_packed(np.random.default_rng(rows), fmt, rows, cols, 32, "f16u")
    _run(spec, None, m, "float16", "float32", "auto")


@pytest.mark.parametrize("rows", [4736, 4768])
@pytest.mark.parametrize("fmt,kind,scale", [("fp4_e2m1", "e8m0", "e8m0"), ("fp6_e3m2", "f16u", None),
                                            ("int4", "f16u", None)])
@pytest.mark.parametrize("m", [1, 2])
def test_decode_gemv_consumer_counts(rows, fmt, kind, scale, m):
    """148 and 149 row blocks of 32 rows: on a 148-SM B200 the streamed GEMV runs 16 consumer
    warps per CTA in the first case (one row block per CTA) and 8 in the second."""
    spec = _spec(fmt, rows, 1024, 32, kind, 5)
    _run(spec, scale, m, "bfloat16", "bfloat16", "gemv")


@pytest.mark.parametrize("ydt", ["float16", "bfloat16", "float32"])
def test_output_dtypes(ydt):
    spec = ref.make_packed(np.random.default_rng(11), "fp4_e2m1", 512, 1024, 32, "e8m0")
    _run(spec, "e8m0", 4, "bfloat16", ydt)


def test_public_api_call_forms():
    """matmul(W, x.T).T and matvec(W, v) give the same numbers as the fused call."""
    import tinygrad_dx12_b200 as tg

    spec = ref.make_packed(np.random.default_rng(5), "int4", 256, 512, 32, "f16u")
    w = to_device(spec, DEV)
    x = torch.randn(3, 512, device=DEV, dtype=torch.float16)
    y = tg.matmul(w, x.t())
    assert y.shape == (256, 3) and y.dtype == torch.float32
    r = ref.packed_linear_ref(spec, x.float().cpu().numpy())
    assert_close(y.t().cpu().numpy(), r, "float32")
    v = tg.matvec(w, x[0])
    assert v.shape == (256,) and v.dtype == torch.float32
    assert_close(v.cpu().numpy()[None], r[:1], "float32")
    v16 = tg.matvec(w, x[0], torch.float16)
    assert v16.dtype == torch.float16
    vt = tg.matvec(w, x[0], thread=True)
    assert_close(vt.cpu().numpy()[None], r[:1], "float32")
    vf = tg.matvec(w, x[0], thread=False)
    assert_close(vf.cpu().numpy()[None], r[:1], "float32")
    yt = tg.matmul(w, x.t(), scope="tiled")
    assert_close(yt.t().cpu().numpy(), r, "float32")
    # a non-transposed (K, M) right operand is staged and gives the same result
    yc = tg.matmul(w, x.t().contiguous(), dtype=torch.float16)
    assert yc.dtype == torch.float16
    assert_close(yc.t().float().cpu().numpy(), r, "float16")


@pytest.mark.parametrize("m", [1, 2, 8])
def test_e8m0_special_bytes(m):
    """E8M0 byte 0 (2^-127, an fp32 subnormal), byte 255 (NaN) and extreme exponents next to
    ordinary ones: the decode kernels (one or two tokens; eight) convert bytes 1..254 with a shift
    and must take the exact conversion for bytes 0 and 255. Row 0 is scaled by 2^-127 everywhere and is compared after
    rescaling; row 3 has one NaN block scale, so its outputs are NaN."""
    from tinygrad_dx12_b200.linalg import _packed_linear

    rng = np.random.default_rng(21)
    base = ref.make_packed(rng, "fp4_e2m1", 256, 2048, 32, None)
    e = rng.integers(-10, 11, size=(256, 64))
    e[0, :] = -127
    e[1:, ::7] = -127
    e[5, 3] = -120
    spec = ref.PackedSpec(base.data, base.format, base.shape, np.exp2(e.astype(np.float64)).astype(np.float32), 32,
                          "float32")
    w = to_device(spec, DEV, "e8m0")
    w.scales.view(torch.uint8)[3, 5] = 255
    x = torch.from_numpy(rng.standard_normal((m, 2048)).astype(np.float32)).to(DEV).to(torch.bfloat16)
    y = _packed_linear(w, x, torch.float32, "gemv").cpu().numpy()
    wf = ref.dequant(spec.data, spec.format, spec.shape, spec.scales, 32, "float32", "float32")
    r = x.float().cpu().numpy() @ wf.T
    assert np.isnan(y[:, 3]).all()
    keep = np.arange(256) != 3
    assert_close(y[:, 1:][:, keep[1:]], r[:, 1:][:, keep[1:]], "float32")
    y0, r0 = y[:, 0].astype(np.float64) * 2.0**127, r[:, 0].astype(np.float64) * 2.0**127
    assert np.all(np.abs(y0 - r0) <= 1e-3 * np.maximum(np.abs(r0), 1.0))


@pytest.mark.parametrize("m", [1, 2])
@pytest.mark.parametrize("edge", ["finite", "beyond"])
def test_gemv_bf16_beyond_fp16(m, edge):
    """The decode GEMV stages bf16 x as fp16: 65280 (the largest bf16 below 2^16) stays finite,
    65536 and beyond take the power-of-two prescale; both match the oracle."""
    from tinygrad_dx12_b200.linalg import _packed_linear

    rng = np.random.default_rng(23)
    spec = ref.make_packed(rng, "fp4_e2m1", 512, 2048, 32, "e8m0")
    w = to_device(spec, DEV, "e8m0")
    x = rng.standard_normal((m, 2048)).astype(np.float32)
    x[:, 7] = 65280.0 if edge == "finite" else 65536.0
    x[:, 900] = -65280.0 if edge == "finite" else -3.0e6
    xt = torch.from_numpy(x).to(DEV).to(torch.bfloat16)
    y = _packed_linear(w, xt, torch.float32, "gemv").cpu().numpy()
    wf = ref.dequant(spec.data, spec.format, spec.shape, oracle_scales(spec, "e8m0")[0], 32, "float32",
                     oracle_scales(spec, "e8m0")[1])
    assert_close(y, xt.float().cpu().numpy() @ wf.T, "float32")


@pytest.mark.parametrize("bs", [64, 128, 256, 512])
@pytest.mark.parametrize("scale", ["float16", "bfloat16", "float32"])
@pytest.mark.parametrize("m", [1, 2])
@pytest.mark.parametrize("fmt", ["int4", "fp6_e3m2"])
def test_group_scales_decode_gemv(bs, scale, m, fmt):
    """Group scales wider than one 32-payload block (c4 uses 128) on the decode GEMV."""
    spec = _spec(fmt, 320, 2048, bs, "f16u", 31)
    plan, *_ = _run(spec, scale, m, "float16", "float16", "gemv")
    assert plan == "gemv"


@pytest.mark.parametrize("rows,cols", [(4096, 14336), (4768, 4096), (4736, 4096), (320, 4096)])
@pytest.mark.parametrize("bs,scale", [(64, "bfloat16"), (128, "float16"), (256, "float32"), (512, "float32")])
@pytest.mark.parametrize("m", [1, 2])
def test_group_scales_streamed_gemv(rows, cols, bs, scale, m):
    """Group scales on the streamed decode GEMV (c4 projections use INT4 with fp16 group-128
    scales): each stage stages a 16-byte-aligned box of group scales per row and indexes the
    stage's groups inside it; both consumer-warp counts (4736 / 4768 rows)."""
    spec = _spec("int4", rows, cols, bs, "f16u", 43)
    plan, *_ = _run(spec, scale, m, "float16", "float16", "gemv")
    assert plan == "gemv"


@pytest.mark.parametrize("bs", [32, 128])
def test_gemm_rejects_inexact_group_scales(bs):
    """Non-power-of-two group scales cannot be folded exactly into a 16-bit tcgen05 operand
    (weight x scale needs up to 15 significant bits); the GEMM path declines them. The decode
    kernel's 64-token tile takes them up to 64 tokens (config c4 at M=64), the fp32 SIMT kernel
    beyond."""
    import tinygrad_dx12_b200 as tg  # noqa: F401
    from tinygrad_dx12_b200.linalg import linear_plan

    spec = _spec("int4", 512, 4096, bs, "f16u", 41)
    w = to_device(spec, DEV, "float16")
    assert linear_plan(w, torch.float16, 64, torch.float16, "gemm") is None
    assert linear_plan(w, torch.float16, 64, torch.float16, "auto") == "gemv"
    assert linear_plan(w, torch.float16, 65, torch.float16, "auto") == "simt"


@pytest.mark.parametrize("m", [1, 8, 64])
@pytest.mark.parametrize("dt", [torch.bfloat16, torch.float16])
def test_dtype_argument_and_cast_call_forms(m, dt):
    """The two call forms of a low-precision output: ``matmul(W, x.T, dtype=dt)`` and
    ``matmul(W, x.T).cast(dt)`` (the form the benchmark configs name: fp32 accumulate, 16-bit
    output). The reference's ``dtype=`` also makes tinygrad accumulate in ``dt``
    (codegen/linalg.py:173-174); here every fused kernel accumulates in fp32 and rounds once, so
    both forms are checked against the fp32 oracle rounded to ``dt`` and agree to one ulp."""
    import tinygrad_dx12_b200 as tg

    spec = _spec("fp4_e2m1", 2048, 4096, 32, "e8m0", 9)
    w = to_device(spec, DEV, "e8m0")
    x = torch.randn((m, 4096), device=DEV).to(dt)
    y_dtype = tg.matmul(w, x.t(), dtype=dt)
    y_cast = tg.matmul(w, x.t()).to(dt)
    assert y_dtype.dtype == dt and y_cast.dtype == dt and y_dtype.shape == (2048, m)
    r = x.float().cpu().numpy() @ _wref(spec, "e8m0").T
    name = "bfloat16" if dt == torch.bfloat16 else "float16"
    assert_close(y_dtype.t().float().cpu().numpy(), r, name)
    assert_close(y_cast.t().float().cpu().numpy(), r, name)
    ulp = 2.0 ** (-8 if dt == torch.bfloat16 else -11)
    diff = (y_dtype.float() - y_cast.float()).abs()
    assert torch.all(diff <= ulp * y_cast.float().abs() * 2 + 1e-30)


def test_profile_hook_reports_kernel_and_estimates():
    """set_profile_hook sees every matmul with the kernel that ran and its Estimates."""
    import tinygrad_dx12_b200 as tg

    rng = np.random.default_rng(11)
    spec = ref.make_packed(rng, "fp4_e2m1", 256, 512, 32, "e8m0")
    w = to_device(spec, "cuda:0", "e8m0")
    x = torch.randn((2, 512), device="cuda:0").to(torch.bfloat16)
    seen = []
    tg.set_profile_hook(lambda kernel, est: seen.append((kernel, est)))
    try:
        tg.matmul(w, x.t(), dtype=torch.bfloat16)
        tg.matmul(w, x.t(), scope="tiled", dtype=torch.bfloat16)
    finally:
        tg.set_profile_hook(None)
    torch.cuda.synchronize()
    assert [k for k, _ in seen][1] == "generic" and seen[0][0] in ("mx", "gemv", "gemm", "simt")
    assert seen[0][1] == tg.estimates(w, x.t(), dtype=torch.bfloat16)
    assert seen[0][1].ops == 2 * 256 * 2 * 512


@pytest.mark.parametrize("afmt,akind,bfmt,bkind", [("fp4_e2m1", None, "fp4_e2m1", None),
                                                   ("fp6_e3m2", "e8m0", "fp4_e2m1", None),
                                                   ("fp4_e2m1", "e8m0", "fp6_e2m3", "e8m0")])
@pytest.mark.parametrize("n", [1, 3, 64, 300])
def test_packed_pair_runs_fused(afmt, akind, bfmt, bkind, n):
    """Packed x packed (dx12.py:115-138): the right operand's FP4 / FP6 codes (unscaled or E8M0)
    decode exactly to bf16 and the product runs on the fused tensor-core kernels with the left
    operand as the weights; the result matches the oracle's float32 product of both decodes, in
    the float32 accumulator dtype. The tiled scope keeps the ordinary kernel."""
    import tinygrad_dx12_b200 as tg

    sa = _spec(afmt, 256, 512, 32, akind, 21)
    sb = _spec(bfmt, 512, n, 32, bkind, 22)
    a = to_device(sa, DEV, "e8m0" if akind else None)
    b = to_device(sb, DEV, "e8m0" if bkind else None)
    seen = []
    tg.set_profile_hook(lambda kernel, est: seen.append(kernel))
    try:
        y = tg.matmul(a, b)
        yt = tg.matmul(a, b, scope="tiled")
    finally:
        tg.set_profile_hook(None)
    torch.cuda.synchronize()
    assert y.dtype == torch.float32 and seen[0] in ("mx", "gemv", "gemm", "simt") and seen[1] == "generic"
    r = _wref(sa, "e8m0" if akind else None) @ _wref(sb, "e8m0" if bkind else None)
    assert_close(y.cpu().numpy(), r, "float32")
    assert_close(yt.float().cpu().numpy(), r, "float32")


@pytest.mark.parametrize("m,fmt,sk", [(1, "fp4_e2m1", "e8m0"), (2, "fp4_e2m1", "e8m0"), (8, "int4", "f16u"),
                                      (64, "fp6_e3m2", "f16row")])
def test_host_activation_and_out(m, fmt, sk):
    """Pinned host x and a pinned host out (decode steps fed from and returning to the host):
    the result equals the all-device call bit for bit (same kernel), whether the kernel stores
    into out itself (decode kernels) or through a device buffer (the GEMM)."""
    import tinygrad_dx12_b200 as tg

    spec = _spec(fmt, 1024, 2048, 2048 if sk == "f16row" else 32, sk, 31)
    w = to_device(spec, DEV, "e8m0" if sk == "e8m0" else None)
    xdt = torch.bfloat16 if sk == "e8m0" else torch.float16
    xd = torch.randn((m, 2048), device=DEV).to(xdt)
    ref_y = tg.matmul(w, xd.t(), dtype=xdt)
    xh = xd.cpu().pin_memory()
    yh = torch.full((m, 1024), float("nan"), dtype=xdt).pin_memory()
    for _ in range(2):  # the staging buffer and out reused across calls
        got = tg.matmul(w, xh.t(), dtype=xdt, out=yh.t())
        torch.cuda.synchronize()
        assert got.data_ptr() == yh.data_ptr()
        assert torch.equal(yh, ref_y.t().cpu())
    yd = torch.empty((1024, m), device=DEV, dtype=xdt)
    assert tg.matmul(w, xh.t(), dtype=xdt, out=yd) is yd
    torch.cuda.synchronize()
    assert torch.equal(yd.cpu(), ref_y.cpu())
    with pytest.raises(ValueError):
        tg.matmul(w, xd.cpu().t(), dtype=xdt)  # host operand not pinned
    with pytest.raises(ValueError):
        tg.matmul(w, xh.t(), dtype=xdt, out=torch.empty((1024, m), dtype=torch.float32).pin_memory())
