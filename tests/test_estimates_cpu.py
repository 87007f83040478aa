"""Cost estimates of the matrix calls (the reference's Estimates(2*m*n*k, bytes) on its LinAlg
program, tinygrad-dx12 src/tinygrad_dx12/codegen/linalg.py:50-56), on CPU tensors: the
reference's figure at the operand dtypes its matrix program sees, and the bytes the fused
kernels move (the bench's algorithmic bytes)."""

import torch

import tinygrad_dx12_b200 as tg


def _fp4_e8m0(n, k):
    codes = torch.zeros(n * k // 2, dtype=torch.uint8)
    scales = torch.full((n, k // 32), 120, dtype=torch.uint8).view(torch.float8_e8m0fnu)
    return tg.PackedTensor(codes, "fp4_e2m1", (n, k), scales, 32)


def test_c2_headline_bytes():
    w = _fp4_e8m0(8192, 8192)
    x = torch.zeros((1, 8192), dtype=torch.bfloat16)
    e = tg.estimates(w, x.t(), dtype=torch.bfloat16)
    assert e.ops == 2 * 8192 * 8192
    # the reference's matrix program sees the scaled FP4 operand decoded to float32
    assert e.mem == 8192 * 2 + 8192 * 8192 * 4 + 8192 * 2
    # packed codes + E8M0 scales + x + y: the bench's algorithmic bytes for c2 M=1
    assert e.packed_mem == 35_684_352


def test_unscaled_fp6_pair_and_plain_tensors():
    from tinygrad_dx12_b200 import dtypes as D

    size = lambda dt: torch.empty((), dtype=dt).element_size()  # noqa: E731
    a = tg.PackedTensor(torch.zeros(64 * 96 * 6 // 8, dtype=torch.uint8), "fp6_e3m2", (64, 96))
    b = tg.PackedTensor(torch.zeros(96 * 32 * 6 // 8, dtype=torch.uint8), "fp6_e2m3", (96, 32))
    e = tg.estimates(a, b)
    inter = tg.matrix_intermediate(a, b)  # an FP8 type holds both unscaled FP6 operands exactly
    out = D.accumulator(inter, inter)
    assert e.ops == 2 * 64 * 32 * 96
    assert e.mem == 64 * 32 * size(out) + 64 * 96 * size(inter) + 96 * 32 * size(inter)
    assert e.packed_mem == 64 * 32 * size(out) + 64 * 96 * 6 // 8 + 96 * 32 * 6 // 8
    f = tg.estimates(torch.zeros((5, 7), dtype=torch.float16), torch.zeros((7, 3), dtype=torch.float16))
    fo = D.accumulator(torch.float16, torch.float16)
    assert f.ops == 2 * 5 * 3 * 7 and f.mem == f.packed_mem == 5 * 7 * 2 + 7 * 3 * 2 + 5 * 3 * size(fo)


def test_profile_hook_is_optional():
    seen = []
    tg.set_profile_hook(lambda kernel, est: seen.append((kernel, est)))
    tg.set_profile_hook(None)
    assert seen == []
