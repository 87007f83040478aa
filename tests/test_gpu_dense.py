"""Ordinary fp16 / bf16 matmul (the reference's 'tiled' scope on plain tensors,
codegen/linalg.py:188-189) on the tcgen05 dense GEMM, against a float32 torch reference of
the same product: row- and column-major right operands, ragged M / N / K tails, default
(float32) and explicit output dtypes. Tolerances: tests/helpers.py."""

import numpy as np
import pytest
import torch

from tests.helpers import assert_close

pytestmark = pytest.mark.gpu
DEV = "cuda:0"


@pytest.mark.parametrize("dt", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("m,k,n", [(256, 512, 384), (300, 1000, 200), (33, 64, 1000), (1, 4096, 512), (4096, 256, 4096)])
@pytest.mark.parametrize("rhs_layout", ["row", "col"])
def test_dense_matmul(dt, m, k, n, rhs_layout):
    import tinygrad_dx12_b200 as tg

    g = torch.Generator(device=DEV).manual_seed(m * 7 + n)
    a = torch.randn((m, k), device=DEV, generator=g).to(dt)
    b = torch.randn((k, n), device=DEV, generator=g).to(dt) if rhs_layout == "row" else \
        torch.randn((n, k), device=DEV, generator=g).to(dt).t()
    y = tg.matmul(a, b)
    assert y.dtype == torch.float32  # accumulator dtype by default (renderer/linalg.py:33-35)
    r = a.float() @ b.float()
    assert_close(y.cpu().numpy(), r.cpu().numpy(), "float32")
    y16 = tg.matmul(a, b, dtype=dt)
    assert y16.dtype == dt
    assert_close(y16.float().cpu().numpy(), r.cpu().numpy(), {torch.float16: "float16", torch.bfloat16: "bfloat16"}[dt])


def test_non_16bit_still_tiled():
    import tinygrad_dx12_b200 as tg

    a = torch.randint(-5, 5, (40, 70), device=DEV, dtype=torch.int32)
    b = torch.randint(-5, 5, (70, 30), device=DEV, dtype=torch.int32)
    assert torch.equal(tg.matmul(a, b).cpu(), (a.cpu().long() @ b.cpu().long()).to(tg.matmul(a, b).dtype))
