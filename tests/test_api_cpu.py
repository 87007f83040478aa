"""Host-side API semantics that need no GPU: PackedTensor validation (dx12.py:32-47),
matrix_intermediate and dtype rules (dx12.py:115-138, renderer/linalg.py:33-35),
matmul/matvec argument checks (linalg.py:159-167, 240-241), register() idempotence
(compat.py:79-81), and the no-CPU-fallback rule."""

import pytest
import torch

import tinygrad_dx12_b200 as tg
from tinygrad_dx12_b200 import dtypes as D
from tinygrad_dx12_b200.compat import registered


def u8(vals):
    return torch.tensor(vals, dtype=torch.uint8)


def test_register_idempotent():
    tg.register()
    tg.register()
    assert registered()


@pytest.mark.parametrize("kwargs,msg", [
    (dict(data=u8([0]), format="int3", shape=(1,)), "unknown packed format"),
    (dict(data=u8([0]), format="int4", shape=()), "nonnegative"),
    (dict(data=u8([0]), format="int4", shape=(-1,)), "nonnegative"),
    (dict(data=torch.zeros(2, dtype=torch.int8), format="int4", shape=(2,)), "flat uint8"),
    (dict(data=torch.zeros((1, 2), dtype=torch.uint8), format="int4", shape=(2,)), "flat uint8"),
    (dict(data=u8([0]), format="int4", shape=(3,)), "smaller than the declared shape"),
    (dict(data=u8([0, 0]), format="fp6_e3m2", shape=(3,)), "smaller than the declared shape"),
    (dict(data=u8([0]), format="int4", shape=(2,), block_size=0), "block size must be positive"),
    (dict(data=u8([0]), format="int4", shape=(1, 2), scales=torch.ones(1, 2), block_size=1), None),
    (dict(data=u8([0]), format="int4", shape=(1, 2), scales=torch.ones(1, 1), block_size=1), "incompatible"),
])
def test_packed_validation(kwargs, msg):
    if msg is None:
        tg.PackedTensor(**kwargs)
        return
    with pytest.raises(ValueError, match=msg):
        tg.PackedTensor(**kwargs)


def test_storage_rounding_matches_reference():
    # ceil(prod(shape) * bits / 8): 3 six-bit values need 3 bytes (18 bits)
    tg.PackedTensor(u8([0, 0, 0]), "fp6_e2m3", (3,))
    tg.PackedTensor(u8([0]), "uint4", (2,))


def test_matrix_intermediate_rules():
    w = tg.PackedTensor(u8([0]), "fp6_e2m3", (1, 1))
    assert tg.matrix_intermediate(torch.ones(1, 1, dtype=torch.float32), w) == torch.float32
    assert tg.matrix_intermediate(w, w) == torch.float8_e4m3fn
    e5 = tg.PackedTensor(u8([0]), "fp4_e2m1", (1, 1))
    assert tg.matrix_intermediate(e5, torch.ones(1, 1, dtype=torch.float8_e5m2)) == torch.float8_e5m2
    scaled = tg.PackedTensor(u8([0]), "int4", (1, 1), torch.ones(1, 1, dtype=torch.float16))
    assert tg.matrix_intermediate(scaled, torch.ones(1, 1, dtype=torch.float16)) == torch.float32
    assert tg.matrix_intermediate(scaled, torch.ones(1, 1, dtype=torch.bfloat16)) == torch.float32
    i4 = tg.PackedTensor(u8([0]), "int4", (1, 1))
    assert tg.matrix_intermediate(i4, torch.ones(1, 1, dtype=torch.int32)) == torch.int32
    assert tg.matrix_intermediate(i4, torch.ones(1, 1, dtype=torch.float16)) == torch.float16
    u4 = tg.PackedTensor(u8([0]), "uint4", (1, 1))
    assert tg.matrix_intermediate(u4, torch.ones(1, 1, dtype=torch.uint64)) == torch.uint64
    f64 = tg.PackedTensor(u8([0]), "fp4_e2m1", (1, 1), torch.ones(1, 1, dtype=torch.float64), 1)
    assert tg.matrix_intermediate(f64, f64) == torch.float64
    e8 = tg.PackedTensor(u8([0]), "fp4_e2m1", (1, 1), torch.ones(1, 1).to(torch.float8_e8m0fnu), 1)
    assert tg.matrix_intermediate(e8, torch.ones(1, 1, dtype=torch.bfloat16)) == torch.float32


def test_default_unpack_dtypes():
    assert tg.PackedTensor(u8([0]), "int4", (2,)).default_dtype() == torch.int32
    assert tg.PackedTensor(u8([0]), "fp4_e2m1", (2,)).default_dtype() == torch.float32
    s16 = tg.PackedTensor(u8([0]), "int4", (2,), torch.ones(1, dtype=torch.float16))
    assert s16.default_dtype() == torch.float32
    s64 = tg.PackedTensor(u8([0]), "int4", (2,), torch.ones(1, dtype=torch.float64))
    assert s64.default_dtype() == torch.float64


def test_accumulator_rules():
    assert D.accumulator(torch.float16, torch.float16) == torch.float32
    assert D.accumulator(torch.bfloat16, torch.float16) == torch.float32
    assert D.accumulator(torch.int8, torch.int8) == torch.int32
    assert D.accumulator(torch.uint8, torch.uint8) == torch.uint32
    assert D.accumulator(torch.int64, torch.int64) == torch.int64
    assert D.accumulator(torch.float64, torch.float32) == torch.float64


def test_matmul_argument_checks():
    w = tg.PackedTensor(u8([0, 0]), "int4", (2, 2))
    with pytest.raises(ValueError, match="unknown matrix scope"):
        tg.matmul(w, torch.ones(2, 1), scope="Warp")
    with pytest.raises(ValueError, match="compatible rank-two"):
        tg.matmul(w, torch.ones(3, 1))
    with pytest.raises(ValueError, match="compatible rank-two"):
        tg.matmul(w, torch.ones(2))
    with pytest.raises(ValueError, match="matvec expects"):
        tg.matvec(w, torch.ones(3))


def test_no_cpu_fallback():
    """CPU tensors are rejected, never computed on the host."""
    w = tg.PackedTensor(u8([0x21, 0x43]), "uint4", (2, 2))
    with pytest.raises(ValueError, match="CUDA"):
        tg.matmul(w, torch.ones(2, 1))
    with pytest.raises(ValueError, match="CUDA"):
        w.unpack()
