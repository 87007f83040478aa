"""GraphStep (the counterpart of the reference's TinyJit graph runner, runtime/graph/dx12.py):
a decode step recorded once as a CUDA graph and replayed with new inputs gives the eager result
bit for bit (the same kernels run), on device inputs and on pinned host inputs with a pinned
host output (the host-I/O decode call); wait=True times the replay."""

import numpy as np
import pytest
import torch

from oracle import packed_ref as ref
from tests.helpers import to_device

pytestmark = pytest.mark.gpu
DEV = "cuda:0"


def _weights():
    rng = np.random.default_rng(41)
    w1 = to_device(ref.make_packed(rng, "fp4_e2m1", 512, 1024, 32, "e8m0"), DEV, "e8m0")
    w2 = to_device(ref.make_packed(rng, "int4", 256, 512, 32, "f16u"), DEV)
    return w1, w2


def test_two_projection_step_on_device():
    import tinygrad_dx12_b200 as tg

    w1, w2 = _weights()

    def step(x):
        h = tg.matmul(w1, x.t(), dtype=torch.float16)  # (512, 1)
        return tg.matmul(w2, h, dtype=torch.float16)   # (256, 1)

    xs = [torch.randn((1, 1024), device=DEV).to(torch.float16) for _ in range(3)]
    g = tg.GraphStep(step, xs[0])
    for x in xs:
        want = step(x).clone()
        got = g(x)
        torch.cuda.synchronize()
        assert torch.equal(got, want)
    out, seconds = g(xs[1], wait=True)
    assert torch.equal(out, step(xs[1])) and seconds > 0


def test_host_io_step():
    import tinygrad_dx12_b200 as tg

    w1, _ = _weights()
    yh = torch.empty((1, 512), dtype=torch.bfloat16).pin_memory()

    def step(xh):
        return tg.matmul(w1, xh.t(), dtype=torch.bfloat16, out=yh.t())

    xs = [torch.randn((1, 1024)).to(torch.bfloat16).pin_memory() for _ in range(3)]
    g = tg.GraphStep(step, xs[0])
    for x in xs:
        want = tg.matmul(w1, x.to(DEV).t(), dtype=torch.bfloat16).t().cpu()
        g(x)
        torch.cuda.synchronize()
        assert torch.equal(yh, want)
    with pytest.raises(ValueError):
        g(torch.randn((1, 1024)).to(torch.float16).pin_memory())
