"""tinygrad device module for ``B200`` (installed as ``tinygrad.runtime.ops_b200`` by
``compat.register()``; imported only when tinygrad is installed).

tinygrad looks a device up by importing ``tinygrad.runtime.ops_<name>`` and taking its
``<Name>Device`` class. The reference supplies a whole DX12 device there
(``src/tinygrad_dx12/runtime/ops_dx12.py:150-338``); a B200 is a CUDA device, so ``B200Device``
is tinygrad's CUDA device under the B200 name, and ordinary kernels use tinygrad's CUDA
renderer, compiler and graph runner. Packed matmuls go through this package's library.
"""

from __future__ import annotations

from tinygrad.runtime.ops_cuda import CUDADevice


class B200Device(CUDADevice):
    """tinygrad's CUDA device, addressed as ``B200`` / ``B200:<ordinal>``."""

    def __init__(self, device: str):
        super().__init__(device)
