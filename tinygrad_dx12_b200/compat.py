"""Plugin surface: ``register()`` (tinygrad-dx12 ``src/tinygrad_dx12/compat.py:69-177``).

The reference's ``register()`` is idempotent and opens no hardware. When tinygrad is installed
it makes the backend's runtime module importable under tinygrad's device-module name
(``sys.modules["tinygrad.runtime.ops_dx12"]``, ``compat.py:93-94``), appends the device to
``Device._devices`` (``:95-96``) and puts it first in ``ALL_DEVICES`` (``:175-176``), so
tinygrad tries it first when it picks a default device. This module does the same for the
device ``B200``: its runtime module is ``tinygrad_dx12_b200.runtime_b200``, whose ``B200Device``
is tinygrad's own CUDA device (a B200 is a CUDA device; the DX12 device, allocator, queues and
graph runner that the reference has to supply have a complete counterpart there), registered
under the B200 name. The packed path itself -- ``PackedTensor``, ``matmul``, ``matvec`` -- runs
through this package's library on torch CUDA tensors.

Not built: the reference also wraps five tinygrad compiler hooks (``compat.py:97-174``) to
rewrite scheduled matmuls into its LinAlg kernels. tinygrad is not installable in this build
environment (no network; the pinned revision needs Python 3.14), so there is nothing to write
those hooks against, and registration stops at the device tables. Without tinygrad,
``register()`` only records that it ran.
"""

from __future__ import annotations

import importlib
import sys

DEVICE = "B200"
RUNTIME_MODULE = "tinygrad.runtime.ops_b200"
_registered = False


def register() -> None:
    """Register B200 for explicit use and automatic device selection.

    Repeated calls have no effect. Opens no hardware and changes no installed file. Without a
    tinygrad installation this records the registration and returns.
    """
    global _registered
    if _registered:
        return
    try:
        device = importlib.import_module("tinygrad.device")
    except ImportError:
        _registered = True
        return
    runtime = importlib.import_module("tinygrad_dx12_b200.runtime_b200")
    sys.modules[RUNTIME_MODULE] = runtime
    devices = device.Device._devices
    if DEVICE not in devices:
        devices.append(DEVICE)
    if DEVICE not in device.ALL_DEVICES:
        device.ALL_DEVICES.insert(0, DEVICE)
    _registered = True


def registered() -> bool:
    return _registered
