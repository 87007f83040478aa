"""Plugin surface: ``register()`` (tinygrad-dx12 ``src/tinygrad_dx12/compat.py:69-177``).

The reference's ``register()`` is idempotent, opens no hardware, injects its runtime module
into ``sys.modules``, appends its device to tinygrad's ``Device._devices`` and puts it first in
``ALL_DEVICES``. This module keeps those semantics for the device name ``B200`` when
tinygrad is importable; without tinygrad (this image has none) registration only records
that it happened, and the torch-tensor API in ``packed`` / ``linalg`` is the whole surface.
"""

from __future__ import annotations

import importlib
import sys

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
    if tinygrad_available():
        from tinygrad.device import ALL_DEVICES, Device  # noqa: WPS433 (optional dependency)

        runtime = importlib.import_module("tinygrad_dx12_b200.runtime")
        sys.modules["tinygrad.runtime.ops_b200"] = runtime
        if DEVICE not in Device._devices:
            Device._devices.append(DEVICE)
        if DEVICE not in ALL_DEVICES:
            ALL_DEVICES.insert(0, DEVICE)
    _registered = True


def registered() -> bool:
    return _registered
