"""Stand-in for tinygrad.device: the device registries (tests only)."""

ALL_DEVICES = ["METAL", "AMD", "NV", "CUDA", "QCOM", "GPU", "CPU", "LLVM", "WEBGPU"]


class _Device:
    def __init__(self):
        self._devices = ["CPU", "CUDA", "NV", "PYTHON"]


Device = _Device()
