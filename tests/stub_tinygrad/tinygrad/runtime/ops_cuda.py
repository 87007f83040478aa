"""Stand-in for tinygrad.runtime.ops_cuda (tests only): records the device string."""


class CUDADevice:
    def __init__(self, device: str):
        self.device = device
