"""Record a decode step once, replay it many times: the counterpart of the reference's TinyJit
graph runner (tinygrad-dx12 src/tinygrad_dx12/runtime/graph/dx12.py:49-253, ``DX12Graph``).

The reference records a kernel sequence into a D3D12 command list and replays it with patched
buffer descriptors, optionally timing the replay (``__call__(..., wait=True)`` returns seconds).
Here the step is any Python function over this library's calls on CUDA tensors (``matmul``,
``matvec``, the layer stacks); it is captured once as a CUDA graph with static input and output
buffers, and each call copies the new inputs into the static ones and replays the graph: every
launch of the step (the fused kernels, the staging copy of host inputs, the reductions) goes out
as one graph launch instead of one host call each.
"""

from __future__ import annotations

import ctypes
import time

import torch


class GraphStep:
    """``step = GraphStep(fn, *inputs)``; ``outputs = step(*new_inputs, wait=False)``.

    ``inputs`` are example tensors (CUDA, or pinned host for the host-I/O decode calls); the step
    keeps static copies of them and captures ``fn(*static_inputs)`` after ``warmup`` eager runs
    on a side stream. A call copies each new input into its static buffer unless it is that
    buffer, replays on the current stream and returns the static outputs (overwritten by the
    next call). ``wait=True`` synchronises and returns ``(outputs, seconds)`` of the replay.
    Host inputs are rewritten only after the previous replay has finished reading them."""

    def __init__(self, fn, *inputs: torch.Tensor, warmup: int = 2):
        if not inputs:
            raise ValueError("GraphStep needs at least one example input")
        self.fn = fn
        self.static = []
        for t in inputs:
            if t.device.type == "cpu":
                if not t.is_pinned():
                    raise ValueError("host inputs of a graph step must be in pinned memory")
                s = torch.empty_like(t, memory_format=torch.contiguous_format).pin_memory()
                s.copy_(t)
            else:
                s = t.clone()
            self.static.append(s)
        # per input: (static buffer, is host, bytes) -- a host input is copied with one memmove
        self._slots = [(s, s.device.type == "cpu", s.numel() * s.element_size()) for s in self.static]
        self._host = any(h for _, h, _ in self._slots)
        self.device = next((t.device for t in inputs if t.device.type == "cuda"), torch.device("cuda", torch.cuda.current_device()))
        side = torch.cuda.Stream(self.device)
        side.wait_stream(torch.cuda.current_stream(self.device))
        with torch.cuda.stream(side):
            for _ in range(warmup):
                fn(*self.static)
        torch.cuda.current_stream(self.device).wait_stream(side)
        torch.cuda.synchronize(self.device)
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph, stream=side):
            self.outputs = fn(*self.static)
        torch.cuda.synchronize(self.device)
        self._done = torch.cuda.Event()
        self._done.record(torch.cuda.current_stream(self.device))

    def __call__(self, *inputs: torch.Tensor, wait: bool = False):
        if len(inputs) not in (0, len(self._slots)):
            raise ValueError(f"GraphStep takes {len(self._slots)} inputs")
        waited = False
        for new, (s, host, nbytes) in zip(inputs, self._slots):
            if new is s:
                continue
            if new.shape != s.shape or new.dtype != s.dtype:
                raise ValueError(f"input of shape {tuple(new.shape)} {new.dtype}, recorded {tuple(s.shape)} {s.dtype}")
            if host:
                if new.device.type != "cpu" or not new.is_contiguous():
                    raise ValueError("a host input of a graph step must be a contiguous host tensor")
                if not waited:  # the previous replay's staging copy has read the old host inputs
                    self._done.synchronize()
                    waited = True
                ctypes.memmove(s.data_ptr(), new.data_ptr(), nbytes)
            else:
                s.copy_(new, non_blocking=True)
        if torch.cuda.current_device() != self.device.index:
            with torch.cuda.device(self.device):
                return self._replay(wait)
        return self._replay(wait)

    def _replay(self, wait: bool):
        if not wait:
            self.graph.replay()
            if self._host:
                self._done.record()  # this device's current stream
            return self.outputs
        stream = torch.cuda.current_stream(self.device)
        t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        t0.record(stream)
        self.graph.replay()
        t1.record(stream)
        self._done.record(stream)
        t1.synchronize()
        return self.outputs, t0.elapsed_time(t1) / 1e3


def time_replays(step: GraphStep, n: int) -> float:
    """Average wall seconds per replay over ``n`` back-to-back replays (inputs unchanged)."""
    torch.cuda.synchronize(step.device)
    t0 = time.perf_counter()
    for _ in range(n):
        step()
    torch.cuda.synchronize(step.device)
    return (time.perf_counter() - t0) / n
