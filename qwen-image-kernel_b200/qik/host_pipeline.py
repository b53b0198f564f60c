"""Host-buffer pipeline: a device function run over a sequence of batches that live in
pinned host memory, with the host->device copy of the next batch and the device->host
copy of the previous one overlapping the current batch's kernels.

A serving process receives activations in host memory and returns results to host
memory.  Done one batch at a time on one stream, the two PCIe copies and the kernels run
back to back.  PCIe is full duplex and the copies run on the copy engines, not the SMs,
so with ``depth`` device slots the three stages overlap and a batch costs
max(h2d, kernels, d2h) instead of their sum.

Ordering, per slot ``s`` (batch ``i`` uses slot ``i % depth``):

* h2d stream: waits until the kernels of batch ``i - depth`` have read ``x[s]``, copies
  the host input into ``x[s]``;
* compute (the caller's current stream): waits for that copy and for the device->host
  copy of batch ``i - depth`` out of ``y[s]``, then runs ``fn(x[s], y[s])``;
* d2h stream: waits for the kernels, copies ``y[s]`` into the host output.

The results are the ones ``fn`` gives when called directly: only the copies move.
"""
from __future__ import annotations

from typing import Callable, Sequence

import torch


class HostPipeline:
    """Runs ``fn(x_dev, y_dev)`` (which must write its whole result into ``y_dev`` on
    torch's current stream) over pinned host batches.

    ``submit(x_host, y_host)`` queues one batch and returns at once with a CUDA event;
    when the event has completed, ``y_host`` holds the batch's result and ``x_host`` may
    be reused.  ``synchronize()`` waits for every queued batch.
    """

    def __init__(self, fn: Callable[[torch.Tensor, torch.Tensor], object], in_shape: Sequence[int],
                 out_shape: Sequence[int], dtype: torch.dtype = torch.bfloat16,
                 device: torch.device | str | int | None = None, depth: int = 2):
        if depth < 1:
            raise ValueError("HostPipeline: depth must be >= 1")
        self.device = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
        if self.device.type != "cuda":
            raise ValueError("HostPipeline: the device must be a CUDA device")
        self.fn = fn
        self.depth = depth
        self.x = [torch.empty(tuple(in_shape), dtype=dtype, device=self.device) for _ in range(depth)]
        self.y = [torch.empty(tuple(out_shape), dtype=dtype, device=self.device) for _ in range(depth)]
        self.h2d_stream = torch.cuda.Stream(self.device)
        self.d2h_stream = torch.cuda.Stream(self.device)
        with torch.cuda.device(self.device):
            # the slots come from the allocator of the current stream: order the copy
            # streams after it once, and keep the memory from being reused while a copy
            # that touches it may still run
            self.h2d_stream.wait_stream(torch.cuda.current_stream(self.device))
        for t in self.x:
            t.record_stream(self.h2d_stream)
        for t in self.y:
            t.record_stream(self.d2h_stream)
        self._x_ready = [torch.cuda.Event() for _ in range(depth)]
        self._computed = [torch.cuda.Event() for _ in range(depth)]
        self._y_free = [torch.cuda.Event() for _ in range(depth)]
        self._count = 0

    def _check_host(self, t: torch.Tensor, dev: torch.Tensor, name: str) -> None:
        if t.device.type != "cpu" or not t.is_pinned():
            raise ValueError(f"HostPipeline: {name} must be a pinned host tensor")
        if t.shape != dev.shape or t.dtype != dev.dtype or not t.is_contiguous():
            raise ValueError(f"HostPipeline: {name} must be contiguous {tuple(dev.shape)} {dev.dtype}")

    def submit(self, x_host: torch.Tensor, y_host: torch.Tensor) -> torch.cuda.Event:
        s = self._count % self.depth
        self._check_host(x_host, self.x[s], "x_host")
        self._check_host(y_host, self.y[s], "y_host")
        reuse = self._count >= self.depth
        with torch.cuda.device(self.device):
            compute = torch.cuda.current_stream(self.device)
            # the copy engine may only overwrite x[s] once batch i - depth's kernels are done
            if reuse:
                self.h2d_stream.wait_event(self._computed[s])
            with torch.cuda.stream(self.h2d_stream):
                self.x[s].copy_(x_host, non_blocking=True)
                self._x_ready[s].record(self.h2d_stream)
            compute.wait_event(self._x_ready[s])
            if reuse:
                compute.wait_event(self._y_free[s])
            self.fn(self.x[s], self.y[s])
            self._computed[s].record(compute)
            self.d2h_stream.wait_event(self._computed[s])
            with torch.cuda.stream(self.d2h_stream):
                y_host.copy_(self.y[s], non_blocking=True)
                self._y_free[s].record(self.d2h_stream)
                done = torch.cuda.Event(enable_timing=True)
                done.record(self.d2h_stream)
        self._count += 1
        return done

    def synchronize(self) -> None:
        self.d2h_stream.synchronize()
        torch.cuda.current_stream(self.device).synchronize()
