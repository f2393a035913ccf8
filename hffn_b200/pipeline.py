"""Host-to-host forward over a sequence of batches, with the host<->device copies overlapped with the kernels.

A serving loop hands the FFN one batch of tokens after another from pinned host memory and wants each output back in
host memory. Done step by step, a step costs copy in + kernels + copy out; PCIe moves about as many bytes per second
as the kernels consume, so two thirds of the time would be copies. ``HostPipeline`` runs three streams: batch k + 1
is copied in (host-to-device copy engine) while the kernels of batch k run on the caller's stream and the output of
batch k - 1 is copied out (device-to-host copy engine). Device batches are double-buffered; events order every reuse
(a device input is overwritten only after the kernels that read it, a device output only after its copy out). Each
batch's output is the same bits that a plain call gives: the kernels, their order and their inputs are unchanged.

``forward(x, out)`` is any device forward that queues its work on the current stream and writes ``out``:
``HFFNRuntime.forward`` (``runtime_forward``) or a sharded forward.
"""
from __future__ import annotations

from typing import Callable, Sequence

import torch


class HostPipeline:
    def __init__(self, forward: Callable[[torch.Tensor, torch.Tensor], object], d_in: int, d_out: int,
                 max_tokens: int, dtype: torch.dtype, device, depth: int = 2) -> None:
        if depth < 1:
            raise ValueError("depth must be at least 1")
        self.forward = forward
        self.d_in, self.d_out, self.max_tokens, self.dtype = d_in, d_out, max_tokens, dtype
        self.device = torch.device(device)
        self.depth = depth
        self._x = [torch.empty(max_tokens, d_in, dtype=dtype, device=self.device) for _ in range(depth)]
        self._y = [torch.empty(max_tokens, d_out, dtype=dtype, device=self.device) for _ in range(depth)]
        self._copy_in = torch.cuda.Stream(self.device)
        self._copy_out = torch.cuda.Stream(self.device)
        self._loaded = [torch.cuda.Event() for _ in range(depth)]
        self._computed = [torch.cuda.Event() for _ in range(depth)]
        self._drained = [torch.cuda.Event() for _ in range(depth)]
        self._used = [False] * depth

    def _check(self, x: torch.Tensor, y: torch.Tensor) -> int:
        n = x.shape[0] if x.dim() == 2 else -1
        if x.dim() != 2 or x.shape[1] != self.d_in or x.dtype != self.dtype or x.device.type != "cpu" \
                or not x.is_contiguous() or not 1 <= n <= self.max_tokens:
            raise ValueError(f"inputs must be contiguous {self.dtype} [N <= {self.max_tokens}, {self.d_in}] host tensors")
        if y.shape != (n, self.d_out) or y.dtype != self.dtype or y.device.type != "cpu" or not y.is_contiguous():
            raise ValueError(f"outputs must be contiguous {self.dtype} [N, {self.d_out}] host tensors")
        if not (x.is_pinned() and y.is_pinned()):
            raise ValueError("host batches must be in pinned memory (asynchronous copies)")
        return n

    def run(self, xs: Sequence[torch.Tensor], ys: Sequence[torch.Tensor], wait: bool = True) -> None:
        """ys[k] = forward(xs[k]) for every k (pinned host tensors); ``wait``: return once the last output is in host
        memory (else the caller synchronises the device)."""
        if len(xs) != len(ys):
            raise ValueError("as many outputs as inputs")
        sizes = [self._check(x, y) for x, y in zip(xs, ys)]
        compute = torch.cuda.current_stream(self.device)
        for k, (x_host, y_host, n) in enumerate(zip(xs, ys, sizes)):
            b = k % self.depth
            x_dev, y_dev = self._x[b][:n], self._y[b][:n]
            if self._used[b]:
                self._copy_in.wait_event(self._computed[b])      # the kernels that read x_dev are done
                compute.wait_event(self._drained[b])             # the copy out of y_dev is done
            with torch.cuda.stream(self._copy_in):
                x_dev.copy_(x_host, non_blocking=True)
                self._loaded[b].record(self._copy_in)
            compute.wait_event(self._loaded[b])
            self.forward(x_dev, y_dev)
            self._computed[b].record(compute)
            self._copy_out.wait_event(self._computed[b])
            with torch.cuda.stream(self._copy_out):
                y_host.copy_(y_dev, non_blocking=True)
                self._drained[b].record(self._copy_out)
            self._used[b] = True
        # the caller's stream follows the last copy out (its later work and events see the outputs in host memory)
        for b in range(self.depth):
            if self._used[b]:
                compute.wait_event(self._drained[b])
        if wait:
            compute.synchronize()


def runtime_forward(runtime, index: int) -> Callable[[torch.Tensor, torch.Tensor], object]:
    """The device forward of layer ``index`` of an ``HFFNRuntime`` in the form ``HostPipeline`` takes."""
    return lambda x, out: runtime.forward(index, x, out=out)
