"""CUDA-graph capture of convrot calls, for the small-M shapes where launches, not kernels, set the time.

At config 5's sizes (cross-attention K/V projections at 256 or 333 text tokens) a convrot linear is three kernels of a
few microseconds each; the host work around them (the module's checks, tensor allocations, the library's argument
checks and tensor-map encoding) costs more than the kernels.  ``CapturedCall`` records the whole call once into a
CUDA graph and replays it: one launch of prerecorded kernels, their tensor maps and launch shapes baked in.

The library is capturable: the calls record kernel launches only (no allocation, no synchronisation inside the
library; outputs come from torch's graph pool), provided each kind of call ran once on the device before the capture
(that first run sets kernel attributes and caches launch facts).  ``CapturedCall`` does that warm-up itself.

A replay reads its inputs from the captured input buffers and writes the same output tensors every time: copy new
inputs in (``__call__`` does) and read or clone the outputs before the next replay.
"""

from __future__ import annotations

from collections.abc import Callable

import torch
from torch import Tensor


class CapturedCall:
    """``fn(*inputs)`` recorded once into a CUDA graph and replayed per call.

    ``example_inputs`` fix the shapes, dtypes and devices of the inputs; ``fn`` must return a tensor (or a tuple of
    tensors) and may use anything captured in its closure (layers, weights) as long as it stays alive.
    """

    def __init__(self, fn: Callable[..., Tensor | tuple[Tensor, ...]], *example_inputs: Tensor, warmup: int = 2):
        if not example_inputs or not all(t.is_cuda for t in example_inputs):
            raise ValueError("CapturedCall needs CUDA example inputs")
        self.inputs = [t.detach().clone() for t in example_inputs]
        side = torch.cuda.Stream(device=self.inputs[0].device)
        side.wait_stream(torch.cuda.current_stream(self.inputs[0].device))
        with torch.cuda.stream(side):
            for _ in range(max(1, warmup)):  # first launches set kernel attributes and launch caches
                fn(*self.inputs)
        torch.cuda.current_stream(self.inputs[0].device).wait_stream(side)
        torch.cuda.synchronize(self.inputs[0].device)
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph):
            self.outputs = fn(*self.inputs)

    def __call__(self, *inputs: Tensor) -> Tensor | tuple[Tensor, ...]:
        if len(inputs) != len(self.inputs):
            raise ValueError(f"expected {len(self.inputs)} inputs, got {len(inputs)}")
        for dst, src in zip(self.inputs, inputs, strict=True):
            if src.shape != dst.shape:
                raise ValueError(f"input shape {tuple(src.shape)} != captured {tuple(dst.shape)}")
            if src.data_ptr() != dst.data_ptr():
                dst.copy_(src, non_blocking=True)
        self.graph.replay()
        return self.outputs


__all__ = ["CapturedCall"]
