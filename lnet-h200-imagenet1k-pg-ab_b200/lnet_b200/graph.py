"""CUDA-graph serving of a prepared B200Alphabet (the role of the reference's
compiled / CUDA-graph inference wrapper, src/lnet/alphabet_backbone.py:1210-1333).

One forward of a fixed request shape is captured once and replayed: the host
issues one graph launch per request instead of the module's Python and seven
kernel launches, which is what dominates small-batch latency.  The fused
route is capture-safe: every per-call tag and counter lives in the prepared
workspace and is advanced on the device.
"""

from __future__ import annotations

import torch
from torch import Tensor


class CudaGraphForward:
    """``runner(x)`` = ``model(x)`` for inputs of ``example``'s shape and dtype
    (or ``model.forward_images`` with ``images=True``), by graph replay.

    The model is prepared (``prepare_for_inference_``) for that shape.  The
    returned logits tensor is the runner's static output buffer: copy it if it
    must survive the next call.  Parameters must not change after capture.
    """

    def __init__(self, model, example: Tensor, *, images: bool = False, warmup: int = 2):
        if not example.is_cuda:
            raise RuntimeError("CudaGraphForward needs a CUDA example input")
        b = example.shape[0]
        steps = (example.shape[1] // 4) * (example.shape[2] // 4) if images else example.shape[1]
        model.prepare_for_inference_(sequence_length=steps, batch_size=b)
        self.model = model
        self.fn = model.forward_images if images else model
        self.static_in = example.clone()
        side = torch.cuda.Stream(example.device)
        side.wait_stream(torch.cuda.current_stream(example.device))
        with torch.no_grad(), torch.cuda.stream(side):
            for _ in range(max(1, warmup)):  # allocations and preparation outside capture
                self.fn(self.static_in)
        torch.cuda.current_stream(example.device).wait_stream(side)
        self.graph = torch.cuda.CUDAGraph()
        with torch.no_grad(), torch.cuda.graph(self.graph):
            self.static_out = self.fn(self.static_in)

    def __call__(self, x: Tensor) -> Tensor:
        if x.shape != self.static_in.shape or x.dtype != self.static_in.dtype:
            raise ValueError(f"captured for {tuple(self.static_in.shape)} {self.static_in.dtype}, "
                             f"got {tuple(x.shape)} {x.dtype}")
        self.static_in.copy_(x, non_blocking=True)
        self.graph.replay()
        return self.static_out


__all__ = ["CudaGraphForward"]
