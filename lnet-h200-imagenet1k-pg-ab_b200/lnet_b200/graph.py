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
from torch import Tensor, nn


class CudaGraphForward:
    """``runner(x)`` = ``model(x)`` for inputs of ``example``'s shape and dtype
    (or ``model.forward_images`` with ``images=True``), by graph replay.

    An unprepared model is prepared (``prepare_for_inference_``) for that shape.  The
    returned logits tensor is the runner's static output buffer: copy it if it
    must survive the next call.  Parameters must not change after capture.
    """

    def __init__(self, model, example: Tensor, *, images: bool = False, warmup: int = 2):
        if not example.is_cuda:
            raise RuntimeError("CudaGraphForward needs a CUDA example input")
        b = example.shape[0]
        steps = (example.shape[1] // 4) * (example.shape[2] // 4) if images else example.shape[1]
        if getattr(model, "_prepare_spec", None) is None:
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
        # the workspace the graph was captured over stays alive with the graph, even
        # if a later, larger request makes the module allocate a new one
        self._workspace = (getattr(model, "_prep", None) or {}).get("ws")

    def __call__(self, x: Tensor) -> Tensor:
        if x.shape != self.static_in.shape or x.dtype != self.static_in.dtype:
            raise ValueError(f"captured for {tuple(self.static_in.shape)} {self.static_in.dtype}, "
                             f"got {tuple(x.shape)} {x.dtype}")
        self.static_in.copy_(x, non_blocking=True)
        self.graph.replay()
        return self.static_out


def _input_signature(x: Tensor):
    return (tuple(x.shape), x.stride(), x.dtype, x.device, int(x.storage_offset()))


class BorrowedInputCudaGraphInference(nn.Module):
    """Replay one graph over a caller-owned CUDA input allocation (the reference's
    ``BorrowedInputCudaGraphInference``, src/lnet/pac_tight_frame_runtime.py:63-118).

    The first call captures against ``inputs`` itself; later calls must pass that
    same tensor (its contents updated in place), else ``ValueError``.  The output
    is the graph's own buffer unless ``copy_output``.  Metadata is not accepted.
    """

    def __init__(self, model: nn.Module, *, copy_output: bool = False, warmup: int = 2) -> None:
        super().__init__()
        self.model = model
        self.copy_output = copy_output
        self.warmup = warmup
        self.graph: torch.cuda.CUDAGraph | None = None
        self.captured_input: Tensor | None = None
        self.captured_signature = None
        self.captured_ptr: int | None = None
        self.output: Tensor | None = None

    @torch.no_grad()
    def forward(self, inputs: Tensor) -> Tensor:
        if not inputs.is_cuda:
            raise ValueError("manual CUDA Graph inference requires CUDA inputs")
        if self.graph is None:
            side = torch.cuda.Stream(inputs.device)
            side.wait_stream(torch.cuda.current_stream(inputs.device))
            with torch.cuda.stream(side):
                for _ in range(max(1, self.warmup)):
                    self.model(inputs)
            torch.cuda.current_stream(inputs.device).wait_stream(side)
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph):
                self.output = self.model(inputs)
            self.graph = graph
            self._workspace = (getattr(self.model, "_prep", None) or {}).get("ws")
            self.captured_input = inputs
            self.captured_ptr = inputs.data_ptr()
            self.captured_signature = _input_signature(inputs)
        elif inputs is not self.captured_input or inputs.data_ptr() != self.captured_ptr:
            raise ValueError("manual CUDA Graph inference requires the captured input allocation")
        elif _input_signature(inputs) != self.captured_signature:
            raise ValueError("manual CUDA Graph inference requires the captured input layout")
        self.graph.replay()
        return self.output.clone() if self.copy_output else self.output


__all__ = ["BorrowedInputCudaGraphInference", "CudaGraphForward"]
