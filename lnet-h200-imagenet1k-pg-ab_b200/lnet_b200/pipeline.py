"""Host-fed serving loop: the host->device copy of batch k+1 overlaps the
forward of batch k (two device input buffers, a copy stream, CUDA events).

Every batch is still copied from (pinned) host memory and every result is
copied back; only the copies of the next batch run while the current batch
computes, so a step costs max(copy, compute) instead of their sum.
"""

from __future__ import annotations

from collections.abc import Callable, Sequence

import torch
from torch import Tensor


def run_pipelined(fn: Callable[[Tensor], Tensor], host_inputs: Sequence[Tensor],
                  host_outputs: Sequence[Tensor], device: torch.device | int | None = None,
                  start_event: torch.cuda.Event | None = None, copy_streams: int = 1) -> None:
    """``host_outputs[k] <- fn(host_inputs[k] on device)`` for every k.

    Inputs and outputs should be pinned host tensors (the copies are
    asynchronous).  ``fn`` runs on the current stream of ``device``; the
    copies of the inputs run on a separate stream, at most two batches ahead
    of the results.  If ``start_event`` is given it is recorded on the
    current stream before the first copy (the copy stream waits for it).
    Returns when every copy is enqueued; synchronise the current stream to
    wait for the results.  ``copy_streams`` > 1 splits each input copy into
    that many contiguous parts on separate streams (several copy engines).
    """
    if len(host_inputs) != len(host_outputs):
        raise ValueError("host_inputs and host_outputs must have the same length")
    if not host_inputs:
        return
    device = torch.device("cuda", torch.cuda.current_device()) if device is None else \
        torch.device(device)
    compute = torch.cuda.current_stream(device)
    copies = [torch.cuda.Stream(device) for _ in range(max(1, copy_streams))]
    copy = copies[0]
    bufs = [torch.empty(host_inputs[0].shape, dtype=host_inputs[0].dtype, device=device)
            for _ in range(2)]
    free = [torch.cuda.Event() for _ in range(2)]
    if start_event is not None:
        start_event.record(compute)
    for c in copies:
        c.wait_stream(compute)
    part_ready = [[torch.cuda.Event() for _ in copies] for _ in range(2)]
    for k, (xh, oh) in enumerate(zip(host_inputs, host_outputs)):
        s = k % 2
        if xh.shape != bufs[s].shape or xh.dtype != bufs[s].dtype:
            raise ValueError("all host inputs must have the same shape and dtype")
        flat_h, flat_d = xh.reshape(-1), bufs[s].view(-1)
        n = flat_h.numel()
        for j, c in enumerate(copies):
            lo, hi = n * j // len(copies), n * (j + 1) // len(copies)
            with torch.cuda.stream(c):
                if k >= 2:
                    c.wait_event(free[s])  # the forward of batch k - 2 has read this buffer
                flat_d[lo:hi].copy_(flat_h[lo:hi], non_blocking=True)
                part_ready[s][j].record(c)
        for e in part_ready[s]:
            compute.wait_event(e)
        y = fn(bufs[s])
        free[s].record(compute)
        oh.copy_(y, non_blocking=True)
    # keep the buffers alive until the compute stream is done with them
    for b in bufs:
        b.record_stream(compute)


__all__ = ["run_pipelined"]
