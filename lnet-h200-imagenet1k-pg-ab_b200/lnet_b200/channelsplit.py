"""Channel (mode) split of the ALPHABET forward over ranks.

BASELINE config 5 (B=16, T=65536, D=256, M=64) has fewer rows than a node has
GPUs; besides the time split (``lnet_b200.timesplit``) its rows can be
partitioned by channel.  Under ALPHABET semantics the D model channels are
mixed by RMSNorm and by the frames, so what splits without an exchange is the
set of complex MODES of each block:

1. every rank runs the stem on the whole request (x is available to all);
2. the writer: each rank computes the drive, the scan and the lag moments of
   its contiguous slice of modes only (``lnet_b200_block_drive`` /
   ``_scan`` / ``_moment_sums`` on a mode-subset parameter set), and its
   partial synthesis s_r (ls W_r)^T; rank 0 adds the residual base
   x + ls ds xhat.  One all-reduce of [B, T, D] fp32 sums the partials into
   the writer stream v -- the only large exchange;
3. the reader: every rank applies the conv to the full v, then drive, scan
   and moments of its modes;
4. one all-gather of the per-rank moment sums [2, B, 7 M_r] (fp64) assembles
   [2, B, 7M]; every rank divides by T / T - lag and evaluates the head.

The all-reduce carries the fp32 stream, 4 B T D bytes (1.07 GB at config 5),
so this split is measured, not recommended: the time split exchanges kilobytes.  Static poles only (no time_delta or masks), the general
route's pieces (fp32 states, bf16 drive operands for bf16 requests).

The per-rank computation is a generator yielding its collectives, run over NCCL
by :func:`channelsplit_forward` and in lockstep in one process by
:func:`channelsplit_emulate` (checks).
"""

from __future__ import annotations

import torch
import torch.distributed as dist
from torch import Tensor

from . import _lib
from .alphabet import _workspace_bytes
from .sharding import shard_bounds
from .timesplit import LAGS, _call_conv, _call_stem, _Pieces, drive_program, run_lockstep


def mode_bounds(modes: int, world: int, rank: int) -> tuple[int, int]:
    """Contiguous balanced slice [lo, hi) of the complex modes owned by `rank`."""
    return shard_bounds(modes, world, rank)


def _subset(model, device, lo: int, hi: int):
    """(params, tensors) of the model restricted to modes [lo, hi) of both blocks: the
    frames' re and im columns of those modes and their pole parameters."""
    params, tensors = model._effective(device)
    m = model.modes
    cols = torch.cat([torch.arange(lo, hi), torch.arange(m + lo, m + hi)]).to(device)
    sub = dict(tensors)
    for blk in ("writer", "reader"):
        sub[f"{blk}_frame"] = tensors[f"{blk}_frame"].index_select(1, cols).contiguous()
        sub[f"{blk}_raw_decay"] = tensors[f"{blk}_raw_decay"][lo:hi].contiguous()
        sub[f"{blk}_raw_frequency"] = tensors[f"{blk}_raw_frequency"][lo:hi].contiguous()
    p = _lib.AlphabetParams(
        raw_input_dim=params.raw_input_dim, model_dim=params.model_dim, modes=hi - lo,
        output_dim=params.output_dim, conv_kernel=params.conv_kernel,
        conv_dilation=params.conv_dilation,
        **{name: sub[name].data_ptr() for name in _lib.PARAM_POINTER_FIELDS})
    return p, sub


class _SubsetPieces(_Pieces):
    """The block pieces of one rank's modes (B rows, all T steps)."""

    def __init__(self, model, ref: Tensor, batch: int, steps: int, act: int, lo: int, hi: int):
        super().__init__(model, ref, batch, steps, act)
        self.params, self._keep = _subset(model, ref.device, lo, hi)
        self.nbytes = _workspace_bytes(self.params, self.req)
        self.ws = torch.empty(max(self.nbytes, 1), dtype=torch.uint8, device=ref.device)


def _rank_program(model, x: Tensor, rank: int, world: int):
    """One rank's forward; yields ("sum", t) -> sum over ranks, ("gather", t) -> stacked."""
    b, t_len, _ = x.shape
    m, d = model.modes, model.model_dim
    if m < world:
        raise ValueError(f"channel split needs at least one mode per rank (M={m}, ranks={world})")
    dev = x.device
    act = _lib.LNET_BF16 if x.dtype == torch.bfloat16 else _lib.LNET_F32
    bounds = [mode_bounds(m, world, r) for r in range(world)]
    lo, hi = bounds[rank]
    mr = hi - lo
    mmax = max(h - l for l, h in bounds)
    with torch.no_grad():
        first = _call_stem(model, x.contiguous(), act)  # replicated [B, T, D] fp32
        pc = _SubsetPieces(model, first, b, t_len, act, lo, hi)
        sums = torch.zeros(2, b, 7 * mmax, dtype=torch.float64, device=dev)
        # writer block: this rank's modes
        u = torch.empty(b, t_len, 2 * mr, device=dev)
        xhat = torch.empty(b, t_len, d, device=dev)
        pc.drive(0, first, u, xhat)
        pc.scan(0, u, None)
        part = torch.zeros(b, 7 * mr, dtype=torch.float64, device=dev)
        pc.sums(u, None, part)
        sums[0, :, :7 * mr] = part
        partial = torch.empty(b, t_len, d, device=dev)
        if rank == 0:
            pc.writer_output(u, xhat, first, partial)  # base + this rank's synthesis
        else:
            zero = torch.zeros_like(first)
            pc.writer_output(u, zero, zero, partial)  # synthesis only
        stream = yield ("sum", partial)
        # reader block on the full stream
        second = _call_conv(model, stream.contiguous(), act)
        u2 = torch.empty(b, t_len, 2 * mr, device=dev)
        pc.drive(1, second, u2, None)
        pc.scan(1, u2, None)
        part = torch.zeros(b, 7 * mr, dtype=torch.float64, device=dev)
        pc.sums(u2, None, part)
        sums[1, :, :7 * mr] = part
        gathered = yield ("gather", sums)  # [G, 2, B, 7 mmax]
        total = torch.empty(2, b, 7 * m, dtype=torch.float64, device=dev)
        for q, (ql, qh) in enumerate(bounds):
            w = qh - ql
            for k in range(7):
                total[:, :, k * m + ql:k * m + qh] = gathered[q][:, :, k * w:(k + 1) * w]
        counts = torch.tensor([float(t_len)] + [float(max(t_len - lag, 0)) for lag in LAGS
                                                for _ in (0, 1)],
                              dtype=torch.float64, device=dev).repeat_interleave(m)
        moments = torch.where(counts > 0, total / counts.clamp_min(1.0),
                              torch.zeros_like(total)).float().contiguous()
        logits = torch.empty(b, model.head.classifier.out_features, device=dev)
        params, _keep = model._effective(dev)
        _lib.check(_lib.load().lnet_b200_head(ctypes_ref(params), b, moments[0].data_ptr(),
                                              moments[1].data_ptr(), logits.data_ptr(),
                                              torch.cuda.current_stream(dev).cuda_stream),
                   "lnet_b200_head")
        return logits


def ctypes_ref(obj):
    import ctypes

    return ctypes.byref(obj)


def channelsplit_forward(model, x: Tensor, group=None) -> Tensor:
    """Logits of the whole batch on every rank of `group`; every rank passes the same
    x [B, T, C] (on its own GPU) and computes its slice of the modes."""
    if not x.is_cuda:
        raise RuntimeError("channelsplit_forward runs on CUDA only")
    world = dist.get_world_size(group) if dist.is_initialized() else 1
    rank = dist.get_rank(group) if dist.is_initialized() else 0
    return drive_program(_rank_program(model, x, rank, world), world, group)


def channelsplit_emulate(model, x: Tensor, world: int) -> list[Tensor]:
    """The `world` rank programs in lockstep in this process; every rank's logits."""
    return run_lockstep([_rank_program(model, x, r, world) for r in range(world)])


__all__ = ["channelsplit_emulate", "channelsplit_forward", "mode_bounds"]
