"""Sequence (time) split of the ALPHABET forward over ranks.

For requests with fewer rows than GPUs (long sequences, small batch) the steps
of every row are split into contiguous balanced slices, one per rank.  The
recurrence and the lag moments cross the slice boundaries, so each block
(writer, reader) takes one exchange step:

1. the rank scans its slice from a zero state (``lnet_b200_block_scan``) and
   all-gathers a summary: the local states at its last four steps [B, 4, 2M];
2. every rank combines the summaries in rank order, with the transition power
   a^L of each slice (static poles), into its carry-in (the true state before
   its slice) and the true states at the four steps before it (lag history);
3. it rescans from the carry-in and forms raw moment sums with that history
   (``lnet_b200_block_moment_sums``).

The stem's ±8-step conv halo comes from overlapping input slices (x is
available to every rank); the reader's comes from the neighbours' writer
stream rows (one all-gather of 8 boundary rows per side).  The moment sums of
both blocks are summed across ranks (one all-reduce of [2, B, 7M] fp64) and
divided by T and T - lag; every rank then evaluates the head and returns the
logits of the whole batch.

Static poles only (no time_delta, no masks): the general-route pieces run in
fp32 with TF32 GEMMs for bf16 inputs.  Requires at least 8 steps per rank.

The per-rank computation is a generator that yields its collectives, so the
same code runs under ``torch.distributed`` (:func:`timesplit_forward`) and as
G ranks in lockstep in one process (:func:`timesplit_emulate`, for checks).
"""

from __future__ import annotations

import ctypes
import math

import torch
import torch.distributed as dist
from torch import Tensor

from . import _lib
from .alphabet import _workspace_bytes
from .sharding import shard_bounds

HALO = 8  # K5 dilation-4 depthwise conv: 8 steps on each side
LAGS = (1, 2, 4)


def _pole_powers(raw_decay: Tensor, raw_freq: Tensor, lengths) -> dict[int, Tensor]:
    """a^L for every slice length L in `lengths` and L - k (k = 0..3), and a itself;
    complex128 [M].
    a = exp(p) with p = -d + i w, d = 1e-3 + (2 - 1e-3) sigmoid(raw_decay),
    w = pi tanh(raw_frequency), rounded to fp32 as the scan kernels use it."""
    r = raw_decay.double()
    d = 1e-3 + (2.0 - 1e-3) / (1.0 + torch.exp(-r))
    w = math.pi * torch.tanh(raw_freq.double())
    a = torch.complex(torch.exp(-d) * torch.cos(w), torch.exp(-d) * torch.sin(w))
    a = torch.complex(a.real.float().double(), a.imag.float().double())
    out = {1: a}
    for n in lengths:
        for k in range(4):
            if n - k >= 0 and (n - k) not in out:
                out[n - k] = a ** (n - k)
    return out


def _to_complex(v: Tensor, m: int) -> Tensor:
    """[..., 2M] re | im -> complex128 [..., M]."""
    v = v.double()
    return torch.complex(v[..., :m], v[..., m:])


def _from_complex(z: Tensor) -> Tensor:
    return torch.cat([z.real, z.imag], dim=-1).float().contiguous()


def _carry(summaries: Tensor, lengths, rank: int, powers, m: int):
    """Carry-in [B, 2M] and lag history [B, 4, 2M] of `rank` from the gathered local
    summaries [G, B, 4, 2M] (local states at the last four steps of each slice)."""
    local = _to_complex(summaries, m)  # [G, B, 4, M]
    s_in = torch.zeros_like(local[0, :, 0])
    hist = None
    for q in range(rank):
        n = lengths[q]
        true_last = torch.stack([local[q, :, k] + powers[n - k] * s_in for k in range(4)], dim=1)
        s_in = powers[n] * s_in + local[q, :, 0]
        hist = true_last
    return _from_complex(s_in), (None if hist is None else _from_complex(hist))


class _Pieces:
    """C-ABI calls of one rank's slice (B rows, Ts steps)."""

    def __init__(self, model, ref: Tensor, batch: int, steps: int, act: int):
        self.lib = _lib.load()
        self.params, self._keep = model._effective(ref.device)
        self.req = _lib.AlphabetRequest(batch=batch, steps=steps, x_dtype=_lib.LNET_F32,
                                        act_dtype=act, x=ref.data_ptr(), obs_channels=1)
        self.nbytes = _workspace_bytes(self.params, self.req)
        self.ws = torch.empty(max(self.nbytes, 1), dtype=torch.uint8, device=ref.device)
        self.stream = torch.cuda.current_stream(ref.device).cuda_stream

    def _p(self):
        return ctypes.byref(self.params), ctypes.byref(self.req)

    def drive(self, block: int, x: Tensor, u: Tensor, xhat: Tensor | None):
        _lib.check(self.lib.lnet_b200_block_drive(*self._p(), block, x.data_ptr(),
                                                  self.ws.data_ptr(), self.nbytes, u.data_ptr(),
                                                  None if xhat is None else xhat.data_ptr(),
                                                  self.stream), "lnet_b200_block_drive")

    def scan(self, block: int, u: Tensor, init: Tensor | None):
        _lib.check(self.lib.lnet_b200_block_scan(*self._p(), block, u.data_ptr(),
                                                 None if init is None else init.data_ptr(),
                                                 self.ws.data_ptr(), self.nbytes, self.stream),
                   "lnet_b200_block_scan")

    def sums(self, states: Tensor, hist: Tensor | None, out: Tensor):
        _lib.check(self.lib.lnet_b200_block_moment_sums(
            *self._p(), states.data_ptr(), None if hist is None else hist.data_ptr(),
            self.ws.data_ptr(), self.nbytes, out.data_ptr(), self.stream),
            "lnet_b200_block_moment_sums")

    def writer_output(self, states: Tensor, xhat: Tensor, first: Tensor, out: Tensor):
        _lib.check(self.lib.lnet_b200_writer_output(*self._p(), states.data_ptr(),
                                                    xhat.data_ptr(), first.data_ptr(),
                                                    self.ws.data_ptr(), self.nbytes,
                                                    out.data_ptr(), self.stream),
                   "lnet_b200_writer_output")


def _call_stem(model, x_ext: Tensor, act: int) -> Tensor:
    lib = _lib.load()
    params, _keep = model._effective(x_ext.device)
    req = model._request(x_ext, None, None, None, act)
    nbytes = _workspace_bytes(params, req)
    ws = torch.empty(max(nbytes, 1), dtype=torch.uint8, device=x_ext.device)
    out = torch.empty(x_ext.shape[0], x_ext.shape[1], model.model_dim, device=x_ext.device)
    stream = torch.cuda.current_stream(x_ext.device).cuda_stream
    _lib.check(lib.lnet_b200_stem(ctypes.byref(params), ctypes.byref(req), ws.data_ptr(), nbytes,
                                  out.data_ptr(), stream), "lnet_b200_stem")
    return out


def _call_conv(model, x_ext: Tensor, act: int) -> Tensor:
    lib = _lib.load()
    params, _keep = model._effective(x_ext.device)
    req = _lib.AlphabetRequest(batch=x_ext.shape[0], steps=x_ext.shape[1], x_dtype=_lib.LNET_F32,
                               act_dtype=act, x=x_ext.data_ptr(), obs_channels=1)
    out = torch.empty_like(x_ext)
    stream = torch.cuda.current_stream(x_ext.device).cuda_stream
    _lib.check(lib.lnet_b200_depthwise_conv_silu(ctypes.byref(params), ctypes.byref(req), 1,
                                                 x_ext.data_ptr(), out.data_ptr(), stream),
               "lnet_b200_depthwise_conv_silu")
    return out


def _rank_program(model, x: Tensor, rank: int, world: int):
    """One rank's forward; yields ("gather", t) -> [world, *t.shape] and ("sum", t) -> sum."""
    b, t_len, _ = x.shape
    if t_len < HALO * world:
        raise ValueError(f"time split needs at least {HALO} steps per rank "
                         f"(T={t_len}, ranks={world})")
    dev = x.device
    m, d = model.modes, model.model_dim
    act = _lib.LNET_BF16 if x.dtype == torch.bfloat16 else _lib.LNET_F32
    bounds = [shard_bounds(t_len, world, r) for r in range(world)]
    lengths = [hi - lo for lo, hi in bounds]
    t0, t1 = bounds[rank]
    ts = t1 - t0
    with torch.no_grad():
        fb, bb = model.forward_block, model.backward_block
        w_pow = _pole_powers(fb.raw_decay.detach().cpu(), fb.raw_frequency.detach().cpu(),
                             lengths)
        r_pow = _pole_powers(bb.raw_decay.detach().cpu(), bb.raw_frequency.detach().cpu(),
                             lengths)
        # stem on the slice with its input halo, cropped to the slice
        e0, e1 = max(0, t0 - HALO), min(t_len, t1 + HALO)
        first_ext = _call_stem(model, x[:, e0:e1].contiguous(), act)
        first = first_ext[:, t0 - e0:t0 - e0 + ts].contiguous()
        pc = _Pieces(model, first, b, ts, act)
        sums = torch.zeros(2, b, 7 * m, dtype=torch.float64, device=dev)
        # writer block
        u = torch.empty(b, ts, 2 * m, device=dev)
        xhat = torch.empty(b, ts, d, device=dev)
        pc.drive(0, first, u, xhat)
        loc = u.clone()
        pc.scan(0, loc, None)
        summary = loc[:, ts - 4:].flip(1).contiguous()  # steps ts-1 .. ts-4
        gathered = yield ("gather", summary)
        init, hist = _carry(gathered.cpu(), lengths, rank, w_pow, m)
        pc.scan(0, u, init.to(dev))
        pc.sums(u, None if hist is None else hist.to(dev), sums[0])
        stream = torch.empty(b, ts, d, device=dev)
        pc.writer_output(u, xhat, first, stream)
        # reader: stream halo from the neighbours, conv, block
        edges = torch.cat([stream[:, :HALO], stream[:, ts - HALO:]], dim=1).contiguous()
        halos = yield ("gather", edges)
        parts = []
        if rank > 0:
            parts.append(halos[rank - 1][:, HALO:])
        parts.append(stream)
        if rank < world - 1:
            parts.append(halos[rank + 1][:, :HALO])
        ext = torch.cat(parts, dim=1).contiguous()
        lo = HALO if rank > 0 else 0
        second = _call_conv(model, ext, act)[:, lo:lo + ts].contiguous()
        u2 = torch.empty(b, ts, 2 * m, device=dev)
        pc.drive(1, second, u2, None)
        loc2 = u2.clone()
        pc.scan(1, loc2, None)
        gathered2 = yield ("gather", loc2[:, ts - 4:].flip(1).contiguous())
        init2, hist2 = _carry(gathered2.cpu(), lengths, rank, r_pow, m)
        pc.scan(1, u2, init2.to(dev))
        pc.sums(u2, None if hist2 is None else hist2.to(dev), sums[1])
        total = yield ("sum", sums)
        counts = torch.tensor([float(t_len)] + [float(max(t_len - lag, 0)) for lag in LAGS for _ in (0, 1)],
                              dtype=torch.float64, device=dev)
        counts = counts.repeat_interleave(m)  # [7M]
        moments = torch.where(counts > 0, total / counts.clamp_min(1.0), torch.zeros_like(total))
        moments = moments.float().contiguous()
        logits = torch.empty(b, model.head.classifier.out_features, device=dev)
        params, _keep = model._effective(dev)
        _lib.check(_lib.load().lnet_b200_head(ctypes.byref(params), b, moments[0].data_ptr(),
                                              moments[1].data_ptr(), logits.data_ptr(),
                                              torch.cuda.current_stream(dev).cuda_stream),
                   "lnet_b200_head")
        return logits


def timesplit_forward(model, x: Tensor, group=None) -> Tensor:
    """Logits of the whole batch on every rank of `group`; every rank passes the
    same x [B, T, C] (on its own GPU) and computes its slice of steps."""
    if not x.is_cuda:
        raise RuntimeError("timesplit_forward runs on CUDA only")
    world = dist.get_world_size(group) if dist.is_initialized() else 1
    rank = dist.get_rank(group) if dist.is_initialized() else 0
    return drive_program(_rank_program(model, x, rank, world), world, group)


def drive_program(prog, world: int, group=None):
    """Runs a rank program, answering its ("gather", t) requests with
    dist.all_gather (stacked [world, ...]) and ("sum", t) with dist.all_reduce."""
    req = next(prog)
    while True:
        kind, t = req
        if kind == "gather":
            parts = [torch.empty_like(t) for _ in range(world)]
            if world > 1:
                dist.all_gather(parts, t, group=group)
            else:
                parts[0].copy_(t)
            res = torch.stack(parts)
        else:
            res = t.clone()
            if world > 1:
                dist.all_reduce(res, group=group)
        try:
            req = prog.send(res)
        except StopIteration as stop:
            return stop.value


def run_lockstep(progs) -> list:
    """Runs rank programs (generators yielding ("gather", t) / ("sum", t)) in lockstep
    in this process, evaluating each collective locally; returns every rank's result."""
    world = len(progs)
    reqs = [next(p) for p in progs]
    while True:
        kinds = {k for k, _ in reqs}
        if len(kinds) != 1:
            raise RuntimeError(f"ranks out of step: {kinds}")
        if reqs[0][0] == "gather":
            res = torch.stack([t for _, t in reqs])
            resps = [res] * world
        else:
            total = torch.stack([t for _, t in reqs]).sum(0)
            resps = [total.clone() for _ in range(world)]
        out, done = [], []
        for p, r in zip(progs, resps):
            try:
                out.append(p.send(r))
            except StopIteration as stop:
                done.append(stop.value)
        if done:
            if len(done) != world:
                raise RuntimeError("ranks finished at different steps")
            return done
        reqs = out


def timesplit_emulate(model, x: Tensor, world: int) -> list[Tensor]:
    """The `world` rank programs run in lockstep in this process (collectives
    evaluated locally); returns every rank's logits."""
    return run_lockstep([_rank_program(model, x, r, world) for r in range(world)])


__all__ = ["drive_program", "run_lockstep", "timesplit_emulate", "timesplit_forward"]
