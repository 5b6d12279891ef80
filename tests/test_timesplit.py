"""Host logic of the sequence split (CPU): the carry combination against a
direct sequential complex scan, and the collective driver on two gloo ranks."""

from __future__ import annotations

import datetime
import math
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from lnet_b200.sharding import shard_bounds
from lnet_b200.timesplit import _carry, _from_complex, _pole_powers, drive_program


def test_carry_matches_sequential_scan():
    g = torch.Generator().manual_seed(0)
    b, t_len, m, world = 3, 61, 5, 4
    raw_decay = torch.randn(m, generator=g) * 2
    raw_freq = torch.randn(m, generator=g)
    bounds = [shard_bounds(t_len, world, r) for r in range(world)]
    lengths = [hi - lo for lo, hi in bounds]
    powers = _pole_powers(raw_decay, raw_freq, lengths)
    a = powers[1]
    u = torch.complex(torch.randn(b, t_len, m, generator=g, dtype=torch.float64),
                      torch.randn(b, t_len, m, generator=g, dtype=torch.float64))
    true = torch.zeros_like(u)
    s = torch.zeros(b, m, dtype=torch.complex128)
    for t in range(t_len):
        s = a * s + u[:, t]
        true[:, t] = s
    summaries = []
    for lo, hi in bounds:  # local scans from zero
        s = torch.zeros(b, m, dtype=torch.complex128)
        loc = []
        for t in range(lo, hi):
            s = a * s + u[:, t]
            loc.append(s)
        loc = torch.stack(loc, 1)
        summaries.append(_from_complex(loc[:, -4:].flip(1)).double())
    summaries = torch.stack(summaries)  # [G, B, 4, 2M]
    for r, (lo, hi) in enumerate(bounds):
        init, hist = _carry(summaries, lengths, r, powers, m)
        want = torch.zeros(b, m, dtype=torch.complex128) if r == 0 else true[:, lo - 1]
        assert torch.allclose(init.double(), _from_complex(want).double(), rtol=1e-5, atol=1e-5)
        if r == 0:
            assert hist is None
        else:
            want_h = torch.stack([true[:, lo - 1 - k] for k in range(4)], 1)
            assert torch.allclose(hist.double(), _from_complex(want_h).double(), rtol=1e-5,
                                  atol=1e-5)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _program(rank, world):
    got = yield ("gather", torch.full((2,), float(rank)))
    assert got.shape == (world, 2) and got[:, 0].tolist() == [float(r) for r in range(world)]
    total = yield ("sum", torch.tensor([rank + 1.0], dtype=torch.float64))
    return float(total.item())


def _worker(rank, world, port, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=30))
    try:
        q.put((rank, drive_program(_program(rank, world), world)))
    finally:
        dist.destroy_process_group()


def test_drive_program_gloo_two_ranks():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
        assert not p.is_alive()
    res = dict(q.get(timeout=5) for _ in procs)
    assert res == {0: 3.0, 1: 3.0}


def test_pole_powers_are_powers():
    p = _pole_powers(torch.tensor([0.3, -1.0]), torch.tensor([0.2, 0.0]), [10])
    assert torch.allclose(p[10], p[1] ** 10) and set(p) >= {7, 8, 9, 10}
    assert not math.isnan(float(p[10].abs().max()))
