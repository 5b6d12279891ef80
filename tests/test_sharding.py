"""Batch-sharding host logic on CPU `gloo` ranks (world size 2).

The per-rank compute is a stand-in linear map on CPU tensors; what is tested
is the split, the metadata slicing, the gather order and that a rank that dies
before the gather makes the others fail fast instead of hanging.
"""

from __future__ import annotations

import datetime
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from lnet_b200.sharding import shard_bounds, sharded_forward


def test_shard_bounds_cover_batch():
    for batch in (0, 1, 5, 256, 257):
        for world in (1, 2, 3, 8):
            spans = [shard_bounds(batch, world, r) for r in range(world)]
            assert spans[0][0] == 0 and spans[-1][1] == batch
            assert all(a[1] == b[0] for a, b in zip(spans, spans[1:]))
            sizes = [s[1] - s[0] for s in spans]
            assert max(sizes) - min(sizes) <= 1
    with pytest.raises(ValueError):
        shard_bounds(4, 2, 2)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _stand_in(x, time_delta=None, observation_mask=None, valid_mask=None):
    w = torch.arange(x.shape[-1] * 3, dtype=torch.float32).reshape(x.shape[-1], 3) / 10
    y = x.mean(dim=1) @ w
    if valid_mask is not None:
        y = y + valid_mask.sum(dim=1, keepdim=True)
    return y


def _seq_stand_in(x):
    """A per-row sequence map without metadata keywords (the Laplace layer's
    forward(inputs) -> [B, T, D] shape)."""
    return torch.cumsum(x, dim=1) * 0.5 + x.sum(dim=-1, keepdim=True)


def _worker(rank, world, port, batch, die_rank, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=10))
    try:
        g = torch.Generator().manual_seed(0)
        x = torch.randn(batch, 6, 4, generator=g)
        valid = (torch.rand(batch, 6, generator=g) < 0.7).float()
        if rank == die_rank:
            raise SystemExit(3)  # this rank leaves before the collective
        out = sharded_forward(_stand_in, x, valid_mask=valid)
        ok = torch.allclose(out, _stand_in(x, valid_mask=valid), atol=1e-6)
        seq = sharded_forward(_seq_stand_in, x)
        ok = ok and seq.shape == x.shape and torch.allclose(seq, _seq_stand_in(x), atol=1e-6)
        q.put((rank, "ok" if ok else "mismatch"))
    except SystemExit:
        q.put((rank, "left"))
    except Exception as exc:  # noqa: BLE001 - the failure of a peer surfaces here
        q.put((rank, f"error:{type(exc).__name__}"))
    finally:
        try:
            dist.destroy_process_group()
        except Exception:  # noqa: BLE001
            pass


def _run(batch, die_rank):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, batch, die_rank, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
        if p.is_alive():
            p.kill()
            pytest.fail("a rank hung")
    return dict(q.get(timeout=5) for _ in procs)


@pytest.mark.parametrize("batch", [7, 8])
def test_sharded_forward_gathers_in_row_order(batch):
    res = _run(batch, die_rank=-1)
    assert res == {0: "ok", 1: "ok"}


def test_dead_rank_fails_fast():
    res = _run(8, die_rank=1)
    assert res[1] == "left"
    assert res[0].startswith("error:")
