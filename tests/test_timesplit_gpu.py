"""Sequence split over ranks (lnet_b200.timesplit) against the unsplit forward.

* emulated ranks (lockstep in one process): 2, 3, 4 ranks on a ragged length
  (T = 203), fp32 and bf16 inputs, every rank returning the logits of the whole
  batch; the split re-associates the fp32 carries (carry-in from the slice
  summaries and a^L powers), so the bound is 1e-5 relative;
* too few steps per rank raises;
* two real ranks over NCCL on two GPUs (skipped with fewer GPUs).
"""

from __future__ import annotations

import datetime
import os
import socket
import sys
from pathlib import Path

import pytest
import torch
import torch.multiprocessing as mp
from conftest import rel_err

from lnet_b200.timesplit import timesplit_emulate, timesplit_forward

sys.path.insert(0, str(Path(__file__).resolve().parents[1]))
import bench  # noqa: E402

pytestmark = pytest.mark.gpu

CFG = dict(workload="timesplit_small", B=3, T=203, C=16, D=32, M=8, K=5, dtype="fp32",
           images=False)


def _model_and_input(device, dtype=torch.float32, t=203):
    cfg = dict(CFG, T=t)
    model = bench.build_model(cfg, device)
    g = torch.Generator().manual_seed(4)
    with torch.no_grad():  # complex poles, so the carries rotate
        for blk in (model.forward_block, model.backward_block):
            blk.raw_frequency.copy_(torch.randn(cfg["M"], generator=g) * 0.8)
    x = torch.randn(cfg["B"], t, cfg["C"], generator=g).to(device=device, dtype=dtype)
    return model, x


@pytest.mark.parametrize("world", [2, 3, 4])
def test_emulated_split_matches_forward(cuda_device, world):
    model, x = _model_and_input(cuda_device)
    with torch.no_grad():
        ref = model(x).cpu().numpy()
        outs = timesplit_emulate(model, x, world)
    for out in outs:
        assert rel_err(out.cpu().numpy(), ref) <= 1e-5


def test_emulated_split_bf16(cuda_device):
    model, x = _model_and_input(cuda_device, torch.bfloat16)
    with torch.no_grad():
        ref = model(x).cpu().numpy()
        out = timesplit_emulate(model, x, 2)[1]
    assert rel_err(out.cpu().numpy(), ref) <= 1e-4


def test_split_needs_eight_steps_per_rank(cuda_device):
    model, x = _model_and_input(cuda_device, t=20)
    with pytest.raises(ValueError):
        timesplit_emulate(model, x, 3)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _nccl_worker(rank, world, port, q):
    import torch.distributed as dist

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev,
                            timeout=datetime.timedelta(seconds=60))
    try:
        model, x = _model_and_input(dev)
        with torch.no_grad():
            out = timesplit_forward(model, x)
            ref = model(x)
        q.put((rank, rel_err(out.cpu().numpy(), ref.cpu().numpy())))
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_two_ranks_nccl():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_nccl_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
        assert not p.is_alive()
    errs = dict(q.get(timeout=5) for _ in procs)
    assert set(errs) == {0, 1} and max(errs.values()) <= 1e-5
