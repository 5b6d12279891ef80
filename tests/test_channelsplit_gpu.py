"""Channel (mode) split over ranks (lnet_b200.channelsplit) against the unsplit forward.

* emulated ranks (lockstep in one process): 2, 3 (uneven mode slices) and 4 ranks,
  fp32 and bf16 inputs, complex poles, every rank returning the logits of the whole
  batch.  The writer stream is the sum of per-rank partial syntheses (one GEMM per
  rank instead of one over all modes), so the bound is 1e-5 relative (fp32);
* more ranks than modes raises;
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

from lnet_b200.channelsplit import channelsplit_emulate, channelsplit_forward

sys.path.insert(0, str(Path(__file__).resolve().parents[1]))
import bench  # noqa: E402

pytestmark = pytest.mark.gpu

CFG = dict(workload="channelsplit_small", B=3, T=203, C=16, D=32, M=8, K=5, dtype="fp32",
           images=False)


def _model_and_input(device, dtype=torch.float32):
    model = bench.build_model(CFG, device)
    g = torch.Generator().manual_seed(4)
    with torch.no_grad():  # complex poles
        for blk in (model.forward_block, model.backward_block):
            blk.raw_frequency.copy_(torch.randn(CFG["M"], generator=g) * 0.8)
    x = torch.randn(CFG["B"], CFG["T"], CFG["C"], generator=g).to(device=device, dtype=dtype)
    return model, x


@pytest.mark.parametrize("world", [2, 3, 4])
def test_emulated_split_matches_forward(cuda_device, world):
    model, x = _model_and_input(cuda_device)
    with torch.no_grad():
        ref = model(x).cpu().numpy()
        outs = channelsplit_emulate(model, x, world)
    assert len(outs) == world
    for out in outs:
        assert rel_err(out.cpu().numpy(), ref) <= 1e-5


def test_emulated_split_bf16(cuda_device):
    model, x = _model_and_input(cuda_device, torch.bfloat16)
    with torch.no_grad():
        ref = model(x).cpu().numpy()
        out = channelsplit_emulate(model, x, 2)[1]
    # bf16 drive operands are rounded after different kernels on the two paths
    # (the unsplit conv + RMSNorm kernel vs the pieces' RMSNorm + conversion)
    assert rel_err(out.cpu().numpy(), ref) <= 2e-4


def test_more_ranks_than_modes_raises(cuda_device):
    model, x = _model_and_input(cuda_device)
    with pytest.raises(ValueError):
        channelsplit_emulate(model, x, CFG["M"] + 1)


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
            out = channelsplit_forward(model, x)
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
