"""Data-parallel training over NCCL: torch DistributedDataParallel around
B200Alphabet (its backward is lnet_b200_alphabet_backward) on two GPUs, each
rank taking half of the batch, reproduces the single-GPU full-batch gradients
(the gradient all-reduce is the only exchange).  Skipped with fewer than two
GPUs; NVLS off, plain NCCL."""

from __future__ import annotations

import datetime
import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _build(dev):
    from lnet_b200 import AlphabetConfig, B200Alphabet

    torch.manual_seed(3)
    model = B200Alphabet(AlphabetConfig(8, 32, 16, 5), 5)
    g = torch.Generator().manual_seed(4)
    with torch.no_grad():
        for blk in (model.forward_block, model.backward_block):
            blk.raw_frequency.copy_(torch.randn(16, generator=g) * 0.8)
        model.forward_block.layer_scale.copy_(0.3 * torch.randn(32, generator=g))
    x = torch.randn(4, 200, 8, generator=g)
    dl = torch.randn(4, 5, generator=g)
    return model.to(dev).train(), x.to(dev), dl.to(dev)


def _worker(rank, world, port, q):
    import torch.distributed as dist
    from torch.nn.parallel import DistributedDataParallel as DDP

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev,
                            timeout=datetime.timedelta(seconds=60))
    try:
        model, x, dl = _build(dev)
        # single-GPU reference on the whole batch (sum loss / world = DDP's mean)
        ref_model, _, _ = _build(dev)
        ((ref_model(x) * dl).sum() / world).backward()
        ref = {n: p.grad.detach().clone() for n, p in ref_model.named_parameters()}
        ddp = DDP(model, device_ids=[rank])
        half = x.shape[0] // world
        rows = slice(rank * half, (rank + 1) * half)
        (ddp(x[rows].contiguous()) * dl[rows]).sum().backward()
        worst = 0.0
        for n, p in model.named_parameters():
            r = ref[n]
            worst = max(worst, float((p.grad - r).abs().max() / r.abs().max().clamp_min(1e-30)))
        q.put((rank, worst))
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_ddp_two_gpus_matches_full_batch():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
        assert not p.is_alive()
    errs = dict(q.get(timeout=5) for _ in procs)
    assert set(errs) == {0, 1} and max(errs.values()) <= 1e-4, errs
