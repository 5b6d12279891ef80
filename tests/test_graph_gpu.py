"""CUDA-graph capture and replay of the fused route.

Replays must track the inputs exactly like eager forwards (the look-back
records are tagged by a device-side epoch, so a replay never reads its
predecessor's records as current): several inputs, repeated replays, and the
image entry point; <= 1e-5 against eager forwards (the look-back
re-association bound).
"""

from __future__ import annotations

import sys
from pathlib import Path

import pytest
import torch
from conftest import rel_err

from lnet_b200.graph import CudaGraphForward

sys.path.insert(0, str(Path(__file__).resolve().parents[1]))
import bench  # noqa: E402

pytestmark = pytest.mark.gpu


def test_graph_replay_tracks_inputs(cuda_device):
    cfg = dict(bench.CONFIGS["4"], B=4)
    model = bench.build_model(cfg, cuda_device)
    xs = [bench.make_inputs(cfg, cuda_device, seed=s) for s in (1, 2, 3)]
    runner = CudaGraphForward(model, xs[0])
    with torch.no_grad():
        for rep in range(2):
            for x in xs:
                got = runner(x).clone()
                torch.cuda.synchronize()
                assert rel_err(got.cpu().numpy(), model(x).cpu().numpy()) <= 1e-5, rep
    with pytest.raises(ValueError):
        runner(xs[0][:2])


def test_graph_replay_images(cuda_device):
    cfg = dict(bench.CONFIGS["4"], B=2)
    model = bench.build_model(cfg, cuda_device)
    imgs = [bench.make_images(cfg, cuda_device, seed=s) for s in (4, 5)]
    runner = CudaGraphForward(model, imgs[0], images=True)
    with torch.no_grad():
        for img in imgs + imgs:
            got = runner(img).clone()
            assert rel_err(got.cpu().numpy(), model.forward_images(img).cpu().numpy()) <= 1e-5


@pytest.mark.parametrize("fill", [0x00, 0xFF])
def test_fresh_workspace_contents_do_not_leak(cuda_device, fill):
    """A workspace of zeros (or of ones) must not read as published look-back
    records: the record tag is never 0 and is fresh per call."""
    import ctypes

    from lnet_b200 import _lib
    from lnet_b200.alphabet import _workspace_bytes

    cfg = dict(bench.CONFIGS["4"], B=3)
    model = bench.build_model(cfg, cuda_device)
    x = bench.make_inputs(cfg, cuda_device)
    lib = _lib.load()
    params, _keep = model._effective(x.device)
    req = model._request(x, None, None, None, _lib.LNET_BF16)
    n = _workspace_bytes(params, req)
    ws = torch.full((n,), fill, dtype=torch.uint8, device=cuda_device)
    out = torch.empty(3, cfg["K"], device=cuda_device)
    _lib.check(lib.lnet_b200_alphabet_forward(ctypes.byref(params), ctypes.byref(req),
                                              ws.data_ptr(), n, out.data_ptr(), None, None,
                                              torch.cuda.current_stream().cuda_stream),
               "lnet_b200_alphabet_forward")
    with torch.no_grad():
        ref = model(x)
    assert rel_err(out.cpu().numpy(), ref.cpu().numpy()) <= 1e-5
