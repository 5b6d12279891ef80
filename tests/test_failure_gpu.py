"""A bounded wait that gives up must surface: the forward's logits become NaN and
the device status word names the wait.

The give-up is made on purpose without faulting anything: the one-shot hook
``lnet_b200_debug_inject_lookback_miss`` makes the next fused forward look for
look-back records under a tag no record carries, with a 64-poll limit, so every
look-back of a chunk > 0 gives up (the kernel records the error bit, continues
with zero carries and returns normally).  The next call is clean again.
"""

from __future__ import annotations

import ctypes
import sys
from pathlib import Path

import pytest
import torch

from lnet_b200 import _lib
from lnet_b200.alphabet import _workspace_bytes

sys.path.insert(0, str(Path(__file__).resolve().parents[1]))
import bench  # noqa: E402

pytestmark = pytest.mark.gpu

LOOKBACK_WRITER, LOOKBACK_READER = 1 << 4, 1 << 5


def _forward(model, x, ws=None):
    lib = _lib.load()
    params, _keep = model._effective(x.device)
    req = model._request(x, None, None, None, _lib.LNET_BF16)
    n = _workspace_bytes(params, req)
    if ws is None:
        ws = torch.empty(n, dtype=torch.uint8, device=x.device)
    logits = torch.empty(x.shape[0], model.head.classifier.out_features, device=x.device)
    _lib.check(lib.lnet_b200_alphabet_forward(ctypes.byref(params), ctypes.byref(req),
                                              ws.data_ptr(), n, logits.data_ptr(), None, None,
                                              torch.cuda.current_stream().cuda_stream),
               "lnet_b200_alphabet_forward")
    status = ctypes.c_uint32(0)
    _lib.check(lib.lnet_b200_alphabet_device_status(ctypes.byref(params), ctypes.byref(req),
                                                    ws.data_ptr(), n, ctypes.byref(status)),
               "lnet_b200_alphabet_device_status")
    assert lib.lnet_b200_alphabet_route(ctypes.byref(params), ctypes.byref(req)) == 0
    return logits, status.value, ws


def test_lookback_give_up_poisons_logits(cuda_device):
    cfg = dict(bench.CONFIGS["4"], B=3, T=700)  # 6 chunks per row: 15 look-backs per block
    model = bench.build_model(cfg, cuda_device)
    x = bench.make_inputs(dict(cfg, images=False), cuda_device)
    with torch.no_grad():
        clean, status, ws = _forward(model, x)
        assert status == 0 and torch.isfinite(clean).all()
        _lib.check(_lib.load().lnet_b200_debug_inject_lookback_miss(), "inject")
        bad, status, _ = _forward(model, x, ws)
        torch.cuda.synchronize()
        assert status & (LOOKBACK_WRITER | LOOKBACK_READER), hex(status)
        assert torch.isnan(bad).all(), "a look-back give-up must not yield finite logits"
        # one shot: the next call on the same workspace is clean and equal to the first
        again, status, _ = _forward(model, x, ws)
        assert status == 0
        assert torch.isfinite(again).all()
        assert (again - clean).abs().max().item() <= 1e-5 * clean.abs().max().item() + 1e-7
