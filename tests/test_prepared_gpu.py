"""Prepared static inference: operands built once (lnet_b200_alphabet_prepare)
and reused by lnet_b200_alphabet_forward_prepared.

* prepared forwards agree with the per-call forward (<= 1e-5, the look-back
  re-association bound of the fused route);
* an in-place parameter change is picked up (the operands are rebuilt);
* batches larger than the prepared size grow the workspace; fp32 inputs (general
  route) on a prepared module still work;
* through the C ABI: one preparation serves requests of several batch sizes.
"""

from __future__ import annotations

import ctypes
import sys
from pathlib import Path

import pytest
import torch
from conftest import rel_err

from lnet_b200 import _lib
from lnet_b200.alphabet import _workspace_bytes

sys.path.insert(0, str(Path(__file__).resolve().parents[1]))
import bench  # noqa: E402

pytestmark = pytest.mark.gpu


def _model(cuda_device, b):
    cfg = dict(bench.CONFIGS["4"], B=b)
    return bench.build_model(cfg, cuda_device), bench.make_inputs(cfg, cuda_device)


def test_prepared_matches_per_call(cuda_device):
    model, x = _model(cuda_device, 8)
    with torch.no_grad():
        ref = model(x)
        assert model.prepare_for_inference_(sequence_length=x.shape[1], batch_size=8) is model
        a = model(x)
        b = model(x)  # second call: operands reused
    assert model._prep is not None and model._prep["fused"]
    assert rel_err(a.cpu().numpy(), ref.cpu().numpy()) <= 1e-5
    assert rel_err(b.cpu().numpy(), ref.cpu().numpy()) <= 1e-5


def test_prepared_picks_up_parameter_changes(cuda_device):
    model, x = _model(cuda_device, 4)
    model.prepare_for_inference_(sequence_length=x.shape[1], batch_size=4)
    with torch.no_grad():
        before = model(x)
        model.forward_block.raw_decay.add_(0.25)   # changes the folded drive operand
        model.backward_block.norm.weight.mul_(1.5)
        after = model(x)
        model._prepare_spec = None  # per-call path on the same parameters
        fresh = model(x)
    assert rel_err(after.cpu().numpy(), fresh.cpu().numpy()) <= 1e-5
    assert rel_err(after.cpu().numpy(), before.cpu().numpy()) > 1e-3


def test_prepared_grows_and_general_route(cuda_device):
    model, x = _model(cuda_device, 6)
    model.prepare_for_inference_(sequence_length=256, batch_size=2)
    with torch.no_grad():
        big = model(x)                       # larger than the prepared size
        ref_fp32 = model(x.float())          # general route on the prepared module
        model._prepare_spec = None
        ref = model(x)
        ref_fp32_call = model(x.float())
    assert rel_err(big.cpu().numpy(), ref.cpu().numpy()) <= 1e-5
    assert rel_err(ref_fp32.cpu().numpy(), ref_fp32_call.cpu().numpy()) <= 1e-6


def test_c_abi_one_preparation_many_batches(cuda_device):
    model, x = _model(cuda_device, 8)
    lib = _lib.load()
    params, _keep = model._effective(x.device)
    delta, obs, valid = model._prepare_metadata(x, None, None, None)
    big_req = model._request(x, delta, obs, valid, _lib.LNET_BF16)
    cap = _workspace_bytes(params, big_req)
    ws = torch.empty(cap, dtype=torch.uint8, device=cuda_device)
    stream = torch.cuda.current_stream().cuda_stream
    _lib.check(lib.lnet_b200_alphabet_prepare(ctypes.byref(params), ctypes.byref(big_req),
                                              ws.data_ptr(), cap, stream),
               "lnet_b200_alphabet_prepare")
    for b in (8, 3, 1):
        xb = x[:b].contiguous()
        req = model._request(xb, None, None, None, _lib.LNET_BF16)
        out = torch.empty(b, model.head.classifier.out_features, device=cuda_device)
        _lib.check(lib.lnet_b200_alphabet_forward_prepared(
            ctypes.byref(params), ctypes.byref(req), ws.data_ptr(), cap, out.data_ptr(), None,
            None, stream), "lnet_b200_alphabet_forward_prepared")
        with torch.no_grad():
            ref = model(xb)
        assert rel_err(out.cpu().numpy(), ref.cpu().numpy()) <= 1e-5
