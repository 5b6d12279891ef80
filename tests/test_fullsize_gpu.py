"""BASELINE configurations at their full sizes, checked through properties that
do not need the oracle to run at that size:

* row independence: every reduction is per row, so a forward over the full
  batch must agree with forwards over row subsets (fp32: <= 1e-5 relative;
  the fused route's look-back may re-associate carries, so the bound is not 0);
* oracle on a row subset: a few full-length rows are recomputed by the float64
  oracle (tolerances as in test_parity_gpu: 1e-4 fp32, 2e-2 bf16);
* route agreement: at config 4 the fused route must agree with the general
  route on the same bf16 inputs (2e-2);
* device status: no bounded wait inside the kernels gave up (fused route at
  config 4, the general route's bulk input copies at config 2).

Config 1 (Laplace layer) is checked entirely against the oracle.
"""

from __future__ import annotations

import ctypes
import math
import sys
from pathlib import Path

import numpy as np
import pytest
import torch
from conftest import record_margin, rel_err

from lnet_b200 import B200PoleResidueTemporalMixing, _lib
from lnet_b200.alphabet import _workspace_bytes
from oracle import alphabet_oracle as A
from oracle import laplace_oracle as L

sys.path.insert(0, str(Path(__file__).resolve().parents[1]))
import bench  # noqa: E402

pytestmark = pytest.mark.gpu


def _model_and_input(cfg, device):
    model = bench.build_model(cfg, device)
    x = bench.make_inputs(cfg, device)
    return model, x


def _forward_with_status(model, x, meta=None):
    """Forward through the C ABI keeping the workspace, then read the device status."""
    meta = meta or {}
    lib = _lib.load()
    act = _lib.LNET_BF16 if x.dtype == torch.bfloat16 else _lib.LNET_F32
    delta, obs, valid = model._prepare_metadata(x, meta.get("time_delta"),
                                                meta.get("observation_mask"),
                                                meta.get("valid_mask"))
    params, _keep = model._effective(x.device)
    req = model._request(x, delta, obs, valid, act)
    n = _workspace_bytes(params, req)
    ws = torch.empty(max(n, 1), dtype=torch.uint8, device=x.device)
    logits = torch.empty(x.shape[0], model.head.classifier.out_features, device=x.device)
    st = lib.lnet_b200_alphabet_forward(ctypes.byref(params), ctypes.byref(req), ws.data_ptr(),
                                        n, logits.data_ptr(), None, None,
                                        torch.cuda.current_stream().cuda_stream)
    _lib.check(st, "lnet_b200_alphabet_forward")
    status = ctypes.c_uint32(0)
    _lib.check(lib.lnet_b200_alphabet_device_status(ctypes.byref(params), ctypes.byref(req),
                                                    ws.data_ptr(), n, ctypes.byref(status)),
               "lnet_b200_alphabet_device_status")
    return logits, status.value


def _oracle_rows(cfg, x, rows, meta=None):
    params = {k: v.numpy().astype(np.float64) for k, v in bench.make_params(cfg).items()}
    xs = x[rows].float().cpu().numpy()
    kw = {}
    for key, value in (meta or {}).items():
        kw[key] = value[rows].cpu().numpy()
    return A.alphabet_forward(xs, params, dtype=np.float64, **kw)


def test_config4_full_fused_route(cuda_device):
    cfg = bench.CONFIGS["4"]
    model, x = _model_and_input(cfg, cuda_device)
    with torch.no_grad():
        logits, status = _forward_with_status(model, x)
    assert status == 0
    assert torch.isfinite(logits).all()
    # row independence against a small subset
    rows = [0, 77, 255]
    with torch.no_grad():
        sub, status_sub = _forward_with_status(model, x[rows].contiguous())
    assert status_sub == 0
    assert rel_err(sub.cpu().numpy(), logits[rows].cpu().numpy()) <= 1e-5
    # oracle (float64) on 32 full-length rows spread over the batch
    rows = [int(r) for r in np.linspace(0, cfg["B"] - 1, 32).round()]
    ref = _oracle_rows(cfg, x, rows)
    nw, _ = record_margin("config4:fused:32rows:logits", logits[rows].cpu().numpy(), ref, 2e-2)
    assert nw <= 2e-2
    # general route on the same bf16 inputs
    _lib.set_route(_lib.ROUTE_GENERAL)
    try:
        with torch.no_grad():
            general = model(x)
    finally:
        _lib.set_route(_lib.ROUTE_AUTO)
    assert rel_err(logits.cpu().numpy(), general.cpu().numpy()) <= 2e-2


def test_config2_full_fp32(cuda_device):
    cfg = bench.CONFIGS["2"]
    model, x = _model_and_input(cfg, cuda_device)
    with torch.no_grad():
        logits, status = _forward_with_status(model, x)  # general route: bulk-copy waits
        sub = model(x[[3, 100]].contiguous())
    assert status == 0
    assert rel_err(sub.cpu().numpy(), logits[[3, 100]].cpu().numpy()) <= 1e-5
    ref = _oracle_rows(cfg, x, [3, 100])
    nw, _ = record_margin("config2:rows3,100:logits", logits[[3, 100]].cpu().numpy(), ref, 1e-4)
    assert nw <= 1e-4


def test_config3_full_irregular_metadata(cuda_device):
    cfg = dict(workload="alphabet_cfg3", B=64, T=2048, C=64, D=64, M=32, K=10, dtype="fp32",
               images=False)
    model, x = _model_and_input(cfg, cuda_device)
    g = torch.Generator().manual_seed(5)
    b, t = cfg["B"], cfg["T"]
    dt = (-torch.log(torch.rand(b, t, generator=g).clamp_min(1e-12))).clamp(0.05, 4.0)
    obs = (torch.rand(b, t, cfg["C"], generator=g) < 0.8).float()
    lengths = torch.randint(t // 2, t + 1, (b,), generator=g)
    valid = (torch.arange(t).view(1, -1) < lengths.view(-1, 1)).float()
    meta = {"time_delta": dt.to(cuda_device), "observation_mask": obs.to(cuda_device),
            "valid_mask": valid.to(cuda_device)}
    with torch.no_grad():
        logits = model(x, **meta)
        rows = [1, 40]
        sub = model(x[rows].contiguous(), **{k: v[rows].contiguous() for k, v in meta.items()})
    assert rel_err(sub.cpu().numpy(), logits[rows].cpu().numpy()) <= 1e-5
    ref = _oracle_rows(cfg, x, rows, {k: v.cpu() for k, v in meta.items()})
    nw, _ = record_margin("config3:rows1,40:logits", logits[rows].cpu().numpy(), ref, 1e-4)
    assert nw <= 1e-4


def test_config5_full_long_sequence(cuda_device):
    cfg = bench.CONFIGS["5"]
    model, x = _model_and_input(cfg, cuda_device)
    with torch.no_grad():
        logits = model(x)
        sub = model(x[[7]].contiguous())
    assert torch.isfinite(logits).all()
    assert rel_err(sub.cpu().numpy(), logits[[7]].cpu().numpy()) <= 1e-5
    ref = _oracle_rows(cfg, x, [7])
    nw, _ = record_margin("config5:row7:logits", logits[[7]].cpu().numpy(), ref, 2e-2)
    assert nw <= 2e-2


def test_config1_full_laplace(cuda_device):
    # C=16 channels x 8 real poles each: 128 block-diagonal modes
    c, per, b, t = 16, 8, 64, 512
    g = torch.Generator().manual_seed(0)
    u = torch.empty(c, per, dtype=torch.float64).uniform_(math.log(0.01), 0.0, generator=g)
    poles = -torch.exp(u).reshape(-1)
    r = torch.randn(c, per, generator=g, dtype=torch.float64) / math.sqrt(per)
    residues = torch.zeros(c, c * per, c, dtype=torch.float64)
    for ch in range(c):
        residues[ch, ch * per:(ch + 1) * per, ch] = r[ch]
    direct = torch.diag(torch.randn(c, generator=g, dtype=torch.float64))
    layer = B200PoleResidueTemporalMixing(c, c * per)
    layer.load_transfer_parameters(poles=poles, residues=residues, direct_term=direct,
                                   bias=torch.zeros(c, dtype=torch.float64))
    x = torch.randn(b, t, c, generator=g)
    y = layer.to(cuda_device)(x.to(cuda_device))
    ref = L.laplace_forward(x.numpy(), layer.raw_decay.detach().cpu().numpy(),
                            residues.numpy(), direct.numpy(), np.zeros(c))
    nw, _ = record_margin("config1:laplace:y", y.cpu().numpy(), ref, 1e-6)
    assert nw <= 1e-6
