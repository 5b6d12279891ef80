"""Fused unit-grid route (tcgen05 writer/reader kernels) vs the float64 oracle.

Config-4 shape (C=48, D=96, M=48, bf16 inputs and activations, fp32 state):
chunk-aligned, ragged and very short sequences, real and complex poles.
Tolerance: max relative error (normwise) <= 2e-2 on logits and raw moments
(bf16 I/O with fp32 state), and the fused route must agree with the general
route run on the same bf16 inputs to the same tolerance.
"""

from __future__ import annotations

import ctypes
import math

import numpy as np
import pytest
import torch
from conftest import rel_err

from lnet_b200 import AlphabetConfig, B200Alphabet, _lib
from oracle import alphabet_oracle as A

pytestmark = pytest.mark.gpu

C, D, M, K = 48, 96, 48, 37


def random_params(seed, real_poles):
    g = torch.Generator().manual_seed(seed)

    def rn(*shape, scale=1.0):
        return torch.randn(*shape, generator=g) * scale

    p = {
        "stem.projection.weight": torch.linalg.qr(rn(D, C))[0],
        "stem.local.weight": rn(D, 1, 5, scale=1 / math.sqrt(5)),
        "stem.local.bias": rn(D, scale=0.1),
        "second_local.weight": rn(D, 1, 5, scale=1 / math.sqrt(5)),
        "second_local.bias": rn(D, scale=0.1),
        "forward_block.direct_scale": rn(D, scale=0.3),
        "forward_block.layer_scale": rn(D, scale=0.3),
        "head.classifier.weight": rn(K, 14 * M, scale=1 / math.sqrt(14 * M)),
        "head.classifier.bias": rn(K, scale=0.1),
    }
    for blk in ("forward_block", "backward_block"):
        if real_poles:
            lam = torch.exp(torch.empty(M).uniform_(math.log(1.1e-3), 0.0, generator=g))
            p[f"{blk}.raw_decay"] = torch.logit((lam - 1e-3) / (2 - 1e-3))
            p[f"{blk}.raw_frequency"] = torch.zeros(M)
        else:
            p[f"{blk}.raw_decay"] = rn(M, scale=2.0)
            p[f"{blk}.raw_frequency"] = rn(M, scale=0.8)
        p[f"{blk}.norm.weight"] = 1 + rn(D, scale=0.1)
        p[f"{blk}.frame.weight"] = torch.linalg.qr(rn(D, 2 * M))[0]
    return {k: v.to(torch.bfloat16).float() for k, v in p.items()}


def build(params, device):
    model = B200Alphabet(AlphabetConfig(C, D, M, K), K).eval()
    model.load_effective_parameters(params)
    return model.to(device)


def route_of(model, x):
    params, _ = model._effective(x.device)
    req = model._request(x, None, None, None, _lib.LNET_BF16)
    return _lib.load().lnet_b200_alphabet_route(ctypes.byref(params), ctypes.byref(req))


@pytest.mark.parametrize("b,t,real", [(3, 256, True), (2, 300, False), (4, 128, True),
                                      (2, 1000, True), (3, 5, False), (2, 1, True),
                                      (5, 129, False)])
def test_fused_route_matches_oracle(b, t, real, cuda_device):
    params = random_params(100 + t, real)
    model = build(params, cuda_device)
    g = torch.Generator().manual_seed(t)
    x = torch.randn(b, t, C, generator=g).to(torch.bfloat16)
    xd = x.to(cuda_device)
    _lib.set_route(_lib.ROUTE_AUTO)
    assert route_of(model, xd) == 0, "the fused route must serve this request"
    with torch.no_grad():
        logits, wm, rm = model(xd, return_moments=True)
    torch.cuda.synchronize()
    pn = {k: v.numpy() for k, v in params.items()}
    st = A.alphabet_forward(x.float().numpy(), pn, dtype=np.float64, return_stages=True)
    assert rel_err(logits.cpu().numpy(), st["logits"]) <= 2e-2
    assert rel_err(wm.cpu().numpy(), st["writer_moments"]) <= 2e-2
    assert rel_err(rm.cpu().numpy(), st["reader_moments"]) <= 2e-2
    _lib.set_route(_lib.ROUTE_GENERAL)
    try:
        with torch.no_grad():
            logits_g = model(xd)
    finally:
        _lib.set_route(_lib.ROUTE_AUTO)
    assert rel_err(logits.cpu().numpy(), logits_g.cpu().numpy()) <= 2e-2


def test_fused_route_long_sequence_carries(cuda_device):
    """Many chunks per row: carries must propagate through the look-back chain."""
    params = random_params(7, True)
    model = build(params, cuda_device)
    g = torch.Generator().manual_seed(9)
    x = torch.randn(2, 4096 + 77, C, generator=g).to(torch.bfloat16)
    with torch.no_grad():
        logits, wm, rm = model(x.to(cuda_device), return_moments=True)
    pn = {k: v.numpy() for k, v in params.items()}
    st = A.alphabet_forward(x.float().numpy(), pn, dtype=np.float64, return_stages=True)
    assert rel_err(wm.cpu().numpy(), st["writer_moments"]) <= 2e-2
    assert rel_err(rm.cpu().numpy(), st["reader_moments"]) <= 2e-2
    assert rel_err(logits.cpu().numpy(), st["logits"]) <= 2e-2


def shape_params(c, d, m, k, seed, real_poles):
    g = torch.Generator().manual_seed(seed)

    def rn(*shape, scale=1.0):
        return torch.randn(*shape, generator=g) * scale

    p = {
        "stem.projection.weight": torch.linalg.qr(rn(d, c))[0] if d >= c
        else torch.linalg.qr(rn(c, d))[0].T,
        "stem.local.weight": rn(d, 1, 5, scale=1 / math.sqrt(5)),
        "stem.local.bias": rn(d, scale=0.1),
        "second_local.weight": rn(d, 1, 5, scale=1 / math.sqrt(5)),
        "second_local.bias": rn(d, scale=0.1),
        "forward_block.direct_scale": rn(d, scale=0.3),
        "forward_block.layer_scale": rn(d, scale=0.3),
        "head.classifier.weight": rn(k, 14 * m, scale=1 / math.sqrt(14 * m)),
        "head.classifier.bias": rn(k, scale=0.1),
    }
    for blk in ("forward_block", "backward_block"):
        if real_poles:
            lam = torch.exp(torch.empty(m).uniform_(math.log(1.1e-3), 0.0, generator=g))
            p[f"{blk}.raw_decay"] = torch.logit((lam - 1e-3) / (2 - 1e-3))
            p[f"{blk}.raw_frequency"] = torch.zeros(m)
        else:
            p[f"{blk}.raw_decay"] = rn(m, scale=2.0)
            p[f"{blk}.raw_frequency"] = rn(m, scale=0.8)
        p[f"{blk}.norm.weight"] = 1 + rn(d, scale=0.1)
        p[f"{blk}.frame.weight"] = torch.linalg.qr(rn(d, 2 * m))[0]
    return {key: v.to(torch.bfloat16).float() for key, v in p.items()}


@pytest.mark.parametrize("c,d,m", [(32, 96, 48), (64, 64, 32), (32, 64, 32), (16, 32, 16)])
@pytest.mark.parametrize("real", [True, False])
def test_other_compiled_shapes(c, d, m, real, cuda_device):
    """The other compiled fused instances against the oracle and the general route."""
    k = 11
    params = shape_params(c, d, m, k, seed=c + d + m, real_poles=real)
    model = B200Alphabet(AlphabetConfig(c, d, m, k), k).eval()
    model.load_effective_parameters(params)
    model = model.to(cuda_device)
    g = torch.Generator().manual_seed(d)
    x = torch.randn(3, 300, c, generator=g).to(torch.bfloat16)
    xd = x.to(cuda_device)
    assert route_of(model, xd) == 0, "the fused route must serve this shape"
    with torch.no_grad():
        logits, wm, rm = model(xd, return_moments=True)
        _lib.set_route(_lib.ROUTE_GENERAL)
        try:
            general = model(xd)
        finally:
            _lib.set_route(_lib.ROUTE_AUTO)
    pn = {key: v.numpy() for key, v in params.items()}
    st = A.alphabet_forward(x.float().numpy(), pn, dtype=np.float64, return_stages=True)
    assert rel_err(logits.cpu().numpy(), st["logits"]) <= 2e-2
    assert rel_err(wm.cpu().numpy(), st["writer_moments"]) <= 2e-2
    assert rel_err(rm.cpu().numpy(), st["reader_moments"]) <= 2e-2
    assert rel_err(logits.cpu().numpy(), general.cpu().numpy()) <= 2e-2
