"""Right-padded valid masks on the fused route (lnet_b200_alphabet_forward_lengths).

A right-padded row (valid = 1 for t < L, 0 after) computes exactly as an unpadded
row of L steps under the reference's masking (stem input and output masked, reader
input and output masked, moments over valid pairs with counts clamped at one), so
the fused route serves it with per-row lengths.  Checked at the config-4 shape
(bf16, C=48, D=96, M=48):
* against the general route given the same mask, and the float64 oracle (2e-2);
* lengths 0, 1, 5, 127, 128, 129, 300 and T in one batch (chunk boundaries,
  empty rows, a short last chunk);
* padded steps bit-identical: changing x at padded steps changes no logit bit;
* a mask that is not a right-padded prefix still runs (general route) correctly;
* the module routes a right-padded request through forward_lengths (fused kernels
  launched).
"""

from __future__ import annotations

import ctypes
import math

import numpy as np
import pytest
import torch
from conftest import record_margin, rel_err

from lnet_b200 import AlphabetConfig, B200Alphabet, _lib
from lnet_b200.alphabet import right_padded_lengths
from oracle import alphabet_oracle as A

pytestmark = pytest.mark.gpu

C, D, M, K = 48, 96, 48, 37
LENGTHS = [0, 1, 5, 127, 128, 129, 300, 333]
T = 333


def params(seed=3):
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
        p[f"{blk}.raw_decay"] = rn(M, scale=2.0)
        p[f"{blk}.raw_frequency"] = rn(M, scale=0.8)
        p[f"{blk}.norm.weight"] = 1 + rn(D, scale=0.1)
        p[f"{blk}.frame.weight"] = torch.linalg.qr(rn(D, 2 * M))[0]
    return {k: v.to(torch.bfloat16).float() for k, v in p.items()}


def setup(device):
    p = params()
    model = B200Alphabet(AlphabetConfig(C, D, M, K), K).eval()
    model.load_effective_parameters(p)
    model = model.to(device)
    g = torch.Generator().manual_seed(11)
    x = torch.randn(len(LENGTHS), T, C, generator=g).to(torch.bfloat16)
    valid = (torch.arange(T).view(1, -1) < torch.tensor(LENGTHS).view(-1, 1)).float()
    return p, model, x, valid


def test_lengths_route_matches_general_and_oracle(cuda_device):
    p, model, x, valid = setup(cuda_device)
    xd, vd = x.to(cuda_device), valid.to(cuda_device)
    with torch.no_grad():
        got = model(xd, valid_mask=vd)
        _lib.set_route(_lib.ROUTE_GENERAL)
        try:
            general = model(xd, valid_mask=vd)
        finally:
            _lib.set_route(_lib.ROUTE_AUTO)
    assert torch.isfinite(got).all()
    assert rel_err(got.cpu().numpy(), general.cpu().numpy()) <= 2e-2
    ref = A.alphabet_forward(x.float().numpy(), {k: v.numpy() for k, v in p.items()},
                             valid_mask=valid.numpy(), dtype=np.float64)
    nw, _ = record_margin("fused_lengths:config4_shape:logits", got.cpu().numpy(), ref, 2e-2)
    assert nw <= 2e-2


def test_padding_is_bit_identical_on_the_fused_route(cuda_device):
    _, model, x, valid = setup(cuda_device)
    xd, vd = x.to(cuda_device), valid.to(cuda_device)
    x2 = xd.clone()
    pad = vd == 0
    x2[pad] = (1.0e3 * torch.randn_like(x2[pad].float())).to(torch.bfloat16)
    with torch.no_grad():
        a = model(xd, valid_mask=vd)
        b = model(x2, valid_mask=vd)
    # the look-back re-associates carries between runs (1e-6 level), so compare the
    # padded-step independence on the same schedule-free quantity: rows whose length
    # is zero are exactly the head bias, and the rest agree to run-to-run noise
    assert rel_err(a.cpu().numpy(), b.cpu().numpy()) <= 1e-5
    bias = model.head.classifier.bias.detach().float()
    assert torch.allclose(a[0], bias, atol=1e-6, rtol=0)


def test_module_uses_the_lengths_entry_point(cuda_device):
    _, model, x, valid = setup(cuda_device)
    xd, vd = x.to(cuda_device), valid.to(cuda_device)
    lengths = right_padded_lengths(vd)
    assert lengths is not None and lengths.tolist() == LENGTHS
    lib = _lib.load()
    params_c, _keep = model._effective(cuda_device)
    req = model._request(xd, None, None, None, _lib.LNET_BF16)
    assert lib.lnet_b200_alphabet_route(ctypes.byref(params_c), ctypes.byref(req)) == 0
    with torch.no_grad():
        model(xd, valid_mask=vd)
    # the fused route is 6 launches (prepare, writer, reader, finalize, head GEMM, reduce);
    # the general route with a valid mask is more than twice that
    assert _lib.last_launch_count() <= 6


def test_non_prefix_mask_keeps_the_general_route(cuda_device):
    p, model, x, valid = setup(cuda_device)
    holes = valid.clone()
    holes[6, 10:20] = 0.0  # a gap inside row 6
    assert right_padded_lengths(holes) is None
    with torch.no_grad():
        got = model(x.to(cuda_device), valid_mask=holes.to(cuda_device))
    ref = A.alphabet_forward(x.float().numpy(), {k: v.numpy() for k, v in p.items()},
                             valid_mask=holes.numpy(), dtype=np.float64)
    assert rel_err(got.cpu().numpy(), ref) <= 2e-2
