"""Pole-residue Laplace layer: the channel-diagonal kernel
(lnet_b200_laplace_forward_channelwise) against the float64 oracle and against the
dense kernel on the same parameters, at BASELINE config 1's layout (C channels x M
real poles each) and at ragged shapes (T not a multiple of the 16 time chunks,
fewer than 16 steps, channels not a multiple of 16, a dense direct term)."""

from __future__ import annotations

import math

import pytest
import torch
from conftest import record_margin, rel_err

from lnet_b200 import B200PoleResidueTemporalMixing
from lnet_b200.laplace import _launch, channel_diagonal_form
from oracle import laplace_oracle as L

pytestmark = pytest.mark.gpu


def per_channel_layer(c, per, seed, direct_dense=False):
    g = torch.Generator().manual_seed(seed)
    u = torch.empty(c, per, dtype=torch.float64).uniform_(math.log(0.01), 0.0, generator=g)
    poles = -torch.exp(u).reshape(-1)
    r = torch.randn(c, per, generator=g, dtype=torch.float64) / math.sqrt(per)
    residues = torch.zeros(c, c * per, c, dtype=torch.float64)
    for ch in range(c):
        residues[ch, ch * per:(ch + 1) * per, ch] = r[ch]
    direct = torch.randn(c, c, generator=g, dtype=torch.float64) if direct_dense else \
        torch.diag(torch.randn(c, generator=g, dtype=torch.float64))
    layer = B200PoleResidueTemporalMixing(c, c * per)
    layer.load_transfer_parameters(poles=poles, residues=residues, direct_term=direct,
                                   bias=torch.randn(c, generator=g, dtype=torch.float64))
    return layer


def _oracle(layer, x):
    return L.laplace_forward(x.numpy(), layer.raw_decay.detach().cpu().numpy(),
                             layer.residues.detach().cpu().numpy(),
                             layer.direct_term.detach().cpu().numpy(),
                             layer.bias.detach().cpu().numpy())


@pytest.mark.parametrize("c,per,b,t,dense_direct", [(16, 8, 64, 512, False), (5, 3, 3, 37, True),
                                                    (20, 16, 2, 9, False), (16, 1, 4, 1000, True)])
@pytest.mark.parametrize("dtype", [torch.float32, torch.float64])
def test_channelwise_matches_oracle_and_dense(c, per, b, t, dense_direct, dtype, cuda_device):
    layer = per_channel_layer(c, per, seed=c * 100 + t, direct_dense=dense_direct)
    assert channel_diagonal_form(layer.residues.detach()) is not None
    layer = layer.to(cuda_device)
    g = torch.Generator().manual_seed(t)
    x = torch.randn(b, t, c, generator=g, dtype=torch.float64).to(dtype)
    xd = x.to(cuda_device)
    y = layer(xd)
    ref = _oracle(layer, x)
    tol = 1e-6 if dtype == torch.float32 else 1e-12
    nw, _ = record_margin(f"laplace_channelwise:{c}x{per}:{b}x{t}:{dtype}", y.cpu().numpy(), ref,
                          tol)
    assert nw <= tol
    dense = _launch(xd, layer.raw_decay.detach(), layer.residues.detach(),
                    layer.direct_term.detach(), layer.bias.detach(), layer.modes, 1.0, 1e-3)
    assert rel_err(y.cpu().numpy(), dense.cpu().numpy()) <= tol


def test_dense_residues_keep_the_dense_kernel(cuda_device):
    layer = B200PoleResidueTemporalMixing(6, 5)  # random dense residues
    assert channel_diagonal_form(layer.residues.detach()) is None
    layer = layer.to(cuda_device)
    x = torch.randn(2, 40, 6, dtype=torch.float64)
    y = layer(x.to(cuda_device))
    assert rel_err(y.cpu().numpy(), _oracle(layer, x)) <= 1e-12
