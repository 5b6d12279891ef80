"""Observation masks on the fused route.

An observation mask scales the raw inputs before the stem and the writer's drive
by the event mask (the mask's amax over its channels); the reader takes none
(src/lnet/alphabet_backbone.py:538-569, 649-676, 1170-1180).  The fused writer
applies both inside the kernel: the landed x tile is scaled in shared memory
before the stem GEMM, and each token's xhat row (the drive GEMM operand) by its
event mask.  Checked at the config-4 shape (bf16, C=48, D=96, M=48):
* [B,T], [B,T,1] and [B,T,C] masks, 0/1 and fractional, against the general
  route given the same mask and against the float64 oracle (2e-2, bf16);
* an observation mask together with a right-padded valid mask (per-row lengths);
* an all-ones mask gives the unmasked logits;
* the request stays on the fused route (six launches).
"""

from __future__ import annotations

import numpy as np
import pytest
import torch
from conftest import record_margin, rel_err
from test_fused_lengths_gpu import LENGTHS, T, setup

from lnet_b200 import _lib
from oracle import alphabet_oracle as A

pytestmark = pytest.mark.gpu


def _mask(kind: str, b: int, c: int, seed: int = 5) -> torch.Tensor:
    g = torch.Generator().manual_seed(seed)
    if kind == "token":
        return (torch.rand(b, T, generator=g) > 0.3).float()
    if kind == "token1":
        return torch.rand(b, T, 1, generator=g)  # fractional
    if kind == "channel":
        m = (torch.rand(b, T, c, generator=g) > 0.5).float()
        m[:, 7:19] = 0.0  # whole events unobserved: no drive there
        return m
    if kind == "channel_frac":
        return torch.rand(b, T, c, generator=g)
    raise ValueError(kind)


def _run(model, x, obs=None, valid=None, general=False):
    if general:
        _lib.set_route(_lib.ROUTE_GENERAL)
    try:
        with torch.no_grad():
            out = model(x, observation_mask=obs, valid_mask=valid)
        return out, _lib.last_launch_count()
    finally:
        _lib.set_route(_lib.ROUTE_AUTO)


@pytest.mark.parametrize("kind", ["token", "token1", "channel", "channel_frac"])
def test_observation_mask_fused_matches_general_and_oracle(cuda_device, kind):
    p, model, x, _ = setup(cuda_device)
    obs = _mask(kind, x.shape[0], x.shape[2])
    xd, od = x.to(cuda_device), obs.to(cuda_device)
    got, launches = _run(model, xd, od)
    assert launches <= 6, "the masked request left the fused route"
    general, _ = _run(model, xd, od, general=True)
    assert torch.isfinite(got).all()
    assert rel_err(got.cpu().numpy(), general.cpu().numpy()) <= 2e-2
    ref = A.alphabet_forward(x.float().numpy(), {k: v.numpy() for k, v in p.items()},
                             observation_mask=obs.numpy(), dtype=np.float64)
    nw, _ = record_margin(f"fused_obs:{kind}:logits", got.cpu().numpy(), ref, 2e-2)
    assert nw <= 2e-2


def test_observation_mask_with_right_padded_valid(cuda_device):
    p, model, x, valid = setup(cuda_device)
    obs = _mask("channel", x.shape[0], x.shape[2], seed=9)
    xd, od, vd = x.to(cuda_device), obs.to(cuda_device), valid.to(cuda_device)
    got, launches = _run(model, xd, od, vd)
    assert launches <= 6
    ref = A.alphabet_forward(x.float().numpy(), {k: v.numpy() for k, v in p.items()},
                             observation_mask=obs.numpy(), valid_mask=valid.numpy(),
                             dtype=np.float64)
    nw, _ = record_margin("fused_obs:channel+lengths:logits", got.cpu().numpy(), ref, 2e-2)
    assert nw <= 2e-2
    assert len(LENGTHS) == x.shape[0]


def test_all_ones_mask_is_the_unmasked_forward(cuda_device):
    _, model, x, _ = setup(cuda_device)
    xd = x.to(cuda_device)
    ones = torch.ones(x.shape[0], T, x.shape[2], device=cuda_device)
    masked, _ = _run(model, xd, ones)
    plain, _ = _run(model, xd)
    # x * 1 and xhat * 1 are exact; what remains is the look-back's run-to-run
    # re-association of carries
    assert rel_err(masked.cpu().numpy(), plain.cpu().numpy()) <= 1e-5
