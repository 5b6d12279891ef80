"""Host logic of the captured training runtime (lnet_b200.train_runtime), on CPU.

* ``capturable_matrix_exp`` (device-chosen squaring count) equals
  ``torch.matrix_exp`` on skew-symmetric and general matrices, small and large
  norms, fp64 and fp32, and so do its autograd gradients;
* the capture-safe frame builder reproduces the module's orthogonally
  parametrised frame weight (``B200Alphabet`` blocks), before and after the
  underlying parameter moves;
* argument checks: unsupported loss kinds, a non-capturable optimizer.
"""

from __future__ import annotations

import pytest
import torch

from lnet_b200 import AlphabetConfig, B200Alphabet
from lnet_b200.train_runtime import (
    AlphabetTrainingRuntime,
    _orthogonal_frame,
    capturable_matrix_exp,
)


@pytest.mark.parametrize("dtype", [torch.float64, torch.float32])
@pytest.mark.parametrize("scale", [1e-3, 0.3, 4.0, 60.0])
def test_matrix_exp_matches_torch(dtype, scale):
    g = torch.Generator().manual_seed(int(scale * 1000) + 7)
    x = torch.randn(24, 24, generator=g, dtype=torch.float64)
    # skew-symmetric (the frames' generators) at every scale; a general matrix
    # where exp stays of moderate size
    cases = [scale * (x - x.T) / 2] + ([scale * x / 24] if scale <= 4.0 else [])
    for a in cases:
        a = a.to(dtype)
        got = capturable_matrix_exp(a)
        want = torch.matrix_exp(a)
        # the squarings amplify rounding by about 2^s (s = 8 at scale 60)
        tol = 1e-12 if dtype == torch.float64 else (2e-5 if scale <= 4.0 else 2e-4)
        assert ((got - want).abs().max() / want.abs().max()).item() <= tol


def test_matrix_exp_gradient_matches_torch():
    g = torch.Generator().manual_seed(3)
    x = torch.randn(16, 16, generator=g, dtype=torch.float64)
    w = torch.randn(16, 16, generator=g, dtype=torch.float64)
    a1 = (2.0 * (x - x.T)).requires_grad_()
    a2 = a1.detach().clone().requires_grad_()
    (capturable_matrix_exp(a1) * w).sum().backward()
    (torch.matrix_exp(a2) * w).sum().backward()
    assert torch.allclose(a1.grad, a2.grad, rtol=0, atol=1e-10 * a2.grad.abs().max().item())


def test_frame_builder_reproduces_the_parametrised_frame():
    torch.manual_seed(0)
    model = B200Alphabet(AlphabetConfig(8, 16, 8, 5), 3)
    for blk in (model.forward_block, model.backward_block):
        want = blk.frame_matrix().detach()
        got = _orthogonal_frame(blk.frame).detach()
        assert torch.allclose(got, want, rtol=0, atol=2e-6)
        with torch.no_grad():  # move the trivialised parameter, as an optimizer would
            blk.frame.parametrizations.weight.original.add_(
                0.05 * torch.randn_like(blk.frame.parametrizations.weight.original))
        assert torch.allclose(_orthogonal_frame(blk.frame).detach(),
                              blk.frame_matrix().detach(), rtol=0, atol=2e-6)


def test_runtime_argument_checks():
    model = B200Alphabet(AlphabetConfig(8, 16, 8, 5), 3)
    x = torch.zeros(2, 4, 8)
    y = torch.zeros(2, dtype=torch.long)
    opt = torch.optim.AdamW(model.parameters(), capturable=False)
    with pytest.raises(ValueError, match="loss_kind"):
        AlphabetTrainingRuntime(model, opt, x, y, loss_kind="hinge")
    with pytest.raises(RuntimeError, match="CUDA"):
        AlphabetTrainingRuntime(model, opt, x, y)
