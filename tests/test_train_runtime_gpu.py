"""The captured training step (lnet_b200.train_runtime) against eager training.

Two copies of one model train on the same batches: one eagerly (module forward,
``loss.backward()``, ``optimizer.step()``), one through the runtime's graph
replays (``step``, ``step_static``, ``step_leased`` in turn).  The captured step
builds the frames with the capture-safe matrix exponential (fp32 rounding away
from ``torch.matrix_exp``), so the comparison is to a tolerance:
* SGD: losses per step and every parameter after the steps (1e-4 relative);
* AdamW (capturable): losses per step (1e-3 relative; Adam's normalised update
  turns rounding-level gradient differences of near-zero entries into
  lr-sized parameter differences, so parameters are not compared);
* the other loss kinds (binary cross-entropy with logits, MSE) and a request
  with an observation and valid mask: the first captured loss equals the eager one.
"""

from __future__ import annotations

import copy

import pytest
import torch
from torch.nn import functional as F

from lnet_b200 import AlphabetConfig, B200Alphabet, prepare_exact_split_training
from lnet_b200.train_runtime import prepare_aggressive_training

pytestmark = pytest.mark.gpu

C, D, M, K, B, T = 16, 32, 16, 7, 4, 96


def _models(dev):
    torch.manual_seed(0)
    m1 = B200Alphabet(AlphabetConfig(C, D, M, 5), K).to(dev).train()
    return m1, copy.deepcopy(m1)


def _batches(dev, n, kind="cross_entropy"):
    g = torch.Generator(device="cpu").manual_seed(4)
    out = []
    for _ in range(n):
        x = torch.randn(B, T, C, generator=g).to(dev)
        if kind == "cross_entropy":
            y = torch.randint(0, K, (B,), generator=g).to(dev)
        else:
            y = torch.rand(B, K, generator=g).to(dev)
        out.append((x, y))
    return out


def _eager(model, opt, x, y, kind="cross_entropy", meta=None):
    opt.zero_grad(set_to_none=False)
    logits = model(x, **(meta or {}))
    if kind == "cross_entropy":
        loss = F.cross_entropy(logits, y)
    elif kind == "binary_cross_entropy":
        loss = F.binary_cross_entropy_with_logits(logits, y)
    else:
        loss = F.mse_loss(logits, y)
    loss.backward()
    opt.step()
    return float(loss.detach())


def _rel(a, b):
    return abs(a - b) / max(abs(b), 1e-30)


@pytest.mark.parametrize("optim", ["sgd", "adamw"])
def test_runtime_matches_eager_training(cuda_device, optim):
    m_rt, m_ea = _models(cuda_device)

    def make(m):
        if optim == "sgd":
            return torch.optim.SGD(m.parameters(), lr=0.05, momentum=0.9)
        return torch.optim.AdamW(m.parameters(), lr=1e-3, capturable=True)

    o_rt, o_ea = make(m_rt), make(m_ea)
    data = _batches(cuda_device, 6)
    ex_x, ex_y = data[0][0].clone(), data[0][1].clone()
    rt = prepare_aggressive_training(m_rt, o_rt, ex_x, ex_y)
    got = []
    for i, (x, y) in enumerate(data):
        if i % 3 == 0:
            loss = rt.step(x, y)
        elif i % 3 == 1:
            rt.static_inputs.copy_(x)
            rt.static_labels.copy_(y)
            loss = rt.step_static()
        else:
            ex_x.copy_(x)
            ex_y.copy_(y)
            loss = rt.step_leased(ex_x, ex_y)
        got.append(float(loss))
    want = [_eager(m_ea, o_ea, x, y) for x, y in data]
    tol = 1e-4 if optim == "sgd" else 1e-3
    for g_, w_ in zip(got, want):
        assert _rel(g_, w_) <= tol, (got, want)
    if optim == "sgd":
        for (name, p1), p2 in zip(m_rt.named_parameters(), m_ea.parameters()):
            err = ((p1 - p2).abs().max() / p2.abs().max().clamp_min(1e-12)).item()
            assert err <= 1e-4, (name, err)
    with pytest.raises(ValueError):
        rt.step_leased(data[1][0], data[1][1])
    rt.close()
    with pytest.raises(RuntimeError):
        rt.step_static()


@pytest.mark.parametrize("kind", ["binary_cross_entropy", "mse"])
def test_runtime_loss_kinds(cuda_device, kind):
    m_rt, m_ea = _models(cuda_device)
    o_rt = torch.optim.SGD(m_rt.parameters(), lr=0.01)
    o_ea = torch.optim.SGD(m_ea.parameters(), lr=0.01)
    (x, y), = _batches(cuda_device, 1, kind)
    with prepare_exact_split_training(m_rt, o_rt, x, y, loss_kind=kind) as rt:
        got = float(rt.step(x, y))
    assert _rel(got, _eager(m_ea, o_ea, x, y, kind)) <= 1e-4


def test_runtime_with_metadata(cuda_device):
    m_rt, m_ea = _models(cuda_device)
    o_rt = torch.optim.SGD(m_rt.parameters(), lr=0.01)
    o_ea = torch.optim.SGD(m_ea.parameters(), lr=0.01)
    (x, y), = _batches(cuda_device, 1)
    g = torch.Generator(device="cpu").manual_seed(8)
    meta = {"observation_mask": (torch.rand(B, T, C, generator=g) > 0.3).float().to(cuda_device),
            "valid_mask": (torch.arange(T).view(1, -1) <
                           torch.tensor([T, 50, 96, 7]).view(-1, 1)).float().to(cuda_device)}
    m_rt.validate_metadata = False  # value checks synchronise the host
    with prepare_exact_split_training(
            m_rt, o_rt, x, y, example_observation_mask=meta["observation_mask"],
            example_valid_mask=meta["valid_mask"]) as rt:
        got = [float(rt.step(x, y)) for _ in range(2)]
    want = [_eager(m_ea, o_ea, x, y, meta=meta) for _ in range(2)]
    for g_, w_ in zip(got, want):
        assert _rel(g_, w_) <= 1e-4, (got, want)
