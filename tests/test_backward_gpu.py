"""Backward pass on the GPU against gradients from the reference's autograd.

``tests/golden/grad_*.npz`` hold dL/dparameter of ``L = sum(logits * dlogits)``
from the reference ``lnet.Alphabet`` in float64 (evaluated at the stored float32
parameters; ``tests/golden/make_grad_golden.py``).  ``B200Alphabet`` in
training mode runs ``lnet_b200_alphabet_train_forward`` and, on
``loss.backward()``, ``lnet_b200_alphabet_backward`` (fp32).  Bounds: logits
1e-5 relative, every parameter gradient 2e-4 relative (normwise per tensor;
fp32 against float64 over sequences up to 300 steps).  Also: the training
forward equals the inference forward; the oracle VJP agrees at a size the
goldens do not cover; return_moments (an inference option) raises in training.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch
from conftest import golden_params, load_golden, rel_err

from lnet_b200 import AlphabetConfig, B200Alphabet
from oracle import alphabet_grad_oracle as G

pytestmark = pytest.mark.gpu

CASES = ["grad_plain", "grad_real_poles", "grad_long", "grad_valid", "grad_obs_channel",
         "grad_obs_event", "grad_delta", "grad_all_meta"]


def _model(z, device):
    b, t, cin, d, m, k = (int(v) for v in z["meta.shape"])
    model = B200Alphabet(AlphabetConfig(cin, d, m, k), k)
    model.load_effective_parameters({k2: torch.from_numpy(v) for k2, v in golden_params(z).items()})
    return model.to(device).train()


def _grads(model, x, dlogits, valid=None, obs=None, delta=None):
    model.zero_grad(set_to_none=True)
    logits = model(x, valid_mask=valid, observation_mask=obs, time_delta=delta)
    (logits * dlogits).sum().backward()
    out = {name: p.grad for name, p in model.named_parameters() if p.grad is not None}
    return logits.detach(), out


@pytest.mark.parametrize("name", CASES)
def test_backward_matches_reference_autograd(name, cuda_device):
    z = load_golden(name)
    model = _model(z, cuda_device)
    x = torch.from_numpy(z["in.x"]).to(cuda_device)
    dl = torch.from_numpy(z["in.dlogits"]).to(cuda_device)
    valid = torch.from_numpy(z["in.valid_mask"]).to(cuda_device) if "in.valid_mask" in z else None
    obs = (torch.from_numpy(z["in.observation_mask"]).to(cuda_device)
           if "in.observation_mask" in z else None)
    delta = torch.from_numpy(z["in.time_delta"]).to(cuda_device) if "in.time_delta" in z else None
    logits, grads = _grads(model, x, dl, valid, obs, delta)
    assert rel_err(logits.cpu().numpy(), z["out.logits"]) <= 1e-5
    checked = 0
    for key in z:
        if not key.startswith("g."):
            continue
        pname = key[2:]
        got = grads[pname].cpu().numpy().reshape(z[key].shape)
        assert rel_err(got, z[key]) <= 2e-4, (pname, rel_err(got, z[key]))
        checked += 1
    assert checked == 17


def test_training_forward_equals_inference(cuda_device):
    z = load_golden("grad_long")
    model = _model(z, cuda_device)
    x = torch.from_numpy(z["in.x"]).to(cuda_device)
    train_logits = model(x).detach()
    with torch.no_grad():
        model.eval()
        infer = model(x)
    assert rel_err(train_logits.cpu().numpy(), infer.cpu().numpy()) <= 1e-5


@pytest.mark.parametrize("shape", [
    dict(b=3, t=517, cin=8, d=32, m=16, k=6, ksize=5, dil=4),  # several chunks, fused conv VJP
    dict(b=2, t=150, cin=5, d=30, m=8, k=4, ksize=3, dil=2),   # generic conv kernels, 4 !| D
])
def test_backward_larger_case_against_oracle(cuda_device, shape):
    """Several scan chunks per row and a valid mask with ragged lengths (and a
    non-canonical conv that takes the generic kernels): the CUDA backward
    against the float64 oracle VJP."""
    g = torch.Generator().manual_seed(21)
    b, t, cin, d, m, k = (shape[n] for n in ("b", "t", "cin", "d", "m", "k"))
    model = B200Alphabet(AlphabetConfig(cin, d, m, k), k, dwconv_kernel_size=shape["ksize"],
                         dwconv_dilation=shape["dil"])
    with torch.no_grad():
        for blk in (model.forward_block, model.backward_block):
            blk.raw_decay.copy_(torch.randn(m, generator=g) * 2.0)
            blk.raw_frequency.copy_(torch.randn(m, generator=g) * 0.8)
            blk.norm.weight.copy_(1.0 + 0.2 * torch.randn(d, generator=g))
        model.forward_block.direct_scale.copy_(0.5 * torch.randn(d, generator=g))
        model.forward_block.layer_scale.copy_(0.5 * torch.randn(d, generator=g))
        for conv in (model.stem.local, model.second_local):
            conv.weight.copy_(torch.randn(conv.weight.shape, generator=g) / 5 ** 0.5)
            conv.bias.copy_(0.1 * torch.randn(d, generator=g))
    for blk in (model.forward_block, model.backward_block):  # plain frames: comparable grads
        B200Alphabet._set_frame(blk, blk.frame_matrix().detach())
    x = torch.randn(b, t, cin, generator=g)
    lengths = torch.tensor([t, 300, 77][:b])
    valid = (torch.arange(t).view(1, -1) < lengths.view(-1, 1)).float()
    dl = torch.randn(b, k, generator=g)
    model = model.to(cuda_device).train()
    _, grads = _grads(model, x.to(cuda_device), dl.to(cuda_device), valid.to(cuda_device))
    params = {n: p.detach().cpu().numpy() for n, p in model.named_parameters()}
    params.update({n: model.get_buffer(n).cpu().numpy()
                   for n in ("backward_block.direct_scale", "backward_block.layer_scale")})
    ref = G.alphabet_backward(x.numpy(), params, dl.numpy(), valid_mask=valid.numpy(),
                              dilation=shape["dil"])
    assert len(ref) == 17
    for name, gref in ref.items():
        got = grads[name].cpu().numpy().reshape(gref.shape)
        assert rel_err(got, gref) <= 5e-4, (name, rel_err(got, gref))


def test_backward_bf16_inputs_tf32(cuda_device):
    """bf16 inputs train with TF32 GEMMs: gradients within 2e-2 of the fp32 ones."""
    z = load_golden("grad_long")
    model = _model(z, cuda_device)
    x = torch.from_numpy(z["in.x"]).to(cuda_device).to(torch.bfloat16)
    dl = torch.from_numpy(z["in.dlogits"]).to(cuda_device)
    _, g16 = _grads(model, x, dl)
    _, g32 = _grads(model, x.float(), dl)
    for name, ref in g32.items():
        assert rel_err(g16[name].cpu().numpy(), ref.cpu().numpy()) <= 2e-2, name


def test_training_rejects_return_moments(cuda_device):
    z = load_golden("grad_plain")
    model = _model(z, cuda_device)
    x = torch.from_numpy(z["in.x"]).to(cuda_device)
    with pytest.raises(NotImplementedError):
        model(x, return_moments=True)
