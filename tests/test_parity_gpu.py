"""CUDA path vs the reference's recorded outputs and the float64 oracle.

Tolerances (max relative error, normwise — max|got - ref| / max|ref|):
  logits, fp32 inputs/params         <= 1e-4
  logits, bf16 inputs with fp32 state <= 2e-2
  raw moments                         <= 5e-4 (fp32) / 2e-2 (bf16)
Padded positions must give bit-identical results: changing x at padded
steps must not change a single bit of the logits.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch
from conftest import golden_names, golden_params, load_golden, record_margin, rel_err

from lnet_b200 import AlphabetConfig, B200Alphabet, B200PoleResidueTemporalMixing
from oracle import alphabet_oracle as A
from oracle import laplace_oracle as L

pytestmark = pytest.mark.gpu


def build_from_golden(z, device):
    b, t, cin, d, m, k = (int(v) for v in z["meta.shape"])
    model = B200Alphabet(AlphabetConfig(cin, d, m, k), k).eval()
    model.load_effective_parameters({k2: torch.from_numpy(v) for k2, v in golden_params(z).items()})
    return model.to(device)


def meta_of(z, device):
    out = {}
    for key in ("time_delta", "observation_mask", "valid_mask"):
        if "in." + key in z:
            out[key] = torch.from_numpy(z["in." + key]).to(device)
    return out


@pytest.mark.parametrize("name", golden_names("alphabet_"))
def test_alphabet_matches_reference_golden(name, cuda_device):
    z = load_golden(name)
    model = build_from_golden(z, cuda_device)
    bf16 = bool(z["meta.bf16"])
    x = torch.from_numpy(z["in.x"]).to(cuda_device)
    if bf16:
        x = x.to(torch.bfloat16)
    with torch.no_grad():
        logits, wm, rm = model(x, **meta_of(z, cuda_device), return_moments=True)
    torch.cuda.synchronize()
    tol_l, tol_m = (2e-2, 2e-2) if bf16 else (1e-4, 5e-4)
    nw, _ = record_margin(f"golden:{name}:logits", logits.cpu().numpy(), z["out.logits"], tol_l)
    assert nw <= tol_l
    nw, _ = record_margin(f"golden:{name}:writer_moments", wm.cpu().numpy(),
                          z["out.writer_moments"], tol_m)
    assert nw <= tol_m
    nw, _ = record_margin(f"golden:{name}:reader_moments", rm.cpu().numpy(),
                          z["out.reader_moments"], tol_m)
    assert nw <= tol_m
    ref64 = A.alphabet_forward(z["in.x"], golden_params(z), time_delta=z.get("in.time_delta"),
                               observation_mask=z.get("in.observation_mask"),
                               valid_mask=z.get("in.valid_mask"), dtype=np.float64)
    nw, _ = record_margin(f"oracle64:{name}:logits", logits.cpu().numpy(), ref64, tol_l)
    assert nw <= tol_l


def test_padding_is_bit_identical(cuda_device):
    z = load_golden("alphabet_valid")
    model = build_from_golden(z, cuda_device)
    meta = meta_of(z, cuda_device)
    x = torch.from_numpy(z["in.x"]).to(cuda_device)
    pad = meta["valid_mask"] == 0
    x2 = x.clone()
    x2[pad] = 1.0e3 * torch.randn_like(x2[pad])
    with torch.no_grad():
        a = model(x, **meta)
        b = model(x2, **meta)
    assert torch.equal(a, b)


@pytest.mark.parametrize("name", golden_names("laplace_"))
@pytest.mark.parametrize("dtype", [torch.float32, torch.float64])
def test_laplace_matches_reference_golden(name, dtype, cuda_device):
    z = load_golden(name)
    d = z["p.residues"].shape[0]
    modes = z["p.residues"].shape[1]
    layer = B200PoleResidueTemporalMixing(d, modes, dt=float(z["p.dt"]),
                                          min_decay=float(z["p.min_decay"]))
    with torch.no_grad():
        layer.raw_decay.copy_(torch.from_numpy(z["p.raw_decay"]))
        layer.residues.copy_(torch.from_numpy(z["p.residues"]))
        layer.direct_term.copy_(torch.from_numpy(z["p.direct_term"]))
        layer.bias.copy_(torch.from_numpy(z["p.bias"]))
    layer = layer.to(cuda_device)
    x = torch.from_numpy(z["in.x"]).to(cuda_device, dtype)
    y = layer(x)
    assert y.dtype == dtype
    tol = 1e-6 if dtype == torch.float32 else 1e-12
    ref = z["out.y"] if dtype == torch.float32 else L.laplace_forward(
        z["in.x"].astype(np.float64), z["p.raw_decay"], z["p.residues"], z["p.direct_term"],
        z["p.bias"], float(z["p.dt"]), float(z["p.min_decay"]))
    assert rel_err(y.cpu().numpy(), ref) <= tol
