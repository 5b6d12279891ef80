"""Generate golden vectors from the reference ``lnet`` package (CPU, fp32).

Run in a container where the reference project is importable:

    LNET_REFERENCE_SRC=<reference>/src python tests/golden/make_golden.py

Each case builds a seeded ``lnet.Alphabet`` (or ``PoleResidueTemporalMixing``),
perturbs its parameters so that every term of the forward path is active,
runs the reference's eager CPU path under ``torch.no_grad()`` and stores, in
``tests/golden/<case>.npz``:

* ``in.*``     inputs and request metadata (``None`` entries are omitted),
* ``p.*``      parameters keyed by ``state_dict`` name, with each block frame
               materialised as ``p.<block>.frame.weight`` ([D, 2M]),
* ``out.*``    stage outputs: first_local, first_stream, encoded,
               writer/reader raw moments and logits,
* ``meta.*``   shapes and flags.

These files are the pins for ``oracle/`` and for the CUDA parity tests; the
GPU box never needs the reference itself.
"""

from __future__ import annotations

import math
import os
import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
# the reference checkout: LNET_REFERENCE_SRC, else a sibling `reference/src` of this repo
sys.path.insert(0, os.environ.get("LNET_REFERENCE_SRC",
                                  str(HERE.parents[2] / "reference" / "src")))

from lnet import Alphabet  # noqa: E402
from lnet.laplace import PoleResidueTemporalMixing  # noqa: E402
from lnet.pac_types import PACExperimentConfig  # noqa: E402

torch.set_num_threads(4)


def build_alphabet(*, cin, d, m, k, t, seed, real_poles=False, bf16=False):
    cfg = PACExperimentConfig(
        sample_count=1,
        validation_count=1,
        test_count=0,
        sequence_length=t,
        raw_input_dim=cin,
        output_dim=k,
        model_dim=d,
        modes=m,
    )
    torch.manual_seed(seed)
    model = Alphabet(cfg, k).eval()
    g = torch.Generator().manual_seed(seed + 1)

    def rn(*shape, scale=1.0):
        return torch.randn(*shape, generator=g) * scale

    with torch.no_grad():
        for blk in (model.forward_block, model.backward_block):
            mm = blk.raw_decay.numel()
            if real_poles:
                lam = torch.exp(torch.empty(mm).uniform_(math.log(1.1e-3), 0.0, generator=g))
                blk.raw_decay.copy_(torch.logit((lam - 1e-3) / (2.0 - 1e-3)))
                blk.raw_frequency.zero_()
            else:
                blk.raw_decay.copy_(rn(mm, scale=2.0))
                blk.raw_frequency.copy_(rn(mm, scale=0.8))
            blk.norm.weight.copy_(1.0 + rn(d, scale=0.2))
            orig = blk.frame.parametrizations.weight.original
            orig.add_(rn(*orig.shape, scale=0.1))
        model.forward_block.direct_scale.copy_(rn(d, scale=0.5))
        model.forward_block.layer_scale.copy_(rn(d, scale=0.5))
        model.stem.local.weight.copy_(rn(d, 1, 5, scale=1.0 / math.sqrt(5.0)))
        model.stem.local.bias.copy_(rn(d, scale=0.1))
        model.second_local.weight.copy_(rn(d, 1, 5, scale=1.0 / math.sqrt(5.0)))
        model.second_local.bias.copy_(rn(d, scale=0.1))
        model.head.classifier.weight.copy_(rn(k, 14 * m, scale=1.0 / math.sqrt(14 * m)))
        model.head.classifier.bias.copy_(rn(k, scale=0.1))
        if bf16:
            for p in model.parameters():
                p.copy_(p.to(torch.bfloat16).float())
    return model


def params_of(model):
    out = {}
    for name, value in model.state_dict().items():
        if ".parametrizations." in name:
            continue
        out["p." + name] = value.detach().float().numpy()
    for blk in ("forward_block", "backward_block"):
        out[f"p.{blk}.frame.weight"] = getattr(model, blk).frame.weight.detach().float().numpy()
    return out


def make_inputs(*, b, t, cin, seed, delta=False, obs=None, valid=False, bf16=False):
    g = torch.Generator().manual_seed(seed + 7)
    x = torch.randn(b, t, cin, generator=g)
    if bf16:
        x = x.to(torch.bfloat16).float()
    meta = {}
    if delta:
        dt = -torch.log(torch.rand(b, t, generator=g).clamp_min(1e-12))
        meta["time_delta"] = dt.clamp(0.05, 4.0)
    if obs == "channel":
        meta["observation_mask"] = (torch.rand(b, t, cin, generator=g) < 0.8).float()
    elif obs == "event":
        meta["observation_mask"] = (torch.rand(b, t, generator=g) < 0.8).float()
    if valid:
        lengths = torch.randint(max(1, t // 2), t + 1, (b,), generator=g)
        lengths[0] = t
        meta["valid_mask"] = (torch.arange(t).view(1, -1) < lengths.view(-1, 1)).float()
    return x, meta


def run_alphabet_case(name, *, b, t, cin, d, m, k, seed, real_poles=False, bf16=False,
                      delta=False, obs=None, valid=False):
    model = build_alphabet(cin=cin, d=d, m=m, k=k, t=t, seed=seed, real_poles=real_poles,
                           bf16=bf16)
    x, meta = make_inputs(b=b, t=t, cin=cin, seed=seed, delta=delta, obs=obs, valid=valid,
                          bf16=bf16)
    with torch.no_grad():
        first_local, a_delta, a_obs, a_valid = model._edge_stem(
            x, meta.get("time_delta"), meta.get("observation_mask"), meta.get("valid_mask")
        )
        first_stream, first_moments = model._writer(first_local, a_delta, a_obs, a_valid)
        encoded, second_moments = model._terminal_reader(first_stream, a_delta, None, a_valid)
        logits = model(x, **meta)
    rec = {"in.x": x.numpy()}
    for key, value in meta.items():
        rec["in." + key] = value.numpy()
    rec.update(params_of(model))
    rec.update(
        {
            "out.first_local": first_local.numpy(),
            "out.first_stream": first_stream.numpy(),
            "out.encoded": encoded.numpy(),
            "out.writer_moments": first_moments.numpy(),
            "out.reader_moments": second_moments.numpy(),
            "out.logits": logits.numpy(),
            "meta.shape": np.array([b, t, cin, d, model.modes, k]),
            "meta.bf16": np.array(int(bf16)),
        }
    )
    np.savez_compressed(HERE / f"{name}.npz", **rec)
    print(f"{name}: logits {tuple(logits.shape)} |max| {logits.abs().max().item():.4g}")


def run_laplace_case(name, *, b, t, d, modes, seed, block_diag_per_channel=None):
    torch.manual_seed(seed)
    layer = PoleResidueTemporalMixing(d, modes if block_diag_per_channel is None
                                      else d * block_diag_per_channel)
    g = torch.Generator().manual_seed(seed + 3)
    if block_diag_per_channel is not None:
        per = block_diag_per_channel
        u = torch.empty(d, per, dtype=torch.float64).uniform_(math.log(0.01), 0.0, generator=g)
        poles = -torch.exp(u).reshape(-1)
        r = torch.randn(d, per, generator=g, dtype=torch.float64) / math.sqrt(per)
        residues = torch.zeros(d, d * per, d, dtype=torch.float64)
        for c in range(d):
            residues[c, c * per : (c + 1) * per, c] = r[c]
        direct = torch.diag(torch.randn(d, generator=g, dtype=torch.float64))
        bias = torch.zeros(d, dtype=torch.float64)
    else:
        poles = -(torch.rand(modes, generator=g, dtype=torch.float64) * 1.5 + 0.01)
        residues = torch.randn(d, modes, d, generator=g, dtype=torch.float64) * 0.3
        direct = torch.randn(d, d, generator=g, dtype=torch.float64) * 0.3
        bias = torch.randn(d, generator=g, dtype=torch.float64) * 0.1
    layer.load_transfer_parameters(poles=poles, residues=residues, direct_term=direct, bias=bias)
    x = torch.randn(b, t, d, generator=g)
    with torch.no_grad():
        y = layer(x)
    np.savez_compressed(
        HERE / f"{name}.npz",
        **{
            "in.x": x.numpy(),
            "p.raw_decay": layer.raw_decay.detach().numpy(),
            "p.residues": layer.residues.detach().numpy(),
            "p.direct_term": layer.direct_term.detach().numpy(),
            "p.bias": layer.bias.detach().numpy(),
            "p.dt": np.array(layer.dt),
            "p.min_decay": np.array(layer.min_decay),
            "out.y": y.numpy(),
        },
    )
    print(f"{name}: y {tuple(y.shape)}")


def main():
    common = {"cin": 6, "d": 16, "m": 8, "k": 7}
    run_alphabet_case("alphabet_plain", b=3, t=50, seed=1, **common)
    run_alphabet_case("alphabet_real_poles", b=2, t=67, seed=2, real_poles=True, **common)
    run_alphabet_case("alphabet_valid", b=4, t=45, seed=3, valid=True, **common)
    run_alphabet_case("alphabet_obs_channel", b=3, t=40, seed=4, obs="channel", **common)
    run_alphabet_case("alphabet_obs_event", b=3, t=40, seed=5, obs="event", **common)
    run_alphabet_case("alphabet_delta", b=3, t=60, seed=6, delta=True, **common)
    run_alphabet_case("alphabet_all_meta", b=4, t=64, seed=7, delta=True, obs="channel",
                      valid=True, real_poles=True, **common)
    run_alphabet_case("alphabet_bf16", b=2, t=70, seed=8, bf16=True, real_poles=True,
                      cin=8, d=24, m=12, k=9)
    run_alphabet_case("alphabet_odd", b=2, t=33, seed=9, cin=5, d=12, m=6, k=3)
    run_alphabet_case("alphabet_long", b=1, t=300, seed=10, real_poles=True, **common)
    for t in (1, 2, 3, 4, 5):
        run_alphabet_case(f"alphabet_short_t{t}", b=2, t=t, seed=20 + t, **common)
        run_alphabet_case(f"alphabet_short_meta_t{t}", b=2, t=t, seed=30 + t, delta=True,
                          obs="channel", valid=True, **common)
    run_laplace_case("laplace_dense", b=2, t=24, d=4, modes=3, seed=40)
    run_laplace_case("laplace_per_channel", b=3, t=40, d=4, modes=0, seed=41,
                     block_diag_per_channel=3)


if __name__ == "__main__":
    main()
