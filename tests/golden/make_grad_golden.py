"""Generate gradient golden vectors from the reference ``lnet`` package (CPU, float64).

Run in a container where the reference project is importable:

    LNET_REFERENCE_SRC=<reference>/src python tests/golden/make_grad_golden.py

Each case builds the same seeded, perturbed ``lnet.Alphabet`` as
``make_golden.py``, converts it to float64, runs the reference's eager CPU
forward with autograd and differentiates ``L = sum(logits * dlogits)`` for a
seeded ``dlogits``.  Stored in ``tests/golden/<case>.npz``:

* ``in.x``, ``in.dlogits`` (and ``in.time_delta`` / ``in.valid_mask`` /
  ``in.observation_mask`` when present),
* ``p.*``  parameters keyed by ``state_dict`` name (float32 values; the
           float64 model is built from exactly these), with each block frame
           materialised as ``p.<block>.frame.weight`` ([D, 2M]),
* ``g.*``  dL/d(parameter) under the same keys; for the frames the gradient
           with respect to the materialised [D, 2M] weight (what flows into
           the orthogonal parametrisation: the float64 model evaluates each
           frame at exactly the stored float32 values),
* ``out.logits``, ``meta.shape``.

These pin the B200 backward (``lnet_b200_alphabet_backward``); the GPU box
never needs the reference itself.
"""

from __future__ import annotations

import os
import sys
from pathlib import Path

import numpy as np
import torch
from torch.nn.utils import parametrize

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE))
# the reference checkout: LNET_REFERENCE_SRC, else a sibling `reference/src` of this repo
sys.path.insert(0, os.environ.get("LNET_REFERENCE_SRC",
                                  str(HERE.parents[2] / "reference" / "src")))

from make_golden import build_alphabet, make_inputs, params_of  # noqa: E402

torch.set_num_threads(4)


def run_grad_case(name, *, b, t, cin, d, m, k, seed, real_poles=False, valid=False, obs=None,
                  delta=False):
    model = build_alphabet(cin=cin, d=d, m=m, k=k, t=t, seed=seed, real_poles=real_poles)
    x, meta = make_inputs(b=b, t=t, cin=cin, seed=seed, valid=valid, obs=obs, delta=delta)
    params = params_of(model)  # float32 values, the pin for both sides
    model = model.double()
    # evaluate the reference's float32 function at exactly these values, in
    # float64 arithmetic: each frame becomes a plain
    # weight holding the stored float32 materialisation, so its gradient is the
    # gradient at the materialised [D, 2M] frame
    for blk in ("forward_block", "backward_block"):
        # nn.RMSNorm(eps=None) takes the eps of its dtype: keep the float32 eps
        getattr(model, blk).norm.eps = float(torch.finfo(torch.float32).eps)
        frame = getattr(model, blk).frame
        parametrize.remove_parametrizations(frame, "weight", leave_parametrized=True)
        with torch.no_grad():
            frame.weight.copy_(torch.from_numpy(params[f"p.{blk}.frame.weight"]).double())
    g = torch.Generator().manual_seed(seed + 11)
    dlogits = torch.randn(b, k, generator=g)
    names = [n for n, _ in model.named_parameters()]
    tensors = [model.get_parameter(n) for n in names]
    logits = model(x.double(), **{key: v.double() for key, v in meta.items()})
    loss = (logits * dlogits.double()).sum()
    grads = torch.autograd.grad(loss, tensors, allow_unused=True)
    rec = {"in.x": x.numpy(), "in.dlogits": dlogits.numpy()}
    for key, value in meta.items():
        rec["in." + key] = value.numpy()
    rec.update(params)
    for n, gr in zip(names, grads):
        if gr is not None:
            rec["g." + n] = gr.detach().numpy()
    rec["out.logits"] = logits.detach().numpy()
    rec["meta.shape"] = np.array([b, t, cin, d, model.modes, k])
    np.savez_compressed(HERE / f"{name}.npz", **rec)
    print(f"{name}: {sum(1 for key in rec if key.startswith('g.'))} gradients, "
          f"|logits| {logits.abs().max().item():.4g}")


def main():
    common = {"cin": 6, "d": 16, "m": 8, "k": 7}
    run_grad_case("grad_plain", b=3, t=50, seed=1, **common)
    run_grad_case("grad_real_poles", b=2, t=67, seed=2, real_poles=True, **common)
    run_grad_case("grad_long", b=2, t=300, seed=8, **common)
    run_grad_case("grad_valid", b=4, t=45, seed=3, valid=True, **common)
    run_grad_case("grad_obs_channel", b=3, t=70, seed=4, obs="channel", valid=True, **common)
    run_grad_case("grad_obs_event", b=3, t=40, seed=5, obs="event", **common)
    run_grad_case("grad_delta", b=3, t=60, seed=6, delta=True, **common)
    run_grad_case("grad_all_meta", b=3, t=64, seed=7, delta=True, obs="channel", valid=True,
                  **common)


if __name__ == "__main__":
    main()
