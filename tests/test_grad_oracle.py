"""The numpy backward oracle against gradients from the reference's autograd.

``tests/golden/grad_*.npz`` hold dL/dparameter of ``L = sum(logits * dlogits)``
computed by the reference ``lnet.Alphabet`` in float64
(``tests/golden/make_grad_golden.py``).  ``oracle.alphabet_grad_oracle``
restates the VJP stage by stage; both sides evaluate the same function in
float64 arithmetic, so they must agree to 1e-9 relative per parameter tensor.
"""

from __future__ import annotations

import numpy as np
import pytest
from conftest import golden_params, load_golden, rel_err

from oracle import alphabet_grad_oracle as G

CASES = ["grad_plain", "grad_real_poles", "grad_long", "grad_valid", "grad_obs_channel",
         "grad_obs_event", "grad_delta", "grad_all_meta"]


@pytest.mark.parametrize("name", CASES)
def test_grad_oracle_matches_reference(name):
    z = load_golden(name)
    params = golden_params(z)
    grads = G.alphabet_backward(z["in.x"], params, z["in.dlogits"],
                                time_delta=z.get("in.time_delta"),
                                observation_mask=z.get("in.observation_mask"),
                                valid_mask=z.get("in.valid_mask"))
    for key in z:
        if not key.startswith("g."):
            continue
        pname = key[2:]
        got = grads[pname].reshape(z[key].shape)
        assert rel_err(got, z[key]) <= 1e-9, (pname, rel_err(got, z[key]))
