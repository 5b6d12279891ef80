"""The CPU oracle against golden vectors recorded from the reference itself."""

from __future__ import annotations

import numpy as np
import pytest
from conftest import golden_names, golden_params, load_golden, rel_err

from oracle import alphabet_oracle as A
from oracle import laplace_oracle as L

STAGES = ("first_local", "first_stream", "encoded", "writer_moments", "reader_moments", "logits")


@pytest.mark.parametrize("name", golden_names("alphabet_"))
@pytest.mark.parametrize("dtype", [np.float32, np.float64])
def test_alphabet_oracle_matches_reference(name, dtype):
    z = load_golden(name)
    out = A.alphabet_forward(
        z["in.x"], golden_params(z), time_delta=z.get("in.time_delta"),
        observation_mask=z.get("in.observation_mask"), valid_mask=z.get("in.valid_mask"),
        dtype=dtype, return_stages=True,
    )
    for stage in STAGES:
        tol = 1e-4 if stage != "logits" else 3e-5
        if "moments" in stage:
            tol = 3e-4
        assert rel_err(out[stage], z["out." + stage]) <= tol, stage


@pytest.mark.parametrize("name", golden_names("laplace_"))
def test_laplace_oracle_matches_reference(name):
    z = load_golden(name)
    y = L.laplace_forward(z["in.x"], z["p.raw_decay"], z["p.residues"], z["p.direct_term"],
                          z["p.bias"], float(z["p.dt"]), float(z["p.min_decay"]))
    assert rel_err(y, z["out.y"]) <= 1e-6


def test_masks_zero_padding_exactly():
    """Padded positions of first_local are exactly zero in oracle and reference."""
    z = load_golden("alphabet_valid")
    out = A.alphabet_forward(z["in.x"], golden_params(z), valid_mask=z["in.valid_mask"],
                             dtype=np.float32, return_stages=True)
    pad = z["in.valid_mask"] == 0
    assert np.all(out["first_local"][pad] == 0) and np.all(z["out.first_local"][pad] == 0)
    assert np.all(out["encoded"][pad] == 0) and np.all(z["out.encoded"][pad] == 0)


def test_zoh_small_branch_and_unit_grid():
    d = np.array([1e-3, 0.5, 2.0])
    w = np.array([0.0, 1.0, -3.0])
    ar, ai, gr, gi = A.discrete_pole_real2d(d, w, 1.0)
    p = -d + 1j * w
    a = np.exp(p)
    assert np.allclose(ar + 1j * ai, a) and np.allclose(gr + 1j * gi, (a - 1) / p)
    ar, ai, gr, gi = A.discrete_pole_real2d(d, w, 0.0)
    assert np.all(gr == 0.0) and np.all(gi == 0.0) and np.all(ar == 1.0)
