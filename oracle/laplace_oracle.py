"""CPU oracle for the pole-residue Laplace layer (numpy restatement).

TEST INFRASTRUCTURE ONLY: imported by the tests, ``__graft_entry__.smoke()``
and ``bench.py``'s CPU-baseline leg as the checker; never by the product.

Restates ``PoleResidueTemporalMixing.forward``
(src/lnet/laplace.py:126-159) in float64: real poles
``p = -(softplus(raw_decay) + min_decay)`` (:78-79), exact ZOH
``a = exp(p dt)``, ``b = dt * phi1(p dt)`` with the series branch of
``_phi1`` for ``|z| < 1e-4`` (:37-42), a per-(mode, channel) state
``state[m, i] = a_m state[m, i] + b_m x_t[i]`` and the readout
``y_t = sum_{m,i} R[o, m, i] state[m, i] + x_t D^T + bias``.
Pinned by ``tests/golden/laplace_*.npz`` (reference outputs).
"""

from __future__ import annotations

import numpy as np


def softplus(x):
    # torch.nn.functional.softplus with beta=1, threshold=20
    return np.where(x > 20.0, x, np.log1p(np.exp(np.minimum(x, 20.0))))


def phi1(z):
    """``_phi1`` (src/lnet/laplace.py:37-42)."""
    small = np.abs(z) < 1.0e-4
    safe = np.where(small, 1.0, z)
    return np.where(small, 1.0 + z / 2.0 + z * z / 6.0, np.expm1(z) / safe)


def zoh_coefficients(raw_decay, dt=1.0, min_decay=1.0e-3):
    poles = -(softplus(np.asarray(raw_decay, np.float64)) + min_decay)
    z = poles * dt
    return np.exp(z), dt * phi1(z)


def laplace_forward(x, raw_decay, residues, direct_term, bias, dt=1.0, min_decay=1.0e-3):
    """``PoleResidueTemporalMixing.forward`` (src/lnet/laplace.py:126-159)."""
    x64 = np.asarray(x, np.float64)
    a, b = zoh_coefficients(raw_decay, dt, min_decay)
    bsz, t, d = x64.shape
    m = a.shape[0]
    state = np.zeros((bsz, m, d))
    r = np.asarray(residues, np.float64).reshape(d, m * d)
    out = np.empty((bsz, t, d))
    dmat = np.asarray(direct_term, np.float64)
    for i in range(t):
        xi = x64[:, i]
        state = a[None, :, None] * state + b[None, :, None] * xi[:, None, :]
        out[:, i] = state.reshape(bsz, m * d) @ r.T + xi @ dmat.T + bias
    return out.astype(np.asarray(x).dtype)
