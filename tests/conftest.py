"""Shared pytest setup: the ``gpu`` marker and import paths.

``-m "not gpu"`` tests run on CPU-only machines (oracle vs golden vectors,
C-ABI symbol checks, host-side validation, gloo multi-process logic);
``-m gpu`` tests need a B200 and exercise the CUDA library.
"""

from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parents[1]
PKG_DIR = ROOT / "lnet-h200-imagenet1k-pg-ab_b200"
GOLDEN = Path(__file__).resolve().parent / "golden"
for p in (str(ROOT), str(PKG_DIR)):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200) and the built library")


def load_golden(name: str) -> dict:
    with np.load(GOLDEN / f"{name}.npz") as z:
        return {k: z[k] for k in z.files}


def golden_names(prefix: str = "alphabet_") -> list[str]:
    return sorted(p.stem for p in GOLDEN.glob(f"{prefix}*.npz"))


def golden_params(z: dict) -> dict:
    return {k[2:]: v for k, v in z.items() if k.startswith("p.")}


def rel_err(got, ref) -> float:
    """Max relative error, normwise: max|got - ref| / max|ref| (the parity metric)."""
    got = np.asarray(got, dtype=np.float64)
    ref = np.asarray(ref, dtype=np.float64)
    scale = max(float(np.abs(ref).max()) if ref.size else 0.0, 1e-30)
    return float(np.abs(got - ref).max()) / scale if ref.size else 0.0


def elem_rel_err(got, ref, floor_frac: float = 1e-3) -> float:
    """Max elementwise relative error, max_i |got_i - ref_i| / max(|ref_i|, floor),
    with the floor at `floor_frac` x max|ref| so that entries near zero (moments of
    nearly silent modes, logits near 0) are measured against a stated absolute
    scale instead of dividing by ~0."""
    got = np.asarray(got, dtype=np.float64)
    ref = np.asarray(ref, dtype=np.float64)
    if not ref.size:
        return 0.0
    floor = max(floor_frac * float(np.abs(ref).max()), 1e-30)
    return float((np.abs(got - ref) / np.maximum(np.abs(ref), floor)).max())


def record_margin(case: str, got, ref, gate: float) -> tuple[float, float]:
    """Normwise and elementwise (floor 1e-3 x max|ref|) errors of one parity check.
    When LNET_PARITY_LOG names a file, one JSON line per check is appended to it
    (case, both errors, the gate), which is how the achieved margins are collected."""
    import json
    import os

    nw, ew = rel_err(got, ref), elem_rel_err(got, ref)
    path = os.environ.get("LNET_PARITY_LOG")
    if path:
        with open(path, "a") as f:
            f.write(json.dumps({"case": case, "normwise": nw, "elementwise": ew,
                                "gate": gate}) + "\n")
    return nw, ew


@pytest.fixture(scope="session")
def cuda_device():
    import torch

    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch.device("cuda:0")
