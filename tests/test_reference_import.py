"""A live reference ``lnet.Alphabet`` converts to :class:`B200Alphabet` with an equal
``state_dict`` (CPU only; no forward).  Skipped when the reference package is not
importable: it is looked for under LNET_REFERENCE_SRC, else in a ``reference/src``
checkout beside this repository."""

from __future__ import annotations

import os
import sys
from pathlib import Path

import pytest
import torch

REF_SRC = os.environ.get("LNET_REFERENCE_SRC",
                         str(Path(__file__).resolve().parents[2] / "reference" / "src"))


def _reference():
    if REF_SRC not in sys.path:
        sys.path.insert(0, REF_SRC)
    try:
        from lnet import Alphabet
        from lnet.pac_types import PACExperimentConfig
    except Exception as exc:  # noqa: BLE001
        pytest.skip(f"reference lnet not importable from {REF_SRC}: {exc}")
    return Alphabet, PACExperimentConfig


@pytest.mark.parametrize("dims", [(6, 16, 4, 5), (48, 96, 48, 1000)])
def test_from_reference_state_dict_equal(dims):
    Alphabet, PACExperimentConfig = _reference()
    from lnet_b200 import B200Alphabet

    cin, d, m, k = dims
    torch.manual_seed(0)
    cfg = PACExperimentConfig(sample_count=1, validation_count=1, test_count=0,
                              sequence_length=32, raw_input_dim=cin, output_dim=k,
                              model_dim=d, modes=m)
    ref = Alphabet(cfg, k).eval()
    ours = B200Alphabet.from_reference(ref)
    a, b = ref.state_dict(), ours.state_dict()
    assert sorted(a) == sorted(b)
    for key in a:
        assert a[key].shape == b[key].shape, key
        assert torch.equal(a[key], b[key]), key
