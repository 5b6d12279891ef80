"""Host-side behaviour of the drop-in modules that needs no GPU."""

from __future__ import annotations

import pytest
import torch

from lnet_b200 import AlphabetConfig, B200Alphabet, B200PoleResidueTemporalMixing
from lnet_b200.laplace import LaplaceParameterError, LaplaceShapeError


def model(cin=3, d=8, m=4, k=5):
    return B200Alphabet(AlphabetConfig(cin, d, m, k), k).eval()


def test_modes_above_half_width_rejected():
    with pytest.raises(RuntimeError):
        B200Alphabet(AlphabetConfig(3, 8, 5, 2), 2)


def test_state_dict_keys_match_reference_layout():
    keys = set(model().state_dict())
    for k in ("stem.projection.weight", "stem.local.weight", "stem.local.bias",
              "forward_block.frame.parametrizations.weight.original",
              "forward_block.direct_scale", "backward_block.layer_scale",
              "head.classifier.weight", "second_local.bias"):
        assert k in keys


@pytest.mark.parametrize(
    "kwargs,msg",
    [
        ({"time_delta": torch.ones(2, 7)}, "time_delta must have shape"),
        ({"time_delta": -torch.ones(2, 6)}, "finite non-negative"),
        ({"time_delta": torch.full((2, 6, 1), float("nan"))}, "finite non-negative"),
        ({"observation_mask": torch.ones(2, 6, 2)}, "observation_mask must have shape"),
        ({"observation_mask": 2 * torch.ones(2, 6, 3)}, "finite values in \\[0,1\\]"),
        ({"valid_mask": torch.ones(2, 6, 3)}, "valid_mask must have shape"),
        ({"valid_mask": -torch.ones(2, 6)}, "finite values in \\[0,1\\]"),
    ],
)
def test_metadata_errors_mirror_reference(kwargs, msg):
    m = model()
    x = torch.randn(2, 6, 3)
    with pytest.raises(ValueError, match=msg):
        m._prepare_metadata(x, kwargs.get("time_delta"), kwargs.get("observation_mask"),
                            kwargs.get("valid_mask"))


def test_metadata_normalisation_shapes():
    m = model()
    x = torch.randn(2, 6, 3)
    d, o, v = m._prepare_metadata(x, torch.ones(2, 6, 1), torch.ones(2, 6), torch.ones(2, 6, 1))
    assert d.shape == (2, 6) and o.shape == (2, 6, 1) and v.shape == (2, 6)
    d, o, v = m._prepare_metadata(x, None, torch.ones(2, 6, 3), None)
    assert d is None and o.shape == (2, 6, 3) and v is None


def test_cpu_inputs_fail_loudly():
    with pytest.raises(RuntimeError, match="CUDA"):
        model()(torch.randn(2, 6, 3))


def test_laplace_errors_mirror_reference():
    layer = B200PoleResidueTemporalMixing(4, 3)
    with pytest.raises(LaplaceShapeError):
        layer(torch.randn(2, 5, 3))
    with pytest.raises(LaplaceParameterError, match="strictly negative"):
        layer.load_transfer_parameters(
            poles=torch.tensor([-1.0, 0.5, -2.0], dtype=torch.float64),
            residues=torch.zeros(4, 3, 4, dtype=torch.float64),
            direct_term=torch.zeros(4, 4, dtype=torch.float64),
            bias=torch.zeros(4, dtype=torch.float64),
        )
    with pytest.raises(LaplaceParameterError, match="residue tensor shape"):
        layer.load_transfer_parameters(
            poles=-torch.ones(3, dtype=torch.float64),
            residues=torch.zeros(4, 2, 4, dtype=torch.float64),
            direct_term=torch.zeros(4, 4, dtype=torch.float64),
            bias=torch.zeros(4, dtype=torch.float64),
        )


def test_training_mode_needs_cuda():
    """Training mode runs the B200 forward/backward; a CPU input is refused, not
    run on a CPU fallback."""
    m = B200Alphabet(AlphabetConfig(3, 8, 4, 5), 5).train()
    with pytest.raises(RuntimeError, match="CUDA"):
        m(torch.randn(2, 6, 3))


def test_patchify_reference_layout():
    """Token channel (i * p + j) * 3 + ch of patch (pr, pc) is pixel (pr p + i, pc p + j, ch),
    normalised as (u / 255 - mean) / std in fp32."""
    from lnet_b200.images import patchify_images_reference

    g = torch.Generator().manual_seed(0)
    img = torch.randint(0, 256, (2, 6, 8, 3), generator=g, dtype=torch.uint8)
    mean, std = (0.1, 0.2, 0.3), (0.5, 0.25, 2.0)
    x = patchify_images_reference(img, mean=mean, std=std, patch=2, dtype=torch.float32)
    assert x.shape == (2, 3 * 4, 12)
    for b, pr, pc, i, j, ch in [(0, 0, 0, 0, 0, 0), (1, 2, 3, 1, 0, 2), (0, 1, 2, 1, 1, 1)]:
        u = torch.tensor(float(img[b, pr * 2 + i, pc * 2 + j, ch]))
        want = (u / 255.0 - torch.tensor(mean[ch])) / torch.tensor(std[ch])
        assert x[b, pr * 4 + pc, (i * 2 + j) * 3 + ch] == want


def test_laplace_channel_diagonal_form():
    """The per-channel (block-diagonal) residue layout is recognised: per output the
    modes with a nonzero R[o, m, o], padded with residue 0; dense residues or too many
    modes per channel fall back to the dense kernel (None)."""
    import torch

    from lnet_b200.laplace import MAX_MODES_PER_CHANNEL, channel_diagonal_form

    d, per = 4, 3
    r = torch.zeros(d, d * per, d, dtype=torch.float64)
    for ch in range(d):
        r[ch, ch * per:(ch + 1) * per, ch] = torch.arange(1, per + 1, dtype=torch.float64) + ch
    r[2, 2 * per + 1, 2] = 0.0  # channel 2 has one mode fewer
    idx, vals = channel_diagonal_form(r)
    assert idx.shape == (d, per) and idx.dtype == torch.int32
    for ch in range(d):
        got = {(int(m), float(v)) for m, v in zip(idx[ch], vals[ch]) if v != 0}
        want = {(m, float(r[ch, m, ch])) for m in range(d * per) if r[ch, m, ch] != 0}
        assert got == want
    assert float(vals[2].abs().min()) == 0.0  # the padding slot adds exactly zero
    dense = r.clone()
    dense[0, 0, 1] = 1.0
    assert channel_diagonal_form(dense) is None
    wide = torch.ones(1, MAX_MODES_PER_CHANNEL + 1, 1, dtype=torch.float64)
    assert channel_diagonal_form(wide) is None
