"""Image input pipeline (uint8 -> normalised 4x4 patch tokens) and the host-fed
serving loop.

* patchify_images is bit-identical to the transform computed by PyTorch on the
  CPU (the reference's data loader: ConvertImageDtype + Normalize, IEEE
  divisions), for bf16 and fp32 tokens, patch 4 (vector kernel) and other
  patch sizes (generic kernel);
* forward_images builds the x tiles inside the fused writer from the uint8
  bytes (lnet_b200_alphabet_forward_images) for the fused shapes: equal to
  forward(patchified tokens) at the config-4 shape, on ragged and tiny images,
  with custom normalisation, returned moments and the prepared operands; other
  shapes patchify first and give the same result;
* forward_images == forward(tokens) and run_pipelined (copies of batch k+1
  overlapping the forward of batch k) == sequential forwards, to <= 1e-5
  relative: the tokens are identical, but the fused route's decoupled
  look-back takes a predecessor's inclusive record or combines aggregates
  depending on timing, which re-associates the fp32 carries (the bound of the
  row-independence checks in test_fullsize_gpu).
"""

from __future__ import annotations

import sys
from pathlib import Path

import pytest
import torch

from conftest import rel_err

from lnet_b200.images import patchify_images, patchify_images_reference
from lnet_b200.pipeline import run_pipelined

sys.path.insert(0, str(Path(__file__).resolve().parents[1]))
import bench  # noqa: E402

pytestmark = pytest.mark.gpu


def _images(b, h, w, seed):
    g = torch.Generator().manual_seed(seed)
    return torch.randint(0, 256, (b, h, w, 3), generator=g, dtype=torch.uint8)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
@pytest.mark.parametrize("shape,patch", [((3, 224, 224), 4), ((2, 8, 12), 2), ((1, 9, 6), 3),
                                         ((2, 16, 16), 4)])
def test_patchify_bit_exact(cuda_device, dtype, shape, patch):
    img = _images(*shape, seed=patch)
    ref = patchify_images_reference(img, patch=patch, dtype=dtype)  # CPU transform
    out = patchify_images(img.to(cuda_device), patch=patch, dtype=dtype)
    assert out.shape == ref.shape
    assert torch.equal(out.cpu().view(torch.int16 if dtype == torch.bfloat16 else torch.int32),
                       ref.view(torch.int16 if dtype == torch.bfloat16 else torch.int32))


def test_patchify_custom_normalisation_and_errors(cuda_device):
    img = _images(2, 8, 8, seed=9)
    kw = dict(mean=(0.5, 0.25, 0.0), std=(0.5, 2.0, 1.0), patch=4, dtype=torch.float32)
    assert torch.equal(patchify_images(img.to(cuda_device), **kw).cpu(),
                       patchify_images_reference(img, **kw))
    with pytest.raises(ValueError):
        patchify_images(img.to(cuda_device), patch=3)
    with pytest.raises(ValueError):
        patchify_images(img.float().to(cuda_device))
    with pytest.raises(ValueError):
        patchify_images(img.to(cuda_device), std=(0.0, 1.0, 1.0))


def test_forward_images_matches_tokens(cuda_device):
    cfg = dict(bench.CONFIGS["4"], B=4)
    model = bench.build_model(cfg, cuda_device)
    img = _images(4, 224, 224, seed=3)
    x = patchify_images_reference(img).to(cuda_device)
    with torch.no_grad():
        a = model.forward_images(img.to(cuda_device))
        b = model(x)
    assert rel_err(a.cpu().numpy(), b.cpu().numpy()) <= 1e-5


def test_run_pipelined_matches_sequential(cuda_device):
    cfg = dict(bench.CONFIGS["4"], B=2)
    model = bench.build_model(cfg, cuda_device)
    hosts = [_images(2, 224, 224, seed=10 + k).pin_memory() for k in range(5)]
    outs = [torch.empty(2, cfg["K"]).pin_memory() for _ in hosts]
    with torch.no_grad():
        run_pipelined(model.forward_images, hosts, outs, cuda_device)
        torch.cuda.synchronize()
        for h, o in zip(hosts, outs):
            ref = model.forward_images(h.to(cuda_device)).cpu()
            assert rel_err(o.numpy(), ref.numpy()) <= 1e-5


def _check_images_vs_tokens(model, img, dev, **kw):
    from lnet_b200.alphabet import images_route_fused

    x = patchify_images_reference(img, **{k: v for k, v in kw.items()
                                          if k in ("mean", "std")}).to(dev)
    with torch.no_grad():
        a, awm, arm = model.forward_images(img.to(dev), return_moments=True, **kw)
        b, bwm, brm = model(x, return_moments=True)
    for got, want in ((a, b), (awm, bwm), (arm, brm)):
        assert rel_err(got.cpu().numpy(), want.cpu().numpy()) <= 1e-5
    return images_route_fused(model, img.to(dev).contiguous())


@pytest.mark.parametrize("shape", [(3, 64, 200), (2, 8, 12), (1, 4, 4), (5, 36, 100)])
def test_forward_images_fused_ragged(cuda_device, shape):
    """Token counts 800 (ragged last chunk), 6, 1 and 225; patch rows of 50, 3, 1
    and 25 tokens, so tiles cross patch rows at every offset."""
    cfg = dict(bench.CONFIGS["4"], B=shape[0])
    model = bench.build_model(cfg, cuda_device)
    img = _images(*shape, seed=sum(shape))
    assert _check_images_vs_tokens(model, img, cuda_device,
                                   mean=(0.5, 0.25, 0.1), std=(0.5, 2.0, 0.75))


def test_forward_images_fused_prepared(cuda_device):
    cfg = dict(bench.CONFIGS["4"], B=3)
    model = bench.build_model(cfg, cuda_device)
    img = _images(3, 96, 224, seed=21)
    model.prepare_for_inference_(sequence_length=24 * 56, batch_size=3)
    for _ in range(2):  # the second call reuses the prepared operands
        assert _check_images_vs_tokens(model, img, cuda_device)


def test_forward_images_other_shapes_patchify_first(cuda_device):
    from lnet_b200 import AlphabetConfig, B200Alphabet

    model = B200Alphabet(AlphabetConfig(48, 64, 16, 7), 7).eval().to(cuda_device)
    img = _images(2, 32, 40, seed=5)
    assert not _check_images_vs_tokens(model, img, cuda_device)
