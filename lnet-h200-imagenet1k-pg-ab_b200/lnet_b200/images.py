"""uint8 images -> normalised, patchified tokens on the GPU (the input pipeline
of the image configuration).

The reference's harness normalises on the host side with
``ConvertImageDtype(float32)`` + ``Normalize(mean, std)``
(scripts/train_alphabet2d_imagenet100.py:292-310) and patchifies 4x4 into
``x [B, (H/4)(W/4), 48]``.  :func:`patchify_images` computes the same fp32
arithmetic in one CUDA kernel (``lnet_b200_patchify_images``), bit-identical
to the PyTorch transform, so a caller copies uint8 images (half the bytes of
bf16 tokens) to the device and patchifies there.
"""

from __future__ import annotations

import ctypes

import torch
from torch import Tensor

from . import _lib

IMAGENET_MEAN = (0.485, 0.456, 0.406)
IMAGENET_STD = (0.229, 0.224, 0.225)


def patchify_images(images: Tensor, *, mean=IMAGENET_MEAN, std=IMAGENET_STD, patch: int = 4,
                    dtype: torch.dtype = torch.bfloat16) -> Tensor:
    """``images`` uint8 [B, H, W, 3] on CUDA -> tokens [B, (H/p)(W/p), 3 p^2] of ``dtype``."""
    if images.dtype != torch.uint8 or images.ndim != 4 or images.shape[-1] != 3:
        raise ValueError(f"images must be uint8 [B, H, W, 3], got {images.dtype} "
                         f"{tuple(images.shape)}")
    if not images.is_cuda:
        raise RuntimeError("patchify_images runs on CUDA only")
    if dtype not in (torch.bfloat16, torch.float32):
        raise TypeError(f"tokens dtype must be bfloat16 or float32, got {dtype}")
    b, h, w, _ = images.shape
    if h % patch or w % patch:
        raise ValueError(f"image {h}x{w} is not divisible by patch {patch}")
    return _launch(images.contiguous(), mean, std, patch, dtype)


def _launch(images: Tensor, mean, std, patch: int, dtype: torch.dtype) -> Tensor:
    """One ``lnet_b200_patchify_images`` call on the current stream (checked arguments)."""
    b, h, w, _ = images.shape
    out = torch.empty(b, (h // patch) * (w // patch), 3 * patch * patch, dtype=dtype,
                      device=images.device)
    m = (ctypes.c_float * 3)(*[float(v) for v in mean])
    s = (ctypes.c_float * 3)(*[float(v) for v in std])
    code = _lib.LNET_BF16 if dtype == torch.bfloat16 else _lib.LNET_F32
    with torch.cuda.device(images.device):
        stream = torch.cuda.current_stream().cuda_stream
        _lib.check(_lib.load().lnet_b200_patchify_images(images.data_ptr(), b, h, w, patch, m, s,
                                                         out.data_ptr(), code, stream),
                   "lnet_b200_patchify_images")
    return out


def patchify_images_reference(images: Tensor, *, mean=IMAGENET_MEAN, std=IMAGENET_STD,
                              patch: int = 4, dtype: torch.dtype = torch.bfloat16) -> Tensor:
    """The same transform in plain PyTorch (the harness form), for checks."""
    b, h, w, _ = images.shape
    mean_t = torch.tensor(mean, device=images.device)
    std_t = torch.tensor(std, device=images.device)
    v = (images.float() / 255.0 - mean_t) / std_t
    v = v.reshape(b, h // patch, patch, w // patch, patch, 3).permute(0, 1, 3, 2, 4, 5)
    return v.reshape(b, (h // patch) * (w // patch), 3 * patch * patch).to(dtype).contiguous()


__all__ = ["IMAGENET_MEAN", "IMAGENET_STD", "patchify_images", "patchify_images_reference"]
