"""``torch.library`` custom ops over the C-ABI library.

The reference's kernels sit behind functional ``torch.library`` ops in the
``lnet::`` namespace (``lnet::pac_real2d_recurrence``,
src/lnet/pac_triton_recurrence_op.py:603-645): they allocate their outputs,
declare ``mutates_args=()`` and carry ``register_fake`` meta kernels
(src/lnet/pac_triton_parallel_static_recurrence_lag124_training.py:1231-1296),
so ``torch.compile`` and FakeTensor tracing treat them as opaque calls with a
known output shape.  This module gives the B200 path the same surface:

* ``lnet_b200::alphabet_forward(x, weights, dims, time_delta, observation_mask,
  valid_mask) -> logits [B, K]`` — one ``lnet_b200_alphabet_forward`` call.
  ``weights`` are the 17 effective fp32 tensors in ``ALPHABET_WEIGHTS`` order
  and ``dims`` = ``[raw_input_dim, model_dim, modes, output_dim, conv_kernel,
  conv_dilation]``; :meth:`lnet_b200.B200Alphabet.op_arguments` builds both.
  Metadata arrives normalised (fp32, ``[B,N]`` / ``[B,N,1 or C]`` / ``[B,N]``);
  the value checks of the reference's request wrapper
  (src/lnet/alphabet_backbone.py:163-201) stay in the module, outside the op.
* ``lnet_b200::laplace_forward(x, raw_decay, residues, direct_term, bias, dt,
  min_decay) -> y [B, T, D]`` — ``lnet_b200_laplace_forward``.
* ``lnet_b200::patchify_images(images, mean, std, patch, dtype) -> tokens`` —
  ``lnet_b200_patchify_images``.

``lnet_b200::alphabet_forward`` also carries ``register_autograd`` (the
reference's ops register their VJPs the same way,
src/lnet/pac_triton_recurrence_op.py:646-684): its backward reruns the fp32
training forward on the saved inputs and calls ``lnet_b200_alphabet_backward``
(the op itself keeps no activations).

Launches are ordered on the current torch stream with no host synchronisation.
There is no CPU implementation: a CPU input raises ``RuntimeError``.
"""

from __future__ import annotations

import ctypes
from typing import Optional

import torch
from torch import Tensor

from . import _lib
from . import images as _images
from . import laplace as _laplace

ALPHABET_WEIGHTS = tuple(_lib.PARAM_POINTER_FIELDS)
ALPHABET_DIMS = ("raw_input_dim", "model_dim", "modes", "output_dim", "conv_kernel",
                 "conv_dilation")


def _weight_shapes(dims: list[int]) -> dict[str, tuple[int, ...]]:
    c, d, m, k, ker, _ = dims
    return {
        "stem_projection": (d, c), "stem_conv_weight": (d, ker), "stem_conv_bias": (d,),
        "writer_norm": (d,), "writer_frame": (d, 2 * m), "writer_raw_decay": (m,),
        "writer_raw_frequency": (m,), "writer_direct_scale": (d,), "writer_layer_scale": (d,),
        "reader_conv_weight": (d, ker), "reader_conv_bias": (d,), "reader_norm": (d,),
        "reader_frame": (d, 2 * m), "reader_raw_decay": (m,), "reader_raw_frequency": (m,),
        "head_weight": (k, 14 * m), "head_bias": (k,),
    }


def _check_alphabet_args(x, weights, dims, time_delta, observation_mask, valid_mask) -> None:
    if len(dims) != len(ALPHABET_DIMS):
        raise ValueError(f"dims must list {ALPHABET_DIMS}, got {list(dims)}")
    if len(weights) != len(ALPHABET_WEIGHTS):
        raise ValueError(f"expected {len(ALPHABET_WEIGHTS)} weights ({ALPHABET_WEIGHTS}), "
                         f"got {len(weights)}")
    if x.ndim != 3 or x.shape[-1] != dims[0]:
        raise ValueError(f"inputs must have shape [B,N,{dims[0]}], got {tuple(x.shape)}")
    if x.dtype not in (torch.float32, torch.bfloat16):
        raise TypeError(f"inputs must be float32 or bfloat16, got {x.dtype}")
    for name, w, shape in zip(ALPHABET_WEIGHTS, weights, _weight_shapes(dims).values()):
        if tuple(w.shape) != shape:
            raise ValueError(f"{name} must have shape {shape}, got {tuple(w.shape)}")
        if w.dtype != torch.float32:
            raise TypeError(f"{name} must be float32, got {w.dtype}")
        if w.device != x.device:
            raise ValueError(f"{name} is on {w.device}, inputs on {x.device}")
    bt = tuple(x.shape[:2])
    for name, t, shapes in (("time_delta", time_delta, (bt,)),
                            ("observation_mask", observation_mask,
                             ((*bt, 1), (*bt, x.shape[2]))),
                            ("valid_mask", valid_mask, (bt,))):
        if t is None:
            continue
        if tuple(t.shape) not in shapes:
            raise ValueError(f"{name} must have shape {' or '.join(map(str, shapes))}, "
                             f"got {tuple(t.shape)}")
        if t.dtype != torch.float32:
            raise TypeError(f"{name} must be float32, got {t.dtype}")
        if t.device != x.device:
            raise ValueError(f"{name} is on {t.device}, inputs on {x.device}")


@torch.library.custom_op("lnet_b200::alphabet_forward", mutates_args=())
def alphabet_forward(x: Tensor, weights: list[Tensor], dims: list[int],
                     time_delta: Optional[Tensor] = None,
                     observation_mask: Optional[Tensor] = None,
                     valid_mask: Optional[Tensor] = None) -> Tensor:
    """ALPHABET logits [B, K] (fp32) for ``x`` [B, N, C] (fp32 or bf16)."""
    _check_alphabet_args(x, weights, dims, time_delta, observation_mask, valid_mask)
    if not x.is_cuda:
        raise RuntimeError("lnet_b200::alphabet_forward runs on CUDA only")
    lib = _lib.load()
    x = x.contiguous()
    ws_keep = [w.contiguous() for w in weights]
    meta = [None if t is None else t.contiguous() for t in (time_delta, observation_mask,
                                                            valid_mask)]
    params = _lib.AlphabetParams(
        **dict(zip(ALPHABET_DIMS, (int(v) for v in dims))),
        **{name: w.data_ptr() for name, w in zip(ALPHABET_WEIGHTS, ws_keep)},
    )
    delta, obs, valid = meta
    dtype = _lib.LNET_BF16 if x.dtype == torch.bfloat16 else _lib.LNET_F32
    req = _lib.AlphabetRequest(
        batch=x.shape[0], steps=x.shape[1], x_dtype=dtype, act_dtype=dtype, x=x.data_ptr(),
        time_delta=None if delta is None else delta.data_ptr(),
        observation_mask=None if obs is None else obs.data_ptr(),
        obs_channels=0 if obs is None else obs.shape[-1],
        valid_mask=None if valid is None else valid.data_ptr(),
    )
    logits = torch.empty(x.shape[0], int(dims[3]), device=x.device, dtype=torch.float32)
    n = ctypes.c_size_t(0)
    _lib.check(lib.lnet_b200_alphabet_workspace_size(ctypes.byref(params), ctypes.byref(req),
                                                     ctypes.byref(n)),
               "lnet_b200_alphabet_workspace_size")
    ws = torch.empty(max(int(n.value), 1), dtype=torch.uint8, device=x.device)
    with torch.cuda.device(x.device):
        stream = torch.cuda.current_stream().cuda_stream
        _lib.check(lib.lnet_b200_alphabet_forward(ctypes.byref(params), ctypes.byref(req),
                                                  ws.data_ptr(), int(n.value), logits.data_ptr(),
                                                  None, None, stream),
                   "lnet_b200_alphabet_forward")
    return logits


@alphabet_forward.register_fake
def _alphabet_forward_fake(x, weights, dims, time_delta=None, observation_mask=None,
                           valid_mask=None):
    _check_alphabet_args(x, weights, dims, time_delta, observation_mask, valid_mask)
    return x.new_empty((x.shape[0], int(dims[3])), dtype=torch.float32)


def _alphabet_setup_context(ctx, inputs, output):
    x, weights, dims, time_delta, observation_mask, valid_mask = inputs
    ctx.save_for_backward(x, *weights)
    ctx.dims = tuple(int(v) for v in dims)
    ctx.meta = (time_delta, observation_mask, valid_mask)


def _alphabet_backward(ctx, dlogits):
    """Gradients for the 17 weights: the training forward is rerun on the saved
    inputs (the op keeps no activations, like activation checkpointing), then
    lnet_b200_alphabet_backward."""
    from .training import AlphabetTrainFunction

    x, *weights = ctx.saved_tensors
    time_delta, obs, valid = ctx.meta
    with torch.enable_grad():
        leaves = [w.detach().requires_grad_(True) for w in weights]
        logits = AlphabetTrainFunction.apply(x, valid, obs, time_delta, ctx.dims, *leaves)
        grads = torch.autograd.grad(logits, leaves, dlogits)
    # the structure of the arguments actually passed (optional arguments left
    # at their defaults are not part of it): x, weights, dims, [metadata...]
    return (None, list(grads)) + (None,) * (len(ctx.needs_input_grad) - 2)


alphabet_forward.register_autograd(_alphabet_backward, setup_context=_alphabet_setup_context)


def _check_laplace_args(x, raw_decay, residues, direct_term, bias) -> None:
    if x.ndim != 3:
        raise ValueError(f"inputs must have shape [B,T,D], got {tuple(x.shape)}")
    d = x.shape[-1]
    m = raw_decay.shape[0] if raw_decay.ndim == 1 else -1
    expect = {"raw_decay": (raw_decay, (m,)), "residues": (residues, (d, m, d)),
              "direct_term": (direct_term, (d, d)), "bias": (bias, (d,))}
    for name, (t, shape) in expect.items():
        if m < 1 or tuple(t.shape) != shape:
            raise ValueError(f"{name} must have shape {shape}, got {tuple(t.shape)}")
        if t.dtype != torch.float64:
            raise TypeError(f"{name} must be float64, got {t.dtype}")
    if x.dtype not in (torch.float32, torch.float64):
        raise TypeError(f"inputs must be float32 or float64, got {x.dtype}")


@torch.library.custom_op("lnet_b200::laplace_forward", mutates_args=())
def laplace_forward(x: Tensor, raw_decay: Tensor, residues: Tensor, direct_term: Tensor,
                    bias: Tensor, dt: float, min_decay: float) -> Tensor:
    """Pole-residue Laplace layer: ``y`` [B, T, D] in the dtype of ``x``."""
    _check_laplace_args(x, raw_decay, residues, direct_term, bias)
    if not x.is_cuda:
        raise RuntimeError("lnet_b200::laplace_forward runs on CUDA only")
    keep = [p.to(x.device).contiguous() for p in (raw_decay, residues, direct_term, bias)]
    return _laplace._launch(x.contiguous(), *keep, raw_decay.shape[0], float(dt),
                            float(min_decay))


@laplace_forward.register_fake
def _laplace_forward_fake(x, raw_decay, residues, direct_term, bias, dt, min_decay):
    _check_laplace_args(x, raw_decay, residues, direct_term, bias)
    return torch.empty_like(x)


def _check_patchify_args(images, mean, std, patch, dtype) -> None:
    if images.dtype != torch.uint8 or images.ndim != 4 or images.shape[-1] != 3:
        raise ValueError(f"images must be uint8 [B, H, W, 3], got {images.dtype} "
                         f"{tuple(images.shape)}")
    if len(mean) != 3 or len(std) != 3:
        raise ValueError("mean and std must have three entries")
    if dtype not in (torch.bfloat16, torch.float32):
        raise TypeError(f"tokens dtype must be bfloat16 or float32, got {dtype}")
    if patch < 1 or images.shape[1] % patch or images.shape[2] % patch:
        raise ValueError(f"image {images.shape[1]}x{images.shape[2]} is not divisible by "
                         f"patch {patch}")


@torch.library.custom_op("lnet_b200::patchify_images", mutates_args=())
def patchify_images(images: Tensor, mean: list[float], std: list[float], patch: int,
                    dtype: torch.dtype) -> Tensor:
    """uint8 images [B, H, W, 3] -> normalised patch tokens [B, (H/p)(W/p), 3 p^2]."""
    _check_patchify_args(images, mean, std, patch, dtype)
    if not images.is_cuda:
        raise RuntimeError("lnet_b200::patchify_images runs on CUDA only")
    return _images._launch(images.contiguous(), mean, std, patch, dtype)


@patchify_images.register_fake
def _patchify_images_fake(images, mean, std, patch, dtype):
    _check_patchify_args(images, mean, std, patch, dtype)
    b, h, w, _ = images.shape
    return images.new_empty((b, (h // patch) * (w // patch), 3 * patch * patch), dtype=dtype)


__all__ = ["ALPHABET_DIMS", "ALPHABET_WEIGHTS", "alphabet_forward", "laplace_forward",
           "patchify_images"]
