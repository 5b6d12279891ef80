"""Training through the B200 kernels: autograd over the ALPHABET forward.

The reference trains ``Alphabet`` with torch autograd through its custom ops
(``register_autograd`` on the ``lnet::`` ops, src/lnet/pac_triton_recurrence_op.py:603-684,
and the fused VJP kernels of
src/lnet/pac_triton_parallel_static_recurrence_lag124_training.py:488-876).
Here one ``torch.autograd.Function`` wraps the two C-ABI calls:

* forward: ``lnet_b200_alphabet_train_forward`` (the general route in fp32,
  every activation the backward needs kept in a workspace owned by the
  autograd context);
* backward: ``lnet_b200_alphabet_backward`` (dL/dparameter of all 17
  effective tensors from dL/dlogits).

The function's inputs are the module's *effective* tensors built with
differentiable torch ops (``frame_matrix()`` through the orthogonal
parametrisation, conv weights reshaped), so torch chains the returned
gradients back to the module's own parameters.  Every metadata combination
(``time_delta``, ``observation_mask``, ``valid_mask``) is supported; with
``time_delta`` the interpolation scatters use float atomics, so those
gradients are reproducible to rounding, not bitwise.
"""

from __future__ import annotations

import ctypes

import torch
from torch import Tensor

from . import _lib


def effective_tensors(model) -> list[Tensor]:
    """The 17 effective fp32 tensors in ``_lib.PARAM_POINTER_FIELDS`` order, built
    differentiably from ``model``'s parameters."""
    fb, bb = model.forward_block, model.backward_block
    d, k = model.model_dim, model.dwconv_kernel_size
    # lnet_b200.train_runtime swaps in a capture-safe frame builder
    frame_fn = getattr(model, "_frame_fn", None)

    def frame(block):
        return frame_fn(block.frame) if frame_fn is not None else block.frame_matrix()

    def f(t: Tensor) -> Tensor:
        return t.float().contiguous()

    return [
        f(model.stem.projection.weight),
        f(model.stem.local.weight.reshape(d, k)),
        f(model.stem.local.bias),
        f(fb.norm.weight),
        f(frame(fb)),
        f(fb.raw_decay),
        f(fb.raw_frequency),
        f(fb.direct_scale),
        f(fb.layer_scale),
        f(model.second_local.weight.reshape(d, k)),
        f(model.second_local.bias),
        f(bb.norm.weight),
        f(frame(bb)),
        f(bb.raw_decay),
        f(bb.raw_frequency),
        f(model.head.classifier.weight),
        f(model.head.classifier.bias),
    ]


class AlphabetTrainFunction(torch.autograd.Function):
    """logits = ALPHABET(x; tensors) with the B200 backward."""

    @staticmethod
    def forward(ctx, x: Tensor, valid: Tensor | None, obs: Tensor | None, delta: Tensor | None,
                dims: tuple, *tensors: Tensor) -> Tensor:
        lib = _lib.load()
        keep = [t.detach().contiguous() for t in tensors]
        params = _lib.AlphabetParams(
            raw_input_dim=dims[0], model_dim=dims[1], modes=dims[2], output_dim=dims[3],
            conv_kernel=dims[4], conv_dilation=dims[5],
            **{name: t.data_ptr() for name, t in zip(_lib.PARAM_POINTER_FIELDS, keep)},
        )
        x = x.detach().contiguous()
        dtype = _lib.LNET_BF16 if x.dtype == torch.bfloat16 else _lib.LNET_F32
        # fp32 inputs: exact fp32 GEMMs; bf16 inputs: TF32 tensor cores (the
        # precision policy of the inference route)
        req = _lib.AlphabetRequest(batch=x.shape[0], steps=x.shape[1], x_dtype=dtype,
                                   act_dtype=dtype, x=x.data_ptr(),
                                   time_delta=None if delta is None else delta.data_ptr(),
                                   observation_mask=None if obs is None else obs.data_ptr(),
                                   obs_channels=1 if obs is None else obs.shape[-1],
                                   valid_mask=None if valid is None else valid.data_ptr())
        n = ctypes.c_size_t(0)
        _lib.check(lib.lnet_b200_alphabet_train_workspace_size(ctypes.byref(params),
                                                                ctypes.byref(req), ctypes.byref(n)),
                   "lnet_b200_alphabet_train_workspace_size")
        ws = torch.empty(max(int(n.value), 1), dtype=torch.uint8, device=x.device)
        logits = torch.empty(x.shape[0], dims[3], device=x.device, dtype=torch.float32)
        with torch.cuda.device(x.device):
            stream = torch.cuda.current_stream().cuda_stream
            _lib.check(lib.lnet_b200_alphabet_train_forward(ctypes.byref(params),
                                                            ctypes.byref(req), ws.data_ptr(),
                                                            int(n.value), logits.data_ptr(),
                                                            stream),
                       "lnet_b200_alphabet_train_forward")
        ctx.state = (params, req, ws, int(n.value), keep, x, valid, obs, delta)
        return logits

    @staticmethod
    def backward(ctx, dlogits: Tensor):
        lib = _lib.load()
        params, req, ws, nbytes, keep, x, valid, obs, delta = ctx.state
        dl = dlogits.detach().float().contiguous()
        grads = [torch.empty_like(t) for t in keep]
        gs = _lib.AlphabetGrads(**{name: g.data_ptr()
                                   for name, g in zip(_lib.PARAM_POINTER_FIELDS, grads)})
        with torch.cuda.device(dl.device):
            stream = torch.cuda.current_stream().cuda_stream
            _lib.check(lib.lnet_b200_alphabet_backward(ctypes.byref(params), ctypes.byref(req),
                                                       ws.data_ptr(), nbytes, dl.data_ptr(),
                                                       ctypes.byref(gs), stream),
                       "lnet_b200_alphabet_backward")
        ctx.state = None  # the workspace is single-use
        return (None, None, None, None, None, *grads)


def train_forward(model, x: Tensor, valid_mask: Tensor | None = None,
                  observation_mask: Tensor | None = None,
                  time_delta: Tensor | None = None) -> Tensor:
    """Differentiable logits of ``model`` (a ``B200Alphabet``) for ``x`` [B, T, C];
    metadata already normalised (fp32; valid [B, T], observation [B, T, 1 or C],
    time_delta [B, T])."""
    dims = (model.raw_input_dim, model.model_dim, model.modes,
            model.head.classifier.out_features, model.dwconv_kernel_size, model.dwconv_dilation)
    valid = None
    if valid_mask is not None:
        valid = valid_mask.to(device=x.device, dtype=torch.float32).reshape(x.shape[:2]).contiguous()
    obs = None
    if observation_mask is not None:
        obs = observation_mask.to(device=x.device, dtype=torch.float32).contiguous()
    delta = None
    if time_delta is not None:
        delta = time_delta.to(device=x.device, dtype=torch.float32).reshape(x.shape[:2]).contiguous()
    return AlphabetTrainFunction.apply(x, valid, obs, delta, dims, *effective_tensors(model))


__all__ = ["AlphabetTrainFunction", "effective_tensors", "train_forward"]
