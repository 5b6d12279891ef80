"""Drop-in ``Alphabet`` whose forward runs on the lnet_b200 CUDA library.

:class:`B200Alphabet` mirrors the reference ``lnet.Alphabet``
(src/lnet/alphabet.py:66-416): the same constructor arguments, the same
module tree and ``state_dict`` keys (so a reference checkpoint loads with
``load_state_dict`` unchanged), the same ``forward(inputs, *, time_delta,
observation_mask, valid_mask)`` signature and the same ``ValueError``
messages for malformed metadata (src/lnet/alphabet_backbone.py:163-201,
522-591).  The forward pass itself is one call into the C ABI
(``lnet_b200_alphabet_forward``); there is no CPU path: non-CUDA inputs raise.

In eval mode (or under ``torch.no_grad``) the forward is that one call.  In
training mode with gradients enabled it runs the autograd function of
``lnet_b200.training`` instead: the fp32 training forward
(``lnet_b200_alphabet_train_forward``) keeps the activations and
``lnet_b200_alphabet_backward`` returns the parameter and input gradients.
"""

from __future__ import annotations

import math
from dataclasses import dataclass

import torch
from torch import Tensor, nn
from torch.nn.utils.parametrizations import orthogonal

from . import _lib


@dataclass(frozen=True)
class AlphabetConfig:
    """The fields of the reference ``PACExperimentConfig`` (src/lnet/pac_types.py:47-67)
    that the ALPHABET forward reads."""

    raw_input_dim: int
    model_dim: int
    modes: int
    output_dim: int = 2
    sequence_length: int = 1


class _RawForcingStem(nn.Module):
    """``Linear(C, D, bias=False)`` + same-length depthwise conv (SiLU applied in forward);
    mirrors src/lnet/pac_laplace_native_input.py:98-138."""

    def __init__(self, input_dim: int, model_dim: int, *, kernel_size: int, dilation: int) -> None:
        super().__init__()
        self.projection = nn.Linear(input_dim, model_dim, bias=False)
        nn.init.orthogonal_(self.projection.weight)
        span = dilation * (kernel_size - 1)
        self.local = nn.Conv1d(model_dim, model_dim, kernel_size=kernel_size, dilation=dilation,
                               padding=span // 2, groups=model_dim)
        with torch.no_grad():
            w = self.projection.weight
            active = w.float() if w.shape[0] >= w.shape[1] else w.float().T
            q, r = torch.linalg.qr(active, mode="reduced")
            signs = torch.where(torch.diagonal(r) >= 0, 1.0, -1.0)
            q = q * signs.unsqueeze(0)
            w.copy_(q if w.shape[0] >= w.shape[1] else q.T)


class _TightFrameBlock(nn.Module):
    """Parameters of one tied pole block (src/lnet/pac_tight_frame_models.py:320-443):
    RMSNorm weight, orthogonally parametrised frame ``[D, 2M]``, raw decay and
    frequency per mode, and the coupled residual scales (parameters in the
    writer, zero buffers in the reader)."""

    def __init__(self, model_dim: int, modes: int, *, residual_parameters: bool) -> None:
        super().__init__()
        self.direction = "forward"
        self.moment_lags = (1, 2, 4)
        self.damping_min = 1.0e-3
        self.damping_max = 2.0
        self.norm = nn.RMSNorm(model_dim)
        self.frame = nn.Linear(2 * modes, model_dim, bias=False)
        nn.init.orthogonal_(self.frame.weight)
        orthogonal(self.frame, "weight", orthogonal_map="matrix_exp", use_trivialization=True)
        self.raw_decay = nn.Parameter(torch.linspace(-3.0, 1.0, modes))
        grid = torch.linspace(0.0, 0.75, modes).clamp(max=0.999)
        self.raw_frequency = nn.Parameter(torch.atanh(grid))
        if residual_parameters:
            self.direct_scale = nn.Parameter(torch.zeros(model_dim))
            self.layer_scale = nn.Parameter(torch.full((model_dim,), 1.0e-2))
        else:
            self.register_buffer("direct_scale", torch.zeros(model_dim))
            self.register_buffer("layer_scale", torch.zeros(model_dim))

    def frame_matrix(self) -> Tensor:
        return self.frame.weight

    def damping_values(self) -> Tensor:
        return self.damping_min + (self.damping_max - self.damping_min) * torch.sigmoid(
            self.raw_decay
        )

    def frequency_values(self) -> Tensor:
        return math.pi * torch.tanh(self.raw_frequency)


class _ModalAffineHead(nn.Module):
    """``Linear(14M, K)`` over ``cat(writer, reader)`` radial-log moments (src/lnet/alphabet.py:49-63)."""

    def __init__(self, modes: int, output_dim: int) -> None:
        super().__init__()
        self.modes = modes
        self.mode_map = None
        self.classifier = nn.Linear(14 * modes, output_dim)


class B200Alphabet(nn.Module):
    """ALPHABET classifier with the forward pass on B200 CUDA kernels."""

    def __init__(
        self,
        config,
        output_dim: int,
        *,
        dwconv_kernel_size: int = 5,
        dwconv_dilation: int = 4,
        objective: str = "classification",
    ) -> None:
        super().__init__()
        if type(dwconv_kernel_size) is not int or dwconv_kernel_size < 1:
            raise ValueError("dwconv_kernel_size must be a positive integer")
        if type(dwconv_dilation) is not int or dwconv_dilation < 1:
            raise ValueError("dwconv_dilation must be a positive integer")
        if (dwconv_dilation * (dwconv_kernel_size - 1)) % 2:
            raise ValueError("odd receptive spans (padding='same') are not supported")
        if objective != "classification":
            raise ValueError("only the classification objective is supported")
        model_dim = int(config.model_dim)
        modes = int(config.modes)
        if modes < 1 or modes > model_dim // 2:
            # The reference constructor fails for modes > model_dim // 2
            # (lag-124 head rebuilt with the unclamped mode count).
            raise RuntimeError(
                f"modes={modes} must lie in [1, model_dim // 2 = {model_dim // 2}]"
            )
        self.model_dim = model_dim
        self.modes = modes
        self.raw_input_dim = int(config.raw_input_dim)
        self.dwconv_kernel_size = dwconv_kernel_size
        self.dwconv_dilation = dwconv_dilation
        self.validate_metadata = True
        self.stem = _RawForcingStem(self.raw_input_dim, model_dim, kernel_size=dwconv_kernel_size,
                                    dilation=dwconv_dilation)
        self.forward_block = _TightFrameBlock(model_dim, modes, residual_parameters=True)
        self.backward_block = _TightFrameBlock(model_dim, modes, residual_parameters=False)
        self.final_norm = None
        self.head = _ModalAffineHead(modes, output_dim)
        span = dwconv_dilation * (dwconv_kernel_size - 1)
        self.second_local = nn.Conv1d(model_dim, model_dim, kernel_size=dwconv_kernel_size,
                                      dilation=dwconv_dilation, padding=span // 2,
                                      groups=model_dim)
        self._cache_key = None
        self._cache = None
        self._prepare_spec = None  # (batch, length) once prepare_for_inference_ ran
        self._prep = None          # persistent workspace of the prepared path

    # ------------------------------------------------------------ construction helpers
    @classmethod
    def from_reference(cls, model: nn.Module) -> B200Alphabet:
        """Build from a reference ``lnet.Alphabet`` and copy its state."""
        for blk in (model.forward_block, model.backward_block):
            if blk._buffers.get("fixed_damping_values") is not None:
                raise NotImplementedError("fixed damping prefixes are not supported")
            if blk._buffers.get("intervention_frame_override") is not None:
                raise NotImplementedError("intervention frames are not supported")
        cfg = AlphabetConfig(
            raw_input_dim=model.stem.projection.in_features,
            model_dim=model.model_dim,
            modes=model.modes,
            output_dim=model.head.classifier.out_features,
        )
        out = cls(cfg, cfg.output_dim, dwconv_kernel_size=model.second_local.kernel_size[0],
                  dwconv_dilation=model.second_local.dilation[0])
        ref_state = model.state_dict()
        out.load_state_dict(ref_state, strict=True)
        return out.to(next(model.parameters()).device)

    def load_effective_parameters(self, params: dict[str, Tensor]) -> None:
        """Load parameters keyed by ``state_dict`` names, with materialised frames given as
        ``<block>.frame.weight`` ([D, 2M]); the frame parametrisation is then bypassed."""
        with torch.no_grad():
            for name, value in params.items():
                if name.endswith("frame.weight"):
                    blk = getattr(self, name.split(".")[0])
                    self._set_frame(blk, torch.as_tensor(value))
                    continue
                target = self.get_parameter(name) if _has_param(self, name) else self.get_buffer(name)
                target.copy_(torch.as_tensor(value, dtype=target.dtype))
        self._cache_key = None

    @staticmethod
    def _set_frame(blk: _TightFrameBlock, weight: Tensor) -> None:
        from torch.nn.utils import parametrize

        if parametrize.is_parametrized(blk.frame, "weight"):
            parametrize.remove_parametrizations(blk.frame, "weight", leave_parametrized=False)
        blk.frame.weight.data = weight.to(blk.frame.weight.device, blk.frame.weight.dtype).clone()

    # ------------------------------------------------------------ parameters for the C ABI
    def _effective(self, device: torch.device):
        key = (device, tuple((p.data_ptr(), p._version) for p in self.parameters()),
               tuple((b.data_ptr(), b._version) for b in self.buffers() if b is not None))
        if self._cache_key == key and self._cache is not None:
            return self._cache

        def f32(t: Tensor) -> Tensor:
            return t.detach().to(device=device, dtype=torch.float32).contiguous()

        fb, bb = self.forward_block, self.backward_block
        k = self.dwconv_kernel_size
        with torch.no_grad():
            tensors = {
                "stem_projection": f32(self.stem.projection.weight),
                "stem_conv_weight": f32(self.stem.local.weight.reshape(self.model_dim, k)),
                "stem_conv_bias": f32(self.stem.local.bias),
                "writer_norm": f32(fb.norm.weight),
                "writer_frame": f32(fb.frame_matrix()),
                "writer_raw_decay": f32(fb.raw_decay),
                "writer_raw_frequency": f32(fb.raw_frequency),
                "writer_direct_scale": f32(fb.direct_scale),
                "writer_layer_scale": f32(fb.layer_scale),
                "reader_conv_weight": f32(self.second_local.weight.reshape(self.model_dim, k)),
                "reader_conv_bias": f32(self.second_local.bias),
                "reader_norm": f32(bb.norm.weight),
                "reader_frame": f32(bb.frame_matrix()),
                "reader_raw_decay": f32(bb.raw_decay),
                "reader_raw_frequency": f32(bb.raw_frequency),
                "head_weight": f32(self.head.classifier.weight),
                "head_bias": f32(self.head.classifier.bias),
            }
        params = _lib.AlphabetParams(
            raw_input_dim=self.raw_input_dim,
            model_dim=self.model_dim,
            modes=self.modes,
            output_dim=self.head.classifier.out_features,
            conv_kernel=k,
            conv_dilation=self.dwconv_dilation,
            **{name: tensors[name].data_ptr() for name in _lib.PARAM_POINTER_FIELDS},
        )
        self._cache_key = key
        self._cache = (params, tensors)
        return self._cache

    # ------------------------------------------------------------ metadata (reference semantics)
    def _prepare_metadata(self, inputs, time_delta, observation_mask, valid_mask):
        """Shape/value validation of src/lnet/alphabet_backbone.py:522-591.  The value
        checks are evaluated on the device and read back with one synchronisation."""
        bt = inputs.shape[:2]
        dev = inputs.device
        delta = obs = valid = None
        checks: list[tuple[Tensor, str]] = []
        if time_delta is not None:
            if time_delta.shape not in (bt, (*bt, 1)):
                raise ValueError("time_delta must have shape [B,N] or [B,N,1]")
            delta = time_delta.to(device=dev, dtype=torch.float32).reshape(bt).contiguous()
            if self.validate_metadata:
                checks.append(((~torch.isfinite(delta)) | (delta < 0),
                               "time_delta must contain finite non-negative values"))
        if observation_mask is not None:
            if observation_mask.shape not in (bt, (*bt, 1), inputs.shape):
                raise ValueError(
                    "observation_mask must have shape [B,N], [B,N,1], or [B,N,C] matching the "
                    "raw input"
                )
            obs = observation_mask.to(device=dev, dtype=torch.float32)
            if obs.ndim == 2:
                obs = obs.unsqueeze(-1)
            obs = obs.contiguous()
            if self.validate_metadata:
                checks.append(((~torch.isfinite(obs)) | (obs < 0) | (obs > 1),
                               "observation_mask must contain finite values in [0,1]"))
        if valid_mask is not None:
            if valid_mask.shape not in (bt, (*bt, 1)):
                raise ValueError("valid_mask must have shape [B,N] or [B,N,1]")
            valid = valid_mask.to(device=dev, dtype=torch.float32).reshape(bt).contiguous()
            if self.validate_metadata:
                checks.append(((~torch.isfinite(valid)) | (valid < 0) | (valid > 1),
                               "valid_mask must contain finite values in [0,1]"))
        if checks:
            bad = torch.stack([c.any() for c, _ in checks]).cpu()  # one synchronisation
            for flag, (_, message) in zip(bad.tolist(), checks):
                if flag:
                    raise ValueError(message)
        return delta, obs, valid

    def _request(self, x: Tensor, delta, obs, valid, act_dtype: int) -> _lib.AlphabetRequest:
        return _lib.AlphabetRequest(
            batch=x.shape[0],
            steps=x.shape[1],
            x_dtype=_lib.LNET_BF16 if x.dtype == torch.bfloat16 else _lib.LNET_F32,
            act_dtype=act_dtype,
            x=x.data_ptr(),
            time_delta=None if delta is None else delta.data_ptr(),
            observation_mask=None if obs is None else obs.data_ptr(),
            obs_channels=0 if obs is None else obs.shape[-1],
            valid_mask=None if valid is None else valid.data_ptr(),
        )

    def forward(
        self,
        inputs: Tensor,
        *,
        time_delta: Tensor | None = None,
        observation_mask: Tensor | None = None,
        valid_mask: Tensor | None = None,
        return_moments: bool = False,
    ):
        if inputs.ndim != 3 or inputs.shape[-1] != self.raw_input_dim:
            raise ValueError(
                f"inputs must have shape [B,N,{self.raw_input_dim}], got {tuple(inputs.shape)}"
            )
        if not inputs.is_cuda:
            raise RuntimeError("B200Alphabet runs on CUDA only; move the inputs to a CUDA device")
        if inputs.dtype not in (torch.float32, torch.bfloat16):
            raise TypeError(f"inputs must be float32 or bfloat16, got {inputs.dtype}")
        if self.training and torch.is_grad_enabled():
            # training: the fp32 forward that keeps its activations, with the
            # B200 backward (lnet_b200.training)
            if return_moments:
                raise NotImplementedError("return_moments is an inference option")
            delta, obs, valid = self._prepare_metadata(inputs, time_delta, observation_mask,
                                                       valid_mask)
            from .training import train_forward

            return train_forward(self, inputs, valid, obs, delta).to(
                self.head.classifier.weight.dtype)
        delta, obs, valid = self._prepare_metadata(inputs, time_delta, observation_mask,
                                                   valid_mask)
        x = inputs.contiguous()
        act = _lib.LNET_BF16 if x.dtype == torch.bfloat16 else _lib.LNET_F32
        logits, wm, rm = alphabet_forward_raw(self, x, delta, obs, valid, act, return_moments)
        out_dtype = self.head.classifier.weight.dtype
        logits = logits.to(out_dtype)
        if return_moments:
            return logits, wm, rm
        return logits

    def op_arguments(self, device: torch.device | None = None) -> tuple[list[Tensor], list[int]]:
        """``(weights, dims)`` for ``torch.ops.lnet_b200.alphabet_forward``: the effective
        fp32 tensors in :data:`lnet_b200.ops.ALPHABET_WEIGHTS` order and the six sizes."""
        device = torch.device(device) if device is not None else self.head.classifier.weight.device
        params, tensors = self._effective(device)
        dims = [params.raw_input_dim, params.model_dim, params.modes, params.output_dim,
                params.conv_kernel, params.conv_dilation]
        return [tensors[name] for name in _lib.PARAM_POINTER_FIELDS], dims

    @torch.no_grad()
    def prepare_for_inference_(self, *, sequence_length: int, batch_size: int,
                               use_static_poles: bool = True) -> B200Alphabet:
        """Prepared static inference (the reference's ``Alphabet.prepare_for_inference_``,
        src/lnet/alphabet.py:190-222): later forwards keep one workspace and build the
        fused route's operands (bf16 GEMM slabs with the ZOH gains folded in, pole
        constants; ``lnet_b200_alphabet_prepare``) once instead of per call, rebuilding
        them only when a parameter changes (version counters) or the workspace grows.
        ``batch_size`` x ``sequence_length`` sizes the workspace up front; larger
        requests grow it.  ``use_static_poles=False`` turns preparation off.  Calls of a
        prepared module must be ordered on one CUDA stream (they share the workspace)."""
        self.eval()
        self._prepare_spec = (int(batch_size), int(sequence_length)) if use_static_poles else None
        self._prep = None
        return self

    def forward_images(self, images: Tensor, *, mean=None, std=None, patch: int = 4,
                       dtype: torch.dtype = torch.bfloat16, return_moments: bool = False):
        """Forward from uint8 images [B, H, W, 3] on CUDA: normalise + patchify on
        the GPU (bit-identical to the harness transform), then the forward on the
        tokens.  Inference requests the fused route serves (4 x 4 patches, bf16,
        48 raw channels) build the tokens inside the fused writer
        (``lnet_b200_alphabet_forward_images``: no token tensor in HBM); every other
        request patchifies first (:func:`lnet_b200.images.patchify_images`) and
        calls :meth:`forward`."""
        from .images import IMAGENET_MEAN, IMAGENET_STD, patchify_images

        mean = IMAGENET_MEAN if mean is None else mean
        std = IMAGENET_STD if std is None else std
        if images.dtype != torch.uint8 or images.ndim != 4 or images.shape[-1] != 3:
            raise ValueError(f"images must be uint8 [B, H, W, 3], got {images.dtype} "
                             f"{tuple(images.shape)}")
        if (patch == 4 and dtype == torch.bfloat16 and images.is_cuda
                and not (self.training and torch.is_grad_enabled())
                and images.shape[1] % 4 == 0 and images.shape[2] % 4 == 0):
            images = images.contiguous()
            if images_route_fused(self, images):
                logits, wm, rm = images_forward_raw(self, images, mean, std, return_moments)
                logits = logits.to(self.head.classifier.weight.dtype)
                return (logits, wm, rm) if return_moments else logits
        x = patchify_images(images, mean=mean, std=std, patch=patch, dtype=dtype)
        return self.forward(x, return_moments=return_moments)


def _has_param(module: nn.Module, name: str) -> bool:
    try:
        module.get_parameter(name)
        return True
    except AttributeError:
        return False


def right_padded_lengths(valid: Tensor) -> Tensor | None:
    """int64 [B] valid lengths when ``valid`` [B, T] is a right-padded 0/1 mask (ones,
    then zeros), else None.  One synchronisation."""
    t = valid.shape[1]
    lengths = (valid != 0).sum(dim=1)
    prefix = torch.arange(t, device=valid.device).unsqueeze(0) < lengths.unsqueeze(1)
    if not torch.equal(valid, prefix.to(valid.dtype)):
        return None
    return lengths.to(torch.int64).contiguous()


def alphabet_forward_raw(model: B200Alphabet, x: Tensor, delta, obs, valid, act_dtype: int,
                         want_moments: bool = False):
    """One ``lnet_b200_alphabet_forward`` call on the current CUDA stream.  A
    right-padded valid mask on a request the fused route serves goes to
    ``lnet_b200_alphabet_forward_lengths`` (per-row lengths; padded chunks skipped),
    which computes the same result."""
    lib = _lib.load()
    params, _keep = model._effective(x.device)
    lengths = None
    if valid is not None and delta is None:
        req0 = model._request(x, None, obs, None, act_dtype)
        if lib.lnet_b200_alphabet_route(ctypes_ref(params), ctypes_ref(req0)) == 0:
            lengths = right_padded_lengths(valid)
    req = model._request(x, delta, obs, None if lengths is not None else valid, act_dtype)
    b = x.shape[0]
    m = model.modes
    logits = torch.empty(b, model.head.classifier.out_features, device=x.device,
                         dtype=torch.float32)
    wm = rm = None
    if want_moments:
        wm = torch.empty(b, 7 * m, device=x.device, dtype=torch.float32)
        rm = torch.empty(b, 7 * m, device=x.device, dtype=torch.float32)
    nbytes = _workspace_bytes(params, req)
    stream = torch.cuda.current_stream(x.device).cuda_stream
    prepared = getattr(model, "_prepare_spec", None) is not None
    if prepared:
        ws, nbytes = _prepared_workspace(model, params, req, nbytes, x.device, stream)
    else:
        ws = torch.empty(max(nbytes, 1), dtype=torch.uint8, device=x.device)
    wm_p = None if wm is None else wm.data_ptr()
    rm_p = None if rm is None else rm.data_ptr()
    with torch.cuda.device(x.device):
        if lengths is not None:
            name = "lnet_b200_alphabet_forward_lengths"
            st = lib.lnet_b200_alphabet_forward_lengths(
                ctypes_ref(params), ctypes_ref(req), lengths.data_ptr(), int(prepared),
                ws.data_ptr(), nbytes, logits.data_ptr(), wm_p, rm_p, stream)
        elif prepared:
            name = "lnet_b200_alphabet_forward_prepared"
            st = lib.lnet_b200_alphabet_forward_prepared(
                ctypes_ref(params), ctypes_ref(req), ws.data_ptr(), nbytes, logits.data_ptr(),
                wm_p, rm_p, stream)
        else:
            name = "lnet_b200_alphabet_forward"
            st = lib.lnet_b200_alphabet_forward(
                ctypes_ref(params), ctypes_ref(req), ws.data_ptr(), nbytes, logits.data_ptr(),
                wm_p, rm_p, stream)
    _lib.check(st, name)
    return logits, wm, rm


def _images_request(images: Tensor):
    """The token request an image forward stands for: [B, (H/4)(W/4), 48] bf16."""
    b, h, w, _ = images.shape
    return _lib.AlphabetRequest(batch=b, steps=(h // 4) * (w // 4), x_dtype=_lib.LNET_BF16,
                                act_dtype=_lib.LNET_BF16, x=images.data_ptr(), obs_channels=0)


def images_route_fused(model: B200Alphabet, images: Tensor) -> bool:
    """Whether ``lnet_b200_alphabet_forward_images`` serves these images (fused route)."""
    if images.shape[0] == 0 or images.data_ptr() % 16 != 0:
        return False
    lib = _lib.load()
    params, _keep = model._effective(images.device)
    return lib.lnet_b200_alphabet_route(ctypes_ref(params),
                                        ctypes_ref(_images_request(images))) == 0


def images_forward_raw(model: B200Alphabet, images: Tensor, mean, std,
                       want_moments: bool = False):
    """One ``lnet_b200_alphabet_forward_images`` call on the current CUDA stream."""
    import ctypes

    lib = _lib.load()
    params, _keep = model._effective(images.device)
    req = _images_request(images)
    b, h, w, _ = images.shape
    m = model.modes
    logits = torch.empty(b, model.head.classifier.out_features, device=images.device,
                         dtype=torch.float32)
    wm = rm = None
    if want_moments:
        wm = torch.empty(b, 7 * m, device=images.device, dtype=torch.float32)
        rm = torch.empty(b, 7 * m, device=images.device, dtype=torch.float32)
    n = ctypes.c_size_t(0)
    _lib.check(lib.lnet_b200_alphabet_images_workspace_size(ctypes_ref(params), b, h, w,
                                                            ctypes.byref(n)),
               "lnet_b200_alphabet_images_workspace_size")
    nbytes = int(n.value)
    stream = torch.cuda.current_stream(images.device).cuda_stream
    prepared = getattr(model, "_prepare_spec", None) is not None
    if prepared:
        ws, nbytes = _prepared_workspace(model, params, req, nbytes, images.device, stream)
    else:
        ws = torch.empty(max(nbytes, 1), dtype=torch.uint8, device=images.device)
    mean_c = (ctypes.c_float * 3)(*[float(v) for v in mean])
    std_c = (ctypes.c_float * 3)(*[float(v) for v in std])
    with torch.cuda.device(images.device):
        st = lib.lnet_b200_alphabet_forward_images(
            ctypes_ref(params), images.data_ptr(), b, h, w, mean_c, std_c, int(prepared),
            ws.data_ptr(), nbytes, logits.data_ptr(), None if wm is None else wm.data_ptr(),
            None if rm is None else rm.data_ptr(), stream)
    _lib.check(st, "lnet_b200_alphabet_forward_images")
    return logits, wm, rm


def _prepared_workspace(model, params, req, need: int, device, stream):
    """The prepared module's persistent workspace, (re)prepared when the parameters
    changed, the request needs more room, or the request takes the fused route and
    the operands have not been built yet."""
    lib = _lib.load()
    fused = lib.lnet_b200_alphabet_route(ctypes_ref(params), ctypes_ref(req)) == 0
    prep = model._prep
    key = (device, model._cache_key)
    if prep is None or prep["key"] != key or prep["cap"] < need:
        b, t = model._prepare_spec
        sized = _lib.AlphabetRequest(batch=b, steps=t, x_dtype=req.x_dtype,
                                     act_dtype=req.act_dtype, x=req.x,
                                     obs_channels=req.obs_channels)
        cap = max(need, _workspace_bytes(params, sized))
        if prep is not None and prep["key"][0] == device and prep["cap"] >= cap:
            ws, cap = prep["ws"], prep["cap"]  # parameters changed: rebuild in place
        else:
            # zero-filled once: no word of a fresh persistent workspace can pose as a
            # look-back record (tag 0 is never used)
            ws = torch.zeros(max(cap, 1), dtype=torch.uint8, device=device)
        prep = model._prep = {"key": key, "ws": ws, "cap": cap, "fused": False}
    if fused and not prep["fused"]:
        with torch.cuda.device(device):
            _lib.check(lib.lnet_b200_alphabet_prepare(ctypes_ref(params), ctypes_ref(req),
                                                      prep["ws"].data_ptr(), prep["cap"], stream),
                       "lnet_b200_alphabet_prepare")
        prep["fused"] = True
    return prep["ws"], prep["cap"]


def _workspace_bytes(params, req) -> int:
    import ctypes

    lib = _lib.load()
    n = ctypes.c_size_t(0)
    _lib.check(lib.lnet_b200_alphabet_workspace_size(ctypes.byref(params), ctypes.byref(req),
                                                     ctypes.byref(n)),
               "lnet_b200_alphabet_workspace_size")
    return int(n.value)


def ctypes_ref(obj):
    import ctypes

    return ctypes.byref(obj)


__all__ = ["AlphabetConfig", "B200Alphabet", "alphabet_forward_raw"]
