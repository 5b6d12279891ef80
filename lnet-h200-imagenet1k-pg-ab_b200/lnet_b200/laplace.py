"""Drop-in ``PoleResidueTemporalMixing`` on the lnet_b200 CUDA library.

Mirrors src/lnet/laplace.py:55-159: the same float64 parameters
(``raw_decay [M]``, ``residues [D, M, D]``, ``direct_term [D, D]``,
``bias [D]``), ``continuous_poles``, ``load_transfer_parameters`` with the
reference's ``LaplaceParameterError`` checks, and ``forward`` raising
``LaplaceShapeError`` for bad ranks/widths.  The recurrence and the readout
run in float64 in one kernel pair (``lnet_b200_laplace_forward``); the state
never reaches HBM.  When the residues are diagonal in channels (each output
reads only its own input channel's states, as with M real poles per channel)
the layer runs ``lnet_b200_laplace_forward_channelwise`` instead: K state
updates per channel and no [D, M D] contraction.  The structure is detected
once per parameter version.
"""

from __future__ import annotations

import ctypes
from dataclasses import dataclass

import torch
from torch import Tensor, nn
from torch.nn import functional

from . import _lib


@dataclass(frozen=True, slots=True)
class LaplaceShapeError(ValueError):
    actual_shape: tuple[int, ...]
    expected_rank: int
    expected_features: int

    def __str__(self) -> str:
        return (
            "expected rank "
            f"{self.expected_rank} with trailing feature size {self.expected_features}, "
            f"received shape {self.actual_shape}"
        )


@dataclass(frozen=True, slots=True)
class LaplaceParameterError(ValueError):
    reason: str

    def __str__(self) -> str:
        return self.reason


def _inverse_softplus(value: Tensor) -> Tensor:
    return torch.log(torch.expm1(value))


class B200PoleResidueTemporalMixing(nn.Module):
    def __init__(self, model_dim: int, modes: int, *, dt: float = 1.0,
                 min_decay: float = 1.0e-3) -> None:
        super().__init__()
        self.model_dim = model_dim
        self.modes = modes
        self.dt = dt
        self.min_decay = min_decay
        initial_decay = torch.linspace(0.2, 1.0, modes, dtype=torch.float64)
        self.raw_decay = nn.Parameter(_inverse_softplus(initial_decay))
        self.residues = nn.Parameter(
            0.05 * torch.randn(model_dim, modes, model_dim, dtype=torch.float64)
        )
        self.direct_term = nn.Parameter(torch.zeros(model_dim, model_dim, dtype=torch.float64))
        self.bias = nn.Parameter(torch.zeros(model_dim, dtype=torch.float64))

    def continuous_poles(self) -> Tensor:
        return -(functional.softplus(self.raw_decay) + self.min_decay)

    def load_transfer_parameters(self, *, poles: Tensor, residues: Tensor, direct_term: Tensor,
                                 bias: Tensor) -> None:
        expected = (self.model_dim, self.modes, self.model_dim)
        if residues.shape != expected:
            raise LaplaceParameterError(
                reason=f"residue tensor shape mismatch: expected {expected}, received "
                f"{tuple(residues.shape)}"
            )
        if direct_term.shape != (self.model_dim, self.model_dim):
            raise LaplaceParameterError(
                reason="direct term shape mismatch: expected "
                f"{(self.model_dim, self.model_dim)}, received {tuple(direct_term.shape)}"
            )
        if bias.shape != (self.model_dim,):
            raise LaplaceParameterError(
                reason=f"bias shape mismatch: expected {(self.model_dim,)}, received "
                f"{tuple(bias.shape)}"
            )
        if poles.shape != (self.modes,):
            raise LaplaceParameterError(
                reason=f"pole shape mismatch: expected {(self.modes,)}, received "
                f"{tuple(poles.shape)}"
            )
        if not torch.all(poles < 0.0):
            raise LaplaceParameterError(reason="all poles must be strictly negative")
        with torch.no_grad():
            self.raw_decay.copy_(_inverse_softplus((-poles) - self.min_decay))
            self.residues.copy_(residues)
            self.direct_term.copy_(direct_term)
            self.bias.copy_(bias)

    @classmethod
    def from_reference(cls, layer: nn.Module) -> B200PoleResidueTemporalMixing:
        out = cls(layer.model_dim, layer.modes, dt=layer.dt, min_decay=layer.min_decay)
        out.load_state_dict(layer.state_dict())
        return out.to(layer.raw_decay.device)

    def forward(self, inputs: Tensor) -> Tensor:
        if inputs.ndim != 3 or inputs.shape[-1] != self.model_dim:
            raise LaplaceShapeError(actual_shape=tuple(inputs.shape), expected_rank=3,
                                    expected_features=self.model_dim)
        if not inputs.is_cuda:
            raise RuntimeError("B200PoleResidueTemporalMixing runs on CUDA only")
        if inputs.dtype not in (torch.float32, torch.float64):
            raise TypeError(f"inputs must be float32 or float64, got {inputs.dtype}")
        return laplace_forward_raw(self, inputs.contiguous())


MAX_MODES_PER_CHANNEL = 16  # bound of lnet_b200_laplace_forward_channelwise


def channel_diagonal_form(residues: Tensor) -> tuple[Tensor, Tensor] | None:
    """(mode_index [D, K] int32, residue [D, K] float64) when ``residues`` [D, M, D]
    is zero off the channel diagonal (R[o, m, i] = 0 for i != o) and every output
    has at most MAX_MODES_PER_CHANNEL nonzero R[o, m, o]; else None.  Padding slots
    carry a valid mode with residue 0 (they add exactly 0)."""
    d, m, d2 = residues.shape
    if d != d2:
        return None
    r = residues.detach()
    eye = torch.eye(d, dtype=torch.bool, device=r.device)
    if bool((r.permute(0, 2, 1)[~eye] != 0).any()):  # [o, i, m] off the diagonal
        return None
    ar = torch.arange(d, device=r.device)
    diag = r[ar, :, ar]  # [o, m] = R[o, m, o]
    nz = diag != 0
    k = max(1, int(nz.sum(dim=1).max()))
    if k > MAX_MODES_PER_CHANNEL:
        return None
    # nonzero modes first (stable order), then padding
    order = torch.argsort((~nz).to(torch.int8), dim=1, stable=True)[:, :k]
    vals = torch.gather(diag, 1, order) * torch.gather(nz, 1, order)
    return order.to(torch.int32).contiguous(), vals.to(torch.float64).contiguous()


def laplace_forward_raw(layer: B200PoleResidueTemporalMixing, x: Tensor) -> Tensor:
    """One ``lnet_b200_laplace_forward`` (or, for channel-diagonal residues,
    ``lnet_b200_laplace_forward_channelwise``) call with ``layer``'s parameters."""
    dev = x.device

    def f64(p: Tensor) -> Tensor:
        return p.detach().to(device=dev, dtype=torch.float64).contiguous()

    key = (dev, layer.residues._version, layer.residues.data_ptr())
    cache = getattr(layer, "_diag_cache", None)
    if cache is None or cache[0] != key:
        layer._diag_cache = cache = (key, channel_diagonal_form(f64(layer.residues)))
    if cache[1] is not None:
        idx, vals = cache[1]
        return _launch_channelwise(x, f64(layer.raw_decay), idx, vals, f64(layer.direct_term),
                                   f64(layer.bias), layer.modes, float(layer.dt),
                                   float(layer.min_decay))
    return _launch(x, f64(layer.raw_decay), f64(layer.residues), f64(layer.direct_term),
                   f64(layer.bias), layer.modes, float(layer.dt), float(layer.min_decay))


def _launch_channelwise(x: Tensor, raw: Tensor, idx: Tensor, vals: Tensor, direct: Tensor,
                        bias: Tensor, modes: int, dt: float, min_decay: float) -> Tensor:
    """The channel-diagonal C-ABI call on the current stream."""
    lib = _lib.load()
    dev = x.device
    b, t, d = x.shape
    y = torch.empty_like(x)
    if b == 0 or t == 0:
        return y
    stream = torch.cuda.current_stream(dev).cuda_stream
    dtype = _lib.LNET_F64 if x.dtype == torch.float64 else _lib.LNET_F32
    with torch.cuda.device(dev):
        st = lib.lnet_b200_laplace_forward_channelwise(
            raw.data_ptr(), idx.data_ptr(), vals.data_ptr(), direct.data_ptr(), bias.data_ptr(),
            d, modes, idx.shape[1], dt, min_decay, dtype, x.data_ptr(), b, t, y.data_ptr(),
            stream)
    _lib.check(st, "lnet_b200_laplace_forward_channelwise")
    return y


def _launch(x: Tensor, raw: Tensor, res: Tensor, direct: Tensor, bias: Tensor, modes: int,
            dt: float, min_decay: float) -> Tensor:
    """The C-ABI call on the current stream: contiguous float64 parameters on x's device."""
    lib = _lib.load()
    dev = x.device
    b, t, d = x.shape
    y = torch.empty_like(x)
    if b == 0 or t == 0:
        return y
    n = ctypes.c_size_t(0)
    _lib.check(lib.lnet_b200_laplace_workspace_size(b, t, d, modes, ctypes.byref(n)),
               "lnet_b200_laplace_workspace_size")
    ws = torch.empty(max(int(n.value), 1), dtype=torch.uint8, device=dev)
    stream = torch.cuda.current_stream(dev).cuda_stream
    dtype = _lib.LNET_F64 if x.dtype == torch.float64 else _lib.LNET_F32
    with torch.cuda.device(dev):
        st = lib.lnet_b200_laplace_forward(
            raw.data_ptr(), res.data_ptr(), direct.data_ptr(), bias.data_ptr(), d, modes, dt,
            min_decay, dtype, x.data_ptr(), b, t, y.data_ptr(), ws.data_ptr(), int(n.value),
            stream,
        )
    _lib.check(st, "lnet_b200_laplace_forward")
    return y


__all__ = [
    "B200PoleResidueTemporalMixing",
    "LaplaceParameterError",
    "LaplaceShapeError",
    "laplace_forward_raw",
]
