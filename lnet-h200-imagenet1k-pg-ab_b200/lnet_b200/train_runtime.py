"""Captured fixed-shape training step: the role of the reference's
``prepare_exact_split_training`` / ``prepare_aggressive_training`` and their
``AlphabetTrainingRuntime`` (src/lnet/alphabet_backbone.py:1336-1673; the loss
objectives of src/lnet/pac_efp16_exact_split_training.py:113-172).

One training step (the B200 training forward ``lnet_b200_alphabet_train_forward``,
the loss, its gradient, ``lnet_b200_alphabet_backward``, the torch autograd tail
from the 17 effective tensors to the module's parameters, and the optimizer step)
is captured once into a CUDA graph over static input / label buffers and
replayed: one graph launch per step instead of a few hundred kernel and Python
dispatches, which is what dominates small training shapes.

Capture needs every op of the step to be free of host synchronisation.  The one
that is not is ``torch.matrix_exp`` of the frames' orthogonal parametrisation
(its CUDA implementation picks the number of squarings on the host), so inside
the runtime the frames are built by :func:`capturable_matrix_exp`: the same
trivialised parametrisation (``base @ exp(A)``, ``A = X.tril() - X.tril()^T``),
with a Taylor / scaling-and-squaring exponential whose squaring count is chosen
on the device.  It agrees with ``torch.matrix_exp`` to fp32 rounding.

The optimizer must be capturable (``torch.optim.AdamW(..., capturable=True)``,
as the reference requires of its outer graph).  Construction runs a few warm-up
steps on a side stream (allocations, library handles) and then restores every
parameter and optimizer state in place, so the first ``step`` is the model's
first update.
"""

from __future__ import annotations

import contextlib
import math

import torch
from torch import Tensor, nn
from torch.nn import functional as F

LOSS_KINDS = ("cross_entropy", "binary_cross_entropy", "mse")

_TAYLOR_DEGREE = 12
_THETA = 0.5  # ||X||_1 after scaling: Taylor remainder below 0.5^13 / 13! (~2e-14)
_MAX_SQUARINGS = 24


def capturable_matrix_exp(a: Tensor) -> Tensor:
    """``exp(a)`` of a square matrix without host synchronisation: scale by 2^-s
    with s = ceil(log2(||a||_1 / theta)) computed on the device, a degree-12
    Taylor polynomial (Horner), then ``_MAX_SQUARINGS`` conditional squarings of
    which the first s are applied.  Differentiable through torch autograd."""
    n = a.shape[-1]
    eye = torch.eye(n, dtype=a.dtype, device=a.device)
    with torch.no_grad():
        norm = a.abs().sum(dim=-2).amax(dim=-1)
        s = torch.ceil(torch.log2(torch.clamp(norm / _THETA, min=1.0)))
        s = torch.clamp(s, 0, _MAX_SQUARINGS)
    x = a * torch.exp2(-s)
    t = eye
    for k in range(_TAYLOR_DEGREE, 0, -1):
        t = eye + (x @ t) / k
    for i in range(_MAX_SQUARINGS):
        t = torch.where(s > i, t @ t, t)
    return t


def _orthogonal_frame(linear: nn.Linear) -> Tensor:
    """The frame weight of an ``orthogonal(..., orthogonal_map="matrix_exp",
    use_trivialization=True)`` parametrised linear, rebuilt with
    :func:`capturable_matrix_exp` (the steps of torch's ``_Orthogonal.forward``)."""
    if not hasattr(linear, "parametrizations"):  # a plain (unparametrised) frame
        return linear.weight
    param = linear.parametrizations.weight
    orth = param[0]
    x = param.original
    n, k = x.shape[-2], x.shape[-1]
    transposed = n < k
    if transposed:
        x = x.mT
        n, k = k, n
    x = x.tril()
    if n != k:
        x = torch.cat([x, x.new_zeros(n, n - k)], dim=-1)
    q = capturable_matrix_exp(x - x.mH)
    if n != k:
        q = q[..., :k]
    if getattr(orth, "base", None) is not None:
        q = orth.base @ q
    return q.mT if transposed else q


@contextlib.contextmanager
def capturable_frames(model):
    """Within the block, ``lnet_b200.training.effective_tensors`` builds the
    frames with :func:`capturable_matrix_exp`."""
    prev = getattr(model, "_frame_fn", None)
    model._frame_fn = _orthogonal_frame
    try:
        yield
    finally:
        model._frame_fn = prev


def _loss(kind: str, logits: Tensor, targets: Tensor, weight: Tensor | None) -> Tensor:
    if kind == "cross_entropy":
        return F.cross_entropy(logits, targets, weight=weight)
    if kind == "binary_cross_entropy":
        return F.binary_cross_entropy_with_logits(logits, targets)
    if kind == "mse":
        return F.mse_loss(logits.reshape_as(targets), targets)
    raise ValueError(f"unsupported loss_kind: {kind}")


class AlphabetTrainingRuntime:
    """Fixed-shape training step replayed from a CUDA graph.

    ``step(inputs, labels)`` copies same-shape CUDA tensors into the static
    buffers and launches the graph; ``step_static()`` launches it on whatever the
    caller wrote into :attr:`static_inputs` / :attr:`static_labels`;
    ``step_leased(inputs, labels)`` takes the construction tensors themselves and
    launches a second graph that also captured their copy.  Each returns the
    runtime's static loss tensor (read it before the next step to keep it).
    """

    def __init__(self, model, optimizer: torch.optim.Optimizer, example_inputs: Tensor,
                 example_labels: Tensor, *, example_time_delta: Tensor | None = None,
                 example_observation_mask: Tensor | None = None,
                 example_valid_mask: Tensor | None = None, loss_kind: str = "cross_entropy",
                 cross_entropy_weight: Tensor | None = None, warmup: int = 3):
        if loss_kind not in LOSS_KINDS:
            raise ValueError(f"unsupported loss_kind: {loss_kind}")
        if not example_inputs.is_cuda or not example_labels.is_cuda:
            raise RuntimeError("the training runtime needs CUDA example tensors")
        for group in optimizer.param_groups:  # optimizers with device step counters
            if group.get("capturable", True) is False:
                raise ValueError("the optimizer must be constructed with capturable=True")
        self.model = model
        self.optimizer = optimizer
        self.loss_kind = loss_kind
        self._meta = dict(time_delta=example_time_delta, observation_mask=example_observation_mask,
                          valid_mask=example_valid_mask)
        self._weight = cross_entropy_weight
        self._lease = (example_inputs, example_labels)
        self.static_inputs = example_inputs.detach().clone()
        self.static_labels = example_labels.detach().clone()
        model.train()
        saved = self._snapshot()
        dev = example_inputs.device
        side = torch.cuda.Stream(dev)
        side.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(side), capturable_frames(model):
            for _ in range(max(1, warmup)):
                self._body(self.static_inputs, self.static_labels)
        torch.cuda.current_stream(dev).wait_stream(side)
        self._restore(saved)
        self.graph = torch.cuda.CUDAGraph()
        self.optimizer.zero_grad(set_to_none=True)
        with capturable_frames(model), torch.cuda.graph(self.graph):
            self.static_loss = self._body(self.static_inputs, self.static_labels)
        self.leased_graph = torch.cuda.CUDAGraph()
        with capturable_frames(model), torch.cuda.graph(self.leased_graph,
                                                        pool=self.graph.pool()):
            self.static_inputs.copy_(example_inputs)
            self.static_labels.copy_(example_labels)
            self.leased_loss = self._body(self.static_inputs, self.static_labels)
        self._destroyed = False

    def _body(self, inputs: Tensor, labels: Tensor) -> Tensor:
        self.optimizer.zero_grad(set_to_none=False)
        logits = self.model(inputs, **{k: v for k, v in self._meta.items() if v is not None})
        loss = _loss(self.loss_kind, logits, labels, self._weight)
        loss.backward()
        self.optimizer.step()
        post = getattr(self.model, "post_optimizer_step", None)
        if callable(post):
            post()
        return loss.detach()

    def _snapshot(self):
        with torch.no_grad():
            params = [p.detach().clone() for p in self.model.parameters()]
            state = {}
            for p, st in self.optimizer.state.items():
                state[p] = {k: (v.clone() if torch.is_tensor(v) else v) for k, v in st.items()}
        return params, state

    def _restore(self, saved) -> None:
        params, state = saved
        with torch.no_grad():
            for p, v in zip(self.model.parameters(), params):
                p.copy_(v)
            for p, st in self.optimizer.state.items():
                old = state.get(p)
                for k, v in st.items():
                    if torch.is_tensor(v):
                        if old is not None and k in old:
                            v.copy_(old[k])
                        else:
                            v.zero_()
        # optimizer state created by the warm-up (first steps) restarts at zero, so
        # the first replay is the first update, as it would be eagerly

    def _check(self, inputs: Tensor, labels: Tensor) -> None:
        if self._destroyed:
            raise RuntimeError("the training runtime was closed")
        if inputs.shape != self.static_inputs.shape or inputs.dtype != self.static_inputs.dtype:
            raise ValueError(f"captured for inputs {tuple(self.static_inputs.shape)} "
                             f"{self.static_inputs.dtype}, got {tuple(inputs.shape)} {inputs.dtype}")
        if labels.shape != self.static_labels.shape or labels.dtype != self.static_labels.dtype:
            raise ValueError(f"captured for labels {tuple(self.static_labels.shape)} "
                             f"{self.static_labels.dtype}, got {tuple(labels.shape)} {labels.dtype}")

    def step(self, inputs: Tensor, labels: Tensor) -> Tensor:
        """Train on same-shape CUDA tensors (copied into the static buffers)."""
        self._check(inputs, labels)
        self.static_inputs.copy_(inputs, non_blocking=True)
        self.static_labels.copy_(labels, non_blocking=True)
        self.graph.replay()
        return self.static_loss

    def step_static(self) -> Tensor:
        """Train on the current contents of the static buffers."""
        if self._destroyed:
            raise RuntimeError("the training runtime was closed")
        self.graph.replay()
        return self.static_loss

    def step_leased(self, inputs: Tensor, labels: Tensor) -> Tensor:
        """Train in one launch from the construction tensors (updated in place)."""
        if self._destroyed:
            raise RuntimeError("the training runtime was closed")
        if inputs is not self._lease[0] or labels is not self._lease[1]:
            raise ValueError("step_leased takes the tensors the runtime was built with")
        self.leased_graph.replay()
        return self.leased_loss

    def close(self) -> None:
        if not self._destroyed:
            self.graph.reset()
            self.leased_graph.reset()
            self._destroyed = True

    destroy = close

    def __enter__(self):
        return self

    def __exit__(self, *_error: object) -> None:
        self.close()


def prepare_exact_split_training(model, optimizer, example_inputs: Tensor,
                                 example_labels: Tensor, *,
                                 example_time_delta: Tensor | None = None,
                                 example_observation_mask: Tensor | None = None,
                                 example_valid_mask: Tensor | None = None,
                                 loss_kind: str = "cross_entropy",
                                 cross_entropy_weight: Tensor | None = None,
                                 **options: object) -> AlphabetTrainingRuntime:
    """Captured training step for a fixed (shape, metadata) signature
    (src/lnet/alphabet_backbone.py:1336-1470).  The reference's kernel-selection
    options (``parallel_static_recurrence_training``, ``fused_*_training``,
    ``memory_efficient_lag124_training`` ...) pick among its Triton kernels; here
    one B200 training path serves every combination, so they are accepted and
    have no effect."""
    del options
    return AlphabetTrainingRuntime(model, optimizer, example_inputs, example_labels,
                                   example_time_delta=example_time_delta,
                                   example_observation_mask=example_observation_mask,
                                   example_valid_mask=example_valid_mask, loss_kind=loss_kind,
                                   cross_entropy_weight=cross_entropy_weight)


def prepare_aggressive_training(model, optimizer, example_inputs: Tensor,
                                example_labels: Tensor, *, loss_kind: str = "cross_entropy",
                                **options: object) -> AlphabetTrainingRuntime:
    """The reference's production training runtime
    (src/lnet/alphabet_backbone.py:1574-1673): the exact-split runtime with the
    optimizer inside the captured graph.  Here the optimizer step is always
    captured, so this is :func:`prepare_exact_split_training` without metadata."""
    return prepare_exact_split_training(model, optimizer, example_inputs, example_labels,
                                        loss_kind=loss_kind, **options)


__all__ = ["AlphabetTrainingRuntime", "LOSS_KINDS", "capturable_matrix_exp",
           "prepare_aggressive_training", "prepare_exact_split_training"]
