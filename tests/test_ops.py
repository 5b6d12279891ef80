"""The ``torch.library`` op surface and the inference runners, on CPU.

Mirrors the reference's op-level contract (functional ``lnet::`` ops with
``register_fake`` meta kernels, src/lnet/pac_triton_recurrence_op.py:603-684):
the ops are registered, FakeTensor tracing gives the output shapes and dtypes
without a GPU, bad arguments raise the reference's exception types
(``ValueError`` shapes, ``TypeError`` dtypes), and a CPU input raises
``RuntimeError`` instead of falling back.  The request-metadata validation of
the compiled-inference wrapper (src/lnet/alphabet_backbone.py:163-201) keeps
the reference's messages.
"""

from __future__ import annotations

import pytest
import torch
from torch._subclasses.fake_tensor import FakeTensorMode

from lnet_b200 import (AlphabetConfig, B200Alphabet, B200PoleResidueTemporalMixing, ops,
                       prepare_compiled_inference)
from lnet_b200.inference import validate_request_metadata


def _model():
    return B200Alphabet(AlphabetConfig(raw_input_dim=48, model_dim=64, modes=32,
                                       output_dim=10), 10).eval()


def test_ops_registered():
    for name in ("alphabet_forward", "laplace_forward", "patchify_images"):
        assert hasattr(torch.ops.lnet_b200, name)
        schema = str(getattr(torch.ops.lnet_b200, name).default._schema)
        assert "!" not in schema.split("->")[0], schema  # functional: no mutated arguments


def test_alphabet_op_fake_shapes():
    weights, dims = _model().op_arguments("cpu")
    assert dims == [48, 64, 32, 10, 5, 4]
    assert [tuple(w.shape) for w in weights][-2:] == [(10, 14 * 32), (10,)]
    with FakeTensorMode():
        wf = [torch.empty(w.shape) for w in weights]
        for dtype in (torch.float32, torch.bfloat16):
            x = torch.empty(3, 17, 48, dtype=dtype)
            y = torch.ops.lnet_b200.alphabet_forward(x, wf, dims)
            assert y.shape == (3, 10) and y.dtype == torch.float32
        y = torch.ops.lnet_b200.alphabet_forward(
            torch.empty(3, 17, 48), wf, dims, torch.empty(3, 17), torch.empty(3, 17, 48),
            torch.empty(3, 17))
        assert y.shape == (3, 10)


def test_alphabet_op_errors():
    weights, dims = _model().op_arguments("cpu")
    with FakeTensorMode():
        wf = [torch.empty(w.shape) for w in weights]
        with pytest.raises(ValueError):
            torch.ops.lnet_b200.alphabet_forward(torch.empty(3, 17, 40), wf, dims)
        with pytest.raises(TypeError):
            torch.ops.lnet_b200.alphabet_forward(torch.empty(3, 17, 48, dtype=torch.float16),
                                                 wf, dims)
        with pytest.raises(ValueError):
            torch.ops.lnet_b200.alphabet_forward(torch.empty(3, 17, 48), wf[:-1], dims)
        with pytest.raises(TypeError):
            torch.ops.lnet_b200.alphabet_forward(torch.empty(3, 17, 48),
                                                 [w.double() for w in wf], dims)
        with pytest.raises(ValueError):
            torch.ops.lnet_b200.alphabet_forward(torch.empty(3, 17, 48), wf, dims,
                                                 torch.empty(3, 16))
    with pytest.raises(RuntimeError, match="CUDA only"):
        torch.ops.lnet_b200.alphabet_forward(torch.randn(3, 17, 48), weights, dims)


def test_laplace_and_patchify_fake_shapes():
    layer = B200PoleResidueTemporalMixing(8, 12)
    p = [t.detach() for t in (layer.raw_decay, layer.residues, layer.direct_term, layer.bias)]
    with FakeTensorMode():
        pf = [torch.empty(t.shape, dtype=torch.float64) for t in p]
        for dtype in (torch.float32, torch.float64):
            y = torch.ops.lnet_b200.laplace_forward(torch.empty(2, 9, 8, dtype=dtype), *pf,
                                                    1.0, 1e-3)
            assert y.shape == (2, 9, 8) and y.dtype == dtype
        with pytest.raises(ValueError):
            torch.ops.lnet_b200.laplace_forward(torch.empty(2, 9, 7), *pf, 1.0, 1e-3)
        im = torch.empty(2, 32, 48, 3, dtype=torch.uint8)
        t = torch.ops.lnet_b200.patchify_images(im, [0.5] * 3, [0.25] * 3, 4, torch.bfloat16)
        assert t.shape == (2, 8 * 12, 48) and t.dtype == torch.bfloat16
        with pytest.raises(ValueError):
            torch.ops.lnet_b200.patchify_images(im, [0.5] * 3, [0.25] * 3, 5, torch.float32)
        with pytest.raises(TypeError):
            torch.ops.lnet_b200.patchify_images(im, [0.5] * 3, [0.25] * 3, 4, torch.float16)
    with pytest.raises(RuntimeError, match="CUDA only"):
        torch.ops.lnet_b200.laplace_forward(torch.randn(2, 9, 8), *p, 1.0, 1e-3)


def test_prepare_compiled_inference_modes():
    model = _model()
    assert prepare_compiled_inference(model, sequence_length=16, batch_size=2,
                                      compile_mode="none") is model
    assert model._prepare_spec == (2, 16)
    runner = prepare_compiled_inference(model, sequence_length=16, batch_size=2)
    assert runner.uses_cuda_graphs and runner.copy_output
    assert model.validate_metadata is False  # the wrapper validates instead
    with pytest.raises(ValueError):
        prepare_compiled_inference(_model(), sequence_length=16, batch_size=2,
                                   compile_mode="fast")


def test_request_metadata_validation_messages():
    x = torch.zeros(2, 5, 3)
    validate_request_metadata(x, torch.ones(2, 5, 1), torch.ones(2, 5, 3), torch.ones(2, 5))
    cases = [
        (dict(time_delta=torch.ones(2, 4)), "time_delta must have shape"),
        (dict(time_delta=-torch.ones(2, 5)), "finite non-negative"),
        (dict(observation_mask=torch.ones(2, 5, 2)), "observation_mask must have shape"),
        (dict(observation_mask=torch.full((2, 5), 2.0)), "finite values in \\[0,1\\]"),
        (dict(valid_mask=torch.full((2, 5), float("nan"))), "valid_mask must contain"),
    ]
    for kw, message in cases:
        args = {"time_delta": None, "observation_mask": None, "valid_mask": None, **kw}
        with pytest.raises(ValueError, match=message):
            validate_request_metadata(x, **args)
