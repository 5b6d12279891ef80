"""The allocation-free Laplace entry point against the workspace entry point.

``lnet_b200_laplace_forward_noalloc`` serves callers that must not allocate
device memory (a host framework that owns every allocation, a plugin that may
not call cudaMalloc, a real-time loop).  It keeps its scratch in a fixed
array inside the library instead of a caller workspace.  This test calls both
entry points through the C ABI on the same inputs, twice in a row (the second
call reuses the array left over by the first), and requires the results to
agree within the tolerance the Laplace parity tests use.  It also checks that
a shape needing more scratch than the array holds is refused.

The file is named to be collected last, so a run stopping at the first
failure has already run every other test.
"""

from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch
from conftest import rel_err

from lnet_b200 import _lib

pytestmark = pytest.mark.gpu


def _params(d, modes, seed, device):
    g = torch.Generator().manual_seed(seed)
    raw = torch.randn(modes, generator=g, dtype=torch.float64)
    res = torch.randn(d, modes, d, generator=g, dtype=torch.float64) * 0.3
    direct = torch.randn(d, d, generator=g, dtype=torch.float64) * 0.3
    bias = torch.randn(d, generator=g, dtype=torch.float64) * 0.1
    return [t.to(device).contiguous() for t in (raw, res, direct, bias)]


def _with_workspace(lib, p, d, modes, x, y, stream):
    b, t, _ = x.shape
    n = ctypes.c_size_t(0)
    _lib.check(lib.lnet_b200_laplace_workspace_size(b, t, d, modes, ctypes.byref(n)), "size")
    ws = torch.empty(int(n.value), dtype=torch.uint8, device=x.device)
    dtype = _lib.LNET_F64 if x.dtype == torch.float64 else _lib.LNET_F32
    _lib.check(lib.lnet_b200_laplace_forward(
        *(q.data_ptr() for q in p), d, modes, 1.0, 1e-3, dtype, x.data_ptr(), b, t,
        y.data_ptr(), ws.data_ptr(), int(n.value), stream), "laplace_forward")


def _no_alloc(lib, p, d, modes, x, y, stream):
    b, t, _ = x.shape
    dtype = _lib.LNET_F64 if x.dtype == torch.float64 else _lib.LNET_F32
    return lib.lnet_b200_laplace_forward_noalloc(
        *(q.data_ptr() for q in p), d, modes, 1.0, 1e-3, dtype, x.data_ptr(), b, t,
        y.data_ptr(), stream)


@pytest.mark.parametrize("dtype", [torch.float64, torch.float32])
def test_no_alloc_matches_workspace_entry_point(dtype, cuda_device):
    lib = _lib.load()
    stream = torch.cuda.current_stream(cuda_device).cuda_stream
    d, modes = 6, 5
    tol = 1e-12 if dtype == torch.float64 else 1e-6
    for call, (b, t, seed) in enumerate([(3, 70, 1), (2, 41, 2)]):
        p = _params(d, modes, seed, cuda_device)
        x = torch.randn(b, t, d, generator=torch.Generator().manual_seed(10 + call)).to(
            cuda_device, dtype)
        ref = torch.empty_like(x)
        got = torch.full_like(x, float("nan"))
        _with_workspace(lib, p, d, modes, x, ref, stream)
        _lib.check(_no_alloc(lib, p, d, modes, x, got, stream), "laplace_forward_noalloc")
        torch.cuda.synchronize()
        assert torch.isfinite(got).all()
        assert rel_err(got.cpu().numpy(), ref.cpu().numpy()) <= tol


def test_no_alloc_rejects_oversized_shapes(cuda_device):
    lib = _lib.load()
    limit = int(lib.lnet_b200_laplace_noalloc_max_scratch_bytes())
    d, modes = 16, 32  # 2 slices of 256 states: 2 * B * T * 16 * 8 bytes of scratch
    t = limit // (2 * 16 * 8) + 1
    p = _params(d, modes, 3, cuda_device)
    x = torch.zeros(1, t, d, device=cuda_device, dtype=torch.float64)
    y = torch.empty_like(x)
    st = _no_alloc(lib, p, d, modes, x, y, torch.cuda.current_stream(cuda_device).cuda_stream)
    assert st == _lib.LNET_ERR_WORKSPACE
    assert "no-alloc" in _lib.last_error()
    assert np.isfinite(limit) and limit > 0
