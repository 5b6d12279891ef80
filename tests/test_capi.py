"""The C-ABI library loads and exports every entry point the headers declare."""

from __future__ import annotations

import ctypes
import re
from pathlib import Path

from conftest import ROOT

HEADERS = sorted((ROOT / "include").glob("*.h"))


def declared_symbols() -> set[str]:
    names = set()
    for h in HEADERS:
        text = re.sub(r"/\*.*?\*/", "", h.read_text(), flags=re.S)
        names |= set(re.findall(r"\b(lnet_b200_\w+)\s*\(", text))
    return names


def test_headers_declare_entry_points():
    names = declared_symbols()
    assert "lnet_b200_alphabet_forward" in names
    assert "lnet_b200_laplace_forward" in names


def test_library_exports_every_declared_symbol():
    from lnet_b200 import _lib

    lib = _lib.load()
    missing = [n for n in sorted(declared_symbols()) if not hasattr(lib, n)]
    assert not missing, missing
    assert all(n in _lib.SIGNATURES for n in declared_symbols())


def test_error_paths_without_gpu():
    """Argument validation runs before any CUDA call, so it works on CPU hosts."""
    from lnet_b200 import _lib

    lib = _lib.load()
    n = ctypes.c_size_t(0)
    st = lib.lnet_b200_alphabet_workspace_size(None, None, ctypes.byref(n))
    assert st == _lib.LNET_ERR_INVALID_ARGUMENT
    assert "params" in _lib.last_error()
    st = lib.lnet_b200_laplace_workspace_size(2, 8, 0, 3, ctypes.byref(n))
    assert st == _lib.LNET_ERR_INVALID_ARGUMENT
    st = lib.lnet_b200_laplace_workspace_size(2, 8, 4, 3, ctypes.byref(n))
    assert st == _lib.LNET_OK and n.value > 0
    assert lib.lnet_b200_version().startswith(b"lnet_b200")


def test_laplace_scratch_size_overflow_is_refused_without_gpu():
    """A shape whose scratch size wraps 64 bits is refused before any launch, by the
    size query and by both forward entry points (the no-alloc one must not let a
    wrapped size pass its 8 MiB check)."""
    from lnet_b200 import _lib

    lib = _lib.load()
    n = ctypes.c_size_t(0)
    huge = 1 << 62
    st = lib.lnet_b200_laplace_workspace_size(2, huge, 16, 8, ctypes.byref(n))
    assert st == _lib.LNET_ERR_INVALID_ARGUMENT and "overflow" in _lib.last_error()
    dummy = ctypes.c_void_p(256)  # never dereferenced: the shape is refused first
    st = lib.lnet_b200_laplace_forward_noalloc(dummy, dummy, dummy, dummy, 16, 8, 1.0, 0.0,
                                               _lib.LNET_F32, dummy, 2, huge, dummy, None)
    assert st == _lib.LNET_ERR_INVALID_ARGUMENT and "overflow" in _lib.last_error()
    st = lib.lnet_b200_laplace_forward(dummy, dummy, dummy, dummy, 16, 8, 1.0, 0.0,
                                       _lib.LNET_F32, dummy, 2, huge, dummy, dummy, 1 << 20, None)
    assert st == _lib.LNET_ERR_INVALID_ARGUMENT and "overflow" in _lib.last_error()


def _struct_fields(name: str) -> list[str]:
    text = re.sub(r"/\*.*?\*/", "", (ROOT / "include" / "lnet_b200.h").read_text(), flags=re.S)
    body = re.search(r"typedef struct %s \{(.*?)\} %s;" % (name, name), text, flags=re.S)
    assert body, name
    return re.findall(r"(\w+)\s*;", body.group(1))


def test_struct_layouts_match_header():
    """The ctypes mirrors list the header's fields in the header's order."""
    from lnet_b200 import _lib

    for cname, py in (("lnet_b200_alphabet_params", _lib.AlphabetParams),
                      ("lnet_b200_alphabet_request", _lib.AlphabetRequest),
                      ("lnet_b200_alphabet_grads", _lib.AlphabetGrads)):
        assert _struct_fields(cname) == [f for f, _ in py._fields_], cname


def test_training_error_paths_without_gpu():
    """The training entry points validate before any CUDA call: a missing
    workspace and malformed metadata are reported, and the workspace size is
    computed on the host."""
    from lnet_b200 import _lib

    lib = _lib.load()
    dummy = 256  # non-NULL pointers are never dereferenced on these paths
    params = _lib.AlphabetParams(raw_input_dim=4, model_dim=8, modes=4, output_dim=3,
                                 conv_kernel=5, conv_dilation=4,
                                 **{n: dummy for n in _lib.PARAM_POINTER_FIELDS})
    req = _lib.AlphabetRequest(batch=2, steps=10, x_dtype=_lib.LNET_F32, act_dtype=_lib.LNET_F32,
                               x=dummy, obs_channels=1)
    n = ctypes.c_size_t(0)
    assert lib.lnet_b200_alphabet_train_workspace_size(ctypes.byref(params), ctypes.byref(req),
                                                       ctypes.byref(n)) == _lib.LNET_OK
    assert n.value > 0
    st = lib.lnet_b200_alphabet_train_forward(ctypes.byref(params), ctypes.byref(req), None, 0,
                                              dummy, None)
    assert st == _lib.LNET_ERR_WORKSPACE
    req.time_delta = dummy  # physical time is supported: validation reaches the workspace
    st = lib.lnet_b200_alphabet_train_forward(ctypes.byref(params), ctypes.byref(req), None, 0,
                                              dummy, None)
    assert st == _lib.LNET_ERR_WORKSPACE
    req.obs_channels = 3  # neither 1 nor C
    req.observation_mask = dummy
    st = lib.lnet_b200_alphabet_train_forward(ctypes.byref(params), ctypes.byref(req), None, 0,
                                              dummy, None)
    assert st == _lib.LNET_ERR_INVALID_ARGUMENT
