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
