"""ctypes binding of the lnet_b200 C ABI (``include/lnet_b200.h``).

The shared library is built in-tree by :mod:`lnet_b200.build`.  There is no
CPU or Python fallback: if the library cannot be loaded, every entry point
raises.
"""

from __future__ import annotations

import ctypes
import os
import threading
from pathlib import Path

from . import build as _build

LNET_OK = 0
LNET_ERR_INVALID_ARGUMENT = 1
LNET_ERR_UNSUPPORTED = 2
LNET_ERR_WORKSPACE = 3
LNET_ERR_CUDA = 4

LNET_F32 = 0
LNET_BF16 = 1
LNET_F64 = 2

_c_p = ctypes.c_void_p
_i32 = ctypes.c_int32
_i64 = ctypes.c_int64


class AlphabetParams(ctypes.Structure):
    _fields_ = [
        ("raw_input_dim", _i32),
        ("model_dim", _i32),
        ("modes", _i32),
        ("output_dim", _i32),
        ("conv_kernel", _i32),
        ("conv_dilation", _i32),
        ("stem_projection", _c_p),
        ("stem_conv_weight", _c_p),
        ("stem_conv_bias", _c_p),
        ("writer_norm", _c_p),
        ("writer_frame", _c_p),
        ("writer_raw_decay", _c_p),
        ("writer_raw_frequency", _c_p),
        ("writer_direct_scale", _c_p),
        ("writer_layer_scale", _c_p),
        ("reader_conv_weight", _c_p),
        ("reader_conv_bias", _c_p),
        ("reader_norm", _c_p),
        ("reader_frame", _c_p),
        ("reader_raw_decay", _c_p),
        ("reader_raw_frequency", _c_p),
        ("head_weight", _c_p),
        ("head_bias", _c_p),
    ]


PARAM_POINTER_FIELDS = [name for name, _ in AlphabetParams._fields_[6:]]


class AlphabetRequest(ctypes.Structure):
    _fields_ = [
        ("batch", _i64),
        ("steps", _i64),
        ("x_dtype", _i32),
        ("act_dtype", _i32),
        ("x", _c_p),
        ("time_delta", _c_p),
        ("observation_mask", _c_p),
        ("obs_channels", _i32),
        ("valid_mask", _c_p),
    ]


class AlphabetGrads(ctypes.Structure):
    """Output pointers of lnet_b200_alphabet_backward, in PARAM_POINTER_FIELDS order."""
    _fields_ = [(name, _c_p) for name in PARAM_POINTER_FIELDS]


# name -> (restype, argtypes)
SIGNATURES = {
    "lnet_b200_alphabet_train_workspace_size": (
        ctypes.c_int,
        [ctypes.POINTER(AlphabetParams), ctypes.POINTER(AlphabetRequest),
         ctypes.POINTER(ctypes.c_size_t)],
    ),
    "lnet_b200_alphabet_train_forward": (
        ctypes.c_int,
        [ctypes.POINTER(AlphabetParams), ctypes.POINTER(AlphabetRequest), _c_p, ctypes.c_size_t,
         _c_p, _c_p],
    ),
    "lnet_b200_alphabet_backward": (
        ctypes.c_int,
        [ctypes.POINTER(AlphabetParams), ctypes.POINTER(AlphabetRequest), _c_p, ctypes.c_size_t,
         _c_p, ctypes.POINTER(AlphabetGrads), _c_p],
    ),
    "lnet_b200_alphabet_workspace_size": (
        ctypes.c_int,
        [ctypes.POINTER(AlphabetParams), ctypes.POINTER(AlphabetRequest),
         ctypes.POINTER(ctypes.c_size_t)],
    ),
    "lnet_b200_alphabet_forward": (
        ctypes.c_int,
        [ctypes.POINTER(AlphabetParams), ctypes.POINTER(AlphabetRequest), _c_p, ctypes.c_size_t,
         _c_p, _c_p, _c_p, _c_p],
    ),
    "lnet_b200_alphabet_prepare": (
        ctypes.c_int,
        [ctypes.POINTER(AlphabetParams), ctypes.POINTER(AlphabetRequest), _c_p, ctypes.c_size_t,
         _c_p],
    ),
    "lnet_b200_alphabet_forward_prepared": (
        ctypes.c_int,
        [ctypes.POINTER(AlphabetParams), ctypes.POINTER(AlphabetRequest), _c_p, ctypes.c_size_t,
         _c_p, _c_p, _c_p, _c_p],
    ),
    "lnet_b200_alphabet_forward_lengths": (
        ctypes.c_int,
        [ctypes.POINTER(AlphabetParams), ctypes.POINTER(AlphabetRequest), _c_p, _i32, _c_p,
         ctypes.c_size_t, _c_p, _c_p, _c_p, _c_p],
    ),
    "lnet_b200_alphabet_images_workspace_size": (
        ctypes.c_int, [ctypes.POINTER(AlphabetParams), _i64, _i32, _i32,
                       ctypes.POINTER(ctypes.c_size_t)],
    ),
    "lnet_b200_alphabet_forward_images": (
        ctypes.c_int,
        [ctypes.POINTER(AlphabetParams), _c_p, _i64, _i32, _i32, ctypes.POINTER(ctypes.c_float),
         ctypes.POINTER(ctypes.c_float), _i32, _c_p, ctypes.c_size_t, _c_p, _c_p, _c_p, _c_p],
    ),
    "lnet_b200_alphabet_device_status": (
        ctypes.c_int,
        [ctypes.POINTER(AlphabetParams), ctypes.POINTER(AlphabetRequest), _c_p, ctypes.c_size_t,
         ctypes.POINTER(ctypes.c_uint32)],
    ),
    "lnet_b200_set_route": (ctypes.c_int, [ctypes.c_int]),
    "lnet_b200_set_gemm_backend": (ctypes.c_int, [ctypes.c_int]),
    "lnet_b200_debug_inject_lookback_miss": (ctypes.c_int, []),
    "lnet_b200_alphabet_route": (
        ctypes.c_int, [ctypes.POINTER(AlphabetParams), ctypes.POINTER(AlphabetRequest)]
    ),
    "lnet_b200_zoh": (ctypes.c_int, [_c_p, _c_p, _i32, _c_p, _i64, _c_p, _c_p, _c_p, _c_p, _c_p]),
    "lnet_b200_stem": (
        ctypes.c_int,
        [ctypes.POINTER(AlphabetParams), ctypes.POINTER(AlphabetRequest), _c_p, ctypes.c_size_t,
         _c_p, _c_p],
    ),
    "lnet_b200_writer": (
        ctypes.c_int,
        [ctypes.POINTER(AlphabetParams), ctypes.POINTER(AlphabetRequest), _c_p, _c_p,
         ctypes.c_size_t, _c_p, _c_p, _c_p],
    ),
    "lnet_b200_reader": (
        ctypes.c_int,
        [ctypes.POINTER(AlphabetParams), ctypes.POINTER(AlphabetRequest), _c_p, _c_p,
         ctypes.c_size_t, _c_p, _c_p],
    ),
    "lnet_b200_head": (
        ctypes.c_int, [ctypes.POINTER(AlphabetParams), _i64, _c_p, _c_p, _c_p, _c_p]
    ),
    "lnet_b200_patchify_images": (
        ctypes.c_int,
        [_c_p, _i64, _i32, _i32, _i32, ctypes.POINTER(ctypes.c_float),
         ctypes.POINTER(ctypes.c_float), _c_p, _i32, _c_p],
    ),
    "lnet_b200_block_drive": (
        ctypes.c_int, [ctypes.POINTER(AlphabetParams), ctypes.POINTER(AlphabetRequest), _i32, _c_p, _c_p, ctypes.c_size_t, _c_p, _c_p, _c_p],
    ),
    "lnet_b200_block_scan": (
        ctypes.c_int, [ctypes.POINTER(AlphabetParams), ctypes.POINTER(AlphabetRequest), _i32, _c_p, _c_p, _c_p, ctypes.c_size_t, _c_p],
    ),
    "lnet_b200_block_moment_sums": (
        ctypes.c_int, [ctypes.POINTER(AlphabetParams), ctypes.POINTER(AlphabetRequest), _c_p, _c_p, _c_p, ctypes.c_size_t, _c_p, _c_p],
    ),
    "lnet_b200_writer_output": (
        ctypes.c_int, [ctypes.POINTER(AlphabetParams), ctypes.POINTER(AlphabetRequest), _c_p, _c_p, _c_p, _c_p, ctypes.c_size_t, _c_p, _c_p],
    ),
    "lnet_b200_depthwise_conv_silu": (
        ctypes.c_int, [ctypes.POINTER(AlphabetParams), ctypes.POINTER(AlphabetRequest), _i32, _c_p, _c_p, _c_p],
    ),
    "lnet_b200_laplace_workspace_size": (
        ctypes.c_int, [_i64, _i64, _i32, _i32, ctypes.POINTER(ctypes.c_size_t)]
    ),
    "lnet_b200_laplace_forward": (
        ctypes.c_int,
        [_c_p, _c_p, _c_p, _c_p, _i32, _i32, ctypes.c_double, ctypes.c_double, _i32, _c_p, _i64,
         _i64, _c_p, _c_p, ctypes.c_size_t, _c_p],
    ),
    "lnet_b200_laplace_forward_channelwise": (
        ctypes.c_int,
        [_c_p, _c_p, _c_p, _c_p, _c_p, _i32, _i32, _i32, ctypes.c_double, ctypes.c_double, _i32,
         _c_p, _i64, _i64, _c_p, _c_p],
    ),
    "lnet_b200_laplace_noalloc_max_scratch_bytes": (ctypes.c_size_t, []),
    "lnet_b200_laplace_forward_noalloc": (
        ctypes.c_int,
        [_c_p, _c_p, _c_p, _c_p, _i32, _i32, ctypes.c_double, ctypes.c_double, _i32, _c_p, _i64,
         _i64, _c_p, _c_p],
    ),
    "lnet_b200_trace_enable": (ctypes.c_int, [ctypes.c_int]),
    "lnet_b200_trace_read": (ctypes.c_int, [ctypes.POINTER(ctypes.c_ulonglong)]),
    "lnet_b200_trace_read_async": (ctypes.c_int, [ctypes.POINTER(ctypes.c_ulonglong), _c_p]),
    "lnet_b200_last_launch_count": (ctypes.c_int, []),
    "lnet_b200_profile_enable": (None, [ctypes.c_int]),
    "lnet_b200_profile_read": (
        ctypes.c_int,
        [ctypes.c_char_p, ctypes.c_int, ctypes.POINTER(ctypes.c_float),
         ctypes.POINTER(ctypes.c_int), ctypes.c_int],
    ),
    "lnet_b200_last_error": (ctypes.c_char_p, []),
    "lnet_b200_version": (ctypes.c_char_p, []),
}

_lock = threading.Lock()
_lib: ctypes.CDLL | None = None


def library_path() -> Path:
    return _build.LIB


def load(auto_build: bool = True) -> ctypes.CDLL:
    """Load (building first if the library is absent or stale and nvcc exists)."""
    global _lib
    with _lock:
        if _lib is not None:
            return _lib
        # LNET_B200_LIBRARY: load that build of the library instead of the in-tree one
        override = os.environ.get("LNET_B200_LIBRARY")
        path = Path(override) if override else _build.LIB
        if not override and auto_build and _build.needs_build():
            try:
                _build.build()
            except RuntimeError:
                if not path.exists():
                    raise
        if not path.exists():
            raise RuntimeError(
                f"lnet_b200 CUDA library missing at {path}; run lnet_b200.build.build()"
            )
        lib = ctypes.CDLL(str(path))
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        _lib = lib
        return lib


def last_error() -> str:
    return load().lnet_b200_last_error().decode()


def last_launch_count() -> int:
    return int(load().lnet_b200_last_launch_count())


def check(status: int, what: str) -> None:
    """Raise the Python exception matching a C status code."""
    if status == LNET_OK:
        return
    msg = f"{what}: {last_error()}"
    if status == LNET_ERR_INVALID_ARGUMENT:
        raise ValueError(msg)
    if status == LNET_ERR_UNSUPPORTED:
        raise TypeError(msg)
    raise RuntimeError(msg)


def profile_enable(on: bool) -> None:
    load().lnet_b200_profile_enable(1 if on else 0)


def profile_read(max_entries: int = 64) -> dict[str, tuple[float, int]]:
    """Per kernel name: (total milliseconds, launches) since profile_enable(True)."""
    lib = load()
    buf = ctypes.create_string_buffer(1 << 16)
    ms = (ctypes.c_float * max_entries)()
    cnt = (ctypes.c_int * max_entries)()
    n = lib.lnet_b200_profile_read(buf, len(buf), ms, cnt, max_entries)
    names = buf.value.decode().split("\n")
    return {names[i]: (float(ms[i]), int(cnt[i])) for i in range(n)}


ROUTE_AUTO = 0
ROUTE_GENERAL = 1


def set_route(route: int) -> None:
    check(load().lnet_b200_set_route(int(route)), "lnet_b200_set_route")


TRACE_SLOTS = {0: "claim", 1: "tile_load", 2: "first_gemm_wait", 3: "token_epilogue",
               4: "drive_gemm_wait", 5: "scan", 6: "synthesis_wait", 7: "residual_epilogue",
               8: "lookback_prefetch_hits", 9: "lookbacks", 10: "scan_pass1", 11: "lookback", 12: "scan_pass2", 15: "items"}


def trace_enable(on: bool) -> None:
    check(load().lnet_b200_trace_enable(1 if on else 0), "lnet_b200_trace_enable")


def trace_read() -> dict[str, dict[str, int]]:
    """Per kernel (writer, reader): phase -> summed cycles of CTA thread 0."""
    buf = (ctypes.c_ulonglong * 32)()
    check(load().lnet_b200_trace_read(buf), "lnet_b200_trace_read")
    out = {}
    for k, name in enumerate(("fused_writer_kernel", "fused_reader_kernel")):
        out[name] = {TRACE_SLOTS[s]: int(buf[16 * k + s]) for s in TRACE_SLOTS}
    return out
