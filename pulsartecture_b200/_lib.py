"""ctypes binding of libfakla.so (the C ABI in include/fakla.h).

This module only loads the shared library and declares signatures; it never
computes anything itself. Loading does not need a GPU. There is no fallback:
if the library is missing, every entry point raises.
"""
from __future__ import annotations

import ctypes
import os
import threading

_PKG = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_PKG, "lib", "libfakla.so")

FAKLA_F32 = 0
FAKLA_BF16 = 1
FAKLA_STATE_IN = 1
FAKLA_STATE_OUT = 2

# fakla_activation (include/fakla.h)
FAKLA_ACT_ELU1 = 0
FAKLA_ACT_RELU = 1
FAKLA_ACT_SOFTPLUS = 2
FAKLA_ACT_GELU = 3
FAKLA_ACT_IDENTITY = 4
FAKLA_ACT_SIGMOID = 5
FAKLA_ACT_ABS = 6
FAKLA_ACT_COSSIN = 7

STATUS = {
    0: "FAKLA_OK",
    1: "FAKLA_ERR_INVALID_ARG",
    2: "FAKLA_ERR_UNSUPPORTED",
    3: "FAKLA_ERR_ALIGNMENT",
    4: "FAKLA_ERR_CUDA",
    5: "FAKLA_ERR_TIMEOUT",
    6: "FAKLA_ERR_WORKSPACE",
    7: "FAKLA_ERR_NO_DEVICE",
}

# Every exported symbol with (restype, argtypes). Kept in the order of
# include/fakla.h; tests check the header and this table agree.
_p = ctypes.c_void_p
_i64 = ctypes.c_int64
_int = ctypes.c_int
_uint = ctypes.c_uint
_sz = ctypes.c_size_t
SIGNATURES = {
    "fakla_strerror": (ctypes.c_char_p, [_int]),
    "fakla_last_error": (ctypes.c_char_p, []),
    "fakla_version": (_int, []),
    "fakla_attention": (_int, [_p, _p, _p, _p, _p, _p, _p, _i64, _i64, _i64, _i64, _i64, _int, _uint, _p, _sz, _p]),
    "fakla_attention_workspace_bytes": (_sz, [_i64, _i64, _i64, _i64, _i64, _int]),
    "fakla_phi": (_int, [_p, _p, _p, _p, _p, _i64, _i64, _i64, _i64, _int, _p]),
    "fakla_attention_backward": (_int, [_p, _p, _p, _p, _p, _p, _p, _p, _p, _p, _p, _p, _p, _p, _p,
                                        _i64, _i64, _i64, _i64, _i64, _int, _p, _sz, _p]),
    "fakla_attention_backward_workspace_bytes": (_sz, [_i64, _i64, _i64, _i64, _i64, _int]),
    "fakla_phi_backward": (_int, [_p, _p, _p, _i64, _int, _p]),
    "fakla_activation_backward": (_int, [_p, _p, _p, _i64, _i64, _int, ctypes.c_float, _int, _p]),
    "fakla_linear_backward": (_int, [_p, _p, _p, _p, _p, _p, _i64, _i64, _i64, _int, _p, _sz, _p]),
    "fakla_linear_backward_workspace_bytes": (_sz, [_i64, _i64, _i64, _int]),
    "fakla_mix_features_backward": (_int, [_p, _p, _p, _p, _p, _i64, _i64, _i64, _int, _p]),
    "fakla_feature_map": (_int, [_p, _p, _p, _p, _i64, _i64, _i64, _int, ctypes.c_float, _int, _p]),
    "fakla_mix_features": (_int, [_p, _p, _p, _i64, _i64, _i64, _int, _p]),
    "fakla_prefill": (_int, [_p, _p, _p, _p, _p, _p, _p, _p, _p, _i64, _i64, _i64, _i64, _i64, _i64, _int, _uint, _p, _sz, _p]),
    "fakla_prefill_workspace_bytes": (_sz, [_i64, _i64, _i64, _i64, _i64, _i64, _int]),
    "fakla_qkv_prefill": (_int, [_p, _p, _p, _p, _p, _p, _p, _i64, _i64, _i64, _i64, _i64, _i64, _int, _uint, _p, _sz, _p]),
    "fakla_qkv_prefill_workspace_bytes": (_sz, [_i64, _i64, _i64, _i64, _i64, _i64, _int]),
    "fakla_decode_mapped": (_int, [_p, _p, _p, _p, _p, _p, _p, _i64, _i64, _i64, _i64, _int, _p]),
    "fakla_decode": (_int, [_p, _p, _p, _p, _p, _p, _p, _p, _p, _i64, _i64, _i64, _i64, _i64, _int, _p, _sz, _p]),
    "fakla_decode_workspace_bytes": (_sz, [_i64, _i64, _i64, _i64, _i64, _int]),
    "fakla_decode_noalloc": (_int, [_p, _p, _p, _p, _p, _p, _p, _p, _p, _i64, _i64, _i64, _i64, _i64, _int, _p]),
    "fakla_device_status": (_int, [_p]),
}

_lib = None
_lock = threading.Lock()


class FaklaError(RuntimeError):
    """A libfakla call returned an error status (a RuntimeError, like the
    reference's TORCH_CHECK failures)."""

    def __init__(self, status: int, message: str):
        super().__init__(f"{STATUS.get(status, status)}: {message}")
        self.status = status


def lib() -> ctypes.CDLL:
    """Load libfakla.so (once). Raises if it has not been built."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not os.path.isfile(LIB_PATH):
                raise ImportError(
                    f"libfakla.so not found at {LIB_PATH}; build it with "
                    "`python -m pulsartecture_b200.build` (there is no CPU fallback)"
                )
            handle = ctypes.CDLL(LIB_PATH)
            for name, (res, args) in SIGNATURES.items():
                fn = getattr(handle, name)
                fn.restype = res
                fn.argtypes = args
            _lib = handle
    return _lib


def check(rc: int) -> None:
    if rc != 0:
        msg = lib().fakla_last_error().decode(errors="replace")
        raise FaklaError(rc, msg or lib().fakla_strerror(rc).decode())
