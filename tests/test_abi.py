"""The C ABI library: loads without a GPU, exports every symbol the headers
declare, and rejects malformed calls before touching a device (CPU only; no
compute call is made here)."""
import ctypes
import glob
import os
import re

import pytest

from pulsartecture_b200 import _lib

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_functions():
    decls = {}
    for h in sorted(glob.glob(os.path.join(ROOT, "include", "*.h"))):
        text = open(h).read()
        text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
        for m in re.finditer(r"^\s*(?:const\s+)?(?:int|size_t|char\s*\*|void)\s*\*?\s*(fakla_\w+)\s*\(([^;]*?)\)\s*;",
                             text, flags=re.M | re.S):
            args = m.group(2).strip()
            n = 0 if args in ("", "void") else len([a for a in args.split(",") if a.strip()])
            decls[m.group(1)] = n
    return decls


def test_header_declares_the_entry_points():
    d = declared_functions()
    for name in ["fakla_attention", "fakla_phi", "fakla_prefill", "fakla_decode", "fakla_decode_mapped",
                 "fakla_strerror", "fakla_last_error", "fakla_device_status"]:
        assert name in d, name


def test_library_exports_every_declared_symbol():
    lib = _lib.lib()
    for name, nargs in declared_functions().items():
        assert hasattr(lib, name), f"{name} declared in include/ but not exported"
        assert name in _lib.SIGNATURES, f"{name} missing from the ctypes signature table"
        assert len(_lib.SIGNATURES[name][1]) == nargs, f"{name}: header has {nargs} args"


def test_version_and_strerror():
    lib = _lib.lib()
    assert lib.fakla_version() == 1
    for code, name in _lib.STATUS.items():
        assert lib.fakla_strerror(code)
    assert lib.fakla_strerror(99) == b"unknown status"


def test_library_has_no_unresolved_cuda_runtime_dependency():
    # static CUDA runtime: the .so must not pin a libcudart.so version
    import subprocess

    out = subprocess.run(["ldd", _lib.LIB_PATH], capture_output=True, text=True).stdout
    assert "libcudart" not in out


def _no_gpu():
    import torch

    if torch.cuda.is_available():
        pytest.skip("dummy-pointer validation checks run only where no GPU exists; "
                    "the GPU tests cover validation with real buffers")


def test_argument_validation_without_device():
    _no_gpu()
    lib = _lib.lib()
    p = ctypes.c_void_p(16)  # never dereferenced: validation fails first
    # bad dtype
    rc = lib.fakla_attention(p, p, p, None, p, None, None, 1, 1, 1, 8, 8, 7, 0, None, 0, None)
    assert rc == 1 and b"dtype" in lib.fakla_last_error()
    # null inputs
    rc = lib.fakla_attention(None, p, p, None, p, None, None, 1, 1, 1, 8, 8, 0, 0, None, 0, None)
    assert rc == 1
    # non-positive sizes
    rc = lib.fakla_attention(p, p, p, None, p, None, None, 0, 1, 1, 8, 8, 0, 0, None, 0, None)
    assert rc == 1
    # head dim beyond the implemented range
    rc = lib.fakla_attention(p, p, p, None, p, None, None, 1, 1, 1, 512, 8, 0, 0, None, 0, None)
    assert rc == 2
    # state flags without state buffers
    rc = lib.fakla_attention(p, p, p, None, p, None, None, 1, 1, 1, 8, 8, 0, 1, None, 0, None)
    assert rc == 1
    # S without z
    rc = lib.fakla_attention(p, p, p, None, p, p, None, 1, 1, 1, 8, 8, 0, 0, None, 0, None)
    assert rc == 1
    # prefill without workspace
    rc = lib.fakla_prefill(p, p, p, None, p, None, p, None, None, 1, 4, 8, 1, 8, 8, 0, 0, None, 0, None)
    assert rc == 6
    # decode needs state
    rc = lib.fakla_decode_mapped(p, p, p, None, p, None, None, 1, 1, 8, 8, 0, None)
    assert rc == 1
    # no-allocation decode: a step whose phi scratch exceeds the static array
    N, H, M = 1024, 32, 128  # 2*N*H*M*2 B = 16 MiB > 8 MiB
    rc = lib.fakla_decode_noalloc(p, p, p, None, p, None, p, p, p, N, H * M, H, M, M, 1, None)
    assert rc == 2 and b"scratch" in lib.fakla_last_error()
    rc = lib.fakla_decode_noalloc(p, p, p, None, p, None, p, p, p, 0, 1, 1, 1, 1, 1, None)
    assert rc == 1
    # ... and it reports the argument error of an oversized call before its scratch limit
    rc = lib.fakla_decode_noalloc(None, p, p, None, p, None, p, p, p, N, H * M, H, M, M, 1, None)
    assert rc == 1 and b"non-NULL" in lib.fakla_last_error()
    rc = lib.fakla_decode_noalloc(p, p, p, None, p, None, p, p, p, N, H * 512, H, 512, M, 1, None)
    assert rc == 2 and b"head dims" in lib.fakla_last_error()
    # linear-layer gradients: dpre is required, dx needs W, db needs a workspace
    rc = lib.fakla_linear_backward(p, p, None, p, None, None, 8, 8, 8, 1, None, 0, None)
    assert rc == 1
    rc = lib.fakla_linear_backward(p, None, p, p, None, None, 8, 8, 8, 1, None, 0, None)
    assert rc == 1
    rc = lib.fakla_linear_backward(p, p, p, None, None, p, 8, 8, 8, 1, None, 0, None)
    assert rc == 6


def test_workspace_queries():
    lib = _lib.lib()
    B, T, D, H, M, Dv = 8, 4096, 2048, 16, 128, 128
    assert lib.fakla_prefill_workspace_bytes(B, T, D, H, M, Dv, 1) == 2 * B * T * H * M * 2
    assert lib.fakla_prefill_workspace_bytes(B, T, D, H, M, Dv, 0) == 2 * B * T * H * M * 4
    assert lib.fakla_decode_workspace_bytes(256, 4096, 32, 128, 128, 1) == 2 * 256 * 32 * 128 * 2
    assert lib.fakla_attention_workspace_bytes(B, T, H, M, Dv, 1) == 0


def test_call_without_gpu_reports_error_not_crash():
    _no_gpu()
    lib = _lib.lib()
    p = ctypes.c_void_p(16)
    rc = lib.fakla_attention(p, p, p, None, p, None, None, 1, 1, 1, 8, 8, 0, 0, None, 0, None)
    assert rc in (4, 7)  # CUDA error (no device) or no sm_100 device
