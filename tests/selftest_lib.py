"""Build/load tests/_build/libfakla_selftest.so (test-only kernels in
tests/csrc/selftest.cu)."""
from __future__ import annotations

import ctypes
import os
import subprocess

HERE = os.path.dirname(os.path.abspath(__file__))
SRC = os.path.join(HERE, "csrc", "selftest.cu")
OUT = os.path.join(HERE, "_build", "libfakla_selftest.so")
DEPS = [SRC, os.path.join(os.path.dirname(HERE), "pulsartecture_b200", "csrc", "sm100_umma.cuh")]


def build(force: bool = False) -> str:
    if force or not os.path.isfile(OUT) or any(os.path.getmtime(d) > os.path.getmtime(OUT) for d in DEPS):
        from pulsartecture_b200.build import ARCH_FLAGS, nvcc_path

        os.makedirs(os.path.dirname(OUT), exist_ok=True)
        tmp = OUT + ".tmp%d" % os.getpid()
        subprocess.check_call([nvcc_path(), *ARCH_FLAGS, "-O2", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC",
                               "-shared", "-cudart", "static", "-o", tmp, SRC])
        os.replace(tmp, OUT)
    return OUT


def load() -> ctypes.CDLL:
    lib = ctypes.CDLL(build())
    lib.selftest_umma_form.restype = ctypes.c_int
    lib.selftest_umma_form.argtypes = [ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p]
    lib.selftest_wait_timeout.restype = ctypes.c_int
    lib.selftest_wait_timeout.argtypes = [ctypes.c_uint64, ctypes.c_void_p, ctypes.c_void_p]
    return lib
