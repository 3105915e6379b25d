"""Build recipe for ``oracle/_ref``: the reference's own FA-KLA CPU kernel.

Test infrastructure only (the checker, never the product). Compiles the
reference file ``ultra_rwka/backend/cpp/cpu/cpu_kernels.cpp`` *where it lies*
in the read-only reference checkout, unmodified, together with two small files
of ours:

* ``oracle/ref_shim/conv1d_compat.h`` (force-included) so the unrelated
  wavelet function at cpu_kernels.cpp:208-212 compiles against current
  libtorch;
* ``oracle/ref_shim/bind.cpp``, the pybind11 binding the reference lacks
  (its ``backend/cpp/fa_kla_bindings.cpp`` is empty).

The reference includes ``"../../include/common.h"`` but its include directory
is spelled ``backend/ include`` (leading space) on disk, so the relative path
never resolves in the reference tree itself. We provide an include root under
``oracle/_ref/inc`` whose ``include/common.h`` is a *symlink* to the reference
header (no copy) and point ``-I`` two levels below it.

Output: ``oracle/_ref/fakla_ref*.so`` (git-ignored; it travels to GPU hosts
with the rest of the tree). Needs only libtorch at run time. The source tree is
only read here, at build time, when the reference checkout is present.

Do not pass -fopenmp: with it, the ``#pragma omp simd`` inside the
AT_DISPATCH lambda at cpu_kernels.cpp:127 is a hard error. Without it,
``at::parallel_for`` still threads through libtorch's own pool.
"""
from __future__ import annotations

import glob
import os
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
# Root of the reference checkout (the directory holding ultra_rwka/): the
# `ref_root` argument, else this environment variable; with neither, build()
# only reports the prebuilt module.
REF_ENV = "FAKLA_REFERENCE_ROOT"
REF_SRC = "ultra_rwka/backend/cpp/cpu/cpu_kernels.cpp"
REF_HDR = "ultra_rwka/backend/ include/common.h"
OUT_DIR = os.path.join(HERE, "_ref")
NAME = "fakla_ref"


def built_module_path() -> str | None:
    hits = sorted(glob.glob(os.path.join(OUT_DIR, NAME + "*.so")))
    return hits[0] if hits else None


def reference_root(ref_root: str | None = None) -> str | None:
    return ref_root or os.environ.get(REF_ENV) or None


def build(ref_root: str | None = None, verbose: bool = False) -> str | None:
    """Compile the reference kernel; returns the .so path, or the prebuilt
    one (None if never built) when no reference checkout is given or present
    (e.g. on a GPU host, which uses the prebuilt file)."""
    ref_root = reference_root(ref_root)
    if ref_root is None:
        return built_module_path()
    src = os.path.join(ref_root, REF_SRC)
    hdr = os.path.join(ref_root, REF_HDR)
    if not (os.path.isfile(src) and os.path.isfile(hdr)):
        return built_module_path()
    os.makedirs(OUT_DIR, exist_ok=True)
    inc_root = os.path.join(OUT_DIR, "inc")
    deep = os.path.join(inc_root, "a", "b")
    os.makedirs(deep, exist_ok=True)
    os.makedirs(os.path.join(inc_root, "include"), exist_ok=True)
    link = os.path.join(inc_root, "include", "common.h")
    if os.path.islink(link) or os.path.exists(link):
        os.remove(link)
    os.symlink(hdr, link)

    from torch.utils import cpp_extension

    build_dir = os.path.join(OUT_DIR, "build")
    os.makedirs(build_dir, exist_ok=True)
    cpp_extension.load(
        name=NAME,
        sources=[src, os.path.join(HERE, "ref_shim", "bind.cpp")],
        extra_cflags=["-O3", "-include", os.path.join(HERE, "ref_shim", "conv1d_compat.h")],
        extra_include_paths=[deep],
        build_directory=build_dir,
        verbose=verbose,
        is_python_module=True,
        with_cuda=False,
    )
    # cpp_extension leaves the module in build_dir; publish it one level up.
    produced = sorted(glob.glob(os.path.join(build_dir, NAME + "*.so")))
    if not produced:
        raise RuntimeError("reference oracle build produced no shared object")
    dst = os.path.join(OUT_DIR, os.path.basename(produced[0]))
    if os.path.abspath(dst) != os.path.abspath(produced[0]):
        import shutil

        shutil.copy2(produced[0], dst)
    return dst


def load():
    """Import the prebuilt reference module (raises if it was never built)."""
    import importlib.util

    import torch  # noqa: F401  (libtorch must be loaded first)

    path = built_module_path()
    if path is None:
        raise ImportError("oracle/_ref not built: run oracle/build_ref.py where the reference is present")
    spec = importlib.util.spec_from_file_location(NAME, path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


if __name__ == "__main__":
    root = reference_root(sys.argv[1] if len(sys.argv) > 1 else None)
    if root is None:
        sys.exit(f"usage: python oracle/build_ref.py REFERENCE_ROOT (or set {REF_ENV})")
    print(build(root, verbose=True))
