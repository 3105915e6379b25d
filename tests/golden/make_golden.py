"""Generate the golden FA-KLA fixtures from the reference implementation.

Run where the reference checkout is present (it is read, never copied):

    python tests/golden/make_golden.py REFERENCE_ROOT     (or set FAKLA_REFERENCE_ROOT)

It imports the reference's own Python modules (LearnablePositiveMap,
TMLinKernelAttn) and calls the reference's own CPU kernel
``fa_kla_attention_cpu`` (ultra_rwka/backend/cpp/cpu/cpu_kernels.cpp:36-170),
compiled in place by ``oracle/build_ref.py``. The reference has no golden
vectors of its own (every file under its tests/ is empty), so these fixtures
are the pin for the oracle and for the GPU kernels.

Reference import shim (the reference package does not import as shipped):
``attention/tm_kla.py`` was written for ``ultra_rwka/components/attention/``
(its relative imports reach ``..projections`` and ``...backend.interface``),
``kernels/mixer.py`` applies ``torch.jit.script`` to a function typed with
``List[FeatureMap]`` (fails at import) and uses ``warnings`` without importing
it, and ``backend/interface.py`` is empty. The shim registers the modules under
the package paths the relative imports expect, loads ``mixer.py`` with
``torch.jit.script`` temporarily replaced by the identity, and provides
``fa_kla_attention`` = the compiled reference kernel.

Stored values: inputs are regenerated from seeds (torch.Generator on CPU);
parameters are pinned by checksums (our modules must reproduce the reference
initialisation from torch.manual_seed(0)); outputs are stored in float32.
S and z come from the float64 oracle restatement (the reference never returns
its state), cross-checked here against the reference output.
"""
from __future__ import annotations

import importlib.util
import os
import sys
import types

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)

from oracle import build_ref  # noqa: E402
from oracle import fakla_oracle as O  # noqa: E402


def _load_file(name: str, path: str, package: str):
    spec = importlib.util.spec_from_file_location(name, path)
    mod = importlib.util.module_from_spec(spec)
    mod.__package__ = package
    sys.modules[name] = mod
    spec.loader.exec_module(mod)
    return mod


def load_reference(ref_root: str, ref_kernel):
    """Import the reference's LearnablePositiveMap and TMLinKernelAttn."""
    fm, _, tm = load_reference_modules(ref_root, ref_kernel)
    return fm.LearnablePositiveMap, tm.TMLinKernelAttn


def load_reference_modules(ref_root: str, ref_kernel):
    """Import the reference's feature_maps, mixer and tm_kla modules."""
    pkg = os.path.join(ref_root, "ultra_rwka")
    for name, path in [
        ("ultra_rwka", pkg),
        ("ultra_rwka.components", os.path.join(pkg, "components")),
        ("ultra_rwka.components.attention", os.path.join(pkg, "attention")),
        ("ultra_rwka.components.kernels", os.path.join(pkg, "kernels")),
        ("ultra_rwka.backend", os.path.join(pkg, "backend")),
    ]:
        m = types.ModuleType(name)
        m.__path__ = [path]
        sys.modules[name] = m
    iface = types.ModuleType("ultra_rwka.backend.interface")
    iface.fa_kla_attention = ref_kernel.fa_kla_attention_cpu
    sys.modules["ultra_rwka.backend.interface"] = iface
    fm = _load_file("ultra_rwka.components.kernels.feature_maps",
                    os.path.join(pkg, "kernels", "feature_maps.py"), "ultra_rwka.components.kernels")
    import warnings

    real_script = torch.jit.script
    torch.jit.script = lambda f, *a, **k: f
    builtins_mod = sys.modules["builtins"]
    had_warnings = hasattr(builtins_mod, "warnings")
    builtins_mod.warnings = warnings  # mixer.py:183 uses `warnings` without importing it
    try:
        mx = _load_file("ultra_rwka.components.kernels.mixer", os.path.join(pkg, "kernels", "mixer.py"),
                        "ultra_rwka.components.kernels")
    finally:
        torch.jit.script = real_script
        if not had_warnings:
            del builtins_mod.warnings
    _load_file("ultra_rwka.components.projections", os.path.join(pkg, "components", "projections.py"),
               "ultra_rwka.components")
    tm = _load_file("ultra_rwka.components.attention.tm_kla", os.path.join(pkg, "attention", "tm_kla.py"),
                    "ultra_rwka.components.attention")
    return fm, mx, tm


def gen(shape, seed, kind="normal", lo=0.0, hi=1.0):
    g = torch.Generator().manual_seed(seed)
    if kind == "normal":
        return torch.randn(*shape, generator=g)
    return torch.rand(*shape, generator=g) * (hi - lo) + lo


def checksum(t: torch.Tensor) -> np.ndarray:
    a = t.detach().double().reshape(-1)
    return np.array([a.sum().item(), (a * a).sum().item(), a[:16].sum().item(), float(a.numel())])


def main(ref_root: str) -> None:
    ref = build_ref.load() if build_ref.built_module_path() else None
    if ref is None:
        build_ref.build(ref_root)
        ref = build_ref.load()
    LPM, TMLKA = load_reference(ref_root, ref)
    out = {}

    # -- small fp32 case: B=2, H=4, T=256, Dk=Dv=M=64, fp32; LearnablePositiveMap(256, 256) from seed 0
    B, T, H, D = 2, 256, 4, 64
    torch.manual_seed(0)
    lpm = LPM(H * D, H * D)
    W = lpm.mlp[0].weight.detach().clone()
    bvec = lpm.mlp[0].bias.detach().clone()
    q, k, v = gen((B, T, H, D), 101), gen((B, T, H, D), 102), gen((B, T, H, D), 103)
    with torch.no_grad():
        pq = lpm(q.reshape(B, T, H * D)).reshape(B, T, H, D).contiguous()
        pk = lpm(k.reshape(B, T, H * D)).reshape(B, T, H, D).contiguous()
    temp = torch.ones(B, T, H)
    o_ref = ref.fa_kla_attention_cpu(pq, pk, v.contiguous(), temp)
    o64, S64, z64 = O.prefill(q.numpy(), k.numpy(), v.numpy(), W.numpy(), bvec.numpy())
    assert O.rel_l2(o_ref.numpy(), o64) < 1e-5, "oracle restatement disagrees with the reference"
    out["small_W_checksum"] = checksum(W)
    out["small_b_checksum"] = checksum(bvec)
    out["small_phi_q_checksum"] = checksum(pq)
    out["small_out"] = o_ref.numpy().astype(np.float32)
    out["small_S"] = S64.astype(np.float32)
    out["small_z"] = z64.astype(np.float32)

    # -- small ragged case with a temperature: B=1, H=3, T=37, Df=16, Dv=24
    q = gen((1, 37, 3, 16), 201, "uniform", 0.1, 1.5)
    k = gen((1, 37, 3, 16), 202, "uniform", 0.1, 1.5)
    v = gen((1, 37, 3, 24), 203)
    tp = gen((1, 37, 3), 204, "uniform", 0.5, 1.5)
    o_ref = ref.fa_kla_attention_cpu(q, k, v, tp)
    o64, S64, z64 = O.attention(q.numpy(), k.numpy(), v.numpy(), tp.numpy())
    assert O.rel_l2(o_ref.numpy(), o64) < 1e-5
    out["ragged_out"] = o_ref.numpy().astype(np.float32)
    out["ragged_S"] = S64.astype(np.float32)
    out["ragged_z"] = z64.astype(np.float32)

    # -- single token, single head: T=1 (first-step behaviour, cpu_kernels.cpp:78-79 zero state)
    q = gen((3, 1, 1, 8), 301, "uniform", 0.1, 1.0)
    k = gen((3, 1, 1, 8), 302, "uniform", 0.1, 1.0)
    v = gen((3, 1, 1, 8), 303)
    tp = gen((3, 1, 1), 304, "uniform", 0.5, 1.5)
    out["t1_out"] = ref.fa_kla_attention_cpu(q, k, v, tp).numpy().astype(np.float32)

    # -- module: TMLinKernelAttn(256, LPM(256,256), H=4, qk=64, v=64), x (2, 64, 256)
    torch.manual_seed(0)
    mapper = LPM(256, 256)
    mod = TMLKA(256, mapper, num_heads=4, qk_dim=64, v_dim=64)
    x = gen((2, 64, 256), 401)
    with torch.no_grad():
        y = mod(x)
    out["module_state_checksum"] = np.stack([checksum(p) for _, p in sorted(mod.state_dict().items())])
    out["module_state_names"] = np.array(sorted(mod.state_dict().keys()))
    out["module_out"] = y.numpy().astype(np.float32)

    path = os.path.join(HERE, "fakla_golden.npz")
    np.savez_compressed(path, **out)
    print("wrote", path, os.path.getsize(path), "bytes")


if __name__ == "__main__":
    from oracle.build_ref import REF_ENV, reference_root

    root = reference_root(sys.argv[1] if len(sys.argv) > 1 else None)
    if root is None:
        sys.exit(f"usage: python {sys.argv[0]} REFERENCE_ROOT (or set {REF_ENV})")
    main(root)
