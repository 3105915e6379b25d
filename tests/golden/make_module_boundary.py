"""Capture the reference module's own call into its FA-KLA backend.

Run where the reference checkout is present (it is read, never copied):

    python tests/golden/make_module_boundary.py REFERENCE_ROOT     (or set FAKLA_REFERENCE_ROOT)

The reference's TMLinKernelAttn (ultra_rwka/attention/tm_kla.py:110-337) is
imported through the loader shim of make_golden.py and run on the CPU. Its
backend name `fa_kla_attention` (imported at tm_kla.py:15, called at :319) is
bound to a recorder that stores the four tensors the module passes, calls the
reference's own CPU kernel fa_kla_attention_cpu (cpu_kernels.cpp:36-170,
compiled in place by oracle/build_ref.py) and stores what it returns. The
module's final output is stored as well. tests/test_gpu_reference_module.py
replays those exact arguments through this library's fa_kla_attention on the
GPU; the reference checkout is not needed there.

Two module configurations, fp32, from fixed seeds:
  * default map: TMLinKernelAttn(128, LearnablePositiveMap(128, 128), num_heads=4,
    qk_dim=32, v_dim=32), x (2, 48, 128);
  * with temperature: the same plus temp_input_dim=16 (TemperatureFunction,
    softplus), temp_input (2, 48, 16).
"""
from __future__ import annotations

import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)
sys.path.insert(0, HERE)

from oracle import build_ref  # noqa: E402
from oracle import fakla_oracle as O  # noqa: E402


def main(ref_root: str) -> None:
    import make_golden

    ref = build_ref.load() if build_ref.built_module_path() else None
    if ref is None:
        build_ref.build(ref_root)
        ref = build_ref.load()
    fm, _, tm = make_golden.load_reference_modules(ref_root, ref)
    calls = []

    def recorder(q_mapped, k_mapped, v_reshaped, temp):
        out = ref.fa_kla_attention_cpu(q_mapped, k_mapped, v_reshaped, temp)
        calls.append([t.detach().clone() for t in (q_mapped, k_mapped, v_reshaped, temp, out)])
        return out

    tm.fa_kla_attention = recorder  # the name tm_kla.py:319 calls
    out = {}
    for tag, temp_dim in (("plain", 0), ("temp", 16)):
        torch.manual_seed(0)
        mapper = fm.LearnablePositiveMap(128, 128)
        mod = tm.TMLinKernelAttn(128, mapper, num_heads=4, qk_dim=32, v_dim=32, temp_input_dim=temp_dim)
        g = torch.Generator().manual_seed(7 + temp_dim)
        x = torch.randn(2, 48, 128, generator=g)
        ti = torch.randn(2, 48, temp_dim, generator=g) if temp_dim else None
        calls.clear()
        with torch.no_grad():
            y = mod(x, ti) if temp_dim else mod(x)
        assert len(calls) == 1, "the module calls its backend once per forward"
        qm, km, vv, tp, o = calls[0]
        e64, _, _ = O.attention(qm.numpy(), km.numpy(), vv.numpy(), tp.numpy())
        assert O.rel_l2(o.numpy(), e64) < 1e-5, "oracle disagrees with the reference kernel"
        for name, t in (("q_mapped", qm), ("k_mapped", km), ("v", vv), ("temp", tp), ("backend_out", o),
                        ("module_out", y)):
            out[f"{tag}/{name}"] = t.numpy().astype(np.float32)
    path = os.path.join(HERE, "module_boundary.npz")
    np.savez_compressed(path, **out)
    print("wrote", path, os.path.getsize(path), "bytes")


if __name__ == "__main__":
    from oracle.build_ref import REF_ENV, reference_root

    root = reference_root(sys.argv[1] if len(sys.argv) > 1 else None)
    if root is None:
        sys.exit(f"usage: python {sys.argv[0]} REFERENCE_ROOT (or set {REF_ENV})")
    main(root)
