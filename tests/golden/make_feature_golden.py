"""Generate golden fixtures of the feature-map family from the reference.

Run where the reference checkout is present (it is read, never copied):

    python tests/golden/make_feature_golden.py REFERENCE_ROOT     (or set FAKLA_REFERENCE_ROOT)

Imports the reference's own RandomFourierFeatures, OrthogonalRandomFeatures,
LearnablePositiveMap (ultra_rwka/kernels/feature_maps.py), GateNet and
KernelFeatureMixer (ultra_rwka/kernels/mixer.py), TemperatureFunction and
TMLinKernelAttn (ultra_rwka/attention/tm_kla.py) through the loader shim of
make_golden.py, builds each from a fixed torch.manual_seed, and stores its
parameters/buffers (all small) and its float32 output on seeded inputs in
feature_maps_golden.npz. The module case runs the reference's own compiled
fa_kla_attention_cpu. Inputs are regenerated from their seeds by the tests.
"""
from __future__ import annotations

import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, HERE)
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))

from make_golden import checksum, gen, load_reference_modules  # noqa: E402
from oracle import build_ref  # noqa: E402

LPM_CASES = [("elu+1", 1), ("relu", 1), ("softplus", 1), ("gelu", 1), ("elu+1", 2), ("softplus", 3)]
TEMP_CASES = ["softplus", "relu", "sigmoid", "abs"]


def state(prefix, module, out):
    for k, v in module.state_dict().items():
        out[f"{prefix}/{k}"] = v.detach().numpy().astype(np.float32)


def state_checksums(prefix, module, out):
    names = sorted(module.state_dict())
    out[f"{prefix}/names"] = np.array(names)
    out[f"{prefix}/checksums"] = np.stack([checksum(module.state_dict()[k]) for k in names])


def main(ref_root: str) -> None:
    if not build_ref.built_module_path():
        build_ref.build(ref_root)
    ref = build_ref.load()
    fm, mx, tm = load_reference_modules(ref_root, ref)
    out = {}
    with torch.no_grad():
        # random Fourier / orthogonal random features
        torch.manual_seed(11)
        m = fm.RandomFourierFeatures(64, 128, gamma=0.5)
        state("rff", m, out)
        out["rff/out"] = m(gen((3, 5, 64), 501)).numpy()
        torch.manual_seed(12)
        m = fm.OrthogonalRandomFeatures(64, 128, gamma=0.5)
        state("orf", m, out)
        out["orf/out"] = m(gen((3, 5, 64), 502)).numpy()
        torch.manual_seed(13)
        m = fm.OrthogonalRandomFeatures(96, 256, gamma=0.2)  # in_dim < num_projections
        state("orf_wide", m, out)
        out["orf_wide/out"] = m(gen((4, 96), 503)).numpy()

        # LearnablePositiveMap: every final activation, deeper MLPs
        for i, (act, layers) in enumerate(LPM_CASES):
            torch.manual_seed(20 + i)
            m = fm.LearnablePositiveMap(64, 96, num_layers=layers, activation=act)
            state(f"lpm{i}", m, out)
            out[f"lpm{i}/out"] = m(gen((4, 7, 64), 600 + i) * 3.0).numpy()

        # KernelFeatureMixer with a two-layer gate over [x, context], then
        # with a (B, C) context expanded over T, then without context
        torch.manual_seed(30)
        maps = [fm.RandomFourierFeatures(64, 128, gamma=0.5), fm.LearnablePositiveMap(64, 128),
                fm.OrthogonalRandomFeatures(64, 128, gamma=0.3)]
        m = mx.KernelFeatureMixer(maps, gate_input_dim=80, gate_hidden_dim=32, gate_layers=2)
        m.eval()
        state("mix", m, out)
        x = gen((2, 6, 64), 701)
        out["mix/out_ctx"] = m(x, gen((2, 6, 16), 702)).numpy()
        out["mix/out_ctx2d"] = m(x, gen((2, 16), 703)).numpy()
        torch.manual_seed(31)
        m = mx.KernelFeatureMixer([fm.LearnablePositiveMap(64, 128, activation="softplus"),
                                   fm.RandomFourierFeatures(64, 128)], gate_input_dim=64)
        m.eval()
        state("mix1", m, out)
        out["mix1/out"] = m(gen((5, 64), 704)).numpy()

        # TemperatureFunction, every final activation
        for i, act in enumerate(TEMP_CASES):
            torch.manual_seed(40 + i)
            m = tm.TemperatureFunction(32, 4, num_layers=2, final_activation=act)
            state(f"temp{i}", m, out)
            out[f"temp{i}/out"] = m(gen((3, 5, 32), 800 + i)).numpy()

        # TMLinKernelAttn with a KernelFeatureMixer mapper (reference CPU kernel)
        torch.manual_seed(50)
        mixer = mx.KernelFeatureMixer([fm.LearnablePositiveMap(256, 256),
                                       fm.RandomFourierFeatures(256, 256, gamma=0.2)], gate_input_dim=256)
        mod = tm.TMLinKernelAttn(256, mixer, num_heads=4, qk_dim=64, v_dim=64)
        mod.eval()
        state_checksums("attn_mix", mod, out)
        out["attn_mix/out"] = mod(gen((2, 32, 256), 901)).numpy()

    for k in list(out):
        if out[k].dtype.kind != "U":
            out[k] = np.asarray(out[k], dtype=np.float64 if k.endswith("checksums") else np.float32)
            assert np.isfinite(out[k]).all(), k
    path = os.path.join(HERE, "feature_maps_golden.npz")
    np.savez_compressed(path, **out)
    print("wrote", path, os.path.getsize(path), "bytes,", len(out), "arrays")


if __name__ == "__main__":
    from oracle.build_ref import REF_ENV, reference_root

    root = reference_root(sys.argv[1] if len(sys.argv) > 1 else None)
    if root is None:
        sys.exit(f"usage: python {sys.argv[0]} REFERENCE_ROOT (or set {REF_ENV})")
    main(root)
