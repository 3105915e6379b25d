"""Feature-map family on CPU: the oracle restatements against the reference's
own outputs (tests/golden/feature_maps_golden.npz, made by
make_feature_golden.py from the reference modules), and this package's
modules against the reference's initialisation (same seed -> same
parameters). No GPU: module forwards run in the GPU tests."""
import os

import numpy as np
import pytest
import torch

from oracle import fakla_oracle as O
from oracle import feature_maps_oracle as F
from tests.golden.make_golden import checksum, gen

GOLD = np.load(os.path.join(os.path.dirname(__file__), "golden", "feature_maps_golden.npz"))
LPM_CASES = [("elu+1", 1), ("relu", 1), ("softplus", 1), ("gelu", 1), ("elu+1", 2), ("softplus", 3)]
TEMP_CASES = ["softplus", "relu", "sigmoid", "abs"]


def rel(a, b):
    return O.rel_l2(a, b)


def params(prefix):
    return {k[len(prefix) + 1:]: GOLD[k] for k in GOLD.files if k.startswith(prefix + "/") and not k.endswith("out")
            and "/out_" not in k}


def mlp_layers(p, key):
    """[(W, b), ...] of the Linear layers of Sequential `key` in a state dict."""
    depth = key.count(".") + 1
    n = sorted({int(k.split(".")[depth]) for k in p if k.startswith(key + ".") and k.endswith(".weight")})
    return [(p[f"{key}.{i}.weight"], p.get(f"{key}.{i}.bias")) for i in n]


# ----------------------------------------------------------------- oracle vs reference outputs
@pytest.mark.parametrize("name,seed,shape", [("rff", 501, (3, 5, 64)), ("orf", 502, (3, 5, 64)),
                                             ("orf_wide", 503, (4, 96))])
def test_fourier_oracle_matches_reference(name, seed, shape):
    p = params(name)
    P = p["W"].shape[1]
    got = F.fourier(gen(shape, seed).numpy(), p["W"], p["b"], np.sqrt(1.0 / P))
    assert rel(got, GOLD[f"{name}/out"]) < 1e-6


@pytest.mark.parametrize("i", range(len(LPM_CASES)))
def test_mlp_oracle_matches_reference_lpm(i):
    act, _ = LPM_CASES[i]
    p = params(f"lpm{i}")
    got = F.mlp(gen((4, 7, 64), 600 + i).numpy() * 3.0, mlp_layers(p, "mlp"), act)
    assert rel(got, GOLD[f"lpm{i}/out"]) < 1e-6


@pytest.mark.parametrize("i", range(len(TEMP_CASES)))
def test_mlp_oracle_matches_reference_temperature(i):
    p = params(f"temp{i}")
    got = F.mlp(gen((3, 5, 32), 800 + i).numpy(), mlp_layers(p, "network"), TEMP_CASES[i])
    assert rel(got, GOLD[f"temp{i}/out"]) < 1e-6


def _mixer_oracle(p, x, ctx, kinds):
    feats = []
    for i, kind in enumerate(kinds):
        if kind == "fourier":
            W, b = p[f"feature_maps.{i}.W"], p[f"feature_maps.{i}.b"]
            feats.append(F.fourier(x, W, b, np.sqrt(1.0 / W.shape[1])))
        else:
            feats.append(F.mlp(x, mlp_layers(p, f"feature_maps.{i}.mlp"), kind))
    gin = x if ctx is None else np.concatenate([x, ctx], axis=-1)
    logits = F.mlp(gin, mlp_layers(p, "gate_net.network"), "identity")
    return F.mix(np.stack(feats), logits)


def test_mixer_oracle_matches_reference():
    p = params("mix")
    x = gen((2, 6, 64), 701).numpy()
    kinds = ["fourier", "elu+1", "fourier"]
    assert rel(_mixer_oracle(p, x, gen((2, 6, 16), 702).numpy(), kinds), GOLD["mix/out_ctx"]) < 1e-6
    c2 = np.broadcast_to(gen((2, 16), 703).numpy()[:, None, :], (2, 6, 16))
    assert rel(_mixer_oracle(p, x, c2, kinds), GOLD["mix/out_ctx2d"]) < 1e-6
    p1 = params("mix1")
    got = _mixer_oracle(p1, gen((5, 64), 704).numpy(), None, ["softplus", "fourier"])
    assert rel(got, GOLD["mix1/out"]) < 1e-6


def _attn_mix_module():
    from pulsartecture_b200.attention import TMLinKernelAttn
    from pulsartecture_b200.kernels import KernelFeatureMixer, LearnablePositiveMap, RandomFourierFeatures

    torch.manual_seed(50)
    mixer = KernelFeatureMixer([LearnablePositiveMap(256, 256), RandomFourierFeatures(256, 256, gamma=0.2)],
                               gate_input_dim=256)
    return TMLinKernelAttn(256, mixer, num_heads=4, qk_dim=64, v_dim=64)


def test_module_with_mixer_oracle_matches_reference():
    """TMLinKernelAttn with a KernelFeatureMixer mapper: projections, mixed
    features, head split and FA-KLA restated on this package's parameters
    (equal to the reference's, checked below) reproduce the reference output."""
    mod = _attn_mix_module()
    sd = {k: v.detach().double().numpy() for k, v in mod.state_dict().items()}
    x = gen((2, 32, 256), 901).numpy()

    def proj(name):
        return x @ sd[f"{name}.linear.weight"].T + sd[f"{name}.linear.bias"]

    p = {k[len("feature_mapper."):]: v for k, v in sd.items() if k.startswith("feature_mapper.")}
    qm = _mixer_oracle(p, proj("proj_q"), None, ["elu+1", "fourier"]).reshape(2, 32, 4, 64)
    km = _mixer_oracle(p, proj("proj_k"), None, ["elu+1", "fourier"]).reshape(2, 32, 4, 64)
    v = proj("proj_v").reshape(2, 32, 4, 64)
    out, _, _ = O.attention(qm, km, v)
    assert rel(out.reshape(2, 32, 256), GOLD["attn_mix/out"]) < 1e-5


# ----------------------------------------------------------------- initialisation = reference's
def _assert_state(prefix, module):
    for k, v in module.state_dict().items():
        np.testing.assert_array_equal(v.detach().numpy().astype(np.float32), GOLD[f"{prefix}/{k}"], err_msg=k)


def test_fourier_maps_reproduce_reference_init():
    from pulsartecture_b200.kernels import OrthogonalRandomFeatures, RandomFourierFeatures

    torch.manual_seed(11)
    _assert_state("rff", RandomFourierFeatures(64, 128, gamma=0.5))
    torch.manual_seed(12)
    _assert_state("orf", OrthogonalRandomFeatures(64, 128, gamma=0.5))
    torch.manual_seed(13)
    _assert_state("orf_wide", OrthogonalRandomFeatures(96, 256, gamma=0.2))


def test_learnable_positive_maps_reproduce_reference_init():
    from pulsartecture_b200.kernels import LearnablePositiveMap

    for i, (act, layers) in enumerate(LPM_CASES):
        torch.manual_seed(20 + i)
        _assert_state(f"lpm{i}", LearnablePositiveMap(64, 96, num_layers=layers, activation=act))


def test_mixers_and_temperature_reproduce_reference_init():
    from pulsartecture_b200.attention import TemperatureFunction
    from pulsartecture_b200.kernels import (KernelFeatureMixer, LearnablePositiveMap, OrthogonalRandomFeatures,
                                            RandomFourierFeatures)

    torch.manual_seed(30)
    maps = [RandomFourierFeatures(64, 128, gamma=0.5), LearnablePositiveMap(64, 128),
            OrthogonalRandomFeatures(64, 128, gamma=0.3)]
    _assert_state("mix", KernelFeatureMixer(maps, gate_input_dim=80, gate_hidden_dim=32, gate_layers=2))
    torch.manual_seed(31)
    _assert_state("mix1", KernelFeatureMixer([LearnablePositiveMap(64, 128, activation="softplus"),
                                              RandomFourierFeatures(64, 128)], gate_input_dim=64))
    for i, act in enumerate(TEMP_CASES):
        torch.manual_seed(40 + i)
        _assert_state(f"temp{i}", TemperatureFunction(32, 4, num_layers=2, final_activation=act))
    mod = _attn_mix_module()
    names = sorted(mod.state_dict())
    assert names == list(GOLD["attn_mix/names"])
    got = np.stack([checksum(mod.state_dict()[k]) for k in names])
    np.testing.assert_allclose(got, GOLD["attn_mix/checksums"], rtol=1e-12)


def test_feature_modules_raise_on_cpu_tensors():
    """No CPU path: a forward on CPU tensors raises instead of computing."""
    from pulsartecture_b200.kernels import RandomFourierFeatures

    m = RandomFourierFeatures(8, 16)
    with pytest.raises(RuntimeError, match="CUDA"):
        m(torch.zeros(2, 8))
