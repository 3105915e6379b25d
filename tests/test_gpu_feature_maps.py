"""Feature-map family on the GPU (fakla_feature_map, fakla_mix_features and
the module classes) against the oracle and the reference's golden outputs.

Bars: fp32 -> rel-L2 <= 1e-5 against the reference's outputs; bf16 (inputs
rounded to bf16 first, fp32 accumulation, one rounding of the output) ->
|err| <= 2^-8 |exact| + atol per element against the float64 oracle.
"""
import os

import numpy as np
import pytest
import torch

from oracle import feature_maps_oracle as F
from tests.golden.make_golden import gen
from tests.helpers import F32_REL_L2, rel_l2, to_np

pytestmark = pytest.mark.gpu
GOLD = np.load(os.path.join(os.path.dirname(__file__), "golden", "feature_maps_golden.npz"))
LPM_CASES = [("elu+1", 1), ("relu", 1), ("softplus", 1), ("gelu", 1), ("elu+1", 2), ("softplus", 3)]
TEMP_CASES = ["softplus", "relu", "sigmoid", "abs"]
ACTS = ["elu+1", "relu", "softplus", "gelu", "identity", "sigmoid", "abs"]


def _bf16_close(got, exp, atol=2e-3):
    got = np.asarray(got, np.float64)
    assert np.all(np.abs(got - exp) <= 2.0 ** -8 * np.abs(exp) + atol), float(np.abs(got - exp).max())


def _inputs(rows, K, N, seed, dtype, dev, xscale=1.0):
    g = torch.Generator().manual_seed(seed)
    x = (torch.randn(rows, K, generator=g) * xscale).to(dtype)
    W = (torch.randn(N, K, generator=g) / np.sqrt(K)).to(dtype)
    b = (torch.randn(N, generator=g) * 0.5).to(dtype)
    return x.to(dev), W.to(dev), b.to(dev)


# ----------------------------------------------------------------- fakla_feature_map
@pytest.mark.parametrize("act", ACTS)
@pytest.mark.parametrize("rows,K,N,dtype", [
    (1000, 256, 512, torch.bfloat16),    # tensor-core tiles (128 wide: 16 tiles of 256 would idle SMs)
    (4000, 128, 1024, torch.bfloat16),   # tensor-core tiles 256 wide
    (600, 192, 384, torch.bfloat16),     # tensor-core tiles, N an odd multiple of 128
    (20000, 128, 1024, torch.bfloat16),  # CTA-pair 256x256 tiles (316 of them)
    (19999, 192, 512, torch.bfloat16),   # CTA-pair tiles, last one ragged (rank 1 partly past the end)
    (5000, 2048, 3, torch.bfloat16),     # narrow output (a gate): one warp per row
    (333, 40, 16, torch.float32),        # narrow output, fp32, K smaller than a warp's 256-wide step
    (64, 36, 5, torch.bfloat16),         # narrow output with K % 8 != 0: the tiled CUDA-core path
    (77, 96, 40, torch.bfloat16),        # CUDA-core shape
    (300, 200, 96, torch.float32),       # fp32
])
def test_feature_map_activations(cuda, act, rows, K, N, dtype):
    from pulsartecture_b200.backend.interface import feature_map

    x, W, b = _inputs(rows, K, N, 11, dtype, cuda, xscale=3.0)
    got = feature_map(x, W, b, act)
    exp = F.linear_act(to_np(x), to_np(W), to_np(b), act)
    if dtype == torch.float32:
        assert rel_l2(to_np(got), exp) < 1e-6
    else:
        _bf16_close(to_np(got), exp)


@pytest.mark.parametrize("rows,K,P,dtype", [
    (1000, 256, 256, torch.bfloat16),    # tensor cores, cos/sin epilogue
    (19001, 128, 512, torch.bfloat16),   # CTA-pair tiles, cos/sin epilogue
    (50, 64, 40, torch.bfloat16),
    (300, 200, 96, torch.float32),
])
def test_feature_map_cos_sin(cuda, rows, K, P, dtype):
    from pulsartecture_b200.backend.interface import feature_map

    x, W, b = _inputs(rows, K, P, 12, dtype, cuda)
    b = (b.float() + 3.0).to(dtype)  # phases spread over (0, 2 pi) like the reference's U(0, 2 pi)
    scale = float(np.sqrt(1.0 / P))
    got = feature_map(x, W, b, "cossin", scale)
    assert tuple(got.shape) == (rows, 2 * P)
    exp = F.fourier(to_np(x), to_np(W).T, to_np(b), scale)
    if dtype == torch.float32:
        assert rel_l2(to_np(got), exp) < 1e-6
    else:
        _bf16_close(to_np(got), exp, atol=1e-3)


# ----------------------------------------------------------------- fakla_mix_features
@pytest.mark.parametrize("n,rows,Fdim,dtype", [(3, 500, 128, torch.bfloat16), (2, 37, 33, torch.float32),
                                               (5, 64, 256, torch.float32),
                                               (6, 300, 64, torch.bfloat16),   # bf16, 5-8 maps: 8 features a thread
                                               (4, 100, 24, torch.bfloat16),   # bf16, F % 16 != 0
                                               (12, 40, 32, torch.bfloat16)])  # bf16, more than 8 maps
def test_mix_features(cuda, n, rows, Fdim, dtype):
    from pulsartecture_b200.backend.interface import mix_features

    g = torch.Generator().manual_seed(13)
    feats = torch.randn(n, rows, Fdim, generator=g).to(dtype).to(cuda)
    logits = (torch.randn(rows, n, generator=g) * 2).to(dtype).to(cuda)
    got = mix_features(feats, logits)
    if dtype == torch.float32:
        exp = F.mix(to_np(feats), to_np(logits))
        assert rel_l2(to_np(got), exp) < 1e-6
    else:
        rnd = lambda w: torch.from_numpy(w).float().bfloat16().float().numpy()  # noqa: E731
        _bf16_close(to_np(got), F.mix(to_np(feats), to_np(logits), rnd), atol=1e-2)


def test_mix_features_rejects_too_many_maps(cuda):
    from pulsartecture_b200.backend.interface import mix_features

    with pytest.raises(RuntimeError, match="at most 32"):
        mix_features(torch.zeros(33, 4, 8, device=cuda), torch.zeros(4, 33, device=cuda))


# ----------------------------------------------------------------- modules vs the reference (fp32)
def test_fourier_modules_match_reference(cuda):
    from pulsartecture_b200.kernels import OrthogonalRandomFeatures, RandomFourierFeatures

    torch.manual_seed(11)
    m = RandomFourierFeatures(64, 128, gamma=0.5).to(cuda)
    assert rel_l2(to_np(m(gen((3, 5, 64), 501).to(cuda))), GOLD["rff/out"]) < F32_REL_L2
    torch.manual_seed(12)
    m = OrthogonalRandomFeatures(64, 128, gamma=0.5).to(cuda)
    assert rel_l2(to_np(m(gen((3, 5, 64), 502).to(cuda))), GOLD["orf/out"]) < F32_REL_L2
    torch.manual_seed(13)
    m = OrthogonalRandomFeatures(96, 256, gamma=0.2).to(cuda)
    assert rel_l2(to_np(m(gen((4, 96), 503).to(cuda))), GOLD["orf_wide/out"]) < F32_REL_L2


@pytest.mark.parametrize("i", range(len(LPM_CASES)))
def test_learnable_positive_map_matches_reference(cuda, i):
    from pulsartecture_b200.kernels import LearnablePositiveMap

    act, layers = LPM_CASES[i]
    torch.manual_seed(20 + i)
    m = LearnablePositiveMap(64, 96, num_layers=layers, activation=act).to(cuda)
    got = m(gen((4, 7, 64), 600 + i).to(cuda) * 3.0)
    assert rel_l2(to_np(got), GOLD[f"lpm{i}/out"]) < F32_REL_L2


def test_mixer_matches_reference(cuda):
    from pulsartecture_b200.kernels import (KernelFeatureMixer, LearnablePositiveMap, OrthogonalRandomFeatures,
                                            RandomFourierFeatures)

    torch.manual_seed(30)
    maps = [RandomFourierFeatures(64, 128, gamma=0.5), LearnablePositiveMap(64, 128),
            OrthogonalRandomFeatures(64, 128, gamma=0.3)]
    m = KernelFeatureMixer(maps, gate_input_dim=80, gate_hidden_dim=32, gate_layers=2).to(cuda).eval()
    x = gen((2, 6, 64), 701).to(cuda)
    assert rel_l2(to_np(m(x, gen((2, 6, 16), 702).to(cuda))), GOLD["mix/out_ctx"]) < F32_REL_L2
    assert rel_l2(to_np(m(x, gen((2, 16), 703).to(cuda))), GOLD["mix/out_ctx2d"]) < F32_REL_L2
    torch.manual_seed(31)
    m = KernelFeatureMixer([LearnablePositiveMap(64, 128, activation="softplus"), RandomFourierFeatures(64, 128)],
                           gate_input_dim=64).to(cuda).eval()
    assert rel_l2(to_np(m(gen((5, 64), 704).to(cuda))), GOLD["mix1/out"]) < F32_REL_L2


@pytest.mark.parametrize("i", range(len(TEMP_CASES)))
def test_temperature_function_matches_reference(cuda, i):
    from pulsartecture_b200.attention import TemperatureFunction

    torch.manual_seed(40 + i)
    m = TemperatureFunction(32, 4, num_layers=2, final_activation=TEMP_CASES[i]).to(cuda)
    assert rel_l2(to_np(m(gen((3, 5, 32), 800 + i).to(cuda))), GOLD[f"temp{i}/out"]) < F32_REL_L2


def test_attention_module_with_mixer_matches_reference(cuda):
    from pulsartecture_b200.attention import TMLinKernelAttn
    from pulsartecture_b200.kernels import KernelFeatureMixer, LearnablePositiveMap, RandomFourierFeatures

    torch.manual_seed(50)
    mixer = KernelFeatureMixer([LearnablePositiveMap(256, 256), RandomFourierFeatures(256, 256, gamma=0.2)],
                               gate_input_dim=256)
    mod = TMLinKernelAttn(256, mixer, num_heads=4, qk_dim=64, v_dim=64).to(cuda).eval()
    with torch.no_grad():
        y = mod(gen((2, 32, 256), 901).to(cuda))
    assert rel_l2(to_np(y), GOLD["attn_mix/out"]) < F32_REL_L2


def test_mixer_bf16_tensor_core_shapes(cuda):
    """bf16 mixer at FA-KLA sizes (in 2048 -> 2048 features: the maps run on the
    tcgen05 GEMM) against the oracle on the same bf16 parameters."""
    from pulsartecture_b200.kernels import KernelFeatureMixer, LearnablePositiveMap, RandomFourierFeatures

    torch.manual_seed(60)
    maps = [LearnablePositiveMap(2048, 2048), RandomFourierFeatures(2048, 2048, gamma=0.02)]
    m = KernelFeatureMixer(maps, gate_input_dim=2048).to(cuda).to(torch.bfloat16).eval()
    x = (gen((512, 2048), 61) / np.sqrt(128)).bfloat16().to(cuda)
    got = m(x)
    sd = {k: to_np(v) for k, v in m.state_dict().items()}
    xs = to_np(x)
    f0 = F.linear_act(xs, sd["feature_maps.0.mlp.0.weight"], sd["feature_maps.0.mlp.0.bias"], "elu+1")
    f1 = F.fourier(xs, sd["feature_maps.1.W"], sd["feature_maps.1.b"], np.sqrt(1.0 / 1024))
    rb = lambda a: torch.from_numpy(np.asarray(a)).float().bfloat16().double().numpy()  # noqa: E731
    logits = rb(F.linear_act(xs, sd["gate_net.network.0.weight"], sd["gate_net.network.0.bias"], "identity"))
    exp = F.mix(np.stack([rb(f0), rb(f1)]), logits, rb)
    _bf16_close(to_np(got), exp, atol=5e-3)
