"""Fused phi + FA-KLA prefill and the module API against the oracle and the
reference's golden outputs (GPU only)."""
import os

import numpy as np
import pytest
import torch

from oracle import fakla_oracle as O
from tests.helpers import BF16_MAX_ABS, BF16_REL_L2, F32_REL_L2, lpm_params, rel_l2, to_np

pytestmark = pytest.mark.gpu
GOLDEN = os.path.join(os.path.dirname(__file__), "golden", "fakla_golden.npz")


def gen(shape, seed):
    g = torch.Generator().manual_seed(seed)
    return torch.randn(*shape, generator=g)


def test_prefill_f32_small_matches_reference_golden(cuda):
    """Config 1: B=2, H=4, T=256, Dk=Dv=M=64, fp32; LearnablePositiveMap(256,256)
    from seed 0; output and final state S, z against the reference."""
    from pulsartecture_b200.attention import fa_kla
    from pulsartecture_b200.kernels import LearnablePositiveMap

    gold = np.load(GOLDEN)
    B, T, H, D = 2, 256, 4, 64
    torch.manual_seed(0)
    m = LearnablePositiveMap(H * D, H * D).to(cuda)
    q, k, v = gen((B, T, H, D), 101), gen((B, T, H, D), 102), gen((B, T, H, D), 103)
    out, (S, z) = fa_kla(q.to(cuda), k.to(cuda), v.to(cuda), phi_weight=m.weight.detach(), phi_bias=m.bias.detach())
    assert rel_l2(to_np(out), gold["small_out"]) < F32_REL_L2
    assert rel_l2(to_np(S), gold["small_S"]) < F32_REL_L2
    assert rel_l2(to_np(z), gold["small_z"]) < F32_REL_L2


def test_module_f32_matches_reference_module_golden(cuda):
    from pulsartecture_b200.attention import TMLinKernelAttn
    from pulsartecture_b200.kernels import LearnablePositiveMap

    gold = np.load(GOLDEN)
    torch.manual_seed(0)
    mapper = LearnablePositiveMap(256, 256)
    mod = TMLinKernelAttn(256, mapper, num_heads=4, qk_dim=64, v_dim=64)
    assert sorted(mod.state_dict().keys()) == list(gold["module_state_names"])
    mod = mod.to(cuda)
    x = gen((2, 64, 256), 401).to(cuda)
    with torch.no_grad():
        y = mod(x)
    assert y.shape == (2, 64, 256)
    assert rel_l2(to_np(y), gold["module_out"]) < F32_REL_L2


@pytest.mark.parametrize("B,T,H,in_heads,with_temp", [
    (2, 256, 4, 4, False),
    (1, 200, 2, 4, True),
    (2, 1024, 16, 16, False),
])
def test_prefill_bf16_fused(cuda, B, T, H, in_heads, with_temp):
    from pulsartecture_b200.attention import fa_kla

    D = 128
    in_dim = in_heads * D
    q = (gen((B, T, in_heads, D), 70) / np.sqrt(D)).bfloat16().to(cuda)
    k = (gen((B, T, in_heads, D), 71) / np.sqrt(D)).bfloat16().to(cuda)
    v = (gen((B, T, H, D), 72) / np.sqrt(D)).bfloat16().to(cuda)
    W, b = lpm_params(in_dim, H * D, seed=73, dtype=torch.bfloat16)
    tp = None
    if with_temp:
        g = torch.Generator().manual_seed(74)
        tp = (torch.rand(B, T, H, generator=g) + 0.5).bfloat16().to(cuda)
    out, (S, z) = fa_kla(q, k, v, phi_weight=W.to(cuda), phi_bias=b.to(cuda), temp=tp)
    eo, eS, ez = O.prefill(to_np(q), to_np(k), to_np(v), to_np(W), to_np(b), None if tp is None else to_np(tp))
    assert rel_l2(to_np(out), eo) < BF16_REL_L2
    assert np.abs(to_np(out) - eo).max() < BF16_MAX_ABS
    assert rel_l2(to_np(S), eS) < BF16_REL_L2
    assert rel_l2(to_np(z), ez) < BF16_REL_L2


def test_prefill_state_handoff_is_exact(cuda):
    """prefill(T1) then prefill(T2, state) equals prefill(T1+T2) bit for bit when
    T1 is a multiple of the 128-token chunk (same arithmetic, state in fp32)."""
    from pulsartecture_b200.attention import fa_kla

    B, T, H, D = 2, 512, 4, 128
    q = (gen((B, T, H, D), 80) / np.sqrt(D)).bfloat16().to(cuda)
    k = (gen((B, T, H, D), 81) / np.sqrt(D)).bfloat16().to(cuda)
    v = (gen((B, T, H, D), 82) / np.sqrt(D)).bfloat16().to(cuda)
    W, b = lpm_params(H * D, H * D, seed=83, dtype=torch.bfloat16)
    W, b = W.to(cuda), b.to(cuda)
    full, (S, z) = fa_kla(q, k, v, phi_weight=W, phi_bias=b)
    o1, st1 = fa_kla(q[:, :256], k[:, :256], v[:, :256], phi_weight=W, phi_bias=b)
    o2, (S2, z2) = fa_kla(q[:, 256:], k[:, 256:], v[:, 256:], st1, phi_weight=W, phi_bias=b)
    assert torch.equal(torch.cat([o1, o2], 1), full)
    assert torch.equal(S2, S) and torch.equal(z2, z)


def test_prefill_bf16_b8h16t4096_full_size(cuda):
    """Config 2 at full size (B=8, H=16, T=4096, D=M=128, bf16): oracle on three
    (b, h) sequences, size-independent checks on all of them."""
    from pulsartecture_b200.attention import fa_kla
    from pulsartecture_b200.backend.interface import phi_map

    B, T, H, D = 8, 4096, 16, 128
    g = torch.Generator(device=cuda).manual_seed(90)
    q = (torch.randn(B, T, H, D, generator=g, device=cuda) / np.sqrt(D)).bfloat16()
    k = (torch.randn(B, T, H, D, generator=g, device=cuda) / np.sqrt(D)).bfloat16()
    v = (torch.randn(B, T, H, D, generator=g, device=cuda) / np.sqrt(D)).bfloat16()
    W, b = lpm_params(H * D, H * D, seed=0, dtype=torch.bfloat16)
    W, b = W.to(cuda), b.to(cuda)
    out, (S, z) = fa_kla(q, k, v, phi_weight=W, phi_bias=b)
    assert torch.isfinite(out).all() and torch.isfinite(S).all()
    # z is the column sum of phi(k) over the whole sequence
    pk = phi_map(k.reshape(B, T, H * D), W, b).float().reshape(B, T, H, D)
    assert rel_l2(to_np(z), to_np(pk.sum(1))) < 1e-5
    for bb, hh in [(0, 0), (3, 7), (7, 15)]:
        Wh, bh = to_np(W)[hh * D:(hh + 1) * D], to_np(b)[hh * D:(hh + 1) * D]
        pq = O.phi(to_np(q[bb]).reshape(T, H * D), Wh, bh)
        pkk = O.phi(to_np(k[bb]).reshape(T, H * D), Wh, bh)
        eo, eS, ez = O.attention(pq[None, :, None], pkk[None, :, None], to_np(v[bb, :, hh])[None, :, None])
        got = to_np(out[bb, :, hh])
        assert rel_l2(got, eo[0, :, 0]) < BF16_REL_L2
        assert np.abs(got - eo[0, :, 0]).max() < BF16_MAX_ABS
        assert rel_l2(to_np(S[bb, hh]), eS[0, 0]) < BF16_REL_L2


def test_module_bf16_fused_path(cuda):
    from pulsartecture_b200.attention import TMLinKernelAttn
    from pulsartecture_b200.kernels import LearnablePositiveMap

    torch.manual_seed(1)
    E, H, D = 512, 4, 128
    mapper = LearnablePositiveMap(H * D, H * D, dtype=torch.bfloat16)
    mod = TMLinKernelAttn(E, mapper, num_heads=H, qk_dim=D, v_dim=D, temp_input_dim=32,
                          dtype=torch.bfloat16).to(cuda)
    x = (gen((2, 300, E), 95)).bfloat16().to(cuda)
    ti = gen((2, 300, 32), 96).bfloat16().to(cuda)
    with torch.no_grad():
        y, (S, z) = mod(x, temp_input=ti, return_state=True)
        qp, kp, vp = mod.proj_q(x), mod.proj_k(x), mod.proj_v(x)
        temp = mod.temp_func(ti).bfloat16()
    eo, eS, ez = O.prefill(to_np(qp), to_np(kp), to_np(vp).reshape(2, 300, H, D), to_np(mapper.weight),
                           to_np(mapper.bias), to_np(temp))
    assert rel_l2(to_np(y).reshape(2, 300, H, D), eo) < BF16_REL_L2
    # decode continues from the returned state like more prefill would
    xs = gen((2, E), 97).bfloat16().to(cuda)
    ts = gen((2, 32), 98).bfloat16().to(cuda)
    with torch.no_grad():
        ys = mod.step(xs, (S, z), temp_input=ts)
        y2 = mod(torch.cat([x, xs[:, None]], 1), temp_input=torch.cat([ti, ts[:, None]], 1))
    assert rel_l2(to_np(ys), to_np(y2[:, -1])) < BF16_REL_L2


def test_native_library_is_loaded(cuda):
    from pulsartecture_b200 import _lib

    _lib.lib()
    maps = open("/proc/self/maps").read()
    assert "libfakla.so" in maps


@pytest.mark.parametrize("micro_batch", [1, 2, None])
def test_prefill_host_streaming_matches_device_and_oracle(cuda, micro_batch):
    """fa_kla_host: host q/k/v/temp in, host out, copies overlapped with compute
    over groups of sequences (the last group ragged; None: the default size,
    here one sequence, half of the batch rounded down); same results as the
    device call and the oracle, initial state carried per sequence."""
    from pulsartecture_b200.attention import fa_kla, fa_kla_host

    B, T, H, D = 3, 300, 2, 128
    q = (gen((B, T, H, D), 120) / np.sqrt(D)).bfloat16()
    k = (gen((B, T, H, D), 121) / np.sqrt(D)).bfloat16()
    v = (gen((B, T, H, D), 122) / np.sqrt(D)).bfloat16()
    g = torch.Generator().manual_seed(123)
    tp = (torch.rand(B, T, H, generator=g) + 0.5).bfloat16()
    W, b = lpm_params(H * D, H * D, seed=124, dtype=torch.bfloat16)
    W, b = W.to(cuda), b.to(cuda)
    S0 = (gen((B, H, D, D), 125) * 0.02 + 0.05).to(cuda)
    z0 = (torch.rand(B, H, D, generator=g) * 20 + 10).to(cuda)
    hq, hk, hv, ht = q.pin_memory(), k.pin_memory(), v.pin_memory(), tp.pin_memory()
    out_h, (S_h, z_h) = fa_kla_host(hq, hk, hv, (S0, z0), phi_weight=W, phi_bias=b, temp=ht,
                                    micro_batch=micro_batch)
    torch.cuda.synchronize()
    assert out_h.device.type == "cpu" and S_h.is_cuda
    out_d, (S_d, z_d) = fa_kla(q.to(cuda), k.to(cuda), v.to(cuda), (S0, z0), phi_weight=W, phi_bias=b,
                               temp=tp.to(cuda))
    assert rel_l2(to_np(out_h), to_np(out_d)) < 2e-3
    assert rel_l2(to_np(S_h), to_np(S_d)) < 1e-5
    assert rel_l2(to_np(z_h), to_np(z_d)) < 1e-6
    eo, eS, ez = O.prefill(to_np(q), to_np(k), to_np(v), to_np(W), to_np(b), to_np(tp), to_np(S0), to_np(z0))
    assert rel_l2(to_np(out_h), eo) < BF16_REL_L2
    assert np.abs(to_np(out_h) - eo).max() < BF16_MAX_ABS
    assert rel_l2(to_np(S_h), eS) < BF16_REL_L2


def test_prefill_host_back_to_back_unordered_calls(cuda):
    """Consecutive fa_kla_host calls with ordered=False share the kept device
    slots: each call's input copies wait only for the slot they refill. Four
    calls on different inputs, queued without a synchronisation, each equal
    the device call on their own inputs."""
    from pulsartecture_b200.attention import fa_kla, fa_kla_host
    from pulsartecture_b200.backend.interface import release_host_pipelines

    B, T, H, D = 5, 260, 2, 128
    W, b = lpm_params(H * D, H * D, seed=130, dtype=torch.bfloat16)
    W, b = W.to(cuda), b.to(cuda)
    ins, outs = [], []
    for c in range(4):
        q = (gen((B, T, H, D), 131 + 3 * c) / np.sqrt(D)).bfloat16().pin_memory()
        k = (gen((B, T, H, D), 132 + 3 * c) / np.sqrt(D)).bfloat16().pin_memory()
        v = (gen((B, T, H, D), 133 + 3 * c) / np.sqrt(D)).bfloat16().pin_memory()
        ins.append((q, k, v))
    for q, k, v in ins:
        o, _ = fa_kla_host(q, k, v, phi_weight=W, phi_bias=b, micro_batch=2, ordered=False)
        outs.append(o)
    torch.cuda.synchronize()
    for (q, k, v), o in zip(ins, outs):
        ref, _ = fa_kla(q.to(cuda), k.to(cuda), v.to(cuda), phi_weight=W, phi_bias=b)
        assert rel_l2(to_np(o), to_np(ref)) < 2e-3
    release_host_pipelines()


def test_prefill_host_rejects_device_inputs(cuda):
    from pulsartecture_b200.attention import fa_kla_host

    W, b = lpm_params(256, 256, seed=1, dtype=torch.bfloat16)
    x = torch.zeros(1, 4, 256, dtype=torch.bfloat16)
    with pytest.raises(RuntimeError, match="host"):
        fa_kla_host(x.to(cuda), x, torch.zeros(1, 4, 2, 128, dtype=torch.bfloat16), phi_weight=W.to(cuda))
    with pytest.raises(RuntimeError, match="CUDA"):
        fa_kla_host(x, x, torch.zeros(1, 4, 2, 128, dtype=torch.bfloat16), phi_weight=W)


@pytest.mark.parametrize("T,with_temp,H,D", [(300, True, 4, 128), (1024, False, 4, 128),
                                               (300, True, 8, 64), (777, False, 16, 64),
                                               (500, True, 3, 128), (3000, False, 3, 128),
                                               (4096, True, 4, 128)])
def test_module_qkv_folded_into_phi(cuda, T, with_temp, H, D):
    """Inference through fakla_qkv_prefill (projections folded into the feature
    map, one GEMM for [phi(q) | phi(k) temp | v]): equal to the projections,
    map and attention of the reference restated in float64 on the same bf16
    parameters, within the bf16 bars; the returned state too. Heads of 128 and
    of 64; 3 heads of 128 give a [q|k|v] width of 1152, an odd multiple of 128
    (128-wide GEMM tiles), at 6 and at 47 row tiles; 2 x 4096 tokens of 4 heads
    of 128 run the GEMM as CTA pairs (192 tiles of 256 x 256)."""
    from pulsartecture_b200.attention import TMLinKernelAttn
    from pulsartecture_b200.kernels import LearnablePositiveMap

    torch.manual_seed(7)
    E = 512 if H * D == 512 else H * D
    mapper = LearnablePositiveMap(H * D, H * D, dtype=torch.bfloat16)
    mod = TMLinKernelAttn(E, mapper, num_heads=H, qk_dim=D, v_dim=D, temp_input_dim=16 if with_temp else 0,
                          dtype=torch.bfloat16).to(cuda).eval()
    x = (gen((2, T, E), 140) * 0.5).bfloat16().to(cuda)
    ti = gen((2, T, 16), 141).bfloat16().to(cuda) if with_temp else None
    with torch.no_grad():
        assert mod._qkv_foldable(x)
        y, (S, z) = mod(x, temp_input=ti, return_state=True)
        temp = mod.temp_func(ti) if with_temp else None
    sd = {k: to_np(v).astype(np.float64) for k, v in mod.state_dict().items()}
    xd = to_np(x).astype(np.float64)

    def lin(name):
        return xd @ sd[f"{name}.linear.weight"].T + sd[f"{name}.linear.bias"]

    eo, eS, ez = O.prefill(lin("proj_q"), lin("proj_k"), lin("proj_v").reshape(2, T, H, D),
                           sd["feature_mapper.mlp.0.weight"], sd["feature_mapper.mlp.0.bias"],
                           None if temp is None else to_np(temp))
    got = to_np(y).reshape(2, T, H, D)
    assert rel_l2(got, eo) < BF16_REL_L2
    assert np.abs(got - eo).max() < BF16_MAX_ABS
    assert rel_l2(to_np(S), eS) < BF16_REL_L2
    assert rel_l2(to_np(z), ez) < BF16_REL_L2


def test_module_qkv_fold_only_where_supported(cuda):
    """The fold needs bf16 and heads of 64 or 128; other modules keep the
    unfused path, and training keeps the autograd path."""
    from pulsartecture_b200.attention import TMLinKernelAttn
    from pulsartecture_b200.kernels import LearnablePositiveMap

    x = torch.zeros(1, 8, 384, dtype=torch.bfloat16, device=cuda)
    mod = TMLinKernelAttn(384, LearnablePositiveMap(288, 288, dtype=torch.bfloat16), num_heads=3, qk_dim=96,
                          v_dim=96, dtype=torch.bfloat16).to(cuda).eval()
    assert not mod._qkv_foldable(x)  # heads of 96
    with torch.no_grad():
        assert mod(x).shape == (1, 8, 288)
    mod4 = TMLinKernelAttn(512, LearnablePositiveMap(512, 512, dtype=torch.bfloat16), num_heads=4, qk_dim=128,
                           v_dim=128, dtype=torch.bfloat16).to(cuda)
    x4 = torch.zeros(1, 8, 512, dtype=torch.bfloat16, device=cuda)
    assert not mod4._qkv_foldable(x4)  # grad enabled with trainable parameters
    with torch.no_grad():
        assert mod4._qkv_foldable(x4)
