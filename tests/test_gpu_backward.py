"""Gradients of FA-KLA on the GPU (fakla_attention_backward, fakla_phi_backward
and the autograd path) against the float64 autograd oracle
(oracle/fakla_grad_oracle.py, pinned by finite differences on CPU).

Bars: fp32 -> rel-L2 <= 2e-5 per gradient; bf16 inputs (gradients rounded to
bf16, fp32 accumulation) -> rel-L2 <= 5e-3.
"""
import numpy as np
import pytest
import torch

from oracle import fakla_grad_oracle as G
from tests.helpers import BF16_REL_L2, lpm_params, rel_l2, to_np

pytestmark = pytest.mark.gpu
F32_GRAD = 2e-5


def _inputs(B, T, H, Df, Dv, dtype, dev, seed, temp=True, state=True):
    g = torch.Generator().manual_seed(seed)
    q = (torch.rand(B, T, H, Df, generator=g) + 0.5).to(dtype)
    k = (torch.rand(B, T, H, Df, generator=g) + 0.5).to(dtype)
    v = (torch.randn(B, T, H, Dv, generator=g) / np.sqrt(Dv)).to(dtype)
    tp = (torch.rand(B, T, H, generator=g) + 0.5).to(dtype) if temp else None
    S0 = (torch.randn(B, H, Df, Dv, generator=g) * 0.02 + 0.05) if state else None
    z0 = (torch.rand(B, H, Df, generator=g) * 20 + 10) if state else None
    ts = [q, k, v, tp, S0, z0]
    return [None if t is None else t.to(dev).requires_grad_() for t in ts]


def _loss_weights(B, T, H, Df, Dv, seed):
    g = torch.Generator().manual_seed(seed)
    return (torch.randn(B, T, H, Dv, generator=g, dtype=torch.float64),
            torch.randn(B, H, Df, Dv, generator=g, dtype=torch.float64) * 0.01,
            torch.randn(B, H, Df, generator=g, dtype=torch.float64) * 0.01)


def _oracle_grads(args, weights, use_final):
    xs = [None if t is None else t.detach().double().cpu().requires_grad_() for t in args]
    out, S, z = G.attention(*xs)
    Ro, RS, Rz = weights
    loss = (out * Ro).sum()
    if use_final:
        loss = loss + (S * RS).sum() + (z * Rz).sum()
    loss.backward()
    return [None if t is None else t.grad.numpy() for t in xs]


@pytest.mark.parametrize("B,T,H,Df,Dv,temp,state,final", [
    (2, 64, 3, 16, 24, True, True, True),
    (1, 300, 2, 128, 128, True, False, False),
    (2, 37, 2, 7, 200, False, True, True),
    (1, 50, 1, 256, 64, True, True, False),
    (1, 1, 2, 32, 32, True, True, True),
])
def test_attention_backward_fp32(cuda, B, T, H, Df, Dv, temp, state, final):
    from pulsartecture_b200.backend.interface import fa_kla_attention_with_state

    args = _inputs(B, T, H, Df, Dv, torch.float32, cuda, 10 + T, temp, state)
    weights = _loss_weights(B, T, H, Df, Dv, 20 + T)
    q, k, v, tp, S0, z0 = args
    out, (S, z) = fa_kla_attention_with_state(q, k, v, tp, None if S0 is None else (S0, z0), True)
    Ro, RS, Rz = [w.float().to(cuda) for w in weights]
    loss = (out * Ro).sum()
    if final:
        loss = loss + (S * RS).sum() + (z * Rz).sum()
    loss.backward()
    exp = _oracle_grads(args, weights, final)
    for name, t, e in zip(["q", "k", "v", "temp", "S0", "z0"], args, exp):
        if t is None:
            continue
        assert rel_l2(to_np(t.grad), e) < F32_GRAD, name


def test_attention_backward_bf16(cuda):
    from pulsartecture_b200.backend.interface import fa_kla_attention_with_state

    B, T, H, D = 1, 256, 2, 128
    args = _inputs(B, T, H, D, D, torch.bfloat16, cuda, 7, True, False)
    weights = _loss_weights(B, T, H, D, D, 8)
    q, k, v, tp, _, _ = args
    out, _ = fa_kla_attention_with_state(q, k, v, tp, None, True)
    (out.float() * weights[0].float().to(cuda)).sum().backward()
    exp = _oracle_grads(args, weights, False)
    for name, t, e in zip(["q", "k", "v", "temp"], args[:4], exp[:4]):
        assert t.grad.dtype == torch.bfloat16
        assert rel_l2(to_np(t.grad), e) < BF16_REL_L2, name


@pytest.mark.parametrize("D", [128, 64])
@pytest.mark.parametrize("B,T,H,temp,state,final", [
    (1, 300, 3, True, True, True),     # ragged last chunk, every gradient
    (2, 129, 2, False, True, False),   # one token past a chunk, no temperature
    (1, 1, 2, True, True, True),       # a single token
    (1, 700, 2, True, False, True),    # six chunks, final-state gradients only
    (1, 128, 1, False, False, False),  # exactly one chunk
])
def test_attention_backward_bf16_chunked(cuda, B, T, H, temp, state, final, D):
    """bf16 heads of 128 and 64 take the tensor-core backward (chunked
    scans): every gradient, including those of the initial state, against
    the float64 oracle."""
    from pulsartecture_b200.backend.interface import fa_kla_attention_with_state

    args = _inputs(B, T, H, D, D, torch.bfloat16, cuda, 50 + T, temp, state)
    weights = _loss_weights(B, T, H, D, D, 60 + T)
    q, k, v, tp, S0, z0 = args
    out, (S, z) = fa_kla_attention_with_state(q, k, v, tp, None if S0 is None else (S0, z0), True)
    Ro, RS, Rz = [w.float().to(cuda) for w in weights]
    loss = (out.float() * Ro).sum()
    if final:
        loss = loss + (S * RS).sum() + (z * Rz).sum()
    loss.backward()
    exp = _oracle_grads(args, weights, final)
    for name, t, e in zip(["q", "k", "v", "temp", "S0", "z0"], args, exp):
        if t is None:
            continue
        assert rel_l2(to_np(t.grad), e) < BF16_REL_L2, name


def test_phi_backward_kernel(cuda):
    from pulsartecture_b200 import _lib

    g = torch.Generator().manual_seed(3)
    pre = torch.randn(1000, 77, generator=g).to(cuda)
    phi = torch.nn.functional.elu(pre) + 1
    dphi = torch.randn(1000, 77, generator=g).to(cuda)
    dpre = torch.empty_like(phi)
    L = _lib.lib()
    _lib.check(L.fakla_phi_backward(phi.data_ptr(), dphi.data_ptr(), dpre.data_ptr(), phi.numel(),
                                    _lib.FAKLA_F32, torch.cuda.current_stream().cuda_stream))
    exp = dphi * torch.where(pre > 0, torch.ones_like(pre), torch.exp(pre))
    assert rel_l2(to_np(dpre), to_np(exp)) < 1e-6


def test_prefill_autograd_fp32(cuda):
    """fa_kla (phi fused with the scan) under autograd: gradients of q, k, v,
    the map's W and b, and temp against the oracle's autograd."""
    from pulsartecture_b200.attention import fa_kla

    B, T, H, Dk = 2, 96, 2, 32
    g = torch.Generator().manual_seed(30)
    q = (torch.randn(B, T, H * Dk, generator=g) * 0.5).to(cuda).requires_grad_()
    k = (torch.randn(B, T, H * Dk, generator=g) * 0.5).to(cuda).requires_grad_()
    v = torch.randn(B, T, H, Dk, generator=g).to(cuda).requires_grad_()
    W, b = lpm_params(H * Dk, H * Dk, seed=31)
    W, b = W.to(cuda).requires_grad_(), b.to(cuda).requires_grad_()
    tp = (torch.rand(B, T, H, generator=g) + 0.5).to(cuda).requires_grad_()
    R = torch.randn(B, T, H, Dk, generator=g, dtype=torch.float64)
    out, _ = fa_kla(q, k, v, phi_weight=W, phi_bias=b, temp=tp)
    (out * R.float().to(cuda)).sum().backward()
    xs = [t.detach().double().cpu().requires_grad_() for t in (q, k, v, W, b, tp)]
    eo, _, _ = G.prefill(xs[0], xs[1], xs[2], xs[3], xs[4], xs[5])
    (eo * R).sum().backward()
    for name, t, e in zip(["q", "k", "v", "W", "b", "temp"], (q, k, v, W, b, tp), xs):
        assert rel_l2(to_np(t.grad), e.grad.numpy()) < F32_GRAD, name


def test_module_training_step_fp32(cuda):
    """One training step of TMLinKernelAttn (fp32): parameter gradients equal
    those of the same module restated in float64 torch."""
    from pulsartecture_b200.attention import TMLinKernelAttn
    from pulsartecture_b200.kernels import LearnablePositiveMap

    torch.manual_seed(5)
    E, H, D = 128, 4, 32
    mod = TMLinKernelAttn(E, LearnablePositiveMap(H * D, H * D), num_heads=H, qk_dim=D, v_dim=D,
                          temp_input_dim=16).to(cuda)
    g = torch.Generator().manual_seed(6)
    x = torch.randn(2, 50, E, generator=g).to(cuda)
    ti = torch.randn(2, 50, 16, generator=g).to(cuda)
    y = mod(x, temp_input=ti)
    R = torch.randn(2, 50, H * D, generator=g, dtype=torch.float64)
    (y * R.float().to(cuda)).sum().backward()

    sd = {n: p.detach().double().cpu().requires_grad_() for n, p in mod.named_parameters()}
    xd, td = x.double().cpu(), ti.double().cpu()

    def lin(name, inp):
        return inp @ sd[f"{name}.linear.weight"].T + sd[f"{name}.linear.bias"]

    qp, kp, vp = lin("proj_q", xd), lin("proj_k", xd), lin("proj_v", xd).reshape(2, 50, H, D)
    hidden = torch.nn.functional.gelu(td @ sd["temp_func.network.0.weight"].T + sd["temp_func.network.0.bias"])
    temp = torch.nn.functional.softplus(hidden @ sd["temp_func.network.2.weight"].T + sd["temp_func.network.2.bias"]) \
        if "temp_func.network.2.weight" in sd else \
        torch.nn.functional.softplus(td @ sd["temp_func.network.0.weight"].T + sd["temp_func.network.0.bias"])
    eo, _, _ = G.prefill(qp, kp, vp, sd["feature_mapper.mlp.0.weight"], sd["feature_mapper.mlp.0.bias"], temp)
    (eo.reshape(2, 50, H * D) * R).sum().backward()
    for n, p in mod.named_parameters():
        assert rel_l2(to_np(p.grad), sd[n].grad.numpy()) < 1e-4, n


@pytest.mark.parametrize("act", ["elu+1", "relu", "softplus", "gelu", "identity", "sigmoid", "abs", "cossin"])
def test_feature_map_autograd_fp32(cuda, act):
    from pulsartecture_b200.backend.interface import feature_map

    g = torch.Generator().manual_seed(40)
    x = (torch.randn(70, 48, generator=g) * 2).to(cuda).requires_grad_()
    W = (torch.randn(40, 48, generator=g) / 7).to(cuda).requires_grad_()
    b = (torch.randn(40, generator=g) * 0.5).to(cuda).requires_grad_()
    y = feature_map(x, W, b, act, 0.3)
    R = torch.randn(*y.shape, generator=g, dtype=torch.float64)
    (y * R.float().to(cuda)).sum().backward()
    xd, Wd, bd = [t.detach().double().cpu().requires_grad_() for t in (x, W, b)]
    p = xd @ Wd.T + bd
    fns = {"elu+1": lambda t: torch.nn.functional.elu(t) + 1, "relu": torch.relu,
           "softplus": torch.nn.functional.softplus, "gelu": torch.nn.functional.gelu, "identity": lambda t: t,
           "sigmoid": torch.sigmoid, "abs": torch.abs,
           "cossin": lambda t: torch.cat([torch.cos(t), torch.sin(t)], -1) * 0.3}
    (fns[act](p) * R).sum().backward()
    for name, t, e in (("x", x, xd), ("W", W, Wd), ("b", b, bd)):
        assert rel_l2(to_np(t.grad), e.grad.numpy()) < 1e-5, name


def test_mixer_autograd_fp32(cuda):
    """KernelFeatureMixer under autograd: gradients of the input, context and
    every parameter (gate, LearnablePositiveMap, learnable RFF) against the
    same mixer restated in float64 torch."""
    import warnings

    from pulsartecture_b200.kernels import KernelFeatureMixer, LearnablePositiveMap, RandomFourierFeatures

    torch.manual_seed(41)
    with warnings.catch_warnings():
        warnings.simplefilter("ignore")
        maps = [LearnablePositiveMap(32, 64, activation="softplus"), RandomFourierFeatures(32, 64, learnable=True)]
    m = KernelFeatureMixer(maps, gate_input_dim=40, gate_hidden_dim=16, gate_layers=2).to(cuda)
    g = torch.Generator().manual_seed(42)
    x = torch.randn(3, 11, 32, generator=g).to(cuda).requires_grad_()
    c = torch.randn(3, 11, 8, generator=g).to(cuda).requires_grad_()
    y = m(x, c)
    R = torch.randn(3, 11, 64, generator=g, dtype=torch.float64)
    (y * R.float().to(cuda)).sum().backward()
    sd = {n: p.detach().double().cpu().requires_grad_() for n, p in m.named_parameters()}
    xd, cd = x.detach().double().cpu().requires_grad_(), c.detach().double().cpu().requires_grad_()
    f0 = torch.nn.functional.softplus(xd @ sd["feature_maps.0.mlp.0.weight"].T + sd["feature_maps.0.mlp.0.bias"])
    pr = xd @ sd["feature_maps.1.W"] + sd["feature_maps.1.b"]
    f1 = torch.cat([torch.cos(pr), torch.sin(pr)], -1) * np.sqrt(1 / 32)
    gin = torch.cat([xd, cd], -1)
    h = torch.nn.functional.gelu(gin @ sd["gate_net.network.0.weight"].T + sd["gate_net.network.0.bias"])
    w = torch.softmax(h @ sd["gate_net.network.2.weight"].T + sd["gate_net.network.2.bias"], -1)
    yd = w[..., 0:1] * f0 + w[..., 1:2] * f1
    (yd * R).sum().backward()
    assert rel_l2(to_np(y), yd.detach().numpy()) < 1e-5
    assert rel_l2(to_np(x.grad), xd.grad.numpy()) < 1e-5
    assert rel_l2(to_np(c.grad), cd.grad.numpy()) < 1e-5
    for n, p in m.named_parameters():
        assert rel_l2(to_np(p.grad), sd[n].grad.numpy()) < 1e-5, n
