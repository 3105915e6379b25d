"""The gradient oracle (float64 torch restatement, CPU): its forward equals
the C oracle (itself pinned to the reference), and its autograd gradients
equal finite differences (torch.autograd.gradcheck)."""
import torch

from oracle import fakla_grad_oracle as G
from oracle import fakla_oracle as O


def _case(seed, B=2, T=9, H=2, Df=5, Dv=4, state=True):
    g = torch.Generator().manual_seed(seed)
    q = torch.rand(B, T, H, Df, generator=g, dtype=torch.float64) + 0.2
    k = torch.rand(B, T, H, Df, generator=g, dtype=torch.float64) + 0.2
    v = torch.randn(B, T, H, Dv, generator=g, dtype=torch.float64)
    tp = torch.rand(B, T, H, generator=g, dtype=torch.float64) + 0.5
    S0 = torch.randn(B, H, Df, Dv, generator=g, dtype=torch.float64) * 0.1 if state else None
    z0 = torch.rand(B, H, Df, generator=g, dtype=torch.float64) + 1.0 if state else None
    return q, k, v, tp, S0, z0


def test_grad_oracle_forward_equals_c_oracle():
    q, k, v, tp, S0, z0 = _case(1, T=40, Df=7, Dv=6)
    out, S, z = G.attention(q, k, v, tp, S0, z0)
    eo, eS, ez = O.attention(q.numpy(), k.numpy(), v.numpy(), tp.numpy(), S0.numpy(), z0.numpy())
    assert O.rel_l2(out.numpy(), eo) < 1e-12
    assert O.rel_l2(S.numpy(), eS) < 1e-12
    assert O.rel_l2(z.numpy(), ez) < 1e-12


def test_grad_oracle_gradients_equal_finite_differences():
    args = [t.requires_grad_() for t in _case(2)]

    def f(q, k, v, tp, S0, z0):
        out, S, z = G.attention(q, k, v, tp, S0, z0)
        return out, S, z

    assert torch.autograd.gradcheck(f, tuple(args), eps=1e-6, atol=1e-7, rtol=1e-5)


def test_grad_oracle_prefill_gradients_equal_finite_differences():
    g = torch.Generator().manual_seed(3)
    B, T, H, D = 1, 6, 2, 3
    q = torch.randn(B, T, H * D, generator=g, dtype=torch.float64, requires_grad=True)
    k = torch.randn(B, T, H * D, generator=g, dtype=torch.float64, requires_grad=True)
    v = torch.randn(B, T, H, D, generator=g, dtype=torch.float64, requires_grad=True)
    W = (torch.randn(H * D, H * D, generator=g, dtype=torch.float64) * 0.5).requires_grad_()
    b = (torch.randn(H * D, generator=g, dtype=torch.float64) * 0.1).requires_grad_()
    assert torch.autograd.gradcheck(lambda *a: G.prefill(*a)[0], (q, k, v, W, b), eps=1e-6, atol=1e-7, rtol=1e-5)
