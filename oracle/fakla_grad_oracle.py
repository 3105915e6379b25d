"""float64 torch restatement of FA-KLA whose autograd gives the gradients.

TEST INFRASTRUCTURE ONLY: the checker of libfakla's backward kernels
(fakla_attention_backward, fakla_phi_backward) and of the autograd path of
pulsartecture_b200. The product path never imports this module.

The reference has no backward. This restates its forward recurrence
(ultra_rwka/backend/cpp/cpu/cpu_kernels.cpp:107-164: k~ = k*temp, z += k~,
S += k~ v^T, out = q^T S / (q.z + 1e-12)) with cumulative sums, so that
torch.autograd differentiates exactly that function; its forward is checked
against the C oracle and its gradients against finite differences
(tests/test_grad_oracle.py). Memory is O(B*T*H*Df*Dv): small cases only.
"""
from __future__ import annotations

import torch

EPS = 1e-12  # K_EPSILON, cpu_kernels.cpp:22


def attention(q, k, v, temp=None, S0=None, z0=None):
    """q, k: (B,T,H,Df); v: (B,T,H,Dv); temp: (B,T,H); S0: (B,H,Df,Dv); z0: (B,H,Df).
    Returns (out, S_T, z_T), differentiable in every input."""
    kt = k * temp[..., None] if temp is not None else k
    S = torch.cumsum(kt[..., :, None] * v[..., None, :], dim=1)
    z = torch.cumsum(kt, dim=1)
    if S0 is not None:
        S = S + S0[:, None]
        z = z + z0[:, None]
    num = torch.einsum("bthf,bthfd->bthd", q, S)
    den = (q * z).sum(-1) + EPS
    return num / den[..., None], S[:, -1], z[:, -1]


def phi(x, W, b=None):
    """elu(x W^T + b) + 1 (feature_maps.py:248, 259-268)."""
    y = x @ W.T
    if b is not None:
        y = y + b
    return torch.nn.functional.elu(y) + 1.0


def prefill(q, k, v, W, b=None, temp=None, S0=None, z0=None):
    """phi on the flattened (B,T,H*Dk) rows, head split, attention (tm_kla.py:268-319)."""
    B, T = q.shape[:2]
    H = v.shape[2]
    M = W.shape[0] // H
    pq = phi(q.reshape(B, T, -1), W, b).reshape(B, T, H, M)
    pk = phi(k.reshape(B, T, -1), W, b).reshape(B, T, H, M)
    return attention(pq, pk, v, temp, S0, z0)
