"""Input, weight and bias gradients of a linear layer (fakla_linear_backward,
through the C ABI and through autograd) against float64 (GPU).

These are the gradients of the nn.Linear inside the feature maps (the
reference has no backward). bf16 shapes with in_dim % 128 == 0 run both
products on the tensor cores (dx = dpre W with W as an MN-major operand,
dW = dpre^T x with both operands MN-major), including ragged row counts,
which make dW's reduction dimension ragged; fp32 and other shapes run on the
CUDA cores.
"""
import numpy as np
import pytest
import torch

from pulsartecture_b200 import _lib
from tests.helpers import BF16_REL_L2, F32_REL_L2, rel_l2, to_np

pytestmark = pytest.mark.gpu


def _run(dev, rows, in_dim, n_out, dtype, seed):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(rows, in_dim, generator=g).to(dtype)
    W = (torch.randn(n_out, in_dim, generator=g) / in_dim ** 0.5).to(dtype)
    dpre = torch.randn(rows, n_out, generator=g).to(dtype)
    L = _lib.lib()
    code = _lib.FAKLA_BF16 if dtype == torch.bfloat16 else _lib.FAKLA_F32
    xd, Wd, dd = x.to(dev), W.to(dev), dpre.to(dev)
    dx = torch.empty(rows, in_dim, device=dev, dtype=dtype)
    dW = torch.empty(n_out, in_dim, device=dev, dtype=dtype)
    db = torch.empty(n_out, device=dev, dtype=dtype)
    wsb = L.fakla_linear_backward_workspace_bytes(rows, in_dim, n_out, code)
    ws = torch.empty(wsb, device=dev, dtype=torch.uint8)
    stream = torch.cuda.current_stream().cuda_stream
    _lib.check(L.fakla_linear_backward(xd.data_ptr(), Wd.data_ptr(), dd.data_ptr(), dx.data_ptr(), dW.data_ptr(),
                                       db.data_ptr(), rows, in_dim, n_out, code, ws.data_ptr(), wsb, stream))
    _lib.check(L.fakla_device_status(stream))
    x64, W64, d64 = x.double(), W.double(), dpre.double()
    return (to_np(dx), to_np(dW), to_np(db)), ((d64 @ W64).numpy(), (d64.T @ x64).numpy(), d64.sum(0).numpy())


@pytest.mark.parametrize("rows,in_dim,n_out", [
    (3000, 256, 512),     # ragged rows (ragged K of dW), single-CTA tiles
    (8192, 2048, 2048),   # the prefill's map at a quarter of config 2's rows: CTA pairs
    (65, 128, 128),       # fewer rows than one tile (dW's K is 65)
    (1000, 384, 64),      # single 64-wide row tile of dW
    (1024, 4096, 4096),   # dW on CTA pairs with both operands MN-major
])
def test_linear_backward_bf16_tensor_cores(cuda, rows, in_dim, n_out):
    got, exp = _run(cuda, rows, in_dim, n_out, torch.bfloat16, seed=rows)
    for name, g, e in zip(("dx", "dW", "db"), got, exp):
        assert rel_l2(g, e) < BF16_REL_L2, (name, rel_l2(g, e))


@pytest.mark.parametrize("rows,in_dim,n_out,dtype", [
    (70, 48, 40, torch.float32),
    (513, 256, 96, torch.float32),
    (300, 200, 72, torch.bfloat16),   # in_dim % 128 != 0: the CUDA-core path in bf16
    (1000, 384, 40, torch.bfloat16),  # n_out < 64: the CUDA-core path in bf16
])
def test_linear_backward_cuda_cores(cuda, rows, in_dim, n_out, dtype):
    got, exp = _run(cuda, rows, in_dim, n_out, dtype, seed=7 + rows)
    tol = F32_REL_L2 if dtype == torch.float32 else BF16_REL_L2
    for name, g, e in zip(("dx", "dW", "db"), got, exp):
        assert rel_l2(g, e) < tol, (name, rel_l2(g, e))


def test_linear_backward_subsets(cuda):
    """Only the requested gradients are written (NULL pointers for the others)."""
    L = _lib.lib()
    rows, in_dim, n_out = 512, 256, 256
    x = torch.randn(rows, in_dim, device=cuda).bfloat16()
    W = torch.randn(n_out, in_dim, device=cuda).bfloat16()
    dpre = torch.randn(rows, n_out, device=cuda).bfloat16()
    dx = torch.full((rows, in_dim), 7.0, device=cuda).bfloat16()
    stream = torch.cuda.current_stream().cuda_stream
    _lib.check(L.fakla_linear_backward(None, W.data_ptr(), dpre.data_ptr(), dx.data_ptr(), None, None, rows, in_dim,
                                       n_out, _lib.FAKLA_BF16, None, 0, stream))
    _lib.check(L.fakla_device_status(stream))
    assert rel_l2(to_np(dx), (dpre.double() @ W.double()).cpu().numpy()) < BF16_REL_L2
    # the bias gradient without a workspace is refused
    db = torch.empty(n_out, device=cuda).bfloat16()
    rc = L.fakla_linear_backward(None, None, dpre.data_ptr(), None, None, db.data_ptr(), rows, in_dim, n_out,
                                 _lib.FAKLA_BF16, None, 0, stream)
    assert rc == 6


def test_feature_map_autograd_bf16_on_tensor_cores(cuda):
    """LearnablePositiveMap-shaped map (elu+1) in bf16 through autograd: the
    input, weight and bias gradients against float64 autograd."""
    from pulsartecture_b200.backend.interface import feature_map

    g = torch.Generator().manual_seed(5)
    x = (torch.randn(2000, 256, generator=g) * 0.5).bfloat16()
    W = (torch.randn(512, 256, generator=g) / 16).bfloat16()
    b = (torch.randn(512, generator=g) * 0.1).bfloat16()
    R = torch.randn(2000, 512, generator=g).bfloat16()
    xs = [t.to(cuda).requires_grad_() for t in (x, W, b)]
    y = feature_map(xs[0], xs[1], xs[2], "elu+1")
    (y.float() * R.to(cuda).float()).sum().backward()
    xd = [t.double().requires_grad_() for t in (x, W, b)]
    yd = torch.nn.functional.elu(xd[0] @ xd[1].T + xd[2]) + 1
    (yd * R.double()).sum().backward()
    for a, e in zip(xs, xd):
        assert rel_l2(to_np(a.grad), e.grad.numpy()) < BF16_REL_L2
