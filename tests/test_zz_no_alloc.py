"""fakla_decode_noalloc through the C ABI against fakla_decode (GPU only).

The no-allocation decode entry point exists for callers that cannot hand the
library a workspace (bare C FFI hosts without a device allocator, per-token
loops where cudaMalloc is off limits). It must give the same step as
fakla_decode -- checked here on two calls in a row, so the second call also
sees scratch left over from the first -- and refuse steps whose scratch would
not fit in the static array. This file sorts last so a failure here cannot
hide any other test in a run that stops at the first failure.
"""
import math

import numpy as np
import pytest
import torch

from pulsartecture_b200 import _lib
from tests.helpers import BF16_MAX_ABS, BF16_REL_L2, F32_REL_L2, lpm_params, rel_l2, to_np

pytestmark = pytest.mark.gpu


def _inputs(dev, N, H, Dk, M, dtype, seed):
    g = torch.Generator().manual_seed(seed)
    in_dim = H * Dk
    q = (torch.randn(2, N, in_dim, generator=g) / math.sqrt(Dk)).to(dtype).to(dev)
    k = (torch.randn(2, N, in_dim, generator=g) / math.sqrt(Dk)).to(dtype).to(dev)
    v = (torch.randn(2, N, H, M, generator=g) / math.sqrt(Dk)).to(dtype).to(dev)
    temp = (torch.rand(2, N, H, generator=g) + 0.5).to(dtype).to(dev)
    W, b = lpm_params(in_dim, H * M, seed=seed + 1, dtype=dtype)
    S = (torch.randn(N, H, M, M, generator=g) * 0.02).to(dev)
    z = (torch.rand(N, H, M, generator=g) + 0.5).to(dev)
    return q, k, v, temp, W.to(dev), b.to(dev), S, z


@pytest.mark.parametrize("dtype,N,H,Dk,M", [
    (torch.bfloat16, 256, 32, 128, 128),  # the decode configuration: 4 MiB of scratch
    (torch.float32, 96, 4, 64, 64),
])
def test_noalloc_decode_matches_workspace_decode_twice(cuda, dtype, N, H, Dk, M):
    L = _lib.lib()
    code = _lib.FAKLA_BF16 if dtype == torch.bfloat16 else _lib.FAKLA_F32
    q, k, v, temp, W, b, S, z = _inputs(cuda, N, H, Dk, M, dtype, seed=11)
    in_dim = H * Dk
    S_ref, z_ref = S.clone(), z.clone()
    S_na, z_na = S.clone(), z.clone()
    ws_bytes = L.fakla_decode_workspace_bytes(N, in_dim, H, M, M, code)
    ws = torch.empty(ws_bytes, device=cuda, dtype=torch.uint8)
    stream = torch.cuda.current_stream().cuda_stream
    tol = BF16_REL_L2 if dtype == torch.bfloat16 else F32_REL_L2
    for step in range(2):
        o_ref = torch.empty(N, H, M, device=cuda, dtype=dtype)
        o_na = torch.empty(N, H, M, device=cuda, dtype=dtype)
        args = (q[step].data_ptr(), k[step].data_ptr(), v[step].data_ptr(), temp[step].data_ptr(),
                W.data_ptr(), b.data_ptr())
        _lib.check(L.fakla_decode(*args, o_ref.data_ptr(), S_ref.data_ptr(), z_ref.data_ptr(),
                                  N, in_dim, H, M, M, code, ws.data_ptr(), ws_bytes, stream))
        _lib.check(L.fakla_decode_noalloc(*args, o_na.data_ptr(), S_na.data_ptr(), z_na.data_ptr(),
                                          N, in_dim, H, M, M, code, stream))
        torch.cuda.synchronize()
        assert rel_l2(to_np(o_na), to_np(o_ref)) < tol
        if dtype == torch.bfloat16:
            assert np.abs(to_np(o_na) - to_np(o_ref)).max() < BF16_MAX_ABS
        assert rel_l2(to_np(S_na), to_np(S_ref)) < F32_REL_L2
        assert rel_l2(to_np(z_na), to_np(z_ref)) < F32_REL_L2
    _lib.check(L.fakla_device_status(stream))


def test_noalloc_decode_rejects_oversized_step(cuda):
    """N=1024, H=32, M=128 in bf16 needs 2*1024*32*128*2 B = 16 MiB of scratch,
    twice the static array: rejected before any launch. Every caller buffer is
    allocated at its full size anyway, so nothing here could touch memory it
    does not own even if the size check were wrong."""
    L = _lib.lib()
    N, H, M = 1024, 32, 128
    in_dim = H * M
    assert L.fakla_decode_workspace_bytes(N, in_dim, H, M, M, _lib.FAKLA_BF16) == 16 << 20
    bf = dict(device=cuda, dtype=torch.bfloat16)
    q = torch.zeros(N, in_dim, **bf)
    k = torch.zeros(N, in_dim, **bf)
    v = torch.zeros(N, H, M, **bf)
    W = torch.zeros(H * M, in_dim, **bf)
    out = torch.zeros(N, H, M, **bf)
    S = torch.zeros(N, H, M, M, device=cuda)
    z = torch.zeros(N, H, M, device=cuda)
    rc = L.fakla_decode_noalloc(q.data_ptr(), k.data_ptr(), v.data_ptr(), None, W.data_ptr(), None,
                                out.data_ptr(), S.data_ptr(), z.data_ptr(), N, in_dim, H, M, M,
                                _lib.FAKLA_BF16, torch.cuda.current_stream().cuda_stream)
    assert rc == 2  # FAKLA_ERR_UNSUPPORTED
    assert b"scratch" in L.fakla_last_error()
    torch.cuda.synchronize()
    assert not out.any()


def test_noalloc_decode_full_shape_against_oracle(cuda):
    """The decode shape (batch 256, H=32, LearnablePositiveMap(4096 -> 4096),
    bf16) once against the oracle itself rather than against fakla_decode, so
    an error common to both entry points would not pass unseen."""
    from oracle import fakla_oracle as O

    L = _lib.lib()
    N, H, D = 256, 32, 128
    in_dim = H * D
    g = torch.Generator(device=cuda).manual_seed(43)
    W, b = lpm_params(in_dim, H * D, seed=44, dtype=torch.bfloat16)
    W, b = W.to(cuda), b.to(cuda)
    S = torch.randn(N, H, D, D, generator=g, device=cuda) * 0.02
    z = torch.rand(N, H, D, generator=g, device=cuda) + 0.5
    q = (torch.randn(N, in_dim, generator=g, device=cuda) / math.sqrt(D)).bfloat16()
    k = (torch.randn(N, in_dim, generator=g, device=cuda) / math.sqrt(D)).bfloat16()
    v = (torch.randn(N, H, D, generator=g, device=cuda) / math.sqrt(D)).bfloat16()
    idx = torch.tensor([0, 77, 128, 255], device=cuda)
    S0, z0 = to_np(S[idx]).astype(np.float64), to_np(z[idx]).astype(np.float64)
    out = torch.empty(N, H, D, device=cuda, dtype=torch.bfloat16)
    stream = torch.cuda.current_stream().cuda_stream
    _lib.check(L.fakla_decode_noalloc(q.data_ptr(), k.data_ptr(), v.data_ptr(), None, W.data_ptr(), b.data_ptr(),
                                      out.data_ptr(), S.data_ptr(), z.data_ptr(), N, in_dim, H, D, D,
                                      _lib.FAKLA_BF16, stream))
    _lib.check(L.fakla_device_status(stream))
    pq = O.phi(to_np(q[idx]), to_np(W), to_np(b)).reshape(len(idx), H, D)
    pk = O.phi(to_np(k[idx]), to_np(W), to_np(b)).reshape(len(idx), H, D)
    eo, eS, ez = O.decode_step(pq, pk, to_np(v[idx]), S0, z0)
    got = to_np(out[idx])
    assert rel_l2(got, eo) < BF16_REL_L2
    assert np.abs(got - eo).max() < BF16_MAX_ABS
    assert rel_l2(to_np(S[idx]), eS) < BF16_REL_L2 and rel_l2(to_np(z[idx]), ez) < BF16_REL_L2
