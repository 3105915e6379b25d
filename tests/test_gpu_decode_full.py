"""The recurrent decode step at its full benchmark shape against the oracle (GPU).

Batch 256, H=32, Dk=Dv=M=128, LearnablePositiveMap(4096 -> 4096) in bf16,
state S ~ N(0, 0.02) and z ~ U(0.5, 1.5) in fp32 -- the shape whose feature-map
GEMM takes the mixed 128/256-wide tile schedule. All 256 sequences run through
fakla_decode (the C ABI) for 64 chained steps with the state updated in place;
the oracle (phi on the bf16 inputs in float64, then the loop body of
cpu_kernels.cpp:121-162 per token) follows a sample of the sequences from the
same initial state. Every step's output and the final state of the sample are
compared, so drift over the chain would show.
"""
import math

import numpy as np
import pytest
import torch

from oracle import fakla_oracle as O
from pulsartecture_b200 import _lib
from tests.helpers import BF16_MAX_ABS, BF16_REL_L2, lpm_params, rel_l2, to_np

pytestmark = pytest.mark.gpu

N, H, D = 256, 32, 128
IN_DIM = H * D
STEPS = 64
# sequences followed by the oracle: both ends, the middle and a few in between
SAMPLE = [0, 1, 63, 64, 127, 128, 200, 255]


def _setup(dev, seed):
    g = torch.Generator(device=dev).manual_seed(seed)
    W, b = lpm_params(IN_DIM, H * D, seed=seed + 1, dtype=torch.bfloat16)
    S = torch.randn(N, H, D, D, generator=g, device=dev) * 0.02
    z = torch.rand(N, H, D, generator=g, device=dev) + 0.5
    q = (torch.randn(STEPS, N, IN_DIM, generator=g, device=dev) / math.sqrt(D)).bfloat16()
    k = (torch.randn(STEPS, N, IN_DIM, generator=g, device=dev) / math.sqrt(D)).bfloat16()
    v = (torch.randn(STEPS, N, H, D, generator=g, device=dev) / math.sqrt(D)).bfloat16()
    return W.to(dev), b.to(dev), S, z, q, k, v


def _oracle_step(q, k, v, W, b, S, z):
    pq = O.phi(q, W, b).reshape(len(SAMPLE), H, D)
    pk = O.phi(k, W, b).reshape(len(SAMPLE), H, D)
    return O.decode_step(pq, pk, v, S, z)


def _check(out, expect, what):
    err = rel_l2(out, expect)
    mx = float(np.abs(out - expect).max())
    assert err < BF16_REL_L2, f"{what}: rel-L2 {err:.2e}"
    assert mx < BF16_MAX_ABS, f"{what}: max-abs {mx:.2e}"
    return err


def test_decode_full_shape_chained_against_oracle(cuda):
    L = _lib.lib()
    W, b, S, z, q, k, v = _setup(cuda, seed=41)
    Wn, bn = to_np(W), to_np(b)
    idx = torch.tensor(SAMPLE, device=cuda)
    S_o = to_np(S[idx]).astype(np.float64)
    z_o = to_np(z[idx]).astype(np.float64)
    ws_bytes = L.fakla_decode_workspace_bytes(N, IN_DIM, H, D, D, _lib.FAKLA_BF16)
    ws = torch.empty(ws_bytes, device=cuda, dtype=torch.uint8)
    out = torch.empty(N, H, D, device=cuda, dtype=torch.bfloat16)
    stream = torch.cuda.current_stream().cuda_stream
    errs = []
    for t in range(STEPS):
        _lib.check(L.fakla_decode(q[t].data_ptr(), k[t].data_ptr(), v[t].data_ptr(), None, W.data_ptr(),
                                  b.data_ptr(), out.data_ptr(), S.data_ptr(), z.data_ptr(), N, IN_DIM, H, D, D,
                                  _lib.FAKLA_BF16, ws.data_ptr(), ws_bytes, stream))
        got = to_np(out[idx])
        eo, S_o, z_o = _oracle_step(to_np(q[t, idx]), to_np(k[t, idx]), to_np(v[t, idx]), Wn, bn, S_o, z_o)
        errs.append(_check(got, eo, f"step {t}"))
    _lib.check(L.fakla_device_status(stream))
    # final state of the sampled sequences after 64 steps
    assert rel_l2(to_np(S[idx]), S_o) < BF16_REL_L2
    assert rel_l2(to_np(z[idx]), z_o) < BF16_REL_L2
    # no drift: the last step is not worse than a few times the first
    assert errs[-1] < max(4 * errs[0], 1e-3), errs
