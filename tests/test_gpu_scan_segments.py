"""Segmented tensor-core scan (GPU only): long sequences with few (b, h)
pairs are split into segments run by separate CTAs, with each segment's
initial state built from the sums of the segments before it. Checked against
the oracle, against the unsegmented scan (same call without workspace), and
at the long-context configuration's full size (B=1, H=32, T=65536, D=M=128).
"""
import numpy as np
import pytest
import torch

from oracle import fakla_oracle as O
from tests.helpers import BF16_MAX_ABS, BF16_REL_L2, lpm_params, rel_l2, to_np

pytestmark = pytest.mark.gpu


def _phi_like(shape, seed, dev):
    g = torch.Generator().manual_seed(seed)
    return (torch.rand(*shape, generator=g) + 0.5).bfloat16().to(dev)


def _normal(shape, seed, dev, scale):
    g = torch.Generator().manual_seed(seed)
    return (torch.randn(*shape, generator=g) * scale).to(dev)


def _attention_abi(q, k, v, tp, S, z, flags, use_workspace):
    """fakla_attention through the C ABI; returns (out, workspace bytes used)."""
    from pulsartecture_b200 import _lib

    L = _lib.lib()
    B, T, H, D = q.shape
    ws_bytes = L.fakla_attention_workspace_bytes(B, T, H, D, D, _lib.FAKLA_BF16) if use_workspace else 0
    ws = torch.empty(max(ws_bytes, 1), device=q.device, dtype=torch.uint8)
    out = torch.empty_like(v)
    _lib.check(L.fakla_attention(q.data_ptr(), k.data_ptr(), v.data_ptr(), None if tp is None else tp.data_ptr(),
                                 out.data_ptr(), S.data_ptr(), z.data_ptr(), B, T, H, D, D, _lib.FAKLA_BF16,
                                 flags, ws.data_ptr() if ws_bytes else None, ws_bytes,
                                 torch.cuda.current_stream().cuda_stream))
    _lib.check(L.fakla_device_status(torch.cuda.current_stream().cuda_stream))
    return out, ws_bytes


def test_workspace_query_segments_only_when_sms_would_idle(cuda):
    from pulsartecture_b200 import _lib

    L = _lib.lib()
    bf = _lib.FAKLA_BF16
    # 128 sequences of the prefill benchmark fill the GPU: no segments
    assert L.fakla_attention_workspace_bytes(8, 4096, 16, 128, 128, bf) == 0
    # 32 long sequences: 4 segments each, one (S, z) record per segment
    rec = (128 * 128 + 128) * 4
    assert L.fakla_attention_workspace_bytes(1, 65536, 32, 128, 128, bf) == 32 * 4 * rec
    # 64-wide heads run in the same tiles: the same records
    assert L.fakla_attention_workspace_bytes(1, 65536, 32, 64, 64, bf) == 32 * 4 * rec
    # fp32 and other head dims run on the CUDA-core scan: no workspace
    assert L.fakla_attention_workspace_bytes(1, 65536, 32, 128, 128, _lib.FAKLA_F32) == 0
    assert L.fakla_attention_workspace_bytes(1, 65536, 2, 32, 32, bf) == 0


@pytest.mark.parametrize("B,T,H,with_temp,with_state", [
    (1, 3000, 3, True, True),     # ragged last chunk inside the last segment
    (1, 8192, 1, False, False),   # 32 segments of two chunks
    (2, 2048, 2, True, False),
])
def test_segmented_matches_oracle_and_single_cta(cuda, B, T, H, with_temp, with_state):
    from pulsartecture_b200 import _lib

    D = 128
    q = _phi_like((B, T, H, D), 20, cuda)
    k = _phi_like((B, T, H, D), 21, cuda)
    v = _normal((B, T, H, D), 22, cuda, 1 / np.sqrt(D)).bfloat16()
    tp = _phi_like((B, T, H), 23, cuda) if with_temp else None
    S0 = _normal((B, H, D, D), 24, cuda, 0.02) + 0.05
    z0 = (torch.rand(B, H, D, generator=torch.Generator().manual_seed(25)) * 20 + 10).to(cuda)
    flags = _lib.FAKLA_STATE_OUT | (_lib.FAKLA_STATE_IN if with_state else 0)
    S_a, z_a = S0.clone(), z0.clone()
    S_b, z_b = S0.clone(), z0.clone()
    out_a, ws = _attention_abi(q, k, v, tp, S_a, z_a, flags, True)
    assert ws > 0, "this shape must take the segmented path"
    out_b, _ = _attention_abi(q, k, v, tp, S_b, z_b, flags, False)
    eo, eS, ez = O.attention(to_np(q), to_np(k), to_np(v), None if tp is None else to_np(tp),
                             to_np(S0) if with_state else None, to_np(z0) if with_state else None)
    for out, S, z in ((out_a, S_a, z_a), (out_b, S_b, z_b)):
        assert rel_l2(to_np(out), eo) < BF16_REL_L2
        assert np.abs(to_np(out) - eo).max() < BF16_MAX_ABS
        assert rel_l2(to_np(S), eS) < BF16_REL_L2
        # k~ = k * temp is rounded to bf16 before it is summed into z
        assert rel_l2(to_np(z), ez) < (1e-4 if with_temp else 1e-5)
    # the two schedules differ only in the fp32 summation order of the state
    assert rel_l2(to_np(S_a), to_np(S_b)) < 1e-5
    assert rel_l2(to_np(z_a), to_np(z_b)) < 1e-6
    assert rel_l2(to_np(out_a), to_np(out_b)) < 2e-3


def test_long_context_b1h32t65536_full_size(cuda):
    """Long-context prefill at full size: B=1, H=32, T=65536, Dk=Dv=M=128,
    bf16, LearnablePositiveMap(4096 -> 4096) from seed 0. The scan is checked
    against the oracle on two whole sequences (fed the kernel's own phi, which
    the phi tests check separately); z = sum_t phi(k_t) on all 32."""
    from pulsartecture_b200.attention import fa_kla
    from pulsartecture_b200.backend.interface import phi_map

    B, T, H, D = 1, 65536, 32, 128
    g = torch.Generator(device=cuda).manual_seed(130)
    q = (torch.randn(B, T, H * D, generator=g, device=cuda) / np.sqrt(D)).bfloat16()
    k = (torch.randn(B, T, H * D, generator=g, device=cuda) / np.sqrt(D)).bfloat16()
    v = (torch.randn(B, T, H, D, generator=g, device=cuda) / np.sqrt(D)).bfloat16()
    W, b = lpm_params(H * D, H * D, seed=0, dtype=torch.bfloat16)
    W, b = W.to(cuda), b.to(cuda)
    out, (S, z) = fa_kla(q, k, v, phi_weight=W, phi_bias=b)
    assert torch.isfinite(out).all() and torch.isfinite(S).all()
    pq = phi_map(q.reshape(T, H * D), W, b).reshape(B, T, H, D)
    pk = phi_map(k.reshape(T, H * D), W, b).reshape(B, T, H, D)
    assert rel_l2(to_np(z), to_np(pk.float().sum(1))) < 1e-5
    for hh in (0, 31):
        eo, eS, _ = O.attention(to_np(pq[:, :, hh:hh + 1]), to_np(pk[:, :, hh:hh + 1]), to_np(v[:, :, hh:hh + 1]))
        got = to_np(out[:, :, hh:hh + 1])
        assert rel_l2(got, eo) < BF16_REL_L2
        assert np.abs(got - eo).max() < BF16_MAX_ABS
        assert rel_l2(to_np(S[:, hh:hh + 1]), eS) < BF16_REL_L2


@pytest.mark.parametrize("B,h0,h1", [
    (1, 0, 16),   # one GPU's part of an 8-way batch split of B=8, H=16: 16 sequences, 8 segments of 4 chunks
    (2, 0, 16),   # ... of a 4-way batch split: 32 sequences, 4 segments of 8 chunks
    (8, 6, 8),    # ... of an 8-way head split (heads 6-7, the map's rows of those heads, q and k rows whole)
])
def test_prefill_shard_shapes_against_oracle(cuda, B, h0, h1):
    """fa_kla at the per-GPU shapes of the multi-GPU prefill bench (T=4096,
    D=M=128, bf16, LearnablePositiveMap(2048 -> 2048) rows of the shard's
    heads, with temperature): the scan runs segmented, and two sequences are
    checked against the oracle fed the oracle's own phi."""
    from pulsartecture_b200.attention import fa_kla

    T, H, D = 4096, 16, 128
    Hs = h1 - h0
    g = torch.Generator(device=cuda).manual_seed(140 + B + h0)
    q = (torch.randn(B, T, H * D, generator=g, device=cuda) / np.sqrt(D)).bfloat16()
    k = (torch.randn(B, T, H * D, generator=g, device=cuda) / np.sqrt(D)).bfloat16()
    v = (torch.randn(B, T, Hs, D, generator=g, device=cuda) / np.sqrt(D)).bfloat16()
    tp = (torch.rand(B, T, Hs, generator=g, device=cuda) + 0.5).bfloat16()
    W, b = lpm_params(H * D, H * D, seed=0, dtype=torch.bfloat16)
    Ws, bs = W[h0 * D:h1 * D].contiguous().to(cuda), b[h0 * D:h1 * D].contiguous().to(cuda)
    from pulsartecture_b200 import _lib

    assert _lib.lib().fakla_attention_workspace_bytes(B, T, Hs, D, D, _lib.FAKLA_BF16) > 0, "segmented"
    out, (S, z) = fa_kla(q, k, v, phi_weight=Ws, phi_bias=bs, temp=tp)
    assert torch.isfinite(out).all() and torch.isfinite(S).all()
    for bb, hh in [(0, 0), (B - 1, Hs - 1)]:
        Wh, bh = to_np(Ws)[hh * D:(hh + 1) * D], to_np(bs)[hh * D:(hh + 1) * D]
        pq = O.phi(to_np(q[bb]), Wh, bh)
        pk = O.phi(to_np(k[bb]), Wh, bh)
        eo, eS, ez = O.attention(pq[None, :, None], pk[None, :, None], to_np(v[bb, :, hh])[None, :, None],
                                 to_np(tp[bb, :, hh])[None, :, None])
        got = to_np(out[bb, :, hh])
        assert rel_l2(got, eo[0, :, 0]) < BF16_REL_L2
        assert np.abs(got - eo[0, :, 0]).max() < BF16_MAX_ABS
        assert rel_l2(to_np(S[bb, hh]), eS[0, 0]) < BF16_REL_L2
        assert rel_l2(to_np(z[bb, hh]), ez[0, 0]) < BF16_REL_L2
