"""Parity of the CUDA kernels with the oracle, through the C ABI (GPU only).

Bars: bf16 inputs with fp32 accumulation -> rel-L2 <= 5e-3 and max-abs <= 2e-2;
fp32 mode -> rel-L2 <= 1e-5 (tests/helpers.py). The oracle computes in float64
on exactly the values the kernels see (bf16 inputs rounded first).
"""
import numpy as np
import pytest
import torch

from oracle import fakla_oracle as O
from tests.helpers import BF16_MAX_ABS, BF16_REL_L2, F32_REL_L2, lpm_params, rel_l2, to_np

pytestmark = pytest.mark.gpu


def _phi_like(shape, seed, dev, dtype):
    g = torch.Generator().manual_seed(seed)
    return (torch.rand(*shape, generator=g) + 0.5).to(dtype).to(dev)


def _normal(shape, seed, dev, dtype, scale=1.0):
    g = torch.Generator().manual_seed(seed)
    return (torch.randn(*shape, generator=g) * scale).to(dtype).to(dev)


# ----------------------------------------------------------------- building blocks
@pytest.mark.parametrize("form", [0, 1, 2, 3])
def test_umma_operand_forms(cuda, form):
    from tests import selftest_lib

    lib = selftest_lib.load()
    A = _normal((128, 128), 1, cuda, torch.bfloat16)
    B = _normal((128, 128), 2, cuda, torch.bfloat16)
    D = torch.empty(128, 128, device=cuda, dtype=torch.float32)
    rc = lib.selftest_umma_form(form, A.data_ptr(), B.data_ptr(), D.data_ptr(), torch.cuda.current_stream().cuda_stream)
    assert rc == 0
    torch.cuda.synchronize()
    a, b = A.double(), B.double()
    exp = {0: a @ b.T, 1: a.T @ b, 2: a @ b, 3: a @ b}[form]
    assert rel_l2(to_np(D), exp.cpu().numpy()) < 1e-6


def test_bounded_wait_times_out_and_context_survives(cuda):
    from tests import selftest_lib

    lib = selftest_lib.load()
    st = torch.full((1,), -1, device=cuda, dtype=torch.int32)
    rc = lib.selftest_wait_timeout(20_000_000, st.data_ptr(), torch.cuda.current_stream().cuda_stream)
    assert rc == 0
    torch.cuda.synchronize()
    assert int(st.item()) == 5  # FAKLA_ERR_TIMEOUT
    x = torch.ones(1000, device=cuda)
    assert float(x.sum().item()) == 1000.0


def test_device_status_clean(cuda):
    from pulsartecture_b200.backend.interface import device_status

    device_status()


# ----------------------------------------------------------------- phi
@pytest.mark.parametrize("rows,K,N,heads,use_bias,use_temp", [
    (512, 256, 256, 4, True, False),
    (1000, 2048, 2048, 16, True, True),
    (1, 256, 512, 2, False, True),
    (130, 4096, 512, 4, True, False),
    (4096, 2048, 2048, 16, True, True),
    (5000, 1024, 512, 4, False, True),    # ragged last row tile
    (32, 4096, 4096, 32, True, True),     # small row sets: 64-row A stages, 8 stages
    (64, 2048, 2048, 16, True, False),    # ... at their largest
    (65, 2048, 2048, 16, True, True),     # one row past them: the plain 128-row tile
])
def test_phi_bf16_tensor_core(cuda, rows, K, N, heads, use_bias, use_temp):
    from pulsartecture_b200.backend.interface import phi_map

    x = _normal((rows, K), 3, cuda, torch.bfloat16, 1 / np.sqrt(128))
    W, b = lpm_params(K, N, seed=4, dtype=torch.bfloat16)
    W, b = W.to(cuda), b.to(cuda)
    temp = _phi_like((rows, heads), 5, cuda, torch.bfloat16) if use_temp else None
    got = phi_map(x, W, b if use_bias else None, temp, heads)
    exp = O.phi(to_np(x), to_np(W), to_np(b) if use_bias else None, to_np(temp) if use_temp else None, heads)
    g = to_np(got)
    # output is rounded to bf16 once: |err| <= half an ulp (2^-9 relative) + accumulation noise
    assert np.all(np.abs(g - exp) <= 2.0 ** -8 * np.abs(exp) + 1e-4)


@pytest.mark.parametrize("rows,nsets", [(8192, 1), (4096, 2)])
def test_phi_split_tail_against_oracle(cuda, rows, nsets):
    """256 tiles of 256 x 256 on the CTA pairs leave a last wave a third full:
    those tiles run as two 256 x 128 halves each (the per-GPU feature map of
    an 8-way split of B=8, H=16, T=4096: 2 x 4096 rows x 2048 -> 2048). The
    rows of the tail (the last 1280 rows of the last row set) and some of the
    first are checked against the oracle, with the k-side temperature."""
    from pulsartecture_b200 import _lib

    L = _lib.lib()
    K = N = 2048
    heads = 16
    x = _normal((nsets, rows, K), 30, cuda, torch.bfloat16, 1 / np.sqrt(128))
    W, b = lpm_params(K, N, seed=31, dtype=torch.bfloat16)
    W, b = W.to(cuda), b.to(cuda)
    temp = _phi_like((rows, heads), 32, cuda, torch.bfloat16)
    out = torch.empty(nsets, rows, N, device=cuda, dtype=torch.bfloat16)
    stream = torch.cuda.current_stream().cuda_stream
    if nsets == 1:
        _lib.check(L.fakla_phi(x.data_ptr(), W.data_ptr(), b.data_ptr(), temp.data_ptr(), out.data_ptr(), rows, K,
                               N, heads, _lib.FAKLA_BF16, stream))
    else:
        # both row sets in one launch, as the prefill runs phi(q) and phi(k) * temp
        B_, T_ = 1, rows
        v = torch.zeros(B_, T_, heads, N // heads, device=cuda, dtype=torch.bfloat16)
        o = torch.empty_like(v)
        wsb = L.fakla_prefill_workspace_bytes(B_, T_, K, heads, N // heads, N // heads, _lib.FAKLA_BF16)
        ws = torch.empty(wsb, device=cuda, dtype=torch.uint8)
        _lib.check(L.fakla_prefill(x[0].data_ptr(), x[1].data_ptr(), v.data_ptr(), temp.data_ptr(), W.data_ptr(),
                                   b.data_ptr(), o.data_ptr(), None, None, B_, T_, K, heads, N // heads, N // heads,
                                   _lib.FAKLA_BF16, 0, ws.data_ptr(), wsb, stream))
        one = rows * N * 2
        out.view(-1).view(torch.uint8).copy_(ws[:2 * one])
    _lib.check(L.fakla_device_status(stream))
    sample = np.r_[0:64, rows - 1280:rows:7]
    for s in range(nsets):
        tp = to_np(temp)[sample] if s == nsets - 1 else None
        exp = O.phi(to_np(x[s])[sample], to_np(W), to_np(b), tp, heads)
        g = to_np(out[s])[sample]
        assert np.all(np.abs(g - exp) <= 2.0 ** -8 * np.abs(exp) + 1e-4), s


def test_phi_f32(cuda):
    from pulsartecture_b200.backend.interface import phi_map

    x = _normal((300, 200), 6, cuda, torch.float32)
    W, b = lpm_params(200, 96, seed=7)
    temp = _phi_like((300, 3), 8, cuda, torch.float32)
    got = phi_map(x, W.to(cuda), b.to(cuda), temp, 3)
    exp = O.phi(to_np(x), W.numpy(), b.numpy(), to_np(temp), 3)
    assert rel_l2(to_np(got), exp) < 1e-6


# ----------------------------------------------------------------- attention (phi given)
ATT_BF16_CASES = [
    (1, 1, 1, False, False),
    (1, 127, 2, True, False),
    (2, 128, 1, False, True),
    (1, 129, 3, True, True),
    (2, 1000, 2, False, True),
    (1, 4096, 1, True, False),
]


@pytest.mark.parametrize("D", [128, 64])
@pytest.mark.parametrize("B,T,H,with_temp,with_state", ATT_BF16_CASES + [(1, 3000, 2, True, True)])
def test_attention_bf16_tensor_core(cuda, B, T, H, with_temp, with_state, D):
    """Heads of 128, and of 64 (run in the 128-wide tiles with the second half
    held at zero); the long few-sequence cases take the segmented scan."""
    from pulsartecture_b200.backend.interface import fa_kla_attention_with_state

    q = _phi_like((B, T, H, D), 10, cuda, torch.bfloat16)
    k = _phi_like((B, T, H, D), 11, cuda, torch.bfloat16)
    v = _normal((B, T, H, D), 12, cuda, torch.bfloat16, 1 / np.sqrt(D))
    tp = _phi_like((B, T, H), 13, cuda, torch.bfloat16) if with_temp else None
    state = None
    S0 = z0 = None
    if with_state:
        S0 = _normal((B, H, D, D), 14, cuda, torch.float32, 0.02) + 0.05
        z0 = _phi_like((B, H, D), 15, cuda, torch.float32) * 20
        state = (S0, z0)
    out, (S, z) = fa_kla_attention_with_state(q, k, v, tp, state, True)
    eo, eS, ez = O.attention(to_np(q), to_np(k), to_np(v), None if tp is None else to_np(tp),
                             None if S0 is None else to_np(S0), None if z0 is None else to_np(z0))
    assert rel_l2(to_np(out), eo) < BF16_REL_L2
    assert np.abs(to_np(out) - eo).max() < BF16_MAX_ABS
    assert rel_l2(to_np(S), eS) < BF16_REL_L2
    assert rel_l2(to_np(z), ez) < BF16_REL_L2
    if state is not None:  # functional API: the input state is untouched
        assert torch.equal(state[0], S0)


@pytest.mark.parametrize("B,T,H,Df,Dv,with_temp", [
    (2, 256, 4, 64, 64, False),
    (1, 37, 3, 16, 24, True),
    (2, 300, 2, 128, 128, True),
    (1, 5, 1, 7, 200, False),
])
def test_attention_f32_cuda_cores(cuda, B, T, H, Df, Dv, with_temp):
    from pulsartecture_b200.backend.interface import fa_kla_attention_with_state

    q = _phi_like((B, T, H, Df), 20, cuda, torch.float32)
    k = _phi_like((B, T, H, Df), 21, cuda, torch.float32)
    v = _normal((B, T, H, Dv), 22, cuda, torch.float32)
    tp = _phi_like((B, T, H), 23, cuda, torch.float32) if with_temp else None
    out, (S, z) = fa_kla_attention_with_state(q, k, v, tp, None, True)
    eo, eS, ez = O.attention(to_np(q), to_np(k), to_np(v), None if tp is None else to_np(tp))
    assert rel_l2(to_np(out), eo) < F32_REL_L2
    assert rel_l2(to_np(S), eS) < F32_REL_L2
    assert rel_l2(to_np(z), ez) < F32_REL_L2


def test_attention_bf16_unaligned_views_take_the_general_path(cuda):
    from pulsartecture_b200.backend.interface import fa_kla_attention

    B, T, H, D = 1, 70, 2, 128
    base = _phi_like((B * T * H * D + 8,), 30, cuda, torch.bfloat16)
    q = base[1:1 + B * T * H * D].view(B, T, H, D)  # 2-byte offset: not 16-byte aligned
    k = _phi_like((B, T, H, D), 31, cuda, torch.bfloat16)
    v = _normal((B, T, H, D), 32, cuda, torch.bfloat16)
    out = fa_kla_attention(q, k, v, None)
    eo, _, _ = O.attention(to_np(q), to_np(k), to_np(v))
    assert rel_l2(to_np(out), eo) < BF16_REL_L2


def test_reference_contract_matches_reference_signature(cuda):
    """fa_kla_attention(q_mapped, k_mapped, v_reshaped, temp) with an explicit
    all-ones temp (what the reference module passes, tm_kla.py:306)."""
    from pulsartecture_b200.backend.interface import fa_kla_attention

    B, T, H, D = 2, 200, 2, 128
    q = _phi_like((B, T, H, D), 40, cuda, torch.bfloat16)
    k = _phi_like((B, T, H, D), 41, cuda, torch.bfloat16)
    v = _normal((B, T, H, D), 42, cuda, torch.bfloat16)
    out_ones = fa_kla_attention(q, k, v, torch.ones(B, T, H, device=cuda, dtype=torch.bfloat16))
    out_none = fa_kla_attention(q, k, v, None)
    assert out_ones.shape == v.shape and out_ones.dtype == v.dtype
    assert torch.equal(out_ones, out_none)  # scaling by 1.0 is exact


def test_interface_errors(cuda):
    from pulsartecture_b200.backend.interface import fa_kla_attention

    q = torch.rand(1, 4, 2, 8, device=cuda)
    with pytest.raises(RuntimeError):
        fa_kla_attention(q[0], q, q, None)
    with pytest.raises(RuntimeError):
        fa_kla_attention(q, q, q.double(), None)
    with pytest.raises(RuntimeError):
        fa_kla_attention(q.transpose(1, 2), q.transpose(1, 2), q.transpose(1, 2), None)
    with pytest.raises(RuntimeError):
        fa_kla_attention(q, q, q, torch.ones(1, 4, 3, device=cuda))
    with pytest.raises(RuntimeError):
        fa_kla_attention(q.cpu(), q.cpu(), q.cpu(), None)


# ----------------------------------------------------------------- decode
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_decode_mapped(cuda, dtype):
    from pulsartecture_b200.backend.interface import fa_kla_decode_step

    N, H, Df, Dv = 5, 3, 128, 128
    q = _phi_like((N, H, Df), 50, cuda, dtype)
    k = _phi_like((N, H, Df), 51, cuda, dtype)
    v = _normal((N, H, Dv), 52, cuda, dtype)
    tp = _phi_like((N, H), 53, cuda, dtype)
    S = _normal((N, H, Df, Dv), 54, cuda, torch.float32, 0.02)
    z = _phi_like((N, H, Df), 55, cuda, torch.float32)
    S0, z0 = to_np(S), to_np(z)
    out = fa_kla_decode_step(q, k, v, (S, z), temp=tp)
    eo, eS, ez = O.decode_step(to_np(q), to_np(k), to_np(v), S0, z0, to_np(tp))
    tol = F32_REL_L2 if dtype == torch.float32 else BF16_REL_L2
    assert rel_l2(to_np(out), eo) < tol
    assert rel_l2(to_np(S), eS) < 1e-6 and rel_l2(to_np(z), ez) < 1e-6


def test_decode_general_head_dims(cuda):
    from pulsartecture_b200.backend.interface import fa_kla_decode_step

    N, H, Df, Dv = 3, 2, 20, 30
    q = _phi_like((N, H, Df), 56, cuda, torch.float32)
    k = _phi_like((N, H, Df), 57, cuda, torch.float32)
    v = _normal((N, H, Dv), 58, cuda, torch.float32)
    S = torch.zeros(N, H, Df, Dv, device=cuda)
    z = torch.zeros(N, H, Df, device=cuda)
    out = fa_kla_decode_step(q, k, v, (S, z))
    eo, eS, ez = O.decode_step(to_np(q), to_np(k), to_np(v), np.zeros((N, H, Df, Dv)), np.zeros((N, H, Df)))
    assert rel_l2(to_np(out), eo) < F32_REL_L2 and rel_l2(to_np(S), eS) < 1e-6


@pytest.mark.parametrize("N,H", [(256, 4), (32, 32)])  # (32, 32): one GPU's share of an 8-way decode split
def test_decode_fused_phi_bf16(cuda, N, H):
    from pulsartecture_b200.backend.interface import fa_kla_decode_step

    Dk, M = 128, 128
    in_dim = H * Dk
    q = _normal((N, in_dim), 60, cuda, torch.bfloat16, 1 / np.sqrt(Dk))
    k = _normal((N, in_dim), 61, cuda, torch.bfloat16, 1 / np.sqrt(Dk))
    v = _normal((N, H, M), 62, cuda, torch.bfloat16, 1 / np.sqrt(Dk))
    W, b = lpm_params(in_dim, H * M, seed=63, dtype=torch.bfloat16)
    S = _normal((N, H, M, M), 64, cuda, torch.float32, 0.02)
    z = _phi_like((N, H, M), 65, cuda, torch.float32)
    S0, z0 = to_np(S), to_np(z)
    out = fa_kla_decode_step(q, k, v, (S, z), W.to(cuda), b.to(cuda))
    pq = O.phi(to_np(q), to_np(W), to_np(b)).reshape(N, H, M)
    pk = O.phi(to_np(k), to_np(W), to_np(b)).reshape(N, H, M)
    eo, eS, ez = O.decode_step(pq, pk, to_np(v), S0, z0)
    assert rel_l2(to_np(out), eo) < BF16_REL_L2
    assert np.abs(to_np(out) - eo).max() < BF16_MAX_ABS
    assert rel_l2(to_np(S), eS) < BF16_REL_L2 and rel_l2(to_np(z), ez) < BF16_REL_L2


@pytest.mark.parametrize("N,H", [(32, 32), (64, 32), (128, 32), (129, 32), (20, 16)])
def test_decode_map_rows_against_oracle(cuda, N, H):
    """The decode step's feature map, read back from the caller's workspace,
    against the oracle at the half-ulp bar, with the k-side temperature, for
    the few-sequence row sets of a split decode batch (fewer than 128 rows per
    A box, one row tile, and one row past it). The step's outputs are checked
    too."""
    from pulsartecture_b200 import _lib

    L = _lib.lib()
    Dk = M = 128
    in_dim = H * Dk
    q = _normal((N, in_dim), 70, cuda, torch.bfloat16, 1 / np.sqrt(Dk))
    k = _normal((N, in_dim), 71, cuda, torch.bfloat16, 1 / np.sqrt(Dk))
    v = _normal((N, H, M), 72, cuda, torch.bfloat16, 1 / np.sqrt(Dk))
    temp = _phi_like((N, H), 73, cuda, torch.bfloat16)
    W, b = lpm_params(in_dim, H * M, seed=74, dtype=torch.bfloat16)
    W, b = W.to(cuda), b.to(cuda)
    S = _normal((N, H, M, M), 75, cuda, torch.float32, 0.02)
    z = _phi_like((N, H, M), 76, cuda, torch.float32)
    S0, z0 = to_np(S), to_np(z)
    out = torch.empty(N, H, M, device=cuda, dtype=torch.bfloat16)
    wsb = L.fakla_decode_workspace_bytes(N, in_dim, H, M, M, _lib.FAKLA_BF16)
    ws = torch.zeros(wsb, device=cuda, dtype=torch.uint8)
    stream = torch.cuda.current_stream().cuda_stream
    _lib.check(L.fakla_decode(q.data_ptr(), k.data_ptr(), v.data_ptr(), temp.data_ptr(), W.data_ptr(), b.data_ptr(),
                              out.data_ptr(), S.data_ptr(), z.data_ptr(), N, in_dim, H, M, M, _lib.FAKLA_BF16,
                              ws.data_ptr(), wsb, stream))
    _lib.check(L.fakla_device_status(stream))
    one = N * H * M * 2
    phq = ws[:one].view(torch.bfloat16).view(N, H * M)
    phk = ws[wsb // 2:wsb // 2 + one].view(torch.bfloat16).view(N, H * M)
    eq = O.phi(to_np(q), to_np(W), to_np(b), None, H)
    ek = O.phi(to_np(k), to_np(W), to_np(b), to_np(temp), H)
    for got, exp in ((phq, eq), (phk, ek)):
        g = to_np(got)
        assert np.all(np.abs(g - exp) <= 2.0 ** -8 * np.abs(exp) + 1e-4)
    eo, eS, ez = O.decode_step(eq.reshape(N, H, M), ek.reshape(N, H, M), to_np(v), S0, z0)
    assert rel_l2(to_np(out), eo) < BF16_REL_L2 and np.abs(to_np(out) - eo).max() < BF16_MAX_ABS
    assert rel_l2(to_np(S), eS) < BF16_REL_L2 and rel_l2(to_np(z), ez) < BF16_REL_L2


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_zero_tokens(cuda, dtype):
    """T = 0 (and B = 0): an empty output, and the state of zero tokens — the
    input state unchanged, or zeros."""
    from pulsartecture_b200.attention import TMLinKernelAttn, fa_kla
    from pulsartecture_b200.backend.interface import fa_kla_attention_with_state
    from pulsartecture_b200.kernels import LearnablePositiveMap

    H, D = 2, 128
    for B, T in ((2, 0), (0, 5)):
        q = torch.rand(B, T, H, D, device=cuda).to(dtype)
        out, (S, z) = fa_kla_attention_with_state(q, q, q, None, None, True)
        assert out.shape == (B, T, H, D)
        assert torch.count_nonzero(S) == 0 and torch.count_nonzero(z) == 0
        S0 = torch.rand(B, H, D, D, device=cuda)
        z0 = torch.rand(B, H, D, device=cuda)
        _, (S1, z1) = fa_kla_attention_with_state(q, q, q, None, (S0, z0), True)
        assert torch.equal(S1, S0) and torch.equal(z1, z0)
        W, b = lpm_params(H * D, H * D, seed=3, dtype=dtype)
        out2, (S2, z2) = fa_kla(q.reshape(B, T, H * D), q.reshape(B, T, H * D), q, phi_weight=W.to(cuda),
                                phi_bias=b.to(cuda))
        assert out2.shape == (B, T, H, D) and torch.count_nonzero(S2) == 0
    mod = TMLinKernelAttn(H * D, LearnablePositiveMap(H * D, H * D, dtype=dtype), num_heads=H, qk_dim=D, v_dim=D,
                          dtype=dtype).to(cuda).eval()
    with torch.no_grad():
        y = mod(torch.zeros(2, 0, H * D, device=cuda, dtype=dtype))
    assert y.shape == (2, 0, H * D)
