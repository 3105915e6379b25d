"""The oracle itself, pinned before it is trusted (CPU only).

* against the golden fixtures made from the reference (tests/golden/);
* against the reference's own fa_kla_attention_cpu compiled in place
  (oracle/_ref), on shapes the fixtures do not cover;
* against size-independent properties: state chaining, decode == T=1 prefill.
"""
import os

import numpy as np
import pytest
import torch

from oracle import build_ref
from oracle import fakla_oracle as O
from tests.helpers import lpm_params, rel_l2

GOLDEN = os.path.join(os.path.dirname(__file__), "golden", "fakla_golden.npz")


@pytest.fixture(scope="module")
def golden():
    return np.load(GOLDEN)


def gen(shape, seed, kind="normal", lo=0.0, hi=1.0):
    g = torch.Generator().manual_seed(seed)
    if kind == "normal":
        return torch.randn(*shape, generator=g)
    return torch.rand(*shape, generator=g) * (hi - lo) + lo


def checksum(t):
    a = torch.as_tensor(t).double().reshape(-1)
    return np.array([a.sum().item(), (a * a).sum().item(), a[:16].sum().item(), float(a.numel())])


def test_lpm_init_matches_reference_checksums(golden):
    from pulsartecture_b200.kernels.feature_maps import LearnablePositiveMap

    torch.manual_seed(0)
    m = LearnablePositiveMap(256, 256)
    np.testing.assert_allclose(checksum(m.weight.detach()), golden["small_W_checksum"], rtol=1e-12)
    np.testing.assert_allclose(checksum(m.bias.detach()), golden["small_b_checksum"], rtol=1e-12)


def test_oracle_small_against_golden(golden):
    B, T, H, D = 2, 256, 4, 64
    torch.manual_seed(0)
    from pulsartecture_b200.kernels.feature_maps import LearnablePositiveMap

    m = LearnablePositiveMap(H * D, H * D)
    W, b = m.weight.detach().numpy(), m.bias.detach().numpy()
    q, k, v = gen((B, T, H, D), 101), gen((B, T, H, D), 102), gen((B, T, H, D), 103)
    out, S, z = O.prefill(q.numpy(), k.numpy(), v.numpy(), W, b)
    assert rel_l2(out, golden["small_out"]) < 1e-6
    assert rel_l2(S, golden["small_S"]) < 1e-6
    assert rel_l2(z, golden["small_z"]) < 1e-6
    pq = O.phi(q.numpy().reshape(B, T, H * D), W, b)
    np.testing.assert_allclose(checksum(torch.from_numpy(pq)), golden["small_phi_q_checksum"], rtol=1e-6)


def test_oracle_ragged_temp_against_golden(golden):
    q = gen((1, 37, 3, 16), 201, "uniform", 0.1, 1.5)
    k = gen((1, 37, 3, 16), 202, "uniform", 0.1, 1.5)
    v = gen((1, 37, 3, 24), 203)
    tp = gen((1, 37, 3), 204, "uniform", 0.5, 1.5)
    for prec in ("f64", "f32"):
        out, S, z = O.attention(q.numpy(), k.numpy(), v.numpy(), tp.numpy(), precision=prec)
        assert rel_l2(out, golden["ragged_out"]) < 1e-6
        assert rel_l2(S, golden["ragged_S"]) < 1e-6
        assert rel_l2(z, golden["ragged_z"]) < 1e-6


def test_oracle_single_token_against_golden(golden):
    q = gen((3, 1, 1, 8), 301, "uniform", 0.1, 1.0)
    k = gen((3, 1, 1, 8), 302, "uniform", 0.1, 1.0)
    v = gen((3, 1, 1, 8), 303)
    tp = gen((3, 1, 1), 304, "uniform", 0.5, 1.5)
    out, _, _ = O.attention(q.numpy(), k.numpy(), v.numpy(), tp.numpy())
    assert rel_l2(out, golden["t1_out"]) < 1e-6


@pytest.fixture(scope="module")
def ref_kernel():
    if build_ref.built_module_path() is None:
        if build_ref.build() is None:
            pytest.skip("reference kernel not built and reference checkout absent")
    return build_ref.load()


@pytest.mark.parametrize("B,T,H,Df,Dv,with_temp", [
    (1, 1, 1, 4, 4, False),
    (2, 129, 3, 32, 16, True),
    (1, 300, 2, 128, 128, True),
    (3, 64, 1, 7, 9, False),
])
def test_oracle_against_compiled_reference(ref_kernel, B, T, H, Df, Dv, with_temp):
    q = gen((B, T, H, Df), 11, "uniform", 0.2, 1.2)
    k = gen((B, T, H, Df), 12, "uniform", 0.2, 1.2)
    v = gen((B, T, H, Dv), 13)
    tp = gen((B, T, H), 14, "uniform", 0.5, 2.0) if with_temp else torch.ones(B, T, H)
    r = ref_kernel.fa_kla_attention_cpu(q, k, v, tp).numpy()
    o64, _, _ = O.attention(q.numpy(), k.numpy(), v.numpy(), tp.numpy() if with_temp else None)
    o32, _, _ = O.attention(q.numpy(), k.numpy(), v.numpy(), tp.numpy(), precision="f32")
    assert rel_l2(r, o64) < 2e-6
    assert rel_l2(r, o32) < 2e-6


def test_reference_rejects_what_the_interface_rejects(ref_kernel):
    """The reference's input checks (cpu_kernels.cpp:43-54) raise RuntimeError;
    the CUDA front end raises the same type for the same mistakes."""
    q = torch.rand(1, 4, 2, 8)
    with pytest.raises(RuntimeError):
        ref_kernel.fa_kla_attention_cpu(q[0], q, q, torch.ones(1, 4, 2))
    with pytest.raises(RuntimeError):
        ref_kernel.fa_kla_attention_cpu(q, q, q, torch.ones(1, 4, 2, dtype=torch.float64))
    with pytest.raises(RuntimeError):
        ref_kernel.fa_kla_attention_cpu(q.transpose(1, 2), q.transpose(1, 2), q.transpose(1, 2),
                                        torch.ones(1, 2, 4))


def test_state_chaining_property():
    rng = np.random.default_rng(5)
    B, T, H, Df, Dv = 2, 90, 2, 12, 10
    q = rng.uniform(0.1, 1, (B, T, H, Df))
    k = rng.uniform(0.1, 1, (B, T, H, Df))
    v = rng.standard_normal((B, T, H, Dv))
    tp = rng.uniform(0.5, 1.5, (B, T, H))
    full, S, z = O.attention(q, k, v, tp)
    o1, S1, z1 = O.attention(q[:, :31], k[:, :31], v[:, :31], tp[:, :31])
    o2, S2, z2 = O.attention(q[:, 31:], k[:, 31:], v[:, 31:], tp[:, 31:], S1, z1)
    assert rel_l2(np.concatenate([o1, o2], 1), full) < 1e-13
    assert rel_l2(S2, S) < 1e-13 and rel_l2(z2, z) < 1e-13


def test_decode_equals_single_token_prefill():
    rng = np.random.default_rng(6)
    N, H, Df, Dv = 4, 3, 8, 6
    S0 = rng.standard_normal((N, H, Df, Dv)) * 0.02
    z0 = rng.uniform(0.5, 1.5, (N, H, Df))
    q = rng.uniform(0.1, 1, (N, H, Df))
    k = rng.uniform(0.1, 1, (N, H, Df))
    v = rng.standard_normal((N, H, Dv))
    out, S1, z1 = O.decode_step(q, k, v, S0, z0)
    S_exp = S0 + k[..., :, None] * v[..., None, :]
    z_exp = z0 + k
    num = np.einsum("nhf,nhfd->nhd", q, S_exp)
    den = np.einsum("nhf,nhf->nh", q, z_exp)
    assert rel_l2(S1, S_exp) < 1e-14 and rel_l2(z1, z_exp) < 1e-14
    assert rel_l2(out, num / (den[..., None] + 1e-12)) < 1e-14


def test_bf16_rounding_matches_torch():
    x = torch.randn(10000) * 10
    ours = O.round_bf16(x.numpy())
    np.testing.assert_array_equal(ours, x.bfloat16().float().numpy())


def test_phi_oracle_matches_torch():
    W, b = lpm_params(48, 32, seed=3, dtype=torch.float64)
    x = torch.randn(5, 7, 48, dtype=torch.float64)
    exp = torch.nn.functional.elu(x @ W.T + b) + 1.0
    got = O.phi(x.numpy(), W.numpy(), b.numpy())
    assert rel_l2(got, exp.numpy()) < 1e-14


def test_oracle_rejects_head_dims_beyond_its_limit():
    """The C restatement returns an error (and writes nothing) for head dims
    above 256 instead of leaving the outputs unset."""
    import ctypes

    lib = O._load()
    for fn, dt, p in ((lib.fakla_oracle_attention_f64, np.float64, ctypes.c_double),
                      (lib.fakla_oracle_attention_f32, np.float32, ctypes.c_float)):
        q = np.zeros((1, 1, 1, 300), dt)
        v = np.zeros((1, 1, 1, 8), dt)
        out = np.full((1, 1, 1, 8), 7, dt)
        ptr = lambda a: a.ctypes.data_as(ctypes.POINTER(p))  # noqa: E731
        rc = fn(ptr(q), ptr(q), ptr(v), None, ptr(out), None, None, None, None, 1, 1, 1, 300, 8)
        assert rc == -1
        assert (out == 7).all()
    with pytest.raises(ValueError):
        O.attention(np.zeros((1, 1, 1, 300)), np.zeros((1, 1, 1, 300)), np.zeros((1, 1, 1, 8)))
