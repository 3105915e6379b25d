"""The fused prefill and the decode step captured in a CUDA graph and replayed:
every call is stream-ordered (no host synchronisation, no allocation outside
torch's caching allocator), so a captured step replays the same kernels.
Replays on fresh inputs equal the eager calls on those inputs bit for bit
(the kernels are deterministic), at sizes that run the single-CTA and the
CTA-pair feature-map GEMMs (GPU only)."""
import pytest
import torch

from tests.helpers import lpm_params

pytestmark = pytest.mark.gpu


def _inputs(B, T, H, D, seed, dev):
    g = torch.Generator().manual_seed(seed)
    mk = lambda *s: (torch.randn(*s, generator=g) / D ** 0.5).bfloat16().to(dev)  # noqa: E731
    return mk(B, T, H * D), mk(B, T, H * D), mk(B, T, H, D)


@pytest.mark.parametrize("B,T,H", [(2, 300, 2), (2, 1024, 16)])
def test_prefill_graph_replay_equals_eager(cuda, B, T, H):
    from pulsartecture_b200.attention import fa_kla

    D = 128
    W, b = lpm_params(H * D, H * D, seed=5, dtype=torch.bfloat16)
    W, b = W.to(cuda), b.to(cuda)
    q, k, v = _inputs(B, T, H, D, 1, cuda)
    # warm-up on a side stream (first-call set-up stays out of the capture)
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        fa_kla(q, k, v, phi_weight=W, phi_bias=b)
    torch.cuda.current_stream().wait_stream(s)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        out_g, (S_g, z_g) = fa_kla(q, k, v, phi_weight=W, phi_bias=b)
    for seed in (2, 3):
        nq, nk, nv = _inputs(B, T, H, D, seed, cuda)
        q.copy_(nq)
        k.copy_(nk)
        v.copy_(nv)
        graph.replay()
        out_e, (S_e, z_e) = fa_kla(nq, nk, nv, phi_weight=W, phi_bias=b)
        torch.cuda.synchronize()
        assert torch.equal(out_g, out_e)
        assert torch.equal(S_g, S_e) and torch.equal(z_g, z_e)


def test_decode_steps_graph_replay_equals_eager(cuda):
    """Four decode tokens captured as one graph; the state evolves in place."""
    from pulsartecture_b200.attention import fa_kla_decode

    N, H, D = 8, 4, 128
    W, b = lpm_params(H * D, H * D, seed=6, dtype=torch.bfloat16)
    W, b = W.to(cuda), b.to(cuda)
    g = torch.Generator().manual_seed(9)
    toks = [tuple((torch.randn(*s, generator=g) / D ** 0.5).bfloat16().to(cuda)
                  for s in ((N, H * D), (N, H * D), (N, H, D))) for _ in range(4)]
    S0 = (torch.randn(N, H, D, D, generator=g) * 0.02).to(cuda)
    z0 = (torch.rand(N, H, D, generator=g) + 0.5).to(cuda)
    S, z = S0.clone(), z0.clone()
    st = torch.cuda.Stream()
    st.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(st):
        fa_kla_decode(*toks[0], (S.clone(), z.clone()), phi_weight=W, phi_bias=b)
    torch.cuda.current_stream().wait_stream(st)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        outs = [fa_kla_decode(*t, (S, z), phi_weight=W, phi_bias=b)[0] for t in toks]
    for _ in range(2):
        S.copy_(S0)
        z.copy_(z0)
        graph.replay()
        Se, ze = S0.clone(), z0.clone()
        eager = [fa_kla_decode(*t, (Se, ze), phi_weight=W, phi_bias=b)[0] for t in toks]
        torch.cuda.synchronize()
        for a, e in zip(outs, eager):
            assert torch.equal(a, e)
        assert torch.equal(S, Se) and torch.equal(z, ze)
