"""The end-to-end LM harness (pulsartecture_b200/lm_harness.py) on the GPU
against the same composition restated in float64 torch on the CPU, with
FA-KLA from the float64 oracle (oracle/fakla_grad_oracle.py).

Bars: fp32 logits rel-L2 <= 1e-4 (a stack of layers: the per-kernel bar is
1e-5); bf16 logits rel-L2 <= 3e-2 (bf16 activations through every layer).
"""
import numpy as np
import pytest
import torch
import torch.nn.functional as F

from oracle import fakla_grad_oracle as G
from tests.helpers import rel_l2, to_np

pytestmark = pytest.mark.gpu


def _restated_logits(model, ids):
    """float64 forward of FaklaLM with the oracle's FA-KLA; expert choice
    taken from the float64 gate logits."""
    sd = {k: v.detach().double().cpu() for k, v in model.state_dict().items()}
    x = sd["embed.weight"][ids.cpu()]
    B, T, _ = x.shape
    for i, blk in enumerate(model.blocks):
        p = f"blocks.{i}."
        H, D = blk.attn.num_heads, blk.attn.qk_head_dim
        h = F.layer_norm(x, x.shape[-1:], sd[p + "ln_attn.weight"], sd[p + "ln_attn.bias"])

        def lin(name):
            return h @ sd[p + f"attn.{name}.linear.weight"].T + sd[p + f"attn.{name}.linear.bias"]

        out, _, _ = G.prefill(lin("proj_q"), lin("proj_k"), lin("proj_v").reshape(B, T, H, D),
                              sd[p + "attn.feature_mapper.mlp.0.weight"], sd[p + "attn.feature_mapper.mlp.0.bias"])
        x = x + out.reshape(B, T, H * D) @ sd[p + "proj_out.weight"].T + sd[p + "proj_out.bias"]
        h = F.layer_norm(x, x.shape[-1:], sd[p + "ln_ff.weight"], sd[p + "ln_ff.bias"]).reshape(B * T, -1)
        logits = h @ sd[p + "ff.gate.weight"].T
        top, idx = torch.topk(logits, blk.ff.top_k, dim=-1)
        w = torch.softmax(top, dim=-1)
        y = torch.zeros_like(h)
        for j in range(blk.ff.top_k):
            for e in range(blk.ff.n_experts):
                rows = (idx[:, j] == e).nonzero().flatten()
                if rows.numel() == 0:
                    continue
                a = F.gelu(h[rows] @ sd[p + "ff.w_in"][e].T + sd[p + "ff.b_in"][e])
                y[rows] += w[rows, j, None] * (a @ sd[p + "ff.w_out"][e].T + sd[p + "ff.b_out"][e])
        x = x + y.reshape(B, T, -1)
    x = F.layer_norm(x, x.shape[-1:], sd["ln_f.weight"], sd["ln_f.bias"])
    return x @ sd["head.weight"].T


@pytest.mark.parametrize("dtype,bar", [(torch.float32, 1e-4), (torch.bfloat16, 3e-2)])
def test_lm_harness_matches_float64_restatement(cuda, dtype, bar):
    from pulsartecture_b200.lm_harness import FaklaLM

    torch.manual_seed(0)
    model = FaklaLM(vocab=500, d_model=256, n_layers=2, n_heads=4, head_dim=64, d_ff=512, n_experts=4,
                    top_k=2, dtype=dtype).to(cuda).eval()
    g = torch.Generator().manual_seed(1)
    ids = torch.randint(0, 500, (2, 200), generator=g).to(cuda)
    with torch.no_grad():
        if dtype == torch.bfloat16:  # the folded q/k/v + map + scan path on tensor cores
            assert model.blocks[0].attn._qkv_foldable(model.embed(ids))
        got = model(ids)
    assert got.dtype == dtype and got.shape == (2, 200, 500)
    exp = _restated_logits(model, ids)
    assert rel_l2(to_np(got), exp.numpy()) < bar
