"""End-to-end language-model harness around FA-KLA.

The reference ships no model: ultra_rwka/models/full.py, base_model.py,
variants/* and configs/* are empty files. This module is this package's own
composition of reference-style parts with FA-KLA (`TMLinKernelAttn`, default
elu+1 map) running on libfakla, and is labelled as such wherever it is
measured:

    x = embed(ids)
    L x [ x += W_o TMLinKernelAttn(LN(x));  x += MoE(LN(x)) ]
    logits = head(LN(x))

The MoE layer follows the reference's top-k gating (ultra_rwka/MoE/gating.py:
112-145: the top-k gate logits, a softmax over those k, no noise at
inference) over GELU MLP experts (the shape of ultra_rwka/MoE/branches.py
MLPBranch). The reference's IDAM memory and wavelet mixing are left out: the
repository gives them no defaults, and the wavelet projection needs a
backend operation the reference does not implement.

Everything but the attention runs on PyTorch / cuBLAS; the attention
sublayers are the FA-KLA kernels of this package.
"""
from __future__ import annotations

import math
import torch
import torch.nn as nn
import torch.nn.functional as F

from .attention import TMLinKernelAttn
from .kernels import LearnablePositiveMap


class MoEFeedForward(nn.Module):
    """Top-k of n_experts GELU MLPs (d_model -> d_ff -> d_model), weights = a
    softmax over the k largest gate logits (gating.py:136-144)."""

    def __init__(self, d_model: int, d_ff: int, n_experts: int = 8, top_k: int = 2, device=None, dtype=None):
        super().__init__()
        if not 1 <= top_k <= n_experts:
            raise ValueError(f"top_k must be in [1, n_experts], got {top_k}")
        fk = {"device": device, "dtype": dtype}
        self.n_experts, self.top_k = n_experts, top_k
        self.gate = nn.Linear(d_model, n_experts, bias=False, **fk)
        self.w_in = nn.Parameter(torch.empty(n_experts, d_ff, d_model, **fk))
        self.b_in = nn.Parameter(torch.zeros(n_experts, d_ff, **fk))
        self.w_out = nn.Parameter(torch.empty(n_experts, d_model, d_ff, **fk))
        self.b_out = nn.Parameter(torch.zeros(n_experts, d_model, **fk))
        for e in range(n_experts):
            nn.init.kaiming_uniform_(self.w_in[e], a=math.sqrt(5))
            nn.init.kaiming_uniform_(self.w_out[e], a=math.sqrt(5))

    def routing(self, x2: torch.Tensor):
        """(rows, d) -> expert indices (rows, k) and weights (rows, k)."""
        logits = self.gate(x2)
        top_logits, top_idx = torch.topk(logits, self.top_k, dim=-1)
        weights = F.softmax(top_logits.float(), dim=-1).to(x2.dtype)
        return top_idx, weights

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        lead = x.shape[:-1]
        x2 = x.reshape(-1, x.shape[-1])
        idx, w = self.routing(x2)
        out = torch.zeros_like(x2)
        flat_idx = idx.reshape(-1)
        flat_w = w.reshape(-1)
        tok = torch.arange(x2.shape[0], device=x.device).repeat_interleave(self.top_k)
        order = torch.argsort(flat_idx)
        counts = torch.bincount(flat_idx, minlength=self.n_experts).tolist()
        start = 0
        for e, n in enumerate(counts):
            if n == 0:
                continue
            sel = order[start:start + n]
            start += n
            rows = tok[sel]
            h = F.gelu(F.linear(x2[rows], self.w_in[e], self.b_in[e]))
            y = F.linear(h, self.w_out[e], self.b_out[e])
            out.index_add_(0, rows, y * flat_w[sel, None])
        return out.reshape(*lead, -1)


class FaklaBlock(nn.Module):
    """Pre-norm block: FA-KLA attention (with an output projection back to
    d_model) and an MoE feed-forward, each added to the residual stream."""

    def __init__(self, d_model: int, n_heads: int, head_dim: int, d_ff: int, n_experts: int, top_k: int,
                 device=None, dtype=None):
        super().__init__()
        fk = {"device": device, "dtype": dtype}
        feat = n_heads * head_dim
        self.ln_attn = nn.LayerNorm(d_model, **fk)
        self.attn = TMLinKernelAttn(d_model, LearnablePositiveMap(feat, feat, **fk), num_heads=n_heads,
                                    qk_dim=head_dim, v_dim=head_dim, **fk)
        self.proj_out = nn.Linear(feat, d_model, **fk)
        self.ln_ff = nn.LayerNorm(d_model, **fk)
        self.ff = MoEFeedForward(d_model, d_ff, n_experts, top_k, **fk)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        x = x + self.proj_out(self.attn(self.ln_attn(x)))
        return x + self.ff(self.ln_ff(x))


class FaklaLM(nn.Module):
    """Token ids (B, T) -> next-token logits (B, T, vocab). Defaults: 12
    layers, d_model 1024, 16 FA-KLA heads of 64, top-2 of 8 experts with
    d_ff 4096, vocabulary 32000."""

    def __init__(self, vocab: int = 32000, d_model: int = 1024, n_layers: int = 12, n_heads: int = 16,
                 head_dim: int = 64, d_ff: int = 4096, n_experts: int = 8, top_k: int = 2, device=None,
                 dtype=None):
        super().__init__()
        fk = {"device": device, "dtype": dtype}
        self.embed = nn.Embedding(vocab, d_model, **fk)
        self.blocks = nn.ModuleList([FaklaBlock(d_model, n_heads, head_dim, d_ff, n_experts, top_k, **fk)
                                     for _ in range(n_layers)])
        self.ln_f = nn.LayerNorm(d_model, **fk)
        self.head = nn.Linear(d_model, vocab, bias=False, **fk)

    def forward(self, ids: torch.Tensor) -> torch.Tensor:
        x = self.embed(ids)
        for blk in self.blocks:
            x = blk(x)
        return self.head(self.ln_f(x))
