"""Q/K/V projection layer feeding FA-KLA.

Same constructor, parameters and forward as the reference's
``LinearProjection`` (ultra_rwka/components/projections.py:8-125): nn.Linear,
optional LayerNorm, optional activation, kaiming/xavier initialisation. The
GEMM itself is a plain library GEMM (cuBLAS through torch); it sits upstream
of the FA-KLA kernels.
"""
from __future__ import annotations

import math
from typing import Optional, Type, Union

import torch
import torch.nn as nn


class LinearProjection(nn.Module):
    def __init__(self, in_dim: int, out_dim: int, use_bias: bool = True,
                 activation_cls: Optional[Type[nn.Module]] = None, use_norm: bool = False,
                 norm_eps: float = 1e-5, norm_affine: bool = True,
                 initialize: Union[str, bool] = "kaiming_uniform", device=None, dtype=None):
        super().__init__()
        self.in_dim = in_dim
        self.out_dim = out_dim
        self.use_bias = use_bias
        self.use_norm = use_norm
        self.factory_kwargs = {"device": device, "dtype": dtype}
        self.linear = nn.Linear(in_dim, out_dim, bias=use_bias, **self.factory_kwargs)
        self.norm: Optional[nn.LayerNorm] = None
        if use_norm:
            self.norm = nn.LayerNorm(out_dim, eps=norm_eps, elementwise_affine=norm_affine, **self.factory_kwargs)
        self.activation: Optional[nn.Module] = activation_cls() if activation_cls is not None else None
        if isinstance(initialize, str):
            self._initialize_weights(initialize)
        elif initialize is True:
            self._initialize_weights("kaiming_uniform")

    def _initialize_weights(self, scheme: str) -> None:
        scheme = scheme.lower()
        if scheme == "kaiming_uniform":
            nn.init.kaiming_uniform_(self.linear.weight, a=math.sqrt(5))
            if self.use_bias and self.linear.bias is not None:
                fan_in, _ = nn.init._calculate_fan_in_and_fan_out(self.linear.weight)
                bound = 1 / math.sqrt(fan_in) if fan_in > 0 else 0
                nn.init.uniform_(self.linear.bias, -bound, bound)
        elif scheme == "xavier_uniform":
            nn.init.xavier_uniform_(self.linear.weight)
            if self.use_bias and self.linear.bias is not None:
                nn.init.zeros_(self.linear.bias)
        else:
            raise ValueError(f"initialize={scheme!r} is not a known scheme (use 'kaiming_uniform', "
                             "'xavier_uniform', True or False)")

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        if x.dtype != self.linear.weight.dtype:
            x = x.to(dtype=self.linear.weight.dtype)
        x = self.linear(x)
        if self.norm is not None:
            x = self.norm(x)
        if self.activation is not None:
            x = self.activation(x)
        return x

    def extra_repr(self) -> str:
        parts = [f"{self.in_dim} -> {self.out_dim}", f"bias={self.use_bias}"]
        if self.norm is not None:
            parts.append(f"layernorm(eps={self.norm.eps}, affine={self.norm.elementwise_affine})")
        if self.activation is not None:
            parts.append(type(self.activation).__name__)
        return ", ".join(parts)
