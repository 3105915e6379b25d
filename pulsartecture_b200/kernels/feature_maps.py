"""Positive feature map phi for FA-KLA, computed by libfakla's phi kernel.

Mirrors ``FeatureMap`` and ``LearnablePositiveMap`` of the reference
(ultra_rwka/kernels/feature_maps.py:15-27 and 176-273): same constructor
arguments, same parameter names/shapes (``mlp.0.weight``, ``mlp.0.bias``, so
reference state dicts load unchanged) and the same initialisation
(kaiming-uniform a=sqrt(5), bias U(+-1/sqrt(fan_in)), feature_maps.py:224-232).

``forward`` runs on the GPU through the fused phi kernel for the map FA-KLA
uses by default: one linear layer followed by 'elu+1'. Other configurations of
the reference class (extra hidden layers, other final activations) are not on
this path and raise NotImplementedError.
"""
from __future__ import annotations

import math
from abc import ABC, abstractmethod

import torch
import torch.nn as nn

from ..backend.interface import phi_map


class FeatureMap(nn.Module, ABC):
    """Abstract base of kernel feature maps (feature_maps.py:15-27)."""

    def __init__(self, in_dim: int, feature_dim: int):
        super().__init__()
        self.in_dim = in_dim
        self.feature_dim = feature_dim

    @abstractmethod
    def forward(self, x: torch.Tensor) -> torch.Tensor:  # pragma: no cover - abstract
        pass

    def extra_repr(self) -> str:
        return f"in_dim={self.in_dim}, feature_dim={self.feature_dim}"


class LearnablePositiveMap(FeatureMap):
    """phi(x) = act(MLP(x)); the fused GPU path covers num_layers=1, act='elu+1'."""

    _supported_activations = {"elu+1", "relu", "softplus", "gelu"}

    def __init__(self, in_dim: int, feature_dim: int, hidden_dim: int | None = None,
                 num_layers: int = 1, activation: str = "elu+1", use_bias: bool = True,
                 initialize_weights: bool = True, device=None, dtype=None):
        super().__init__(in_dim, feature_dim)
        self.activation_type = activation.lower()
        self.factory_kwargs = {"device": device, "dtype": dtype}
        if num_layers < 1:
            raise ValueError("num_layers must be at least 1.")
        if self.activation_type not in self._supported_activations:
            raise ValueError(f"Unsupported activation: {activation}. Choose from {self._supported_activations}")
        _hidden_dim = hidden_dim if hidden_dim is not None else max(in_dim, feature_dim)
        layers = []
        current = in_dim
        for i in range(num_layers):
            last = i == num_layers - 1
            out_dim = feature_dim if last else _hidden_dim
            lin = nn.Linear(current, out_dim, bias=use_bias, **self.factory_kwargs)
            if initialize_weights:
                nn.init.kaiming_uniform_(lin.weight, a=math.sqrt(5))
                if use_bias:
                    fan_in, _ = nn.init._calculate_fan_in_and_fan_out(lin.weight)
                    bound = 1 / math.sqrt(fan_in) if fan_in > 0 else 0
                    nn.init.uniform_(lin.bias, -bound, bound)
            layers.append(lin)
            if not last:
                layers.append(nn.GELU())
                current = _hidden_dim
        self.mlp = nn.Sequential(*layers)
        self.num_layers = num_layers

    # -- what the fused FA-KLA kernels need
    @property
    def fusable(self) -> bool:
        """True when phi is exactly one linear layer followed by elu+1."""
        return self.num_layers == 1 and self.activation_type == "elu+1"

    @property
    def weight(self) -> torch.Tensor:
        return self.mlp[0].weight

    @property
    def bias(self):
        return self.mlp[0].bias

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        if not self.fusable:
            raise NotImplementedError(
                "LearnablePositiveMap on the FA-KLA GPU path supports num_layers=1 with "
                f"activation 'elu+1' (got num_layers={self.num_layers}, activation={self.activation_type!r})")
        p = self.weight
        if x.device != p.device or x.dtype != p.dtype:
            x = x.to(device=p.device, dtype=p.dtype)
        return phi_map(x, p, self.bias)

    def extra_repr(self) -> str:
        n = sum(1 for m in self.mlp if isinstance(m, nn.Linear))
        return f"{super().extra_repr()}, activation={self.activation_type}, mlp_layers={n}"
