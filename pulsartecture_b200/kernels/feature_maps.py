"""Kernel feature maps phi for FA-KLA, computed by libfakla's feature-map GEMMs.

Mirrors the reference's ultra_rwka/kernels/feature_maps.py: ``FeatureMap``
(15-27), ``RandomFourierFeatures`` (39-99), ``OrthogonalRandomFeatures``
(102-172) and ``LearnablePositiveMap`` (176-273). Same constructor arguments,
parameter and buffer names/shapes (reference state dicts load unchanged) and
the same initialisation draws in the same order, so a seed reproduces the
reference's parameters.

Every forward runs on the GPU: each linear layer and its activation is one
``fakla_feature_map`` launch (tcgen05 tensor cores for bf16 tiles, CUDA cores
otherwise); the random-Fourier maps use its cos/sin epilogue. There is no
CPU path.
"""
from __future__ import annotations

import math
import warnings
from abc import ABC, abstractmethod

import torch
import torch.nn as nn

from ..backend.interface import feature_map, phi_map


class FeatureMap(nn.Module, ABC):
    """Abstract base of kernel feature maps (feature_maps.py:15-27)."""

    def __init__(self, in_dim: int, feature_dim: int):
        super().__init__()
        self.in_dim = in_dim
        self.feature_dim = feature_dim

    @abstractmethod
    def forward(self, x: torch.Tensor) -> torch.Tensor:  # pragma: no cover - abstract
        pass

    def forward_into(self, x: torch.Tensor, out: torch.Tensor) -> torch.Tensor:
        """forward(x) written into ``out`` (contiguous, (..., feature_dim)).
        Maps of this package write directly; others are copied."""
        out.copy_(self.forward(x).reshape(out.shape))
        return out

    def extra_repr(self) -> str:
        return f"in_dim={self.in_dim}, feature_dim={self.feature_dim}"


def kernel_activation(module: nn.Module) -> str:
    """The fakla_feature_map activation equal to an activation module."""
    if isinstance(module, nn.GELU) and module.approximate == "none":
        return "gelu"
    if isinstance(module, nn.ReLU):
        return "relu"
    if isinstance(module, nn.Identity):
        return "identity"
    if isinstance(module, nn.Sigmoid):
        return "sigmoid"
    if isinstance(module, nn.Softplus) and module.beta == 1 and module.threshold == 20:
        return "softplus"
    raise NotImplementedError(
        f"activation {module!r} has no fakla_feature_map form (supported: GELU(approximate='none'), "
        "ReLU, Identity, Sigmoid, Softplus(beta=1, threshold=20))")


def run_mlp(x: torch.Tensor, layers: nn.Sequential, final_act: str) -> torch.Tensor:
    """A Sequential of Linear [activation] [Dropout] ... blocks, one
    fakla_feature_map launch per Linear with the activation that follows it
    fused; the last Linear gets ``final_act``."""
    mods = list(layers)
    i = 0
    h = x
    while i < len(mods):
        lin = mods[i]
        if not isinstance(lin, nn.Linear):
            raise NotImplementedError(f"expected nn.Linear in the MLP, got {lin!r}")
        i += 1
        if i == len(mods):
            act = final_act
        elif isinstance(mods[i], (nn.Linear, nn.Dropout)):
            act = "identity"
        else:
            act = kernel_activation(mods[i])
            i += 1
        h = feature_map(h, lin.weight, lin.bias, act)
        if i < len(mods) and isinstance(mods[i], nn.Dropout):
            h = mods[i](h)
            i += 1
    return h


class _TransposedWeight:
    """Row-major (n_proj, in_dim) copy of an (in_dim, n_proj) projection,
    refreshed when the source tensor changes (version counter)."""

    def __init__(self):
        self.key = None
        self.value = None

    def get(self, W: torch.Tensor) -> torch.Tensor:
        key = (W.data_ptr(), W._version, W.dtype, W.device, tuple(W.shape))
        if self.key != key:
            self.value = W.detach().t().contiguous()
            self.key = key
        return self.value


class RandomFourierFeatures(FeatureMap):
    """phi(x) = sqrt(1/P) [cos(x W + b), sin(x W + b)], W ~ N(0, gamma^2),
    b ~ U(0, 2 pi), P = feature_dim / 2 (feature_maps.py:39-99)."""

    def __init__(self, in_dim: int, feature_dim: int, gamma: float = 1.0, learnable: bool = False,
                 device=None, dtype=None):
        super().__init__(in_dim, feature_dim)
        if feature_dim % 2 != 0:
            raise ValueError(f"feature_dim (d_k={feature_dim}) must be even for RFFs using sin/cos pairs.")
        self.gamma = gamma
        self.learnable = learnable
        self.factory_kwargs = {"device": device, "dtype": dtype}
        num_projections = feature_dim // 2
        W_init = torch.randn(in_dim, num_projections, **self.factory_kwargs) * gamma
        b_init = torch.rand(num_projections, **self.factory_kwargs) * 2 * math.pi
        if learnable:
            warnings.warn("Making RFF projection matrix W learnable. This deviates from standard RFF theory.")
            self.W = nn.Parameter(W_init)
            self.b = nn.Parameter(b_init)
        else:
            self.register_buffer("W", W_init)
            self.register_buffer("b", b_init)
        self.scale_factor = math.sqrt(1.0 / num_projections)
        self._wt = _TransposedWeight()

    def _prep(self, x: torch.Tensor) -> torch.Tensor:
        if x.device != self.W.device or x.dtype != self.W.dtype:
            x = x.to(device=self.W.device, dtype=self.W.dtype)
        return x

    def _w_rows(self) -> torch.Tensor:
        # under autograd a learnable W must stay in the graph: transpose it there
        if torch.is_grad_enabled() and self.W.requires_grad:
            return self.W.t().contiguous()
        return self._wt.get(self.W)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        return feature_map(self._prep(x), self._w_rows(), self.b, "cossin", self.scale_factor)

    def forward_into(self, x: torch.Tensor, out: torch.Tensor) -> torch.Tensor:
        return feature_map(self._prep(x), self._w_rows(), self.b, "cossin", self.scale_factor, out=out)

    def extra_repr(self) -> str:
        return f"{super().extra_repr()}, gamma={self.gamma}, learnable={self.learnable}"


class OrthogonalRandomFeatures(RandomFourierFeatures):
    """Random Fourier features with W taken from the Q factor of a Gaussian
    matrix, times gamma (feature_maps.py:102-172)."""

    def __init__(self, in_dim: int, feature_dim: int, gamma: float = 1.0, learnable: bool = False,
                 device=None, dtype=None):
        FeatureMap.__init__(self, in_dim, feature_dim)
        if feature_dim % 2 != 0:
            raise ValueError(f"feature_dim (d_k={feature_dim}) must be even for ORF using sin/cos pairs.")
        if learnable:
            warnings.warn("Making ORF projection matrix W learnable. Orthogonality constraint will likely be "
                          "broken during training.")
        self.gamma = gamma
        self.learnable = learnable
        self.factory_kwargs = {"device": device, "dtype": dtype}
        num_projections = feature_dim // 2
        matrix_dim = max(in_dim, num_projections)
        gaussian_matrix = torch.randn(matrix_dim, matrix_dim, **self.factory_kwargs)
        q, _ = torch.linalg.qr(gaussian_matrix)
        W_init = q[:in_dim, :num_projections] * gamma
        b_init = torch.rand(num_projections, **self.factory_kwargs) * 2 * math.pi
        if learnable:
            self.W = nn.Parameter(W_init)
            self.b = nn.Parameter(b_init)
        else:
            self.register_buffer("W", W_init)
            self.register_buffer("b", b_init)
        self.scale_factor = math.sqrt(1.0 / num_projections)
        self._wt = _TransposedWeight()


class LearnablePositiveMap(FeatureMap):
    """phi(x) = act(MLP(x)) (feature_maps.py:176-273); hidden layers use GELU.
    One layer with 'elu+1' is FA-KLA's default map, which the prefill and
    decode entry points fuse with the scan."""

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

    # -- what the one-call FA-KLA entry points need
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

    def _prep(self, x: torch.Tensor) -> torch.Tensor:
        p = self.mlp[0].weight
        if x.device != p.device or x.dtype != p.dtype:
            x = x.to(device=p.device, dtype=p.dtype)
        return x

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        x = self._prep(x)
        if self.fusable:
            return phi_map(x, self.weight, self.bias)
        return run_mlp(x, self.mlp, self.activation_type)

    def forward_into(self, x: torch.Tensor, out: torch.Tensor) -> torch.Tensor:
        x = self._prep(x)
        if self.num_layers == 1:
            return feature_map(x, self.weight, self.bias, self.activation_type, out=out)
        return super().forward_into(x, out)

    def extra_repr(self) -> str:
        n = sum(1 for m in self.mlp if isinstance(m, nn.Linear))
        return f"{super().extra_repr()}, activation={self.activation_type}, mlp_layers={n}"
