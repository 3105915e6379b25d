"""Dynamic mixture of kernel feature maps, on libfakla.

Mirrors ``GateNet`` and ``KernelFeatureMixer`` of the reference
(ultra_rwka/kernels/mixer.py:11-66 and 153-261): same constructor arguments,
parameter names and initialisation (xavier-uniform weights, zero biases),
same context handling and errors.

    kappa_t = sum_i pi_t^(i) FeatureMap_i(x_t),  pi_t = softmax(GateNet([x_t, context_t]))

GateNet's layers run as fakla_feature_map launches; every base map writes its
features into one (n_maps, rows, F) buffer; fakla_mix_features applies the
softmax and the weighted sum in one pass.
"""
from __future__ import annotations

import warnings
from typing import Optional, Sequence, Type

import torch
import torch.nn as nn

from ..backend.interface import mix_features
from .feature_maps import FeatureMap, run_mlp


class GateNet(nn.Module):
    """MLP producing the mixture logits (mixer.py:11-66)."""

    def __init__(self, input_dim: int, num_outputs: int, hidden_dim: Optional[int] = None,
                 num_layers: int = 1, use_bias: bool = True, activation_cls: Type[nn.Module] = nn.GELU,
                 dropout_p: float = 0.0, initialize_weights: bool = True, device=None, dtype=None):
        super().__init__()
        self.factory_kwargs = {"device": device, "dtype": dtype}
        self.input_dim = input_dim
        self.num_outputs = num_outputs
        self.dropout_p = dropout_p
        if num_layers < 1:
            raise ValueError("GateNet num_layers must be at least 1.")
        if not (0.0 <= dropout_p < 1.0):
            raise ValueError(f"dropout_p must be between 0.0 and 1.0, got {dropout_p}")
        _hidden_dim = hidden_dim if hidden_dim is not None else max(input_dim // 2, num_outputs)
        layers = []
        current = input_dim
        for i in range(num_layers):
            last = i == num_layers - 1
            out_dim = num_outputs if last else _hidden_dim
            lin = nn.Linear(current, out_dim, bias=use_bias, **self.factory_kwargs)
            if initialize_weights:
                nn.init.xavier_uniform_(lin.weight)
                if use_bias and lin.bias is not None:
                    nn.init.zeros_(lin.bias)
            layers.append(lin)
            if not last:
                layers.append(activation_cls())
                if dropout_p > 0.0:
                    layers.append(nn.Dropout(p=dropout_p))
                current = _hidden_dim
        self.network = nn.Sequential(*layers)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        """Gate logits (no activation after the last layer)."""
        return run_mlp(x, self.network, "identity")


class KernelFeatureMixer(nn.Module):
    """kappa_t = sum_i softmax(GateNet(x_t [, context_t]))_i FeatureMap_i(x_t)
    (mixer.py:153-261)."""

    def __init__(self, feature_maps: Sequence[FeatureMap], gate_input_dim: int,
                 gate_hidden_dim: Optional[int] = None, gate_layers: int = 1,
                 gate_activation_cls: Type[nn.Module] = nn.GELU, gate_dropout_p: float = 0.0,
                 device=None, dtype=None):
        super().__init__()
        if not feature_maps:
            raise ValueError("feature_maps list/tuple cannot be empty.")
        self.feature_maps = nn.ModuleList(feature_maps)
        self.num_feature_maps = len(feature_maps)
        self.feature_dim = feature_maps[0].feature_dim
        for i, fm in enumerate(self.feature_maps):
            if not isinstance(fm, FeatureMap):
                warnings.warn(f"Item at index {i} is not an instance of FeatureMap base class.")
            if fm.feature_dim != self.feature_dim:
                raise ValueError(f"Feature map at index {i} has dimension {fm.feature_dim}, "
                                 f"but expected {self.feature_dim} based on the first map.")
        self.gate_net = GateNet(input_dim=gate_input_dim, num_outputs=self.num_feature_maps,
                                hidden_dim=gate_hidden_dim, num_layers=gate_layers,
                                activation_cls=gate_activation_cls, dropout_p=gate_dropout_p,
                                device=device, dtype=dtype)
        self.factory_kwargs = {"device": device, "dtype": dtype}

    def _gate_input(self, x: torch.Tensor, context: Optional[torch.Tensor]) -> torch.Tensor:
        # context handling of mixer.py:217-233
        if context is not None:
            if x.shape[:-1] != context.shape[:-1]:
                if context.ndim == x.ndim - 1 and x.ndim > 1:
                    context = context.unsqueeze(1).expand(-1, x.size(1), -1)
                elif context.ndim != x.ndim:
                    raise ValueError(f"Shape mismatch for concat: x {x.shape}, context {context.shape}")
            if x.shape[:-1] == context.shape[:-1]:
                gate_input = torch.cat([x, context.to(dtype=x.dtype)], dim=-1)
                if gate_input.shape[-1] != self.gate_net.input_dim:
                    raise ValueError(f"Concatenated input dim ({gate_input.shape[-1]}) does not match GateNet "
                                     f"expected input dim ({self.gate_net.input_dim}).")
            else:
                raise ValueError(f"Cannot automatically concatenate x ({x.shape}) and context ({context.shape})")
        else:
            gate_input = x
            if gate_input.shape[-1] != self.gate_net.input_dim:
                raise ValueError(f"Input dim ({gate_input.shape[-1]}) does not match GateNet expected input dim "
                                 f"({self.gate_net.input_dim}) when context is None.")
        return gate_input

    def forward(self, x: torch.Tensor, context: Optional[torch.Tensor] = None) -> torch.Tensor:
        """Mixed features kappa (*, feature_dim) for x (*, in_dim)."""
        gate_input = self._gate_input(x, context)
        gdt = self.gate_net.network[0].weight.dtype
        logits = self.gate_net(gate_input.to(dtype=gdt))
        lead = x.shape[:-1]
        rows = 1
        for s in lead:
            rows *= s
        x2 = x.reshape(rows, -1)
        # The stacked features take the first map's output dtype (mixer.py:106):
        # our maps compute in the dtype of their parameters / buffers.
        first = self.feature_maps[0]
        ref = next(iter(list(first.parameters()) + list(first.buffers())), x)
        if torch.is_grad_enabled() and (x.requires_grad or any(p.requires_grad for p in self.parameters())):
            # autograd: each map's output stays a graph node
            feats = torch.stack([fm(x2).to(dtype=ref.dtype) for fm in self.feature_maps])
        else:
            feats = torch.empty(self.num_feature_maps, rows, self.feature_dim, device=x.device, dtype=ref.dtype)
            for i, fm in enumerate(self.feature_maps):
                fm.forward_into(x2, feats[i])
        mixed = mix_features(feats, logits.reshape(rows, -1).to(dtype=feats.dtype))
        return mixed.reshape(*lead, self.feature_dim)

    def extra_repr(self) -> str:
        s = f"num_feature_maps={self.num_feature_maps}, output_feature_dim={self.feature_dim}\n"
        s += f"  (gate_net): {self.gate_net}\n"
        s += f"  (feature_maps): {self.feature_maps}"
        return s.strip()
