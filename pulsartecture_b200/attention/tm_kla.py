"""TM-KLA attention module and functional FA-KLA ops on libfakla.

``TemperatureFunction`` and ``TMLinKernelAttn`` mirror the reference classes in
ultra_rwka/attention/tm_kla.py:17-107 and :110-357: same constructor arguments,
parameter names and initialisation, same checks and error types, same forward
contract (x (B, T, embed_dim) -> (B, T, H*Dv)). The FA-KLA part of forward
(feature map on q and k, temperature, causal kernelized attention,
tm_kla.py:264-332) runs in libfakla: when the mapper is the default
``LearnablePositiveMap`` (one linear layer + elu+1) phi and the scan run in one
call (``fakla_prefill``: the phi GEMM, then the scan as its dependent launch); any other ``FeatureMap`` is applied first and the mapped
tensors go through ``fakla_attention``.

Extension (the reference is stateless): ``forward(..., state=None,
return_state=False)`` accepts and returns the recurrent state (S, z), and
``step`` runs one decode token against it.
"""
from __future__ import annotations

import warnings
from typing import Optional, Tuple, Type

import torch
import torch.nn as nn
import torch.nn.functional as F

from ..backend.interface import (
    State,
    fa_kla_attention_with_state,
    fa_kla_decode_step,
    _needs_grad,
    fa_kla_prefill,
    fa_kla_prefill_host,
    fa_kla_qkv_prefill,
    new_state,
)
from ..components.projections import LinearProjection
from ..kernels.feature_maps import FeatureMap, LearnablePositiveMap, run_mlp


class TemperatureFunction(nn.Module):
    """Non-negative per-head temperatures from an MLP (tm_kla.py:17-107)."""

    def __init__(self, input_dim: int, output_dim: int, hidden_dim: Optional[int] = None,
                 num_layers: int = 1, activation_cls: Type[nn.Module] = nn.GELU,
                 final_activation: str = "softplus", use_bias: bool = True, dropout_p: float = 0.0,
                 initialize_weights: bool = True, device=None, dtype=None):
        super().__init__()
        self.factory_kwargs = {"device": device, "dtype": dtype}
        self.input_dim = input_dim
        self.output_dim = output_dim
        self.final_activation_type = final_activation.lower()
        if num_layers < 1:
            raise ValueError("TemperatureFunction num_layers must be at least 1.")
        supported = ["softplus", "relu", "sigmoid", "abs"]
        if self.final_activation_type not in supported:
            raise ValueError(f"final_activation must be one of {supported}")
        _hidden = hidden_dim if hidden_dim is not None else max(input_dim // 2, output_dim)
        layers = []
        cur = input_dim
        for i in range(num_layers):
            last = i == num_layers - 1
            lin = nn.Linear(cur, output_dim if last else _hidden, bias=use_bias, **self.factory_kwargs)
            if initialize_weights:
                nn.init.xavier_uniform_(lin.weight)
                if use_bias and lin.bias is not None:
                    nn.init.zeros_(lin.bias)
            layers.append(lin)
            if not last:
                layers.append(activation_cls())
                if dropout_p > 0.0:
                    layers.append(nn.Dropout(p=dropout_p))
                cur = _hidden
        self.network = nn.Sequential(*layers)
        self.final_activation_fn = {
            "softplus": F.softplus, "relu": F.relu, "sigmoid": torch.sigmoid, "abs": torch.abs,
        }[self.final_activation_type]

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        expected = next(self.parameters()).dtype
        if x.dtype != expected:
            x = x.to(dtype=expected)
        # every Linear with the activation after it (the last one with the
        # final activation) is one fakla_feature_map launch
        return run_mlp(x, self.network, self.final_activation_type)


class TMLinKernelAttn(nn.Module):
    """Temperature-Modulated Linear Kernel Attention on the B200 FA-KLA kernels."""

    def __init__(self, embed_dim: int, feature_mapper: nn.Module, num_heads: int = 8,
                 qk_dim: Optional[int] = None, v_dim: Optional[int] = None, temp_input_dim: int = 0,
                 temp_hidden_dim: Optional[int] = None, temp_layers: int = 1,
                 temp_final_activation: str = "softplus", proj_bias: bool = True,
                 proj_init: str = "kaiming_uniform", dropout_p: float = 0.0, device=None, dtype=None):
        super().__init__()
        self.embed_dim = embed_dim
        self.num_heads = num_heads
        self.feature_dim = feature_mapper.feature_dim
        self.factory_kwargs = {"device": device, "dtype": dtype}
        self.qk_head_dim = qk_dim if qk_dim is not None else embed_dim // num_heads
        self.v_head_dim = v_dim if v_dim is not None else embed_dim // num_heads
        if embed_dim % num_heads != 0 and (qk_dim is None or v_dim is None):
            warnings.warn(f"embed_dim ({embed_dim}) is not divisible by num_heads ({num_heads}). "
                          "Head dimensions might not be as expected if qk_dim/v_dim are not specified.")
        self.total_qk_dim = self.num_heads * self.qk_head_dim
        self.total_v_dim = self.num_heads * self.v_head_dim
        if isinstance(feature_mapper, FeatureMap) or hasattr(feature_mapper, "in_dim"):
            actual_in = feature_mapper.in_dim
        elif hasattr(feature_mapper, "feature_maps"):  # a mixer: input dim of its first map
            actual_in = feature_mapper.feature_maps[0].in_dim
        else:
            raise TypeError("feature_mapper must be an instance of FeatureMap or KernelFeatureMixer")
        if actual_in != self.total_qk_dim:
            raise ValueError(f"feature_mapper input dimension ({actual_in}) does not match "
                             f"required Q/K projection dimension ({self.total_qk_dim})")
        self.dropout = nn.Dropout(p=dropout_p) if dropout_p > 0 else nn.Identity()
        self.proj_q = LinearProjection(embed_dim, self.total_qk_dim, use_bias=proj_bias, initialize=proj_init, **self.factory_kwargs)
        self.proj_k = LinearProjection(embed_dim, self.total_qk_dim, use_bias=proj_bias, initialize=proj_init, **self.factory_kwargs)
        self.proj_v = LinearProjection(embed_dim, self.total_v_dim, use_bias=proj_bias, initialize=proj_init, **self.factory_kwargs)
        self.feature_mapper = feature_mapper
        self.temp_func: Optional[TemperatureFunction] = None
        if temp_input_dim > 0:
            self.temp_func = TemperatureFunction(
                input_dim=temp_input_dim, output_dim=self.num_heads, hidden_dim=temp_hidden_dim,
                num_layers=temp_layers, final_activation=temp_final_activation, device=device, dtype=dtype)

    def _temperature(self, B: int, T: int, temp_input, dtype) -> Optional[torch.Tensor]:
        if self.temp_func is None:
            return None  # all ones (tm_kla.py:303-306); the kernels skip the multiply
        if temp_input is None:
            raise ValueError("temp_input is required for TemperatureFunction but was not provided.")
        expected = (B, T, self.temp_func.input_dim)
        if tuple(temp_input.shape) != expected:
            raise ValueError(f"Expected temp_input shape {expected}, got {tuple(temp_input.shape)}")
        temp = self.temp_func(temp_input)
        return temp.to(dtype=dtype).contiguous()

    # ------------------------------------------------------------- q/k/v folded into phi
    def _qkv_foldable(self, x: torch.Tensor) -> bool:
        """Inference with the default map on plain linear projections: the
        projections can be folded into the feature map (fakla_qkv_prefill)."""
        mapper = self.feature_mapper
        if not (isinstance(mapper, LearnablePositiveMap) and mapper.fusable):
            return False
        projs = (self.proj_q, self.proj_k, self.proj_v)
        if any(p.norm is not None or p.activation is not None for p in projs):
            return False
        if self.training and not isinstance(self.dropout, nn.Identity):
            return False
        if _needs_grad(x, *self.parameters()):
            return False
        dt = mapper.weight.dtype
        H, M, Dv = self.num_heads, self.feature_dim // self.num_heads, self.v_head_dim
        return (x.is_cuda and dt == torch.bfloat16 and M == Dv and M in (64, 128) and self.embed_dim % 64 == 0
                and (2 * H * M + H * Dv) % 128 == 0 and self.feature_dim % self.num_heads == 0)

    def _qkv_fold(self):
        """[Wphi Wq; Wphi Wk; Wv] and [Wphi bq + bphi; Wphi bk + bphi; bv], computed
        in fp32 and cached until a parameter changes."""
        mapper = self.feature_mapper
        params = (self.proj_q.linear.weight, self.proj_q.linear.bias, self.proj_k.linear.weight,
                  self.proj_k.linear.bias, self.proj_v.linear.weight, self.proj_v.linear.bias,
                  mapper.weight, mapper.bias)
        key = tuple(None if p is None else (p.data_ptr(), p._version) for p in params) + (mapper.weight.dtype,)
        if getattr(self, "_fold_key", None) != key:
            with torch.no_grad():
                wq, bq, wk, bk, wv, bv, wp, bp = [None if p is None else p.float() for p in params]
                zero = lambda n: torch.zeros(n, device=wp.device)  # noqa: E731
                bq = zero(wq.shape[0]) if bq is None else bq
                bk = zero(wk.shape[0]) if bk is None else bk
                bv = zero(wv.shape[0]) if bv is None else bv
                bp = zero(wp.shape[0]) if bp is None else bp
                W = torch.cat([wp @ wq, wp @ wk, wv]).to(mapper.weight.dtype).contiguous()
                b = torch.cat([wp @ bq + bp, wp @ bk + bp, bv]).to(mapper.weight.dtype).contiguous()
            self._fold = (W, b)
            self._fold_key = key
        return self._fold

    def forward(self, x: torch.Tensor, temp_input: Optional[torch.Tensor] = None,
                mixer_context: Optional[torch.Tensor] = None, state: Optional[State] = None,
                return_state: bool = False):
        """x (B, T, embed_dim) -> (B, T, H*Dv); with return_state also (S, z)."""
        if not x.is_contiguous():
            x = x.contiguous()
        B, T, _ = x.shape
        H, Dv = self.num_heads, self.v_head_dim
        if self._qkv_foldable(x):
            W, b = self._qkv_fold()
            temp = self._temperature(B, T, temp_input, W.dtype)
            out, st = fa_kla_qkv_prefill(self.dropout(x).to(W.dtype), W, b, H, self.feature_dim // H, Dv, temp,
                                         state, return_state)
            out = out.reshape(B, T, self.total_v_dim)
            return (out, st) if return_state else out
        x = self.dropout(x)
        q_proj = self.proj_q(x)
        k_proj = self.proj_k(x)
        v = self.proj_v(x)
        if self.feature_dim % H != 0:
            raise ValueError(f"Feature dim ({self.feature_dim}) must be divisible by num_heads ({H}) for head reshaping.")
        Df = self.feature_dim // H
        v4 = v.reshape(B, T, H, Dv).contiguous()
        mapper = self.feature_mapper
        if isinstance(mapper, LearnablePositiveMap) and mapper.fusable:
            p = mapper.weight
            q_proj = q_proj.to(dtype=p.dtype).contiguous()
            k_proj = k_proj.to(dtype=p.dtype).contiguous()
            v4 = v4.to(dtype=p.dtype)
            temp = self._temperature(B, T, temp_input, p.dtype)
            out, st = fa_kla_prefill(q_proj, k_proj, v4, p, mapper.bias, temp, state, return_state)
        else:
            if hasattr(mapper, "feature_maps"):
                qm = mapper(q_proj, mixer_context)
                km = mapper(k_proj, mixer_context)
            else:
                qm = mapper(q_proj)
                km = mapper(k_proj)
            qm = qm.reshape(B, T, H, Df).contiguous()
            km = km.reshape(B, T, H, Df).contiguous()
            v4 = v4.to(dtype=qm.dtype)
            temp = self._temperature(B, T, temp_input, qm.dtype)
            out, st = fa_kla_attention_with_state(qm, km, v4, temp, state, return_state)
        out = out.reshape(B, T, self.total_v_dim)
        return (out, st) if return_state else out

    def init_state(self, batch: int, device=None) -> State:
        dev = device if device is not None else self.proj_q.linear.weight.device
        return new_state(batch, self.num_heads, self.feature_dim // self.num_heads, self.v_head_dim, dev)

    def step(self, x: torch.Tensor, state: State, temp_input: Optional[torch.Tensor] = None) -> torch.Tensor:
        """One decode token per sequence: x (N, embed_dim) -> (N, H*Dv); state updated in place."""
        N = x.shape[0]
        H, Dv = self.num_heads, self.v_head_dim
        q_proj = self.proj_q(x)
        k_proj = self.proj_k(x)
        v = self.proj_v(x).reshape(N, H, Dv)
        mapper = self.feature_mapper
        if not (isinstance(mapper, LearnablePositiveMap) and mapper.fusable):
            raise NotImplementedError("step() needs the one-call LearnablePositiveMap (1 layer, elu+1)")
        p = mapper.weight
        temp = None
        if self.temp_func is not None:
            if temp_input is None:
                raise ValueError("temp_input is required for TemperatureFunction but was not provided.")
            temp = self.temp_func(temp_input).to(dtype=p.dtype).reshape(N, H).contiguous()
        out = fa_kla_decode_step(q_proj.to(p.dtype).contiguous(), k_proj.to(p.dtype).contiguous(),
                                 v.to(p.dtype).contiguous(), state, p, mapper.bias, temp)
        return out.reshape(N, H * Dv)


def fa_kla(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, state: Optional[State] = None, *,
           phi_weight: torch.Tensor, phi_bias: Optional[torch.Tensor] = None,
           temp: Optional[torch.Tensor] = None, chunk: int = 128) -> Tuple[torch.Tensor, State]:
    """Functional FA-KLA prefill with phi in the same call: ``forward(q, k, v, state) -> (out, state)``.

    q, k: (B, T, H_in, Dk) or (B, T, H_in*Dk) projected rows; v: (B, T, H, Dv);
    phi_weight: (H*M, H_in*Dk); phi_bias: (H*M,); temp: (B, T, H) or None.
    The input state is not modified; a new (S, z) is returned. ``chunk`` is
    accepted for chunked-scan call sites and must be positive; the kernels
    tile by 128 tokens whatever it is (the result does not depend on the
    chunk size beyond fp32 rounding).
    """
    if chunk < 1:
        raise RuntimeError(f"chunk must be positive, got {chunk}")
    out, st = fa_kla_prefill(q.contiguous(), k.contiguous(), v.contiguous(), phi_weight, phi_bias,
                             temp, state, True)
    return out, st


def fa_kla_host(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, state: Optional[State] = None, *,
                phi_weight: torch.Tensor, phi_bias: Optional[torch.Tensor] = None,
                temp: Optional[torch.Tensor] = None, out: Optional[torch.Tensor] = None,
                micro_batch: Optional[int] = None, ordered: bool = True) -> Tuple[torch.Tensor, State]:
    """``fa_kla`` for inputs that live in host memory: q, k, v (and temp) on the
    CPU, phi_weight/phi_bias on the GPU that runs the call; returns the output
    in host memory and the state on the GPU. Transfers in both directions
    overlap the compute of neighbouring groups of ``micro_batch`` sequences.
    The output is complete once the current CUDA stream has reached the call.
    ordered=False lets back-to-back calls overlap their copies (the host
    inputs must not be written by device work still pending on the current
    stream; see fa_kla_prefill_host).
    """
    return fa_kla_prefill_host(q, k, v, phi_weight, phi_bias, temp, state, True, out, micro_batch,
                               ordered=ordered)


def fa_kla_decode(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, state: State, *,
                  phi_weight: Optional[torch.Tensor] = None, phi_bias: Optional[torch.Tensor] = None,
                  temp: Optional[torch.Tensor] = None) -> Tuple[torch.Tensor, State]:
    """One recurrent token; the state is updated in place and returned."""
    out = fa_kla_decode_step(q.contiguous(), k.contiguous(), v.contiguous(), state, phi_weight, phi_bias, temp)
    return out, state
