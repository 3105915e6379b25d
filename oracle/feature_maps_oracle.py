"""numpy (float64) restatement of the reference's feature-map family.

TEST INFRASTRUCTURE ONLY: used by tests/ as the checker of libfakla's
fakla_feature_map / fakla_mix_features kernels and of the module classes in
pulsartecture_b200.kernels. The product path never imports this module.

Each function restates a piece of the reference:

* :func:`activation` -- the final activations of LearnablePositiveMap
  (ultra_rwka/kernels/feature_maps.py:246-254: elu+1, relu, softplus, gelu),
  the GELU of its hidden layers (239), and the final activations of
  TemperatureFunction (ultra_rwka/attention/tm_kla.py:86-94: softplus, relu,
  sigmoid, abs).
* :func:`mlp` -- LearnablePositiveMap.forward (feature_maps.py:259-268),
  GateNet.forward (mixer.py:64-66), TemperatureFunction.forward (tm_kla.py:
  96-107): Linear layers with GELU between them and a final activation.
* :func:`fourier` -- _rff_forward_script (feature_maps.py:30-37), the forward
  of RandomFourierFeatures and OrthogonalRandomFeatures.
* :func:`mix` -- KernelFeatureMixer (mixer.py:118-150): softmax over the gate
  logits, weights cast to the logits' dtype, weighted sum of the maps.
"""
from __future__ import annotations

import numpy as np
from scipy.special import erf


def activation(x, kind: str) -> np.ndarray:
    x = np.asarray(x, dtype=np.float64)
    if kind == "elu+1":
        return np.where(x > 0, x + 1.0, np.exp(np.minimum(x, 0.0)))
    if kind == "relu":
        return np.maximum(x, 0.0)
    if kind == "softplus":  # torch softplus: beta=1, threshold=20
        return np.where(x > 20.0, x, np.log1p(np.exp(np.minimum(x, 20.0))))
    if kind == "gelu":  # exact form (nn.GELU(), approximate='none')
        return 0.5 * x * (1.0 + erf(x / np.sqrt(2.0)))
    if kind == "sigmoid":
        return 1.0 / (1.0 + np.exp(-x))
    if kind == "abs":
        return np.abs(x)
    if kind == "identity":
        return x
    raise ValueError(kind)


def linear_act(x, W, b, kind: str) -> np.ndarray:
    """act(x W^T + b), W in nn.Linear layout (n_out, in_dim)."""
    y = np.asarray(x, np.float64) @ np.asarray(W, np.float64).T
    if b is not None:
        y = y + np.asarray(b, np.float64)
    return activation(y, kind)


def mlp(x, layers, final_act: str, hidden_act: str = "gelu") -> np.ndarray:
    """layers: [(W, b), ...]; hidden_act after every layer but the last."""
    h = np.asarray(x, np.float64)
    for i, (W, b) in enumerate(layers):
        h = linear_act(h, W, b, final_act if i == len(layers) - 1 else hidden_act)
    return h


def fourier(x, W, b, scale: float) -> np.ndarray:
    """scale * [cos(x W + b), sin(x W + b)], W (in_dim, P) as the reference stores it."""
    p = np.asarray(x, np.float64) @ np.asarray(W, np.float64) + np.asarray(b, np.float64)
    return np.concatenate([np.cos(p), np.sin(p)], axis=-1) * scale


def mix(feats, logits, round_weights=None) -> np.ndarray:
    """sum_i softmax(logits)_i feats[i]; feats (n, ..., F), logits (..., n).
    round_weights: the cast of the softmax weights to the logits' dtype
    (identity for float64/float32 references)."""
    lg = np.asarray(logits, np.float64)
    e = np.exp(lg - lg.max(axis=-1, keepdims=True))
    w = e / e.sum(axis=-1, keepdims=True)
    if round_weights is not None:
        w = np.asarray(round_weights(w), np.float64)
    f = np.asarray(feats, np.float64)
    return np.einsum("n...f,...n->...f", f, w)
