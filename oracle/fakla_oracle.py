"""numpy front end for the C oracle in ``fakla_oracle.c``.

TEST INFRASTRUCTURE ONLY: used by tests/, ``__graft_entry__.smoke()`` and the
CPU-baseline leg of bench.py as the checker. The product path
(``pulsartecture_b200``) never imports this module.

Every function restates a piece of the reference and cites it:

* :func:`phi` -- ``LearnablePositiveMap.forward`` (ultra_rwka/kernels/
  feature_maps.py:259-268; 'elu+1' at :248; one nn.Linear at :224).
* :func:`attention` -- ``fa_kla_attention_cpu`` (ultra_rwka/backend/cpp/cpu/
  cpu_kernels.cpp:36-170), extended with an injected initial state and the
  returned final state (S, z).
* :func:`decode_step` -- the loop body of cpu_kernels.cpp:121-162 applied to one
  token with injected state.
* :func:`prefill` -- phi on the flattened (B,T,H*Dk) q and k, head split
  (ultra_rwka/attention/tm_kla.py:268-287), then :func:`attention`
  (tm_kla.py:319).
"""
from __future__ import annotations

import ctypes
import os
import subprocess
import threading

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_SRC = os.path.join(_HERE, "fakla_oracle.c")
_OUT_DIR = os.path.join(_HERE, "_build")
_LIB_PATH = os.path.join(_OUT_DIR, "libfakla_oracle.so")
_lib = None
_lock = threading.Lock()

_f64p = ctypes.POINTER(ctypes.c_double)
_f32p = ctypes.POINTER(ctypes.c_float)
_i64 = ctypes.c_int64


def build(force: bool = False) -> str:
    """Compile the C oracle with gcc (OpenMP over (b,h) sequences)."""
    if force or not os.path.isfile(_LIB_PATH) or os.path.getmtime(_LIB_PATH) < os.path.getmtime(_SRC):
        os.makedirs(_OUT_DIR, exist_ok=True)
        tmp = _LIB_PATH + ".tmp%d" % os.getpid()
        subprocess.check_call(
            ["gcc", "-O3", "-fopenmp", "-fPIC", "-shared", "-o", tmp, _SRC, "-lm"]
        )
        os.replace(tmp, _LIB_PATH)
    return _LIB_PATH


def _load():
    global _lib
    with _lock:
        if _lib is None:
            lib = ctypes.CDLL(build())
            lib.fakla_oracle_phi_f64.argtypes = [_f64p, _f64p, _f64p, _f64p, _f64p, _i64, _i64, _i64, _i64]
            for name, p in (("fakla_oracle_attention_f64", _f64p), ("fakla_oracle_attention_f32", _f32p)):
                fn = getattr(lib, name)
                fn.argtypes = [p] * 9 + [_i64] * 5
                fn.restype = ctypes.c_int
            lib.fakla_oracle_round_bf16.argtypes = [_f32p, _i64]
            _lib = lib
    return _lib


def _ptr(a, p):
    return None if a is None else a.ctypes.data_as(p)


def _c(a, dt):
    return None if a is None else np.ascontiguousarray(a, dtype=dt)


def round_bf16(x) -> np.ndarray:
    """Round float values to bfloat16 (nearest-even) and return them as float32."""
    a = np.array(x, dtype=np.float32, copy=True, order="C")
    _load().fakla_oracle_round_bf16(_ptr(a, _f32p), a.size)
    return a


def phi(x, W, bias=None, temp=None, heads: int = 1) -> np.ndarray:
    """phi(x) = elu(x @ W.T + bias) + 1 in float64, optionally times the
    per-(row, head) temperature. x: (..., in_dim); W: (feat_dim, in_dim);
    temp: (..., heads)."""
    x = np.asarray(x)
    lead = x.shape[:-1]
    in_dim = x.shape[-1]
    W = _c(W, np.float64)
    feat = W.shape[0]
    rows = int(np.prod(lead)) if lead else 1
    xd = _c(x.reshape(rows, in_dim), np.float64)
    bd = _c(bias, np.float64)
    td = None if temp is None else _c(np.asarray(temp).reshape(rows, heads), np.float64)
    out = np.empty((rows, feat), np.float64)
    _load().fakla_oracle_phi_f64(
        _ptr(xd, _f64p), _ptr(W, _f64p), _ptr(bd, _f64p), _ptr(td, _f64p), _ptr(out, _f64p),
        rows, in_dim, feat, heads,
    )
    return out.reshape(*lead, feat)


def attention(q, k, v, temp=None, S0=None, z0=None, precision: str = "f64"):
    """Causal FA-KLA over (B,T,H,D) inputs; returns (out, S, z).

    precision="f64": double arithmetic (the high-accuracy oracle).
    precision="f32": float arithmetic in the reference's statement order.
    """
    q = np.asarray(q)
    B, T, H, Df = q.shape
    Dv = np.asarray(v).shape[-1]
    if Df > 256 or Dv > 256:
        raise ValueError("oracle supports head dims up to 256")
    dt, p, fn = (
        (np.float64, _f64p, "fakla_oracle_attention_f64")
        if precision == "f64"
        else (np.float32, _f32p, "fakla_oracle_attention_f32")
    )
    qd, kd, vd = _c(q, dt), _c(k, dt), _c(v, dt)
    td = _c(temp, dt)
    S0d, z0d = _c(S0, dt), _c(z0, dt)
    out = np.empty((B, T, H, Dv), dt)
    S1 = np.empty((B, H, Df, Dv), dt)
    z1 = np.empty((B, H, Df), dt)
    rc = getattr(_load(), fn)(
        _ptr(qd, p), _ptr(kd, p), _ptr(vd, p), _ptr(td, p), _ptr(out, p),
        _ptr(S0d, p), _ptr(z0d, p), _ptr(S1, p), _ptr(z1, p), B, T, H, Df, Dv,
    )
    if rc != 0:
        raise ValueError(f"oracle attention rejected head dims Df={Df} Dv={Dv}")
    return out, S1, z1


def decode_step(q, k, v, S, z, temp=None, precision: str = "f64"):
    """One recurrent step for a batch of sequences: q,k: (N,H,Df), v: (N,H,Dv),
    S: (N,H,Df,Dv), z: (N,H,Df), temp: (N,H) or None. Returns (out, S', z')."""
    q = np.asarray(q)
    N, H, Df = q.shape
    out, S1, z1 = attention(
        q[:, None], np.asarray(k)[:, None], np.asarray(v)[:, None],
        None if temp is None else np.asarray(temp)[:, None], S, z, precision,
    )
    return out[:, 0], S1, z1


def prefill(q, k, v, W, bias, temp=None, S0=None, z0=None):
    """Fused path restated: phi on flattened q,k rows, head split, attention.

    q, k: (B,T,H*Dk) (or (B,T,H,Dk)); v: (B,T,H,Dv); W: (H*M, H*Dk);
    temp: (B,T,H) or None. Returns (out (B,T,H,Dv), S, z) in float64."""
    q = np.asarray(q)
    B, T = q.shape[:2]
    v = np.asarray(v)
    H = v.shape[2]
    in_dim = int(np.prod(q.shape[2:]))
    feat = np.asarray(W).shape[0]
    M = feat // H
    pq = phi(q.reshape(B, T, in_dim), W, bias).reshape(B, T, H, M)
    pk = phi(np.asarray(k).reshape(B, T, in_dim), W, bias).reshape(B, T, H, M)
    return attention(pq, pk, v, temp, S0, z0, "f64")


def rel_l2(a, b) -> float:
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    den = np.linalg.norm(b.ravel())
    return float(np.linalg.norm((a - b).ravel()) / (den if den > 0 else 1.0))
