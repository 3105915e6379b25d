"""Torch-tensor front end of the FA-KLA C ABI.

Mirrors the reference's backend dispatch for this path:
``ultra_rwka.backend.interface.fa_kla_attention(q_mapped, k_mapped,
v_reshaped, temp)`` as called at ultra_rwka/attention/tm_kla.py:319, whose
native kernel is ``fa_kla_attention_cpu`` (ultra_rwka/backend/cpp/cpu/
cpu_kernels.cpp:36-170). Same argument meaning, layouts (B, T, H, D), returned
tensor (a new (B, T, H, Dv) tensor of the input dtype) and error type
(RuntimeError on a bad shape, dtype or layout).

Differences, all deliberate:
* inputs must be CUDA tensors on an sm_100 GPU (there is no CPU path);
* dtypes float32 and bfloat16 (the reference dispatches float/double/half,
  cpu_kernels.cpp:82; it has no bf16 case);
* ``temp`` may be None (all ones, the module default at tm_kla.py:303-306);
* the ``*_with_state`` / prefill / decode entry points carry the recurrent
  state (S, z), which the reference keeps in locals (cpu_kernels.cpp:78-79).

torch only allocates outputs/workspace and supplies the current stream; all
arithmetic happens in libfakla.so.
"""
from __future__ import annotations

import threading
from typing import Optional, Tuple

import torch

from .. import _lib

State = Tuple[torch.Tensor, torch.Tensor]


def _dtype_code(t: torch.Tensor) -> int:
    if t.dtype == torch.bfloat16:
        return _lib.FAKLA_BF16
    if t.dtype == torch.float32:
        return _lib.FAKLA_F32
    raise RuntimeError(f"FA-KLA supports float32 and bfloat16 inputs, got {t.dtype}")


def _ptr(t: Optional[torch.Tensor]):
    return None if t is None else t.data_ptr()


def _stream(dev: torch.device) -> int:
    return torch.cuda.current_stream(dev).cuda_stream


def _require(cond: bool, msg: str) -> None:
    if not cond:
        raise RuntimeError(msg)


def _check_device(tensors, names) -> torch.device:
    dev = None
    for t, n in zip(tensors, names):
        if t is None:
            continue
        _require(t.is_cuda, f"{n} must be a CUDA tensor (libfakla has no CPU path)")
        if dev is None:
            dev = t.device
        _require(t.device == dev, f"{n} is on {t.device}, expected {dev}")
    return dev


def _check_state(state: Optional[State], B: int, H: int, Df: int, Dv: int, dev) -> None:
    if state is None:
        return
    _require(isinstance(state, (tuple, list)) and len(state) == 2, "state must be a (S, z) pair")
    S, z = state
    _require(tuple(S.shape) == (B, H, Df, Dv), f"state S must be (B, H, Df, Dv) = {(B, H, Df, Dv)}, got {tuple(S.shape)}")
    _require(tuple(z.shape) == (B, H, Df), f"state z must be (B, H, Df) = {(B, H, Df)}, got {tuple(z.shape)}")
    _require(S.dtype == torch.float32 and z.dtype == torch.float32, "state S, z must be float32")
    _require(S.device == dev and z.device == dev, "state must be on the same device as the inputs")
    _require(S.is_contiguous() and z.is_contiguous(), "state S, z must be contiguous")


def new_state(B: int, H: int, Df: int, Dv: int, device) -> State:
    """A zero recurrent state (S, z)."""
    return (torch.zeros(B, H, Df, Dv, device=device, dtype=torch.float32),
            torch.zeros(B, H, Df, device=device, dtype=torch.float32))


def _state_buffers(state: Optional[State], return_state: bool, B, H, Df, Dv, dev):
    """(S, z, flags) for a functional call: the input state is never mutated."""
    flags = 0
    if state is None and not return_state:
        return None, None, 0
    if state is not None:
        S = state[0].clone()
        z = state[1].clone()
        flags |= _lib.FAKLA_STATE_IN
    else:
        S = torch.empty(B, H, Df, Dv, device=dev, dtype=torch.float32)
        z = torch.empty(B, H, Df, device=dev, dtype=torch.float32)
    if return_state:
        flags |= _lib.FAKLA_STATE_OUT
    return S, z, flags


def _no_tokens(out, state: Optional[State], S, z, return_state: bool):
    """The result of a call over zero tokens: the output as allocated (empty)
    and the input state unchanged, or the zero state."""
    if return_state and state is None:
        S.zero_()
        z.zero_()
    return out, ((S, z) if return_state else None)


def fa_kla_attention_with_state(q_mapped: torch.Tensor, k_mapped: torch.Tensor, v_reshaped: torch.Tensor,
                                temp: Optional[torch.Tensor] = None, state: Optional[State] = None,
                                return_state: bool = True):
    """FA-KLA on feature-mapped q, k. Returns ``(out, (S, z))`` (or ``(out, None)``).

    Shapes follow fa_kla_attention_cpu (cpu_kernels.cpp:43-54): q_mapped and
    k_mapped (B, T, H, Df), v_reshaped (B, T, H, Dv), temp (B, T, H) or None.
    """
    _require(q_mapped.dim() == 4, "q_mapped must be 4D (B, T, H, Df)")
    _require(k_mapped.dim() == 4, "k_mapped must be 4D (B, T, H, Df)")
    _require(v_reshaped.dim() == 4, "v_reshaped must be 4D (B, T, H, Dv)")
    _require(temp is None or temp.dim() == 3, "temp must be 3D (B, T, H)")
    _require(q_mapped.shape == k_mapped.shape, "q_mapped and k_mapped shapes must match")
    _require(q_mapped.shape[:3] == v_reshaped.shape[:3], "B, T, H dimensions must match for q/k/v")
    _require(temp is None or tuple(temp.shape) == tuple(q_mapped.shape[:3]),
             "B, T, H dimensions must match for q/k and temp")
    dev = _check_device([q_mapped, k_mapped, v_reshaped, temp], ["q_mapped", "k_mapped", "v_reshaped", "temp"])
    dt = q_mapped.dtype
    _require(all(t is None or t.dtype == dt for t in (k_mapped, v_reshaped, temp)),
             "All inputs must have the same dtype")
    _require(all(t is None or t.is_contiguous() for t in (q_mapped, k_mapped, v_reshaped, temp)),
             "All input tensors must be contiguous for fa_kla_attention")
    code = _dtype_code(q_mapped)
    B, T, H, Df = q_mapped.shape
    Dv = v_reshaped.shape[3]
    _check_state(state, B, H, Df, Dv, dev)
    if _needs_grad(q_mapped, k_mapped, v_reshaped, temp, *(state or ())) and B * T * H > 0:
        S0, z0 = state if state is not None else (None, None)
        out, S, z = _AttentionFn.apply(q_mapped, k_mapped, v_reshaped, temp, S0, z0)
        return out, ((S, z) if return_state else None)
    out = torch.empty_like(v_reshaped)
    S, z, flags = _state_buffers(state, return_state, B, H, Df, Dv, dev)
    if B * T * H == 0:
        return _no_tokens(out, state, S, z, return_state)
    L = _lib.lib()
    with torch.cuda.device(dev):
        # segment records of the tensor-core scan (0 bytes unless few (b, h)
        # pairs would leave SMs idle)
        ws_bytes = L.fakla_attention_workspace_bytes(B, T, H, Df, Dv, code)
        ws = torch.empty(ws_bytes, device=dev, dtype=torch.uint8) if ws_bytes else None
        _lib.check(L.fakla_attention(
            _ptr(q_mapped), _ptr(k_mapped), _ptr(v_reshaped), _ptr(temp), _ptr(out), _ptr(S), _ptr(z),
            B, T, H, Df, Dv, code, flags, _ptr(ws), ws_bytes, _stream(dev)))
    return out, ((S, z) if return_state else None)


def fa_kla_attention(q_mapped: torch.Tensor, k_mapped: torch.Tensor, v_reshaped: torch.Tensor,
                     temp: Optional[torch.Tensor]) -> torch.Tensor:
    """Drop-in for the reference's ``fa_kla_attention`` (tm_kla.py:15,319):
    zero initial state, returns only the (B, T, H, Dv) output."""
    out, _ = fa_kla_attention_with_state(q_mapped, k_mapped, v_reshaped, temp, None, False)
    return out


def phi_map(x: torch.Tensor, weight: torch.Tensor, bias: Optional[torch.Tensor] = None,
            temp: Optional[torch.Tensor] = None, heads: int = 1) -> torch.Tensor:
    """phi(x) = elu(x W^T + b) + 1 (LearnablePositiveMap.forward, feature_maps.py:
    259-268), optionally times temp[..., head]. x: (..., in_dim) -> (..., feat)."""
    _require(weight.dim() == 2, "weight must be (feat_dim, in_dim)")
    feat, in_dim = weight.shape
    _require(x.shape[-1] == in_dim, f"x last dim {x.shape[-1]} != in_dim {in_dim}")
    _require(bias is None or tuple(bias.shape) == (feat,), "bias must be (feat_dim,)")
    _require(feat % heads == 0, "feat_dim must be divisible by heads")
    lead = x.shape[:-1]
    rows = 1
    for s in lead:
        rows *= s
    _require(temp is None or temp.numel() == rows * heads, "temp must hold one value per (row, head)")
    dev = _check_device([x, weight, bias, temp], ["x", "weight", "bias", "temp"])
    if _needs_grad(x, weight, bias, temp) and rows > 0:
        out = _PhiFn.apply(x.reshape(rows, in_dim), weight, bias)
        if temp is not None:
            out = (out.reshape(rows, heads, feat // heads) * temp.reshape(rows, heads, 1)).reshape(rows, feat)
        return out.reshape(*lead, feat)
    dt = x.dtype
    _require(all(t is None or t.dtype == dt for t in (weight, bias, temp)), "x, weight, bias, temp must share a dtype")
    code = _dtype_code(x)
    x = x.contiguous()
    weight = weight.contiguous()
    bias = None if bias is None else bias.contiguous()
    temp = None if temp is None else temp.contiguous()
    out = torch.empty(*lead, feat, device=dev, dtype=dt)
    if rows == 0:
        return out
    L = _lib.lib()
    with torch.cuda.device(dev):
        _lib.check(L.fakla_phi(_ptr(x), _ptr(weight), _ptr(bias), _ptr(temp), _ptr(out),
                               rows, in_dim, feat, heads, code, _stream(dev)))
    return out


def fa_kla_prefill(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, weight: torch.Tensor,
                   bias: Optional[torch.Tensor] = None, temp: Optional[torch.Tensor] = None,
                   state: Optional[State] = None, return_state: bool = True):
    """phi and FA-KLA in one library call (tm_kla.py:268-332 from the projected q/k/v on).

    q, k: (B, T, in_dim) or (B, T, H_in, Dk) projected rows (phi mixes all heads
    of a row); v: (B, T, H, Dv); weight: (H*M, in_dim) -- the map rows of the H
    heads computed here; bias: (H*M,) or None; temp: (B, T, H) or None.
    Returns (out (B, T, H, Dv), (S (B,H,M,Dv), z (B,H,M)) or None).
    """
    _require(q.dim() >= 3 and k.shape == q.shape, "q and k must have the same (B, T, ...) shape")
    _require(v.dim() == 4, "v must be 4D (B, T, H, Dv)")
    B, T = q.shape[0], q.shape[1]
    in_dim = 1
    for s in q.shape[2:]:
        in_dim *= s
    _require(tuple(v.shape[:2]) == (B, T), "B, T dimensions must match for q/k/v")
    H, Dv = v.shape[2], v.shape[3]
    _require(weight.dim() == 2 and weight.shape[1] == in_dim, f"weight must be (H*M, {in_dim})")
    _require(weight.shape[0] % H == 0, "weight rows must be divisible by the number of heads")
    M = weight.shape[0] // H
    _require(bias is None or tuple(bias.shape) == (H * M,), "bias must be (H*M,)")
    _require(temp is None or tuple(temp.shape) == (B, T, H), "temp must be (B, T, H)")
    dev = _check_device([q, k, v, weight, bias, temp], ["q", "k", "v", "weight", "bias", "temp"])
    dt = q.dtype
    _require(all(t is None or t.dtype == dt for t in (k, v, weight, bias, temp)), "All inputs must have the same dtype")
    _require(all(t is None or t.is_contiguous() for t in (q, k, v, weight, bias, temp)), "All inputs must be contiguous")
    code = _dtype_code(q)
    _check_state(state, B, H, M, Dv, dev)
    if _needs_grad(q, k, v, weight, bias, temp, *(state or ())) and B * T > 0:
        # differentiable form: phi(q), phi(k) kept for the backward, then the
        # attention (temperature applied in the scan so that it gets a gradient)
        pq = _PhiFn.apply(q.reshape(B * T, in_dim), weight, bias).reshape(B, T, H, M)
        pk = _PhiFn.apply(k.reshape(B * T, in_dim), weight, bias).reshape(B, T, H, M)
        return fa_kla_attention_with_state(pq, pk, v, temp, state, return_state)
    out = torch.empty(B, T, H, Dv, device=dev, dtype=dt)
    S, z, flags = _state_buffers(state, return_state, B, H, M, Dv, dev)
    if B * T == 0:
        return _no_tokens(out, state, S, z, return_state)
    L = _lib.lib()
    ws_bytes = L.fakla_prefill_workspace_bytes(B, T, in_dim, H, M, Dv, code)
    ws = torch.empty(ws_bytes, device=dev, dtype=torch.uint8)
    with torch.cuda.device(dev):
        _lib.check(L.fakla_prefill(
            _ptr(q), _ptr(k), _ptr(v), _ptr(temp), _ptr(weight), _ptr(bias), _ptr(out), _ptr(S), _ptr(z),
            B, T, in_dim, H, M, Dv, code, flags, _ptr(ws), ws_bytes, _stream(dev)))
    return out, ((S, z) if return_state else None)


def fa_kla_decode_step(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, state: State,
                       weight: Optional[torch.Tensor] = None, bias: Optional[torch.Tensor] = None,
                       temp: Optional[torch.Tensor] = None) -> torch.Tensor:
    """One recurrent token for N sequences; updates ``state`` IN PLACE.

    With ``weight`` (the map, (H*M, in_dim)): q, k are projected rows (N, in_dim)
    or (N, H_in, Dk). Without it, q, k are already mapped: (N, H, Df).
    v: (N, H, Dv); temp: (N, H) or None; state: S (N, H, Df, Dv), z (N, H, Df)
    fp32. Returns out (N, H, Dv) computed from the updated state (the reference
    updates S, z before forming the output, cpu_kernels.cpp:121-162).
    """
    _require(v.dim() == 3, "v must be 3D (N, H, Dv)")
    N, H, Dv = v.shape
    _require(q.shape == k.shape and q.shape[0] == N, "q and k must match and share N with v")
    S, z = state
    dev = _check_device([q, k, v, weight, bias, temp, S, z], ["q", "k", "v", "weight", "bias", "temp", "S", "z"])
    dt = q.dtype
    _require(all(t is None or t.dtype == dt for t in (k, v, weight, bias, temp)), "All inputs must have the same dtype")
    _require(all(t is None or t.is_contiguous() for t in (q, k, v, weight, bias, temp)), "All inputs must be contiguous")
    _require(temp is None or tuple(temp.shape) == (N, H), "temp must be (N, H)")
    code = _dtype_code(q)
    out = torch.empty(N, H, Dv, device=dev, dtype=dt)
    L = _lib.lib()
    if weight is None:
        _require(q.dim() == 3 and q.shape[1] == H, "mapped q, k must be (N, H, Df)")
        Df = q.shape[2]
        _check_state(state, N, H, Df, Dv, dev)
        with torch.cuda.device(dev):
            _lib.check(L.fakla_decode_mapped(_ptr(q), _ptr(k), _ptr(v), _ptr(temp), _ptr(out), _ptr(S), _ptr(z),
                                             N, H, Df, Dv, code, _stream(dev)))
        return out
    in_dim = 1
    for s in q.shape[1:]:
        in_dim *= s
    _require(weight.dim() == 2 and weight.shape[1] == in_dim and weight.shape[0] % H == 0,
             f"weight must be (H*M, {in_dim})")
    M = weight.shape[0] // H
    _require(bias is None or tuple(bias.shape) == (H * M,), "bias must be (H*M,)")
    _check_state(state, N, H, M, Dv, dev)
    ws_bytes = L.fakla_decode_workspace_bytes(N, in_dim, H, M, Dv, code)
    ws = torch.empty(ws_bytes, device=dev, dtype=torch.uint8)
    with torch.cuda.device(dev):
        _lib.check(L.fakla_decode(_ptr(q), _ptr(k), _ptr(v), _ptr(temp), _ptr(weight), _ptr(bias), _ptr(out),
                                  _ptr(S), _ptr(z), N, in_dim, H, M, Dv, code, _ptr(ws), ws_bytes, _stream(dev)))
    return out


def device_status(stream: Optional[torch.cuda.Stream] = None) -> None:
    """Synchronise and raise if a kernel recorded a device-side failure
    (e.g. a bounded wait that expired)."""
    s = stream if stream is not None else torch.cuda.current_stream()
    _lib.check(_lib.lib().fakla_device_status(s.cuda_stream))


class _HostPipeline:
    """Side streams, device slot buffers and per-slot events of
    fa_kla_prefill_host, kept from one call to the next of the same shape
    (one pipeline per device): a call's input copies then only wait for the
    slot they refill, not for the previous call's last output copy."""

    def __init__(self, dev, key, mb, T, q_tail, H, Dv, dt, with_temp, ws_bytes, ns):
        self.key = key
        self.s_in = torch.cuda.Stream(dev)
        self.s_out = torch.cuda.Stream(dev)
        self.bq = [torch.empty((mb,) + q_tail, device=dev, dtype=dt) for _ in range(ns)]
        self.bk = [torch.empty((mb,) + q_tail, device=dev, dtype=dt) for _ in range(ns)]
        self.bv = [torch.empty((mb, T, H, Dv), device=dev, dtype=dt) for _ in range(ns)]
        self.bt = [torch.empty((mb, T, H), device=dev, dtype=dt) for _ in range(ns)] if with_temp else None
        self.bo = [torch.empty((mb, T, H, Dv), device=dev, dtype=dt) for _ in range(ns)]
        self.bw = [torch.empty(ws_bytes, device=dev, dtype=torch.uint8) for _ in range(ns)]
        # the buffers come from the caching allocator on the caller's stream:
        # the side streams start after whatever last used that memory
        born = torch.cuda.Event()
        born.record(torch.cuda.current_stream(dev))
        self.s_in.wait_event(born)
        self.s_out.wait_event(born)
        self.in_free = [None] * ns   # the prefill that last read the slot's inputs
        self.out_free = [None] * ns  # the copy that last read the slot's output


_HOST_PIPES: dict = {}
_HOST_PIPES_LOCK = threading.Lock()  # one caller at a time queues work on a pipeline's slots


def release_host_pipelines() -> None:
    """Free the device buffers fa_kla_prefill_host keeps between calls."""
    with _HOST_PIPES_LOCK:
        _HOST_PIPES.clear()


def fa_kla_prefill_host(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, weight: torch.Tensor,
                        bias: Optional[torch.Tensor] = None, temp: Optional[torch.Tensor] = None,
                        state: Optional[State] = None, return_state: bool = True,
                        out: Optional[torch.Tensor] = None, micro_batch: Optional[int] = None, slots: int = 3,
                        ordered: bool = True):
    """phi and FA-KLA on HOST tensors, transfers overlapped with compute.

    q, k: (B, T, in_dim) or (B, T, H_in, Dk) on the CPU (pin them for
    asynchronous copies); v: (B, T, H, Dv) on the CPU; temp: (B, T, H) on the
    CPU or None; weight, bias and the optional input state on the GPU that
    runs the call. Sequences are independent, so the batch is cut into groups
    of ``micro_batch`` sequences that flow through ``slots`` device buffers:
    the host->device copy of one group, the prefill of the previous one
    and the device->host copy of the one before run on three streams at once
    (the two copy directions use separate copy engines). By default a group
    holds enough sequences for its q copy to reach 64 MiB, and at most half
    the batch: fewer, larger copies keep the link busier (B=8, T=4096,
    in_dim=2048 bf16: groups of 4 ran 3 % faster than single sequences).

    Returns (out, state): ``out`` is a (B, T, H, Dv) host tensor (pinned unless
    given), state (S, z) on the GPU. Like a ``non_blocking`` copy, the call
    returns once the work is queued; ``out`` is complete when the caller's
    current stream reaches this point (e.g. after ``torch.cuda.synchronize()``).

    ordered=True starts the input copies after all work queued so far on the
    caller's stream (as a copy on that stream would). ordered=False starts
    them as soon as their device slot is free, so back-to-back calls overlap
    one call's last output copy with the next call's first input copies; the
    host inputs must then not be written by device work still pending on the
    caller's stream (host-side writes before the call are fine). The device
    buffers are kept for the next call of the same shape
    (release_host_pipelines() frees them).
    """
    _require(weight.is_cuda, "weight must be a CUDA tensor: it selects the GPU that runs the call")
    dev = weight.device
    for t, n in ((q, "q"), (k, "k"), (v, "v"), (temp, "temp")):
        _require(t is None or t.device.type == "cpu", f"{n} must be a host (CPU) tensor")
    _require(q.dim() >= 3 and k.shape == q.shape, "q and k must have the same (B, T, ...) shape")
    _require(v.dim() == 4, "v must be 4D (B, T, H, Dv)")
    B, T = q.shape[0], q.shape[1]
    in_dim = 1
    for s_ in q.shape[2:]:
        in_dim *= s_
    _require(tuple(v.shape[:2]) == (B, T), "B, T dimensions must match for q/k/v")
    H, Dv = v.shape[2], v.shape[3]
    _require(weight.dim() == 2 and weight.shape[1] == in_dim, f"weight must be (H*M, {in_dim})")
    _require(weight.shape[0] % H == 0, "weight rows must be divisible by the number of heads")
    M = weight.shape[0] // H
    _require(bias is None or (bias.device == dev and tuple(bias.shape) == (H * M,)), "bias must be (H*M,) on weight's GPU")
    _require(temp is None or tuple(temp.shape) == (B, T, H), "temp must be (B, T, H)")
    dt = q.dtype
    _require(all(t is None or t.dtype == dt for t in (k, v, weight, bias, temp)), "All inputs must have the same dtype")
    _require(all(t is None or t.is_contiguous() for t in (q, k, v, weight, bias, temp)), "All inputs must be contiguous")
    if micro_batch is None:
        per_seq = max(1, T * in_dim * q.element_size())
        micro_batch = max(1, min(max(1, B // 2), -(-(64 << 20) // per_seq)))
    _require(micro_batch >= 1 and slots >= 2, "micro_batch >= 1 and slots >= 2")
    code = _dtype_code(q)
    _check_state(state, B, H, M, Dv, dev)
    if out is None:
        out = torch.empty(B, T, H, Dv, dtype=dt, pin_memory=True)
    _require(out.device.type == "cpu" and tuple(out.shape) == (B, T, H, Dv) and out.dtype == dt and out.is_contiguous(),
             "out must be a contiguous (B, T, H, Dv) host tensor of the input dtype")
    S, z, flags = _state_buffers(state, return_state, B, H, M, Dv, dev)
    if B * T == 0:
        return _no_tokens(out, state, S, z, return_state)
    L = _lib.lib()
    mb = min(micro_batch, B)
    ngroups = (B + mb - 1) // mb
    ns = min(slots, ngroups)
    ws_bytes = L.fakla_prefill_workspace_bytes(mb, T, in_dim, H, M, Dv, code)
    with torch.cuda.device(dev), _HOST_PIPES_LOCK:
        main = torch.cuda.current_stream(dev)
        key = (mb, T, tuple(q.shape[2:]), H, Dv, dt, temp is not None, ws_bytes, ns)
        pipe = _HOST_PIPES.get(dev)
        if pipe is None or pipe.key != key:
            _HOST_PIPES.pop(dev, None)
            pipe = _HostPipeline(dev, key, mb, T, tuple(q.shape[1:]), H, Dv, dt, temp is not None, ws_bytes, ns)
            _HOST_PIPES[dev] = pipe
        s_in, s_out = pipe.s_in, pipe.s_out
        if ordered:
            ready = torch.cuda.Event()
            ready.record(main)  # inputs and state on the caller's stream precede the copies
            s_in.wait_event(ready)
        last = None
        for j in range(ngroups):
            b0, b1 = j * mb, min(B, (j + 1) * mb)
            n = b1 - b0
            sl = j % ns
            # host -> device, once the prefill that last read this slot is done
            if pipe.in_free[sl] is not None:
                s_in.wait_event(pipe.in_free[sl])
            with torch.cuda.stream(s_in):
                pipe.bq[sl][:n].copy_(q[b0:b1], non_blocking=True)
                pipe.bk[sl][:n].copy_(k[b0:b1], non_blocking=True)
                pipe.bv[sl][:n].copy_(v[b0:b1], non_blocking=True)
                if temp is not None:
                    pipe.bt[sl][:n].copy_(temp[b0:b1], non_blocking=True)
            in_done = torch.cuda.Event()
            in_done.record(s_in)
            # prefill on the caller's stream (slot output free once copied out)
            main.wait_event(in_done)
            if pipe.out_free[sl] is not None:
                main.wait_event(pipe.out_free[sl])
            Sj = None if S is None else S[b0:b1]
            zj = None if z is None else z[b0:b1]
            _lib.check(L.fakla_prefill(
                _ptr(pipe.bq[sl]), _ptr(pipe.bk[sl]), _ptr(pipe.bv[sl]),
                None if temp is None else _ptr(pipe.bt[sl]),
                _ptr(weight), _ptr(bias), _ptr(pipe.bo[sl]), _ptr(Sj), _ptr(zj),
                n, T, in_dim, H, M, Dv, code, flags, _ptr(pipe.bw[sl]), ws_bytes, main.cuda_stream))
            comp = torch.cuda.Event()
            comp.record(main)
            pipe.in_free[sl] = comp
            # device -> host
            s_out.wait_event(comp)
            with torch.cuda.stream(s_out):
                out[b0:b1].copy_(pipe.bo[sl][:n], non_blocking=True)
            last = torch.cuda.Event()
            last.record(s_out)
            pipe.out_free[sl] = last
        # the caller's stream waits for the last copies
        main.wait_event(last)
    return out, ((S, z) if return_state else None)


# ----------------------------------------------------------------------------- feature-map family
ACTIVATIONS = {
    "elu+1": _lib.FAKLA_ACT_ELU1, "relu": _lib.FAKLA_ACT_RELU, "softplus": _lib.FAKLA_ACT_SOFTPLUS,
    "gelu": _lib.FAKLA_ACT_GELU, "identity": _lib.FAKLA_ACT_IDENTITY, "sigmoid": _lib.FAKLA_ACT_SIGMOID,
    "abs": _lib.FAKLA_ACT_ABS, "cossin": _lib.FAKLA_ACT_COSSIN,
}


def feature_map(x: torch.Tensor, weight: torch.Tensor, bias: Optional[torch.Tensor] = None,
                act: str = "elu+1", scale: float = 1.0, out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """act(x W^T + b) in one launch of fakla_feature_map.

    x: (..., in_dim); weight: (n_out, in_dim) (nn.Linear layout); bias: (n_out,)
    or None. Returns (..., n_out), or (..., 2*n_out) for act="cossin" (scale *
    [cos p, sin p], the random-Fourier-feature form of feature_maps.py:30-37).
    ``out`` (contiguous, right shape) is written in place when given.
    """
    _require(act in ACTIVATIONS, f"unknown activation {act!r}; choose from {sorted(ACTIVATIONS)}")
    _require(weight.dim() == 2, "weight must be (n_out, in_dim)")
    if _needs_grad(x, weight, bias):
        if act == "elu+1" and out is None:
            return phi_map(x, weight, bias)
        lead = x.shape[:-1]
        y = _FeatureMapFn.apply(x.reshape(-1, x.shape[-1]), weight, bias, act, float(scale))
        y = y.reshape(*lead, y.shape[-1])
        if out is not None:
            out.copy_(y.reshape(out.shape))
            return out
        return y
    n_out, in_dim = weight.shape
    _require(x.shape[-1] == in_dim, f"x last dim {x.shape[-1]} != in_dim {in_dim}")
    _require(bias is None or tuple(bias.shape) == (n_out,), "bias must be (n_out,)")
    dev = _check_device([x, weight, bias, out], ["x", "weight", "bias", "out"])
    dt = x.dtype
    _require(all(t is None or t.dtype == dt for t in (weight, bias, out)), "All inputs must have the same dtype")
    code = _dtype_code(x)
    x = x.contiguous()
    weight = weight.contiguous()
    bias = None if bias is None else bias.contiguous()
    lead = x.shape[:-1]
    rows = 1
    for s in lead:
        rows *= s
    cols = 2 * n_out if act == "cossin" else n_out
    if out is None:
        out = torch.empty(*lead, cols, device=dev, dtype=dt)
    _require(out.is_contiguous() and out.numel() == rows * cols, "out must be a contiguous (..., n_out) tensor")
    if rows == 0:
        return out
    L = _lib.lib()
    with torch.cuda.device(dev):
        _lib.check(L.fakla_feature_map(_ptr(x), _ptr(weight), _ptr(bias), _ptr(out), rows, in_dim, n_out,
                                       ACTIVATIONS[act], float(scale), code, _stream(dev)))
    return out


def mix_features(feats: torch.Tensor, logits: torch.Tensor, out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """sum_i softmax(logits)_i * feats[i] (KernelFeatureMixer, mixer.py:118-150).

    feats: (n_maps, rows, F); logits: (rows, n_maps), same dtype. Returns (rows, F).
    """
    _require(feats.dim() == 3, "feats must be (n_maps, rows, F)")
    n_maps, rows, F = feats.shape
    _require(tuple(logits.shape) == (rows, n_maps), f"logits must be (rows, n_maps) = {(rows, n_maps)}")
    dev = _check_device([feats, logits, out], ["feats", "logits", "out"])
    _require(logits.dtype == feats.dtype, "feats and logits must have the same dtype")
    code = _dtype_code(feats)
    if _needs_grad(feats, logits) and rows > 0:
        y = _MixFn.apply(feats.contiguous(), logits.contiguous())
        if out is not None:
            out.copy_(y)
            return out
        return y
    feats = feats.contiguous()
    logits = logits.contiguous()
    if out is None:
        out = torch.empty(rows, F, device=dev, dtype=feats.dtype)
    if rows == 0:
        return out
    L = _lib.lib()
    with torch.cuda.device(dev):
        _lib.check(L.fakla_mix_features(_ptr(feats), _ptr(logits), _ptr(out), rows, n_maps, F, code, _stream(dev)))
    return out


# ----------------------------------------------------------------------------- autograd
def _needs_grad(*tensors) -> bool:
    return torch.is_grad_enabled() and any(t is not None and t.requires_grad for t in tensors)


class _AttentionFn(torch.autograd.Function):
    """FA-KLA with gradients: forward fakla_attention (final state always
    returned), backward fakla_attention_backward. The reference has no
    backward; this differentiates its recurrence (cpu_kernels.cpp:107-164)."""

    @staticmethod
    def forward(ctx, q, k, v, temp, S0, z0):
        ctx.set_materialize_grads(False)
        B, T, H, Df = q.shape
        Dv = v.shape[3]
        dev = q.device
        out = torch.empty_like(v)
        S = S0.detach().clone() if S0 is not None else torch.empty(B, H, Df, Dv, device=dev, dtype=torch.float32)
        z = z0.detach().clone() if z0 is not None else torch.empty(B, H, Df, device=dev, dtype=torch.float32)
        flags = _lib.FAKLA_STATE_OUT | (_lib.FAKLA_STATE_IN if S0 is not None else 0)
        L = _lib.lib()
        code = _dtype_code(q)
        with torch.cuda.device(dev):
            ws_bytes = L.fakla_attention_workspace_bytes(B, T, H, Df, Dv, code)
            ws = torch.empty(ws_bytes, device=dev, dtype=torch.uint8) if ws_bytes else None
            _lib.check(L.fakla_attention(_ptr(q), _ptr(k), _ptr(v), _ptr(temp), _ptr(out), _ptr(S), _ptr(z),
                                         B, T, H, Df, Dv, code, flags, _ptr(ws), ws_bytes, _stream(dev)))
        ctx.save_for_backward(q, k, v, temp, S0, z0)
        return out, S, z

    @staticmethod
    def backward(ctx, dout, dS, dz):
        q, k, v, temp, S0, z0 = ctx.saved_tensors
        B, T, H, Df = q.shape
        Dv = v.shape[3]
        dev = q.device
        if dout is None:
            dout = torch.zeros_like(v)
        dout = dout.contiguous().to(dtype=v.dtype)
        if (dS is None) != (dz is None):
            dS = torch.zeros(B, H, Df, Dv, device=dev) if dS is None else dS
            dz = torch.zeros(B, H, Df, device=dev) if dz is None else dz
        dS = None if dS is None else dS.contiguous().float()
        dz = None if dz is None else dz.contiguous().float()
        dq, dk, dv = torch.empty_like(q), torch.empty_like(k), torch.empty_like(v)
        dtemp = torch.empty_like(temp) if temp is not None and ctx.needs_input_grad[3] else None
        want_state = S0 is not None and (ctx.needs_input_grad[4] or ctx.needs_input_grad[5])
        dS0 = torch.empty_like(S0) if want_state else None
        dz0 = torch.empty_like(z0) if want_state else None
        L = _lib.lib()
        code = _dtype_code(q)
        with torch.cuda.device(dev):
            ws_bytes = L.fakla_attention_backward_workspace_bytes(B, T, H, Df, Dv, code)
            ws = torch.empty(ws_bytes, device=dev, dtype=torch.uint8)
            _lib.check(L.fakla_attention_backward(
                _ptr(q), _ptr(k), _ptr(v), _ptr(temp), _ptr(dout), _ptr(S0), _ptr(z0), _ptr(dS), _ptr(dz),
                _ptr(dq), _ptr(dk), _ptr(dv), _ptr(dtemp), _ptr(dS0), _ptr(dz0),
                B, T, H, Df, Dv, code, _ptr(ws), ws_bytes, _stream(dev)))
        return dq, dk, dv, dtemp, dS0, dz0


def _linear_backward(x, W, dpre, want_dx: bool, want_dW: bool, want_db: bool):
    """dx = dpre W, dW = dpre^T x, db = sum_rows dpre of one linear layer
    (fakla_linear_backward: tensor-core GEMMs for bf16, CUDA cores otherwise)."""
    x = None if x is None else x.contiguous()
    W, dpre = W.contiguous(), dpre.contiguous()
    rows, n_out = dpre.shape
    in_dim = W.shape[1]
    dev = dpre.device
    dx = torch.empty(rows, in_dim, device=dev, dtype=dpre.dtype) if want_dx else None
    dW = torch.empty(n_out, in_dim, device=dev, dtype=dpre.dtype) if want_dW else None
    db = torch.empty(n_out, device=dev, dtype=dpre.dtype) if want_db else None
    if not (want_dx or want_dW or want_db) or rows == 0:
        if db is not None:
            db.zero_()
        if dW is not None:
            dW.zero_()
        return dx, dW, db
    L = _lib.lib()
    code = _dtype_code(dpre)
    with torch.cuda.device(dev):
        ws_bytes = L.fakla_linear_backward_workspace_bytes(rows, in_dim, n_out, code) if want_db else 0
        ws = torch.empty(ws_bytes, device=dev, dtype=torch.uint8) if ws_bytes else None
        _lib.check(L.fakla_linear_backward(_ptr(x), _ptr(W), _ptr(dpre), _ptr(dx), _ptr(dW), _ptr(db), rows,
                                           in_dim, n_out, code, _ptr(ws), ws_bytes, _stream(dev)))
    return dx, dW, db


class _PhiFn(torch.autograd.Function):
    """phi(x) = elu(x W^T + b) + 1 with gradients: forward fakla_phi; backward
    fakla_phi_backward (dpre = dphi * min(phi, 1)), then fakla_linear_backward
    (dx = dpre W, dW = dpre^T x, db = sum_rows dpre)."""

    @staticmethod
    def forward(ctx, x, W, b):
        rows, in_dim = x.shape
        feat = W.shape[0]
        dev = x.device
        out = torch.empty(rows, feat, device=dev, dtype=x.dtype)
        L = _lib.lib()
        with torch.cuda.device(dev):
            _lib.check(L.fakla_phi(_ptr(x), _ptr(W), _ptr(b), None, _ptr(out), rows, in_dim, feat, 1,
                                   _dtype_code(x), _stream(dev)))
        ctx.save_for_backward(x, W, out)
        ctx.has_bias = b is not None
        return out

    @staticmethod
    def backward(ctx, dphi):
        x, W, phi = ctx.saved_tensors
        dphi = dphi.contiguous().to(dtype=phi.dtype)
        dpre = torch.empty_like(phi)
        L = _lib.lib()
        dev = phi.device
        with torch.cuda.device(dev):
            _lib.check(L.fakla_phi_backward(_ptr(phi), _ptr(dphi), _ptr(dpre), phi.numel(), _dtype_code(phi),
                                            _stream(dev)))
        return _linear_backward(x, W, dpre, ctx.needs_input_grad[0], ctx.needs_input_grad[1],
                                ctx.has_bias and ctx.needs_input_grad[2])


class _FeatureMapFn(torch.autograd.Function):
    """act(x W^T + b) with gradients for every fakla_feature_map activation:
    the backward recomputes the pre-activation with one identity launch,
    applies fakla_activation_backward, then fakla_linear_backward (dx = dpre W,
    dW = dpre^T x, db = sum_rows dpre)."""

    @staticmethod
    def forward(ctx, x, W, b, act, scale):
        with torch.no_grad():
            y = feature_map(x, W, b, act, scale)
        ctx.save_for_backward(x, W, b)
        ctx.act = act
        ctx.scale = scale
        return y

    @staticmethod
    def backward(ctx, dy):
        x, W, b = ctx.saved_tensors
        with torch.no_grad():
            pre = feature_map(x, W, b, "identity")
        dy = dy.contiguous().to(dtype=pre.dtype)
        dpre = torch.empty_like(pre)
        rows, n = pre.shape
        L = _lib.lib()
        dev = pre.device
        with torch.cuda.device(dev):
            _lib.check(L.fakla_activation_backward(_ptr(pre), _ptr(dy), _ptr(dpre), rows, n, ACTIVATIONS[ctx.act],
                                                   ctx.scale, _dtype_code(pre), _stream(dev)))
        dx, dW, db = _linear_backward(x, W, dpre, ctx.needs_input_grad[0], ctx.needs_input_grad[1],
                                      b is not None and ctx.needs_input_grad[2])
        return dx, dW, db, None, None


class _MixFn(torch.autograd.Function):
    """KernelFeatureMixer combination with gradients (fakla_mix_features /
    fakla_mix_features_backward)."""

    @staticmethod
    def forward(ctx, feats, logits):
        with torch.no_grad():
            y = mix_features(feats, logits)
        ctx.save_for_backward(feats, logits)
        return y

    @staticmethod
    def backward(ctx, dout):
        feats, logits = ctx.saved_tensors
        n_maps, rows, F = feats.shape
        dout = dout.contiguous().to(dtype=feats.dtype)
        dfeats = torch.empty_like(feats) if ctx.needs_input_grad[0] else None
        dlogits = torch.empty_like(logits) if ctx.needs_input_grad[1] else None
        L = _lib.lib()
        dev = feats.device
        with torch.cuda.device(dev):
            _lib.check(L.fakla_mix_features_backward(_ptr(feats), _ptr(logits), _ptr(dout), _ptr(dfeats),
                                                     _ptr(dlogits), rows, n_maps, F, _dtype_code(feats),
                                                     _stream(dev)))
        return dfeats, dlogits


def fa_kla_qkv_prefill(x: torch.Tensor, weight: torch.Tensor, bias: Optional[torch.Tensor], H: int, M: int, Dv: int,
                       temp: Optional[torch.Tensor] = None, state: Optional[State] = None,
                       return_state: bool = True):
    """Projections folded into the feature map, then FA-KLA (fakla_qkv_prefill).

    x: (B, T, embed); weight: (2*H*M + H*Dv, embed) = [Wphi Wq; Wphi Wk; Wv];
    bias: (2*H*M + H*Dv,) or None; temp: (B, T, H) or None. Forward only.
    Returns (out (B, T, H, Dv), (S, z) or None).
    """
    _require(x.dim() == 3, "x must be (B, T, embed)")
    B, T, E = x.shape
    N = 2 * H * M + H * Dv
    _require(tuple(weight.shape) == (N, E), f"weight must be ({N}, {E})")
    _require(bias is None or tuple(bias.shape) == (N,), f"bias must be ({N},)")
    _require(temp is None or tuple(temp.shape) == (B, T, H), "temp must be (B, T, H)")
    dev = _check_device([x, weight, bias, temp], ["x", "weight", "bias", "temp"])
    dt = x.dtype
    _require(all(t is None or t.dtype == dt for t in (weight, bias, temp)), "All inputs must have the same dtype")
    x, weight = x.contiguous(), weight.contiguous()
    bias = None if bias is None else bias.contiguous()
    temp = None if temp is None else temp.contiguous()
    code = _dtype_code(x)
    _check_state(state, B, H, M, Dv, dev)
    out = torch.empty(B, T, H, Dv, device=dev, dtype=dt)
    S, z, flags = _state_buffers(state, return_state, B, H, M, Dv, dev)
    if B * T == 0:
        return _no_tokens(out, state, S, z, return_state)
    L = _lib.lib()
    with torch.cuda.device(dev):
        ws_bytes = L.fakla_qkv_prefill_workspace_bytes(B, T, E, H, M, Dv, code)
        ws = torch.empty(max(ws_bytes, 16), device=dev, dtype=torch.uint8)
        _lib.check(L.fakla_qkv_prefill(_ptr(x), _ptr(weight), _ptr(bias), _ptr(temp), _ptr(out), _ptr(S), _ptr(z),
                                       B, T, E, H, M, Dv, code, flags, _ptr(ws), ws_bytes, _stream(dev)))
    return out, ((S, z) if return_state else None)
