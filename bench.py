#!/usr/bin/env python
"""FA-KLA prefill benchmark (one JSON line on rank 0).

Headline workload: ONE fixed FA-KLA prefill problem, B=8, H=16, T=4096,
Dk=Dv=M=128, bf16 activations, fp32 state, causal, feature map
LearnablePositiveMap(2048 -> 2048) (phi(q), phi(k), then the chunked scan: one
call, two launches); synthetic q, k, v ~ N(0,1)/sqrt(128) drawn per batch
element from fixed seeds, map parameters initialised like the reference
module from torch.manual_seed(0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

N > 1 runs under torchrun, one process per GPU, and splits that same problem
across the ranks by (batch x head) units, which are independent (strong
scaling, no collective on the data path): `batch` gives each rank B/N batch
rows with all heads, `head` gives each rank H/N heads of every row (with the
matching rows of the map; q and k rows stay whole because the map mixes all
heads). Both are timed and the faster is the headline; the step time is the
max over ranks and `value` is the problem's tokens / that time. After timing,
out, S and z are gathered over NCCL and compared on rank 0 with the problem
run whole on one GPU (`gather_check`).

The same line carries, each split the same way: the long-context prefill
(B=1, H=32, T=65536; heads split), the recurrent decode step (batch 256, H=32,
1024 chained steps; batch split) and the forward of this package's LM
composition (batch split); and `e2e` (the headline metric through the public
API with pinned host buffers, host<->device copies inside the timed region;
`e2e.link` times the same bytes copied alone), per-kernel times with a cuBLAS
comparator for the feature-map GEMM, the roofline of the dominant kernel, the
CPU baseline (the reference's own CPU kernel, compiled from its sources into
oracle/_ref, on the whole workload once) and SM clocks sampled through NVML
during the timed region. `--impl reference` times the reference's CPU
implementation alone (rank 0).
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

import torch  # noqa: E402
import torch.distributed as dist  # noqa: E402

B, T, H, D = 8, 4096, 16, 128
IN_DIM = H * D
DEC_N, DEC_H, DEC_STEPS = 256, 32, 1024
DEC_IN = DEC_H * D
METRIC = "FA-KLA prefill tokens/s"
UNIT = "tokens/s"
# DRAM bytes (read + write) per launch of each kernel at the 1-GPU shapes
# (B=8, H=16, T=4096), from one ncu capture each (dram__bytes_read.sum +
# dram__bytes_write.sum).
PROFILED_DRAM_BYTES = {"phi_gemm_sm100": 276.9e6 + 235.5e6, "scan_sm100": 402.7e6 + 112.8e6}


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.isfile(p):
        with open(p) as f:
            j = json.load(f)
        return float(j["hbm_gbs"]), float(j["bf16_tflops"]), float(j.get("bf16_tflops_sustained", j["bf16_tflops"])), "measured"
    return 6650.0, 1590.0, 1400.0, "fallback"


# ----------------------------------------------------------------------------- clocks
class ClockSampler:
    """Samples SM clock and throttle reasons through NVML while running."""

    REASONS = {
        0x1: "gpu_idle", 0x2: "applications_clocks_setting", 0x4: "sw_power_cap",
        0x8: "hw_slowdown", 0x10: "sync_boost", 0x20: "sw_thermal_slowdown",
        0x40: "hw_thermal_slowdown", 0x80: "hw_power_brake_slowdown", 0x100: "display_clock_setting",
    }

    def __init__(self, device_index: int, interval_s: float = 0.002):
        self.idx = device_index
        self.interval = interval_s
        self.samples = []
        self.reasons = 0
        self.max_mhz = None
        self._stop = threading.Event()
        self._t = None
        self.ok = False
        try:
            import pynvml

            pynvml.nvmlInit()
            self.nv = pynvml
            self.h = pynvml.nvmlDeviceGetHandleByIndex(device_index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self.h, pynvml.NVML_CLOCK_SM)
            self.ok = True
        except Exception:
            self.ok = False

    def _run(self):
        while not self._stop.is_set():
            try:
                self.samples.append(self.nv.nvmlDeviceGetClockInfo(self.h, self.nv.NVML_CLOCK_SM))
                self.reasons |= int(self.nv.nvmlDeviceGetCurrentClocksEventReasons(self.h))
            except Exception:
                pass
            time.sleep(self.interval)

    def __enter__(self):
        if self.ok:
            self._t = threading.Thread(target=self._run, daemon=True)
            self._t.start()
        return self

    def __exit__(self, *a):
        if self._t is not None:
            self._stop.set()
            self._t.join()

    def summary(self):
        if not self.ok or not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": [], "samples": 0,
                    "note": "NVML unavailable" if not self.ok else "no samples"}
        names = [n for bit, n in self.REASONS.items() if self.reasons & bit and n != "gpu_idle"]
        return {"sm_mhz": statistics.median(self.samples), "sm_max_mhz": self.max_mhz,
                "reasons": names, "samples": len(self.samples)}


# ----------------------------------------------------------------------------- helpers
def lpm_init(in_dim, feat, seed=0):
    from pulsartecture_b200.kernels import LearnablePositiveMap

    torch.manual_seed(seed)
    m = LearnablePositiveMap(in_dim, feat)
    return m.weight.detach().clone(), m.bias.detach().clone()


def bind_near_gpu(device_index: int):
    """Restrict this process's threads to the CPUs NVML lists as closest to
    the GPU (its NUMA node), so that host buffers first touched afterwards
    live in that node's memory; returns the previous CPU set to restore, or
    None when NVML gives nothing usable. With one process per GPU, every
    rank's pinned copies then come from the memory next to its own GPU."""
    try:
        import pynvml

        pynvml.nvmlInit()
        h = pynvml.nvmlDeviceGetHandleByIndex(device_index)
        words = ((os.cpu_count() or 64) + 63) // 64
        masks = pynvml.nvmlDeviceGetCpuAffinity(h, words)
        cpus = {64 * w + b for w, m in enumerate(masks) for b in range(64) if (int(m) >> b) & 1}
        prev = os.sched_getaffinity(0)
        cpus &= prev
        if not cpus or cpus == prev:
            return None
        os.sched_setaffinity(0, cpus)
        return prev
    except Exception:
        return None


def sync_barrier(world):
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()


def max_over_ranks(x: float, world: int, dev) -> float:
    if world == 1:
        return x
    t = torch.tensor([x], device=dev, dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def time_loop(fn, steps, stream):
    """Device time (ms) of `steps` calls of fn on `stream`, events on that stream."""
    start = torch.cuda.Event(enable_timing=True)
    end = torch.cuda.Event(enable_timing=True)
    start.record(stream)
    for _ in range(steps):
        fn()
    end.record(stream)
    end.synchronize()
    return start.elapsed_time(end)


# ----------------------------------------------------------------------------- CPU baseline
def cpu_model() -> str | None:
    try:
        with open("/proc/cpuinfo") as f:
            for line in f:
                if line.startswith("model name"):
                    return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return None


def cpu_reference_sample(batch: int, t_len: int, threads: int | None = None):
    """The reference's CPU path on `batch` sequences of t_len tokens, all 16
    heads: phi with torch fp32 (LearnablePositiveMap = nn.Linear + elu+1,
    feature_maps.py:259-268) and the reference's own fa_kla_attention_cpu
    (cpu_kernels.cpp:36-170) from oracle/_ref, parallel over (b, h) through
    at::parallel_for. Returns (tokens, seconds, kind, cores)."""
    from oracle import build_ref

    # all host cores this process may run on (torchrun sets OMP_NUM_THREADS=1
    # per rank; the CPU baseline runs on rank 0 alone and should use them all)
    torch.set_num_threads(threads or len(os.sched_getaffinity(0)))
    cores = torch.get_num_threads()
    W, b = lpm_init(IN_DIM, H * D)
    g = torch.Generator().manual_seed(1234)
    q = torch.randn(batch, t_len, IN_DIM, generator=g) / math.sqrt(D)
    k = torch.randn(batch, t_len, IN_DIM, generator=g) / math.sqrt(D)
    v = (torch.randn(batch, t_len, H, D, generator=g) / math.sqrt(D)).contiguous()
    temp = torch.ones(batch, t_len, H)
    try:
        ref = build_ref.load()
        kind = "reference"
        attn = ref.fa_kla_attention_cpu
    except Exception:
        from oracle import fakla_oracle as O

        kind = "port"

        def attn(qm, km, vv, tp):
            return torch.from_numpy(O.attention(qm.numpy(), km.numpy(), vv.numpy(), tp.numpy(), precision="f32")[0])
    t0 = time.perf_counter()
    with torch.no_grad():
        pq = (torch.nn.functional.elu(torch.nn.functional.linear(q, W, b)) + 1.0).reshape(batch, t_len, H, D)
        pk = (torch.nn.functional.elu(torch.nn.functional.linear(k, W, b)) + 1.0).reshape(batch, t_len, H, D)
        out = attn(pq.contiguous(), pk.contiguous(), v, temp)
    dt = time.perf_counter() - t0
    assert torch.isfinite(out).all()
    return batch * t_len, dt, kind, cores


def run_reference_arm(args):
    """The reference's CPU implementation of the path on this host: each timed
    step is the whole config-2 prefill (B=8, T=4096, H=16, all host threads);
    warm-up steps run one sequence batch element (they only warm the thread
    pool and the allocator). Under torchrun rank 0 alone runs it."""
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if rank != 0:
        return 0
    for _ in range(args.warmup):
        cpu_reference_sample(1, T)
    secs = []
    kind = cores = None
    for _ in range(args.steps):
        n, dt, kind, cores = cpu_reference_sample(B, T)
        secs.append(dt)
    total = sum(secs)
    value = args.steps * B * T / total
    line = {
        "impl": "reference",
        "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": 1000 * total / args.steps, "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": workload_config(world, "batch"),
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": cores, "cpu_model": cpu_model(), "kind": kind,
                         "sample": f"the whole workload per timed step: B={B} x T={T} tokens x H={H} heads "
                                   "(phi torch fp32 + reference fa_kla_attention_cpu); warm-up steps run "
                                   "one batch element"},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "gpu_launches": 0,
    }
    print(json.dumps(line), flush=True)
    return 0


def workload_config(world, partition):
    return {
        "workload": f"FA-KLA prefill, one fixed problem: B={B}, H={H}, T={T}, Dk=Dv=M={D}, bf16 in / fp32 state, "
                    "causal, chunk 128, phi = LearnablePositiveMap(2048->2048, elu+1); one call, two launches "
                    "(phi GEMM, then the chunked scan; four when the scan runs segmented)",
        "global_batch": B, "seq_len": T, "heads": H, "head_dim": D,
        "parallelism": (f"{partition}-sharded x{world} ((batch x head) units split across ranks, "
                        "no collective on the data path)") if world > 1 else "1 GPU",
        "l2": "inputs larger than L2 (q,k,v 403 MB + phi workspace 268 MB per step at 1 GPU)",
    }


# ----------------------------------------------------------------------------- single kernel
def run_prefill_only(args):
    """The headline prefill step alone (fakla_prefill: phi GEMM, then the scan),
    for launch lists: the whole B=8, H=16, T=4096 problem, or with --shard-of N
    rank 0's part of an N-way split (--partition batch or head). Prints the mean
    device time per step."""
    from pulsartecture_b200 import _lib

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    L = _lib.lib()
    W, bias = lpm_init(IN_DIM, H * D)
    W, bias = W.bfloat16().to(dev), bias.bfloat16().to(dev)
    part = "batch" if args.partition == "auto" else args.partition
    shard = PrefillShard(L, dev, part, args.shard_of, 0, B, T, H, W, bias, 1000)
    for _ in range(args.warmup):
        shard.step()
    torch.cuda.synchronize()
    ms = time_loop(shard.step, args.steps, torch.cuda.current_stream(dev)) / args.steps
    _lib.check(L.fakla_device_status(shard.sh))
    print(json.dumps({"only": "prefill", "shard_of": args.shard_of, "partition": part, "batch": shard.B,
                      "heads": shard.H, "launches_per_step": shard.launches_per_step(), "ms_per_step": ms}),
          flush=True)
    return 0


def run_decode_step_only(args):
    """The whole decode step (fakla_decode: the map GEMM for q and k, then the
    state kernel) of batch 256, H=32, or with --shard-of N rank 0's 256/N
    sequences of an N-way batch split. Prints the mean device time per step."""
    from pulsartecture_b200 import _lib

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    L = _lib.lib()
    Wd, bd = lpm_init(DEC_IN, DEC_H * D)
    Wd, bd = Wd.bfloat16().to(dev), bd.bfloat16().to(dev)
    sh = DecodeShard(L, dev, args.shard_of, 0, Wd, bd)
    for _ in range(args.warmup):
        sh.step()
    torch.cuda.synchronize()
    ms = time_loop(sh.step, args.steps, torch.cuda.current_stream(dev)) / args.steps
    _lib.check(L.fakla_device_status(sh.sh))
    print(json.dumps({"only": "decode_step", "shard_of": args.shard_of, "sequences": sh.N, "ms_per_step": ms,
                      "tokens_per_s_if_all_ranks": DEC_N / (ms * 1e-3)}), flush=True)
    return 0


def run_only(args):
    """One kernel of the path alone, on the benchmark's shapes: `phi` = the
    phi GEMM for q and k of the B=8, H=16, T=4096 prefill (2*65536 rows), `scan` =
    the chunk scan of that prefill on precomputed phi, `decode` = the decode state
    kernel (batch 256, H=32), `backward` = the attention backward (temperature
    included) on the prefill's mapped shapes. Prints the mean device time per launch."""
    from pulsartecture_b200 import _lib

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    L = _lib.lib()
    sh = torch.cuda.current_stream(dev).cuda_stream
    g = torch.Generator(device=dev).manual_seed(7)
    if args.only in ("phi", "scan"):
        x = (torch.randn(2 * B * T, IN_DIM, generator=g, device=dev) / math.sqrt(D)).bfloat16()
        W, bias = lpm_init(IN_DIM, H * D)
        W, bias = W.bfloat16().to(dev), bias.bfloat16().to(dev)
        ph = torch.empty(2 * B * T, H * D, device=dev, dtype=torch.bfloat16)

        def phi():
            _lib.check(L.fakla_phi(x.data_ptr(), W.data_ptr(), bias.data_ptr(), None, ph.data_ptr(),
                                   2 * B * T, IN_DIM, H * D, H, _lib.FAKLA_BF16, sh))
        fn = phi
        if args.only == "scan":
            phi()
            v = (torch.randn(B, T, H, D, generator=g, device=dev) / math.sqrt(D)).bfloat16()
            out = torch.empty_like(v)
            S = torch.empty(B, H, D, D, device=dev)
            z = torch.empty(B, H, D, device=dev)

            def scan():
                _lib.check(L.fakla_attention(ph.data_ptr(), ph[B * T:].data_ptr(), v.data_ptr(), None,
                                             out.data_ptr(), S.data_ptr(), z.data_ptr(), B, T, H, D, D,
                                             _lib.FAKLA_BF16, _lib.FAKLA_STATE_OUT, None, 0, sh))
            fn = scan
    elif args.only == "backward":
        qm = (torch.rand(B, T, H, D, generator=g, device=dev) + 0.5).bfloat16()
        km = (torch.rand(B, T, H, D, generator=g, device=dev) + 0.5).bfloat16()
        v = (torch.randn(B, T, H, D, generator=g, device=dev) / math.sqrt(D)).bfloat16()
        do = (torch.randn(B, T, H, D, generator=g, device=dev) / math.sqrt(D)).bfloat16()
        tp = (torch.rand(B, T, H, generator=g, device=dev) + 0.5).bfloat16()
        dq, dk, dv = torch.empty_like(qm), torch.empty_like(km), torch.empty_like(v)
        dtp = torch.empty_like(tp)
        wsb = L.fakla_attention_backward_workspace_bytes(B, T, H, D, D, _lib.FAKLA_BF16)
        ws = torch.empty(wsb, device=dev, dtype=torch.uint8)

        def bwd():
            _lib.check(L.fakla_attention_backward(qm.data_ptr(), km.data_ptr(), v.data_ptr(), tp.data_ptr(),
                                                  do.data_ptr(), None, None, None, None, dq.data_ptr(), dk.data_ptr(),
                                                  dv.data_ptr(), dtp.data_ptr(), None, None, B, T, H, D, D,
                                                  _lib.FAKLA_BF16, ws.data_ptr(), wsb, sh))
        fn = bwd
    else:
        S = torch.randn(DEC_N, DEC_H, D, D, generator=g, device=dev) * 0.02
        z = torch.rand(DEC_N, DEC_H, D, generator=g, device=dev) + 0.5
        qm = (torch.rand(DEC_N, DEC_H, D, generator=g, device=dev) + 0.5).bfloat16()
        km = (torch.rand(DEC_N, DEC_H, D, generator=g, device=dev) + 0.5).bfloat16()
        vd = (torch.randn(DEC_N, DEC_H, D, generator=g, device=dev) / math.sqrt(D)).bfloat16()
        od = torch.empty_like(vd)

        def dec():
            _lib.check(L.fakla_decode_mapped(qm.data_ptr(), km.data_ptr(), vd.data_ptr(), None, od.data_ptr(),
                                             S.data_ptr(), z.data_ptr(), DEC_N, DEC_H, D, D, _lib.FAKLA_BF16, sh))
        fn = dec
    for _ in range(args.warmup):
        fn()
    torch.cuda.synchronize()
    ms = time_loop(fn, args.steps, torch.cuda.current_stream(dev)) / args.steps
    _lib.check(L.fakla_device_status(sh))
    print(json.dumps({"only": args.only, "launches": args.warmup + args.steps, "ms_per_launch": ms}), flush=True)
    return 0


def run_sustained(args):
    """phi, scan and the phi+scan step of the B=8, H=16, T=4096 prefill, each launched back to back
    for about 1.5 s while NVML samples SM clock, power and throttle reasons
    every 5 ms (middle half of each run reported): how the kernels behave once
    the part sits at its power cap, next to the burst numbers of the main line."""
    import pynvml
    from pulsartecture_b200 import _lib

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    pynvml.nvmlInit()
    hnd = pynvml.nvmlDeviceGetHandleByIndex(0)
    L = _lib.lib()
    sh = torch.cuda.current_stream(dev).cuda_stream
    g = torch.Generator(device=dev).manual_seed(7)
    x = (torch.randn(2 * B * T, IN_DIM, generator=g, device=dev) / math.sqrt(D)).bfloat16()
    W, bias = lpm_init(IN_DIM, H * D)
    W, bias = W.bfloat16().to(dev), bias.bfloat16().to(dev)
    ph = torch.empty(2 * B * T, H * D, device=dev, dtype=torch.bfloat16)
    v = (torch.randn(B, T, H, D, generator=g, device=dev) / math.sqrt(D)).bfloat16()
    out = torch.empty_like(v)
    S = torch.empty(B, H, D, D, device=dev)
    z = torch.empty(B, H, D, device=dev)

    def phi():
        _lib.check(L.fakla_phi(x.data_ptr(), W.data_ptr(), bias.data_ptr(), None, ph.data_ptr(),
                               2 * B * T, IN_DIM, H * D, H, _lib.FAKLA_BF16, sh))

    def scan():
        _lib.check(L.fakla_attention(ph.data_ptr(), ph[B * T:].data_ptr(), v.data_ptr(), None, out.data_ptr(),
                                     S.data_ptr(), z.data_ptr(), B, T, H, D, D, _lib.FAKLA_BF16,
                                     _lib.FAKLA_STATE_OUT, None, 0, sh))

    def step():
        phi()
        scan()

    res = {}
    for name, fn, n in (("phi_gemm_sm100", phi, 3200), ("scan_sm100", scan, 11000), ("step", step, 2500)):
        for _ in range(5):
            fn()
        torch.cuda.synchronize()
        samples = []
        stop = threading.Event()

        def sample():
            while not stop.is_set():
                samples.append((pynvml.nvmlDeviceGetClockInfo(hnd, pynvml.NVML_CLOCK_SM),
                                pynvml.nvmlDeviceGetPowerUsage(hnd) / 1000.0,
                                int(pynvml.nvmlDeviceGetCurrentClocksEventReasons(hnd))))
                time.sleep(0.005)

        th = threading.Thread(target=sample, daemon=True)
        th.start()
        ms = time_loop(fn, n, torch.cuda.current_stream(dev)) / n
        stop.set()
        th.join()
        mid = samples[len(samples) // 4: 3 * len(samples) // 4] or samples
        bits = 0
        for _, _, r in mid:
            bits |= r
        res[name] = {"ms_per_launch": ms, "sm_mhz": statistics.median(c for c, _, _ in mid),
                     "power_w": statistics.median(p for _, p, _ in mid),
                     "reasons": [nm for bit, nm in ClockSampler.REASONS.items() if bits & bit and nm != "gpu_idle"],
                     "samples": len(mid)}
    _lib.check(L.fakla_device_status(sh))
    print(json.dumps({"only": "sustained", **res}), flush=True)
    return 0


# ----------------------------------------------------------------------------- long context
def run_longctx(args):
    """Long-context prefill on one GPU: B=1, H=32, T=65536, Dk=Dv=M=128, bf16,
    LearnablePositiveMap(4096 -> 4096) (fa_kla: one call, two launches). The 32 sequences would
    leave most SMs idle, so the scan runs segmented (segment sums, a prefix,
    then one CTA per segment). Prints tokens/s, the phi GEMM and scan times
    and the whole prefill's rate against the measured tensor peak."""
    from pulsartecture_b200 import _lib

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    L = _lib.lib()
    sh = torch.cuda.current_stream(dev).cuda_stream
    B_, T_, H_, D_ = 1, 65536, 32, 128
    g = torch.Generator(device=dev).manual_seed(3)
    q = (torch.randn(B_, T_, H_ * D_, generator=g, device=dev) / math.sqrt(D_)).bfloat16()
    k = (torch.randn(B_, T_, H_ * D_, generator=g, device=dev) / math.sqrt(D_)).bfloat16()
    v = (torch.randn(B_, T_, H_, D_, generator=g, device=dev) / math.sqrt(D_)).bfloat16()
    W, bias = lpm_init(H_ * D_, H_ * D_)
    W, bias = W.bfloat16().to(dev), bias.bfloat16().to(dev)
    out = torch.empty_like(v)
    S = torch.empty(B_, H_, D_, D_, device=dev)
    z = torch.empty(B_, H_, D_, device=dev)
    wsb = L.fakla_prefill_workspace_bytes(B_, T_, H_ * D_, H_, D_, D_, _lib.FAKLA_BF16)
    ws = torch.empty(wsb, device=dev, dtype=torch.uint8)

    def prefill():
        _lib.check(L.fakla_prefill(q.data_ptr(), k.data_ptr(), v.data_ptr(), None, W.data_ptr(), bias.data_ptr(),
                                   out.data_ptr(), S.data_ptr(), z.data_ptr(), B_, T_, H_ * D_, H_, D_, D_,
                                   _lib.FAKLA_BF16, _lib.FAKLA_STATE_OUT, ws.data_ptr(), wsb, sh))

    ph = torch.empty(2 * T_, H_ * D_, device=dev, dtype=torch.bfloat16)
    xq = torch.cat([q.reshape(T_, -1), k.reshape(T_, -1)])

    def phi():
        _lib.check(L.fakla_phi(xq.data_ptr(), W.data_ptr(), bias.data_ptr(), None, ph.data_ptr(), 2 * T_,
                               H_ * D_, H_ * D_, H_, _lib.FAKLA_BF16, sh))

    res = {}
    for name, fn in (("prefill", prefill), ("phi", phi)):
        for _ in range(args.warmup):
            fn()
        torch.cuda.synchronize()
        res[name] = time_loop(fn, args.steps, torch.cuda.current_stream(dev)) / args.steps
    _lib.check(L.fakla_device_status(sh))
    _, tflops_burst, _, _ = peaks()
    flops = 2 * (2 * T_) * (H_ * D_) * (H_ * D_) + T_ * H_ * 98304
    line = {"only": "longctx", "workload": "FA-KLA prefill B=1, H=32, T=65536, Dk=Dv=M=128, bf16, phi 4096->4096",
            "ms": round(res["prefill"], 4), "tokens_per_s": round(T_ / res["prefill"] * 1e3, 1),
            "phi_ms": round(res["phi"], 4), "scan_ms": round(res["prefill"] - res["phi"], 4),
            "tflops": round(flops / res["prefill"] / 1e9, 1),
            "frac_of_tensor_peak": round(flops / res["prefill"] / 1e9 / tflops_burst, 4)}
    print(json.dumps(line), flush=True)
    return 0


# ----------------------------------------------------------------------------- feature-map mixer
def run_mixer(args):
    """KernelFeatureMixer forward (inference, bf16) on the prefill's q rows:
    x (8*4096, 2048) -> three base maps of 2048 features each
    (LearnablePositiveMap elu+1, RandomFourierFeatures and
    OrthogonalRandomFeatures, 1024 projections each with cos/sin), a GateNet
    over the same x and the softmax-weighted sum. Prints the time per forward,
    tokens/s, the base-map GEMM rate against the measured tensor peak and the
    mix kernel's HBM rate."""
    from pulsartecture_b200.kernels import (KernelFeatureMixer, LearnablePositiveMap, OrthogonalRandomFeatures,
                                            RandomFourierFeatures)

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    torch.manual_seed(0)
    maps = [LearnablePositiveMap(IN_DIM, H * D), RandomFourierFeatures(IN_DIM, H * D, gamma=0.02),
            OrthogonalRandomFeatures(IN_DIM, H * D, gamma=0.02)]
    m = KernelFeatureMixer(maps, gate_input_dim=IN_DIM).to(dev).to(torch.bfloat16).eval()
    g = torch.Generator(device=dev).manual_seed(5)
    rows = B * T
    x = (torch.randn(rows, IN_DIM, generator=g, device=dev) / math.sqrt(D)).bfloat16()
    stream = torch.cuda.current_stream(dev)
    with torch.no_grad():
        for _ in range(args.warmup):
            m(x)
        torch.cuda.synchronize()
        ms = time_loop(lambda: m(x), args.steps, stream) / args.steps
        map_ms = []
        for fm in m.feature_maps:
            fm(x)
            map_ms.append(time_loop(lambda: fm(x), args.steps, stream) / args.steps)
        y = m(x)
    torch.cuda.synchronize()
    _, tflops_burst, _, _ = peaks()
    F = H * D
    # base maps: the LearnablePositiveMap GEMM (F outputs) and F/2 projections
    # for each of the two Fourier maps; the gate GEMM (3 outputs) is negligible
    gemm_flops = 2.0 * rows * IN_DIM * (F + F // 2 + F // 2)
    mix_bytes = (len(maps) + 1) * rows * F * 2  # read every map's features once, write the mix
    line = {"only": "mixer", "workload": "KernelFeatureMixer([LPM elu+1, RFF, ORF], GateNet) forward, x (32768, 2048) "
                                         "bf16 -> 2048 features",
            "ms": round(ms, 4), "tokens_per_s": round(rows / ms * 1e3, 1),
            "base_map_ms": {"lpm": round(map_ms[0], 4), "rff": round(map_ms[1], 4), "orf": round(map_ms[2], 4)},
            "base_map_gemm_flops": gemm_flops, "gemm_tflops_if_alone": round(gemm_flops / ms / 1e9, 1),
            "frac_of_tensor_peak_whole_forward": round(gemm_flops / ms / 1e9 / tflops_burst, 4),
            "mix_bytes": mix_bytes, "finite": bool(torch.isfinite(y).all().item())}
    print(json.dumps(line), flush=True)
    return 0


# ----------------------------------------------------------------------------- LM harness
def run_lm(args):
    """Forward of the package's own end-to-end LM composition (lm_harness.py:
    the reference ships no model) at 12 layers, d_model 1024, 16 FA-KLA heads
    of 64, top-2 of 8 experts with d_ff 4096, vocabulary 32000, B=16, T=2048,
    bf16, random weights from seed 0 and uniform token ids. Prints tokens/s
    and the share of the time spent in the FA-KLA sublayers (CUDA events
    around each TMLinKernelAttn call on the launching stream)."""
    from pulsartecture_b200.lm_harness import FaklaLM

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    B_, T_ = 16, 2048
    torch.manual_seed(0)
    model = FaklaLM(dtype=torch.bfloat16, device=dev).eval()
    g = torch.Generator(device=dev).manual_seed(1)
    ids = torch.randint(0, 32000, (B_, T_), generator=g, device=dev)
    marks = []

    def pre(mod, inp):
        e = torch.cuda.Event(enable_timing=True)
        e.record()
        marks.append(e)

    def post(mod, inp, out):
        e = torch.cuda.Event(enable_timing=True)
        e.record()
        marks.append(e)

    hooks = []
    for blk in model.blocks:
        hooks.append(blk.attn.register_forward_pre_hook(pre))
        hooks.append(blk.attn.register_forward_hook(post))
    with torch.no_grad():
        assert model.blocks[0].attn._qkv_foldable(model.embed(ids))
        for _ in range(args.warmup):
            model(ids)
        torch.cuda.synchronize()
        marks.clear()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(args.steps):
            logits = model(ids)
        e1.record()
        e1.synchronize()
    for h in hooks:
        h.remove()
    ms = e0.elapsed_time(e1) / args.steps
    attn_ms = sum(marks[i].elapsed_time(marks[i + 1]) for i in range(0, len(marks), 2)) / args.steps
    # one training step: forward, next-token cross entropy, backward (FA-KLA
    # through its tensor-core backward), no optimizer
    targets = torch.randint(0, 32000, (B_, T_), generator=g, device=dev)

    def train_step():
        model.zero_grad(set_to_none=True)
        loss = torch.nn.functional.cross_entropy(model(ids).float().view(-1, 32000), targets.view(-1))
        loss.backward()
        return loss

    for _ in range(2):
        train_step()
    torch.cuda.synchronize()
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0.record()
    n_train = max(2, min(args.steps, 5))
    for _ in range(n_train):
        loss = train_step()
    t1.record()
    t1.synchronize()
    train_ms = t0.elapsed_time(t1) / n_train
    line = {"only": "lm", "model": "FA-KLA LM (this package's composition; no reference model exists)",
            "config": {"layers": 12, "d_model": 1024, "heads": 16, "head_dim": 64, "experts": "top-2 of 8",
                       "d_ff": 4096, "vocab": 32000, "batch": B_, "seq_len": T_, "dtype": "bf16"},
            "ms_per_forward": round(ms, 3), "tokens_per_s": round(B_ * T_ / ms * 1e3, 1),
            "fakla_ms_per_forward": round(attn_ms, 3), "fakla_share": round(attn_ms / ms, 4),
            "logits_finite": bool(torch.isfinite(logits.float()).all().item()),
            "train_step_ms": round(train_ms, 3), "train_tokens_per_s": round(B_ * T_ / train_ms * 1e3, 1),
            "train_loss_finite": bool(torch.isfinite(loss).item())}
    print(json.dumps(line), flush=True)
    return 0


# ----------------------------------------------------------------------------- sharded workloads
def shard_range(n, world, rank):
    from pulsartecture_b200.sharding import shard_range as sr

    return sr(n, world, rank)


def batch_rows(b, dev, t_len, heads, seed0):
    """Projected q, k rows (t_len, heads*D) and v (t_len, heads, D) of batch
    element b, drawn from a generator seeded by (seed0 + b): every rank that
    holds b draws the same numbers, so shards equal slices of the 1-GPU inputs."""
    g = torch.Generator(device=dev).manual_seed(seed0 + b)
    q = (torch.randn(t_len, heads * D, generator=g, device=dev) / math.sqrt(D)).bfloat16()
    k = (torch.randn(t_len, heads * D, generator=g, device=dev) / math.sqrt(D)).bfloat16()
    v = (torch.randn(t_len, heads, D, generator=g, device=dev) / math.sqrt(D)).bfloat16()
    return q, k, v


class PrefillShard:
    """This rank's part of one fixed prefill problem (batch, t_len, heads, D)
    under a (batch x head) partition: `batch` takes batch rows [b0, b1) with
    every head; `head` takes heads [h0, h1) of every batch row, with the
    matching rows of the feature map and the whole q, k rows (the map mixes
    all heads of a row)."""

    def __init__(self, L, dev, partition, world, rank, batch, t_len, heads, W, bias, seed0):
        from pulsartecture_b200 import _lib

        self.L, self.dev, self.partition = L, dev, partition
        if partition == "batch":
            self.b0, self.b1 = shard_range(batch, world, rank)
            self.h0, self.h1 = 0, heads
        else:
            self.b0, self.b1 = 0, batch
            self.h0, self.h1 = shard_range(heads, world, rank)
        self.B, self.T, self.H = self.b1 - self.b0, t_len, self.h1 - self.h0
        self.in_dim = heads * D
        self.q = torch.empty(self.B, t_len, self.in_dim, device=dev, dtype=torch.bfloat16)
        self.k = torch.empty_like(self.q)
        self.v = torch.empty(self.B, t_len, self.H, D, device=dev, dtype=torch.bfloat16)
        for i, b in enumerate(range(self.b0, self.b1)):
            qb, kb, vb = batch_rows(b, dev, t_len, heads, seed0)
            self.q[i].copy_(qb)
            self.k[i].copy_(kb)
            self.v[i].copy_(vb[:, self.h0:self.h1])
            del qb, kb, vb
        self.W = W[self.h0 * D:self.h1 * D].contiguous()
        self.bias = bias[self.h0 * D:self.h1 * D].contiguous()
        self.out = torch.empty(self.B, t_len, self.H, D, device=dev, dtype=torch.bfloat16)
        self.S = torch.empty(self.B, self.H, D, D, device=dev, dtype=torch.float32)
        self.z = torch.empty(self.B, self.H, D, device=dev, dtype=torch.float32)
        self.ws_bytes = L.fakla_prefill_workspace_bytes(self.B, t_len, self.in_dim, self.H, D, D, _lib.FAKLA_BF16)
        self.ws = torch.empty(self.ws_bytes, device=dev, dtype=torch.uint8)
        self.segmented = L.fakla_attention_workspace_bytes(self.B, t_len, self.H, D, D, _lib.FAKLA_BF16) > 0
        self.sh = torch.cuda.current_stream(dev).cuda_stream

    def launches_per_step(self):
        # phi GEMM + scan; a segmented scan adds the segment sums and the prefix
        return 4 if self.segmented else 2

    def step(self):
        from pulsartecture_b200 import _lib

        _lib.check(self.L.fakla_prefill(self.q.data_ptr(), self.k.data_ptr(), self.v.data_ptr(), None,
                                        self.W.data_ptr(), self.bias.data_ptr(), self.out.data_ptr(),
                                        self.S.data_ptr(), self.z.data_ptr(), self.B, self.T, self.in_dim, self.H,
                                        D, D, _lib.FAKLA_BF16, _lib.FAKLA_STATE_OUT, self.ws.data_ptr(),
                                        self.ws_bytes, self.sh))

    def phi_flops(self):
        return 2.0 * (2 * self.B * self.T) * self.in_dim * (self.H * D)

    def free(self):
        for n in ("q", "k", "v", "out", "S", "z", "ws", "W", "bias"):
            setattr(self, n, None)


def timed(fn, steps, warmup, world, dev, stream, sampler=None):
    """Device time (ms, max over ranks) of `steps` calls after `warmup` calls,
    bracketed by a barrier and a synchronize on both sides."""
    for _ in range(warmup):
        fn()
    sync_barrier(world)
    if sampler is not None:
        with sampler:
            ms = time_loop(fn, steps, stream)
    else:
        ms = time_loop(fn, steps, stream)
    sync_barrier(world)
    return max_over_ranks(ms, world, dev)


def gather_cat(t, world, axis):
    """All ranks' equal-shaped shards of t (NCCL all_gather), concatenated
    along `axis` in rank order."""
    parts = [torch.empty_like(t) for _ in range(world)]
    dist.all_gather(parts, t.contiguous())
    return torch.cat(parts, dim=axis)


def compare(got, ref):
    d = got.double() - ref.double()
    den = ref.double().norm().item()
    return {"bit_exact": bool(torch.equal(got, ref)), "max_abs": float(d.abs().max().item()),
            "rel_l2": float(d.norm().item() / (den if den > 0 else 1.0))}


def verify_prefill(shard, world, rank, make_full):
    """Gather this partition's out, S and z to every rank over NCCL and, on
    rank 0, compare them with the same problem run whole on one GPU (outside
    any timed region). Returns the comparison on rank 0, None elsewhere."""
    shard.step()
    torch.cuda.synchronize()
    bax, hax = (0, 0, 0), (2, 1, 1)
    axes = bax if shard.partition == "batch" else hax
    full = [gather_cat(t, world, ax) for t, ax in zip((shard.out, shard.S, shard.z), axes)]
    res = None
    if rank == 0:
        ref = make_full()
        ref.step()
        torch.cuda.synchronize()
        res = {n: compare(g, r) for n, g, r in zip(("out", "S", "z"), full, (ref.out, ref.S, ref.z))}
        res["ok"] = all(v["rel_l2"] < 1e-3 and v["max_abs"] < 2e-2 for v in res.values())
        ref.free()
    del full
    sync_barrier(world)
    return res


def run_prefill_partition(L, dev, partition, world, rank, W, bias, steps, warmup, sampler, verify):
    shard = PrefillShard(L, dev, partition, world, rank, B, T, H, W, bias, 1000)
    stream = torch.cuda.current_stream(dev)
    ms = timed(shard.step, steps, warmup, world, dev, stream, sampler)
    res = {"ms_per_step": ms / steps, "tokens_per_s": B * T * steps / (ms / 1000.0),
           "per_rank": {"batch": shard.B, "heads": shard.H, "seq_len": T},
           "launches_per_step": shard.launches_per_step(), "scan_segmented": shard.segmented}
    check = None
    if verify and world > 1:
        check = verify_prefill(shard, world, rank,
                               lambda: PrefillShard(L, dev, "batch", 1, 0, B, T, H, W, bias, 1000))
    return shard, res, check


def run_longctx_sharded(L, dev, world, rank, steps, warmup, verify, tflops_burst):
    """Long-context prefill B=1, H=32, T=65536 (LearnablePositiveMap(4096 ->
    4096)), heads split across ranks (32/N per GPU, no cross-GPU traffic)."""
    B_, T_, H_ = 1, 65536, 32
    W, bias = lpm_init(H_ * D, H_ * D)
    W, bias = W.bfloat16().to(dev), bias.bfloat16().to(dev)
    shard = PrefillShard(L, dev, "head", world, rank, B_, T_, H_, W, bias, 5000)
    stream = torch.cuda.current_stream(dev)
    n = max(3, min(steps, 10))
    ms = timed(shard.step, n, max(3, min(warmup, 3)), world, dev, stream)
    flops_local = shard.phi_flops() + B_ * T_ * shard.H * 98304
    res = {"workload": f"FA-KLA prefill B=1, H=32, T=65536, Dk=Dv=M=128, bf16, phi 4096->4096; "
                       f"heads split over {world} GPU(s) ({shard.H} per GPU)",
           "ms": ms / n, "tokens_per_s": B_ * T_ * n / (ms / 1000.0),
           "tflops_per_gpu": flops_local / (ms / n * 1e-3) / 1e12,
           "frac_of_tensor_peak": flops_local / (ms / n * 1e-3) / 1e12 / tflops_burst,
           "flops_per_gpu": flops_local, "launches_per_step": shard.launches_per_step()}
    if verify and world > 1:
        res["gather_check"] = verify_prefill(
            shard, world, rank, lambda: PrefillShard(L, dev, "head", 1, 0, B_, T_, H_, W, bias, 5000))
    shard.free()
    del W, bias
    torch.cuda.empty_cache()
    return res


class DecodeShard:
    """This rank's sequences [n0, n1) of the decode batch (256, H=32): the
    state and the token inputs are drawn per sequence / per step from fixed
    seeds, so shards equal slices of the 1-GPU problem."""

    RING = 16  # distinct token inputs, cycled (the state evolves every step regardless)

    def __init__(self, L, dev, world, rank, W, bias):
        from pulsartecture_b200 import _lib

        self.L = L
        self.n0, self.n1 = shard_range(DEC_N, world, rank)
        self.N = self.n1 - self.n0
        self.W, self.bias = W, bias
        self.S = torch.empty(self.N, DEC_H, D, D, device=dev)
        self.z = torch.empty(self.N, DEC_H, D, device=dev)
        self.reset(dev)
        self.q = torch.empty(self.RING, self.N, DEC_IN, device=dev, dtype=torch.bfloat16)
        self.k = torch.empty_like(self.q)
        self.v = torch.empty(self.RING, self.N, DEC_H, D, device=dev, dtype=torch.bfloat16)
        for s in range(self.RING):
            g = torch.Generator(device=dev).manual_seed(3000 + s)
            self.q[s].copy_((torch.randn(DEC_N, DEC_IN, generator=g, device=dev) / math.sqrt(D))[self.n0:self.n1])
            self.k[s].copy_((torch.randn(DEC_N, DEC_IN, generator=g, device=dev) / math.sqrt(D))[self.n0:self.n1])
            self.v[s].copy_((torch.randn(DEC_N, DEC_H, D, generator=g, device=dev) / math.sqrt(D))[self.n0:self.n1])
        self.out = torch.empty(self.N, DEC_H, D, device=dev, dtype=torch.bfloat16)
        self.ws_bytes = L.fakla_decode_workspace_bytes(self.N, DEC_IN, DEC_H, D, D, _lib.FAKLA_BF16)
        self.ws = torch.empty(self.ws_bytes, device=dev, dtype=torch.uint8)
        self.sh = torch.cuda.current_stream(dev).cuda_stream
        self.it = 0

    def reset(self, dev):
        for i, n in enumerate(range(self.n0, self.n1)):
            g = torch.Generator(device=dev).manual_seed(2000 + n)
            self.S[i].copy_(torch.randn(DEC_H, D, D, generator=g, device=dev) * 0.02)
            self.z[i].copy_(torch.rand(DEC_H, D, generator=g, device=dev) + 0.5)
        self.it = 0

    def step(self):
        from pulsartecture_b200 import _lib

        i = self.it % self.RING
        self.it += 1
        _lib.check(self.L.fakla_decode(self.q[i].data_ptr(), self.k[i].data_ptr(), self.v[i].data_ptr(), None,
                                       self.W.data_ptr(), self.bias.data_ptr(), self.out.data_ptr(),
                                       self.S.data_ptr(), self.z.data_ptr(), self.N, DEC_IN, DEC_H, D, D,
                                       _lib.FAKLA_BF16, self.ws.data_ptr(), self.ws_bytes, self.sh))

    def state_only(self):
        from pulsartecture_b200 import _lib

        phq = self.ws.data_ptr()
        phk = self.ws.data_ptr() + self.ws_bytes // 2
        _lib.check(self.L.fakla_decode_mapped(phq, phk, self.v[0].data_ptr(), None, self.out.data_ptr(),
                                              self.S.data_ptr(), self.z.data_ptr(), self.N, DEC_H, D, D,
                                              _lib.FAKLA_BF16, self.sh))


def run_decode_sharded(L, dev, world, rank, verify, hbm_gbs):
    """Recurrent decode, batch 256 split across ranks: 1024 chained steps."""
    Wd, bd = lpm_init(DEC_IN, DEC_H * D)
    Wd, bd = Wd.bfloat16().to(dev), bd.bfloat16().to(dev)
    sh = DecodeShard(L, dev, world, rank, Wd, bd)
    stream = torch.cuda.current_stream(dev)
    dms = timed(sh.step, DEC_STEPS, 5, world, dev, stream)
    for _ in range(3):
        sh.state_only()
    torch.cuda.synchronize()
    st_ms = time_loop(sh.state_only, 200, stream) / 200
    state_bytes = sh.N * DEC_H * (2 * D * D * 4 + 2 * D * 4 + 2 * D * 2 + D * 2 + D * 2)
    step_bytes = state_bytes + DEC_IN * DEC_H * D * 2  # + the map's weight, read once per step
    res = {"workload": f"recurrent decode: batch {DEC_N}, H={DEC_H}, Dk=Dv=M=128, fp32 state, {DEC_STEPS} "
                       f"sequential steps, phi LearnablePositiveMap(4096->4096); batch split over {world} GPU(s) "
                       f"({sh.N} sequences per GPU)",
           "tokens_per_s": DEC_N * DEC_STEPS / (dms / 1000.0), "ms_per_step": dms / DEC_STEPS,
           "step_gbs_per_gpu": step_bytes / (dms / DEC_STEPS * 1e-3) / 1e9,
           "step_frac_of_hbm": step_bytes / (dms / DEC_STEPS * 1e-3) / 1e9 / hbm_gbs,
           "state_kernel_us": st_ms * 1000, "state_kernel_gbs": state_bytes / (st_ms * 1e-3) / 1e9,
           "state_kernel_frac": state_bytes / (st_ms * 1e-3) / 1e9 / hbm_gbs,
           "state_kernel_bytes": state_bytes, "peak_gbs": hbm_gbs}
    if verify and world > 1:
        # 16 steps from the initial state on every rank, gathered, against the
        # whole batch run on one GPU
        sh.reset(dev)
        for _ in range(16):
            sh.step()
        torch.cuda.synchronize()
        full = [gather_cat(t, world, 0) for t in (sh.out, sh.S, sh.z)]
        if rank == 0:
            ref = DecodeShard(L, dev, 1, 0, Wd, bd)
            for _ in range(16):
                ref.step()
            torch.cuda.synchronize()
            chk = {n: compare(g, r) for n, g, r in zip(("out", "S", "z"), full, (ref.out, ref.S, ref.z))}
            chk["ok"] = all(v["rel_l2"] < 1e-3 and v["max_abs"] < 2e-2 for v in chk.values())
            res["gather_check"] = chk
            del ref
        del full
        sync_barrier(world)
    del sh, Wd, bd
    torch.cuda.empty_cache()
    return res


def run_lm_sharded(dev, world, rank, steps, warmup):
    """Forward of the package's own LM composition (lm_harness.py; the
    reference ships no model): 12 layers, d_model 1024, 16 FA-KLA heads of
    64, top-2 of 8 experts (d_ff 4096), vocabulary 32000, B=16, T=2048, bf16,
    random weights from seed 0; the batch is split across ranks."""
    from pulsartecture_b200.lm_harness import FaklaLM

    B_, T_ = 16, 2048
    b0, b1 = shard_range(B_, world, rank)
    torch.manual_seed(0)
    model = FaklaLM(dtype=torch.bfloat16, device=dev).eval()
    g = torch.Generator(device=dev).manual_seed(1)
    ids = torch.randint(0, 32000, (B_, T_), generator=g, device=dev)[b0:b1].contiguous()
    marks = []

    def mark(*_):
        e = torch.cuda.Event(enable_timing=True)
        e.record()
        marks.append(e)

    hooks = []
    for blk in model.blocks:
        hooks.append(blk.attn.register_forward_pre_hook(mark))
        hooks.append(blk.attn.register_forward_hook(mark))
    stream = torch.cuda.current_stream(dev)
    n = max(3, min(steps, 10))
    with torch.no_grad():
        assert model.blocks[0].attn._qkv_foldable(model.embed(ids))
        for _ in range(max(2, min(warmup, 3))):
            logits = model(ids)
        sync_barrier(world)
        marks.clear()
        ms = time_loop(lambda: model(ids), n, stream)
        sync_barrier(world)
        logits = model(ids)
        finite = bool(torch.isfinite(logits.float()).all().item())
    ms_local = ms
    ms = max_over_ranks(ms, world, dev)
    for h in hooks:
        h.remove()
    attn_ms = sum(marks[i].elapsed_time(marks[i + 1]) for i in range(0, len(marks), 2)) / n
    del model, logits
    torch.cuda.empty_cache()
    return {"model": "FA-KLA LM (this package's composition; no reference model exists)",
            "config": {"layers": 12, "d_model": 1024, "heads": 16, "head_dim": 64, "experts": "top-2 of 8",
                       "d_ff": 4096, "vocab": 32000, "batch": B_, "seq_len": T_, "dtype": "bf16",
                       "partition": f"batch split over {world} GPU(s) ({b1 - b0} sequences per GPU)"},
            "ms_per_forward": ms / n, "tokens_per_s": B_ * T_ * n / (ms / 1000.0),
            "fakla_ms_per_forward": attn_ms, "fakla_share": attn_ms / (ms_local / n),
            "logits_finite": finite}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--partition", default="auto", choices=["auto", "batch", "head"],
                    help="how the fixed prefill problem is split across ranks; auto measures both at N > 1 "
                         "and reports the faster as the headline")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-decode", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-module", action="store_true")
    ap.add_argument("--no-longctx", action="store_true")
    ap.add_argument("--no-lm", action="store_true")
    ap.add_argument("--no-verify", action="store_true")
    ap.add_argument("--shard-of", type=int, default=1,
                    help="with --only prefill or decode_step: time rank 0's part of an N-way split on one GPU")
    ap.add_argument("--only", choices=["phi", "scan", "decode", "backward", "sustained", "lm", "longctx", "mixer",
                                       "prefill", "decode_step"],
                    help="launch just one kernel (warmup + steps launches) for profiler captures; "
                         "'sustained' runs each kernel for ~1.5 s and reports clocks and power")
    args = ap.parse_args()
    if args.impl == "reference":
        return run_reference_arm(args)
    if args.only == "sustained":
        return run_sustained(args)
    if args.only == "lm":
        return run_lm(args)
    if args.only == "longctx":
        return run_longctx(args)
    if args.only == "mixer":
        return run_mixer(args)
    if args.only == "prefill":
        return run_prefill_only(args)
    if args.only == "decode_step":
        return run_decode_step_only(args)
    if args.only:
        return run_only(args)
    assert args.warmup >= 3, "at least 3 warm-up steps"

    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta

        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev)
    verify = not args.no_verify

    from pulsartecture_b200 import _lib
    from pulsartecture_b200.attention import fa_kla_host

    L = _lib.lib()
    hbm_gbs, tflops_burst, tflops_sust, peak_kind = peaks()
    stream = torch.cuda.current_stream(dev)
    sh = stream.cuda_stream
    W, bias = lpm_init(IN_DIM, H * D)
    W, bias = W.bfloat16().to(dev), bias.bfloat16().to(dev)

    # ---- config 2: one fixed prefill problem split across the ranks
    if args.partition != "auto":
        parts = [args.partition]
    else:
        parts = ["batch", "head"] if world > 1 else ["batch"]
    partitions = {}
    checks = {}
    best = None
    for part in parts:
        sampler = ClockSampler(local)
        shard, res, check = run_prefill_partition(L, dev, part, world, rank, W, bias, args.steps, args.warmup,
                                                  sampler, verify)
        res["clocks"] = sampler.summary()
        partitions[part] = res
        if check is not None:
            checks[part] = check
        if best is None or res["ms_per_step"] < partitions[best[0]]["ms_per_step"]:
            if best is not None:
                best[1].free()
            best = (part, shard, sampler)
        else:
            shard.free()
        torch.cuda.empty_cache()
    part, shard, sampler = best
    head = partitions[part]
    ms_per_step = head["ms_per_step"]
    value = head["tokens_per_s"]
    _lib.check(L.fakla_device_status(sh))

    # ---- per-kernel device times of this rank's shard (same shapes, launched alone)
    rows2 = 2 * shard.B * T
    # the workspace starts with the phi(q) and phi(k) buffers, each rounded up to 256 bytes
    phq = shard.ws.data_ptr()
    phk = shard.ws.data_ptr() + ((shard.B * T * shard.H * D * 2 + 255) // 256) * 256
    xq = torch.empty(rows2, IN_DIM, device=dev, dtype=torch.bfloat16)
    xq[: shard.B * T].copy_(shard.q.reshape(-1, IN_DIM))
    xq[shard.B * T:].copy_(shard.k.reshape(-1, IN_DIM))
    n_heads_local = shard.H

    def phi_only():
        _lib.check(L.fakla_phi(xq.data_ptr(), shard.W.data_ptr(), shard.bias.data_ptr(), None, phq, rows2, IN_DIM,
                               n_heads_local * D, n_heads_local, _lib.FAKLA_BF16, sh))

    seg_ws = None
    seg_bytes = L.fakla_attention_workspace_bytes(shard.B, T, n_heads_local, D, D, _lib.FAKLA_BF16)
    if seg_bytes:
        seg_ws = torch.empty(seg_bytes, device=dev, dtype=torch.uint8)

    def scan_only():
        _lib.check(L.fakla_attention(phq, phk, shard.v.data_ptr(), None, shard.out.data_ptr(), shard.S.data_ptr(),
                                     shard.z.data_ptr(), shard.B, T, n_heads_local, D, D, _lib.FAKLA_BF16,
                                     _lib.FAKLA_STATE_OUT, None if seg_ws is None else seg_ws.data_ptr(),
                                     seg_bytes, sh))

    Wt = shard.W

    def cublas_only():
        torch.matmul(xq, Wt.t())

    for _ in range(3):
        phi_only()
        scan_only()
        cublas_only()
    torch.cuda.synchronize()
    ksteps = max(args.steps, 20)
    phi_ms = time_loop(phi_only, ksteps, stream) / ksteps
    scan_ms = time_loop(scan_only, ksteps, stream) / ksteps
    cublas_ms = time_loop(cublas_only, ksteps, stream) / ksteps
    del xq, seg_ws
    phi_flops = shard.phi_flops()
    phi_tflops = phi_flops / (phi_ms * 1e-3) / 1e12
    units = shard.B * T * shard.H  # token-heads of this rank
    scan_bytes = units * 4 * D * 2 + shard.B * shard.H * (D * D + D) * 4
    scan_gbs = scan_bytes / (scan_ms * 1e-3) / 1e9
    attn_flops = units * (2 * 128 * D + 2 * 128 * D + 2 * D * D + 2 * D * D + 2 * 128 * D)
    # DRAM bytes per launch from one ncu capture of each kernel at the 1-GPU
    # shapes, scaled by the token-heads this rank processes
    scale = units / (B * T * H)

    # ---- end to end through the public API with host buffers (batch shard of each rank)
    e2e = None
    if not args.no_e2e:
        b0, b1 = shard_range(B, world, rank)
        eb = b1 - b0
        prev_cpus = bind_near_gpu(dev.index if dev.index is not None else 0)
        hq = torch.empty(eb, T, IN_DIM, dtype=torch.bfloat16).pin_memory()
        hk = torch.empty_like(hq).pin_memory()
        hv = torch.empty(eb, T, H, D, dtype=torch.bfloat16).pin_memory()
        for i, b in enumerate(range(b0, b1)):
            qb, kb, vb = batch_rows(b, dev, T, H, 1000)
            hq[i].copy_(qb)
            hk[i].copy_(kb)
            hv[i].copy_(vb)
        hout = torch.empty(eb, T, H, D, dtype=torch.bfloat16).pin_memory()

        def e2e_step():
            # host q, k, v in, host output back; groups of sequences stream
            # through the GPU with both copy directions overlapping compute;
            # the inputs are filled on the host before the timed loop, so the
            # calls may overlap one step's last output copy with the next
            # step's inputs
            fa_kla_host(hq, hk, hv, phi_weight=W, phi_bias=bias, out=hout, ordered=False)

        e_steps = max(3, min(args.steps, 10))
        ems = timed(e2e_step, e_steps, 2, world, dev, stream)
        h2d_bytes, d2h_bytes = 3 * eb * T * H * D * 2, eb * T * H * D * 2

        # the link floor of that step: the same bytes copied with no compute,
        # inputs on one stream and the output on another (both directions at once)
        s_in, s_out = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
        lq, lk, lv = (torch.empty(t.shape, dtype=t.dtype, device=dev) for t in (hq, hk, hv))
        lout = torch.zeros(eb, T, H, D, dtype=torch.bfloat16, device=dev)

        def link_step():
            s_in.wait_stream(stream)
            s_out.wait_stream(stream)
            with torch.cuda.stream(s_in):
                for hsrc, ddst in ((hq, lq), (hk, lk), (hv, lv)):
                    ddst.copy_(hsrc, non_blocking=True)
            with torch.cuda.stream(s_out):
                hout.copy_(lout, non_blocking=True)
            stream.wait_stream(s_in)
            stream.wait_stream(s_out)

        link_step()
        lms = time_loop(link_step, e_steps, stream) / e_steps
        del lq, lk, lv, lout
        e2e = {"value": B * T * e_steps / (ems / 1000.0), "unit": UNIT,
               "h2d_bytes_per_step": h2d_bytes * world, "d2h_bytes_per_step": d2h_bytes * world,
               "ms_per_step": ems / e_steps,
               "api": "pulsartecture_b200.attention.fa_kla_host (pinned host q/k/v in, host out; copies "
                      "overlapped with compute per group of sequences and across steps, ordered=False); each "
                      "rank streams its batch rows",
               "link": {"copies_only_ms_per_step": lms, "h2d_gbs_per_gpu": h2d_bytes / lms / 1e6,
                        "frac": lms / (ems / e_steps),
                        "note": "the step's host<->device bytes copied alone (pinned, both directions "
                                "at once, no compute); frac = that time / the e2e step"}}
        del hq, hk, hv, hout
        from pulsartecture_b200.backend.interface import release_host_pipelines
        release_host_pipelines()
        if prev_cpus is not None:
            os.sched_setaffinity(0, prev_cpus)
        e2e["host_cpus"] = "GPU-local NUMA node (NVML CPU affinity)" if prev_cpus is not None else "unchanged"

    headline_kernels = {
        "phi_gemm_sm100": {"ms": phi_ms, "flops": phi_flops, "tflops": phi_tflops,
                           "frac_of_peak": phi_tflops / tflops_burst},
        "cublas_same_gemm": {"ms": cublas_ms, "tflops": phi_flops / (cublas_ms * 1e-3) / 1e12,
                             "frac_of_peak": phi_flops / (cublas_ms * 1e-3) / 1e12 / tflops_burst,
                             "note": "torch.matmul (cuBLAS) of the same x W^T, no bias or activation; the "
                                     "comparator for phi_gemm_sm100"},
        "scan_sm100": {"ms": scan_ms, "bytes": scan_bytes, "gbs": scan_gbs, "frac_of_hbm": scan_gbs / hbm_gbs,
                       "tflops": attn_flops / (scan_ms * 1e-3) / 1e12,
                       "traffic": PROFILED_DRAM_BYTES["scan_sm100"] * scale,
                       "segmented": shard.segmented},
        "sum_ms": phi_ms + scan_ms,
    }
    shard_desc = f"{shard.B} batch rows x {shard.H} heads per GPU"
    shard.free()
    torch.cuda.empty_cache()

    # ---- config 3: long-context prefill, heads split across ranks
    longctx = None if args.no_longctx else run_longctx_sharded(L, dev, world, rank, args.steps, args.warmup,
                                                               verify, tflops_burst)

    # ---- config 4: decode, batch split across ranks
    decode = None if args.no_decode else run_decode_sharded(L, dev, world, rank, verify, hbm_gbs)

    # ---- module forward (TMLinKernelAttn, embed 2048 -> 16 heads of 128, bf16, inference) at 1 GPU:
    # projections folded into the feature map (one GEMM + scan) against the
    # projections as three library GEMMs followed by fakla_prefill
    module = None
    if not args.no_module and world == 1:
        from pulsartecture_b200.attention import TMLinKernelAttn
        from pulsartecture_b200.backend.interface import fa_kla_prefill
        from pulsartecture_b200.kernels import LearnablePositiveMap

        torch.manual_seed(0)
        mod = TMLinKernelAttn(IN_DIM, LearnablePositiveMap(IN_DIM, H * D, dtype=torch.bfloat16), num_heads=H,
                              qk_dim=D, v_dim=D, dtype=torch.bfloat16).to(dev).eval()
        gm = torch.Generator(device=dev).manual_seed(3000 + rank)
        xm = (torch.randn(B, T, IN_DIM, generator=gm, device=dev) * 0.5).bfloat16()
        with torch.no_grad():
            assert mod._qkv_foldable(xm)

            def folded():
                mod(xm)

            def unfolded():
                qp, kp, vp = mod.proj_q(xm), mod.proj_k(xm), mod.proj_v(xm)
                fa_kla_prefill(qp, kp, vp.reshape(B, T, H, D), mod.feature_mapper.weight, mod.feature_mapper.bias,
                               None, None, False)

            for fn in (folded, unfolded):
                for _ in range(3):
                    fn()
            torch.cuda.synchronize()
            m_steps = max(5, min(args.steps, 20))
            f_ms = time_loop(folded, m_steps, stream) / m_steps
            u_ms = time_loop(unfolded, m_steps, stream) / m_steps
        module = {
            "workload": "TMLinKernelAttn forward (inference): x (8, 4096, 2048) bf16 -> 16 heads of 128, "
                        "LearnablePositiveMap(2048 -> 2048)",
            "folded_ms": f_ms, "folded_tokens_per_s": B * T / (f_ms * 1e-3),
            "unfolded_ms": u_ms, "unfolded_tokens_per_s": B * T / (u_ms * 1e-3),
            "note": "folded = projections folded into the feature map (fakla_qkv_prefill, one GEMM for "
                    "[phi(q) | phi(k) | v] + scan); unfolded = three cuBLAS projections + fakla_prefill",
        }
        del mod, xm
        torch.cuda.empty_cache()

    # ---- config 5: the LM forward, batch split across ranks
    lm = None if args.no_lm else run_lm_sharded(dev, world, rank, args.steps, args.warmup)

    # ---- CPU baseline (rank 0, N=1 only): the whole config-2 workload once
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        n, dt, kind, cores = cpu_reference_sample(B, T)
        cpu = {"value": n / dt, "unit": UNIT, "cores": cores, "cpu_model": cpu_model(), "kind": kind,
               "sample": f"the whole workload once: B={B} x T={T} tokens x H={H} heads (phi torch fp32 + "
                         "reference fa_kla_attention_cpu)"}

    if rank == 0:
        clocks = sampler.summary()
        line = {
            "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms_per_step, "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "bf16", "data": "synthetic (seeded N(0,1)/sqrt(128) per batch element; "
                                                          "map init from seed 0)",
            "config": workload_config(world, part),
            "partitions": partitions,
            "gather_check": checks or None,
            "roofline": {"bound": "tensor",
                         "kernel": f"phi_gemm_sm100 (phi(q), phi(k) of this GPU's shard: {shard_desc}, "
                                   f"{rows2} x {IN_DIM} x {n_heads_local * D})",
                         "achieved": phi_tflops, "peak": tflops_burst, "unit": "TFLOP/s",
                         "frac": phi_tflops / tflops_burst,
                         "traffic": PROFILED_DRAM_BYTES["phi_gemm_sm100"] * scale,
                         "traffic_source": "ncu dram__bytes_read.sum + dram__bytes_write.sum of one launch at the "
                                           "1-GPU shape, scaled by this GPU's share of the token-heads",
                         "peak_source": f"bf16_tflops (burst) of {peak_kind} MEASURED_PEAKS"},
            "kernels": headline_kernels,
            "e2e": e2e,
            "longctx": longctx,
            "decode": decode,
            "lm": lm,
            "module_forward": module,
            "cpu_baseline": cpu,
            "clocks": clocks,
            "gpu_launches": args.steps * head["launches_per_step"],
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
