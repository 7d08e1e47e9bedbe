#!/usr/bin/env python3
"""Benchmark of the B200 retention hot path.

Headline workload (one "step"): one recurrent decode step of a
MultiScaleRetention layer, d_model=2048, 8 heads (head_dim 256), 256
independent streams per GPU, fp32 state [256, 8, 256, 256] (512 MiB, larger
than L2, so every step streams it from HBM), x_t ~ N(0,1) fp32, weights
~ N(0, 0.02), gamma_h = 1 - 2^(-5-h).  Multi-GPU: streams are sharded with no
communication; each rank runs 256 streams (weak scaling).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Prints ONE JSON line (rank 0).  `value` is device-timed tok/s with inputs
resident in HBM (max over ranks); `e2e` is the same metric through the public
API with host buffers (pinned H2D of x_t and D2H of the output every step);
`roofline` is the state-stream kernel's algorithmic bytes / CUDA-event time
against the measured HBM copy peak; `cpu_baseline` is the C restatement of
the reference's SIMD CPU path on this host's cores.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

D_MODEL, HEADS, STREAMS = 2048, 8, 256
# DRAM bytes (read + write) of one state-stream launch at this workload,
# measured with ncu (profiles/retention_step_kernel_decode_b256_d2048.md)
STATE_KERNEL_TRAFFIC = 555.808e6 + 483.676e6
EPS = 1e-6
PEAKS_FALLBACK = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0}


def load_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            return json.load(f), "measured"
    return PEAKS_FALLBACK, "fallback"


def decode_bytes_per_step(B, d, H):
    """Algorithmic HBM bytes of one decode step (fp32): state read+write,
    the four d x d projection weights, x in and out."""
    dh = d // H
    state = 2 * B * H * dh * dh * 4
    weights = 4 * d * d * 4
    act = 2 * B * d * 4
    return state, weights, act


def retention_kernel_bytes(B, d, H):
    """Algorithmic bytes of one retention-step launch: state r+w, q/k/v read,
    o write."""
    dh = d // H
    return 2 * B * H * dh * dh * 4 + 3 * B * d * 4 + B * d * 4


# ---------------------------------------------------------------- clocks
class ClockSampler:
    """Samples SM clock and throttle reasons through NVML while running."""

    REASONS = {
        "gpu_idle": 0x1, "applications_clocks_setting": 0x2, "sw_power_cap": 0x4, "hw_slowdown": 0x8,
        "sync_boost": 0x10, "sw_thermal_slowdown": 0x20, "hw_thermal_slowdown": 0x40,
        "hw_power_brake_slowdown": 0x80, "display_clock_setting": 0x100,
    }

    def __init__(self, index: int, period_s: float = 0.01):
        self.samples, self.reasons, self.max_mhz = [], set(), None
        self._stop = threading.Event()
        self._ok = False
        try:
            import pynvml

            import torch

            pynvml.nvmlInit()
            self._nv = pynvml
            p = torch.cuda.get_device_properties(index)
            bus = f"{p.pci_domain_id:08x}:{p.pci_bus_id:02x}:{p.pci_device_id:02x}.0"
            self._h = pynvml.nvmlDeviceGetHandleByPciBusId(bus)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self._h, pynvml.NVML_CLOCK_SM)
            self._ok = True
        except Exception as e:  # pragma: no cover - no NVML
            self.error = str(e)
        self._period = period_s
        self._t = threading.Thread(target=self._run, daemon=True)

    def _run(self):
        while not self._stop.is_set():
            try:
                self.samples.append(self._nv.nvmlDeviceGetClockInfo(self._h, self._nv.NVML_CLOCK_SM))
                r = self._nv.nvmlDeviceGetCurrentClocksEventReasons(self._h)
                for name, bit in self.REASONS.items():
                    if r & bit and name != "gpu_idle":
                        self.reasons.add(name)
            except Exception:
                pass
            time.sleep(self._period)

    def __enter__(self):
        if self._ok:
            self._t.start()
        return self

    def __exit__(self, *a):
        self._stop.set()
        if self._ok:
            self._t.join()

    def summary(self):
        if not self._ok:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "note": "NVML unavailable"}
        return {"sm_mhz": statistics.median(self.samples) if self.samples else None, "sm_max_mhz": self.max_mhz,
                "reasons": sorted(self.reasons), "samples": len(self.samples)}


# ---------------------------------------------------------------- CPU legs
def cpu_decode_sample(seconds: float, nthreads: int, seed: int = 0):
    """Times the C restatement of the reference CPU path (oracle/cpu_ref.c,
    gemv_avx2 + retention_step_core + rmsnorm_core per stream, OpenMP over
    streams) on a bounded sample of the decode workload: `nthreads` streams
    per step (one per thread), repeated until `seconds` elapse."""
    from oracle import cpu_ref

    rng = np.random.default_rng(seed)
    d, H = D_MODEL, HEADS
    dh = d // H
    B = max(1, nthreads)
    w_qkv = (0.02 * rng.standard_normal((3 * d, d))).astype(np.float32)
    w_o = (0.02 * rng.standard_normal((d, d))).astype(np.float32)
    ret_w = np.ones(d, np.float32)
    gamma = np.array([1.0 - 2.0 ** (-5.0 - h) for h in range(H)], np.float32)
    state = np.zeros((B, H, dh, dh), np.float32)
    x = rng.standard_normal((B, d)).astype(np.float32)
    cpu_ref.msr_decode_step(x, state, gamma, w_qkv, w_o, ret_w, EPS, nthreads)  # warm
    steps, t0 = 0, time.perf_counter()
    while True:
        cpu_ref.msr_decode_step(x, state, gamma, w_qkv, w_o, ret_w, EPS, nthreads)
        steps += 1
        el = time.perf_counter() - t0
        if el >= seconds:
            break
    return B * steps / el, steps, B, el


def host_threads() -> int:
    try:
        return len(os.sched_getaffinity(0))
    except Exception:
        return os.cpu_count() or 1


def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    nthreads = host_threads()
    per_step_secs = []
    from oracle import cpu_ref

    # each step: a bounded sample of the decode step, one stream per thread
    rng = np.random.default_rng(0)
    d, H = D_MODEL, HEADS
    dh = d // H
    B = nthreads
    w_qkv = (0.02 * rng.standard_normal((3 * d, d))).astype(np.float32)
    w_o = (0.02 * rng.standard_normal((d, d))).astype(np.float32)
    ret_w = np.ones(d, np.float32)
    gamma = np.array([1.0 - 2.0 ** (-5.0 - h) for h in range(H)], np.float32)
    state = np.zeros((B, H, dh, dh), np.float32)
    x = rng.standard_normal((B, d)).astype(np.float32)
    for _ in range(args.warmup):
        cpu_ref.msr_decode_step(x, state, gamma, w_qkv, w_o, ret_w, EPS, nthreads)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        s = time.perf_counter()
        cpu_ref.msr_decode_step(x, state, gamma, w_qkv, w_o, ret_w, EPS, nthreads)
        per_step_secs.append(time.perf_counter() - s)
    el = time.perf_counter() - t0
    value = B * args.steps / el
    sample = f"{B} of 256 streams per step (one per host thread), d_model=2048, 8 heads, fp32"
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": "tok/s", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1e3 * el / args.steps, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": WORKLOAD, "streams_per_step_sampled": B},
        "cpu_baseline": {"value": value, "unit": "tok/s", "cores": nthreads, "kind": "port", "sample": sample},
        "e2e": {"value": value, "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


METRIC = "retention decode tok/s (B=256,d=2048)"
WORKLOAD = "MultiScaleRetention recurrent decode step: d_model=2048, 8 heads (head_dim 256), 256 streams/GPU, fp32 state"


# ---------------------------------------------------------------- GPU leg
def run_ours(args):
    import torch
    import torch.distributed as dist

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        import datetime

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)

    from aceflow_b200 import _lib, cuda_ops

    if args.only in ("prefill", "longctx", "stack"):
        # one secondary workload alone (profiling runs); same objects as in the full line
        peaks, _ = load_peaks()

        def barrier1():
            if world > 1:
                dist.barrier()

        def max1(v):
            if world == 1:
                return v
            t = torch.tensor([v], dtype=torch.float64, device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            return float(t.item())

        if args.only == "prefill":
            sec = bench_prefill(dev, args.prefill_passes, peaks)
        elif args.only == "longctx":
            sec = bench_longctx(dev, world, rank, args.longctx_passes, peaks, barrier1, max1)
        else:
            sec = bench_stack(dev, peaks)
        if rank == 0:
            print(json.dumps({"section": args.only, **sec}), flush=True)
        if world > 1:
            dist.barrier()
            dist.destroy_process_group()
        return 0

    d, H, B = D_MODEL, HEADS, STREAMS
    dh = d // H
    g = torch.Generator(device=dev)
    g.manual_seed(1234 + rank)
    w_qkv = torch.randn(3 * d, d, generator=g, device=dev) * 0.02
    w_o = torch.randn(d, d, generator=g, device=dev) * 0.02
    ret_w = torch.ones(d, device=dev)
    gamma = cuda_ops.gammas(H, dev)
    state = torch.zeros(B, H, dh, dh, device=dev)
    n_in = args.steps + args.warmup
    n_pool = min(n_in, 256)  # distinct device-resident inputs, cycled
    xs = torch.randn(n_pool, B, d, generator=g, device=dev)
    out = torch.empty(B, d, device=dev)
    stream = torch.cuda.current_stream(dev)
    # weights are prepared once, at load time, like the module's .to(): fp32
    # split exactly into tf32 hi + lo for the tensor cores
    w_qkv_s, w_o_s = cuda_ops.prepare_decode_weights(w_qkv, w_o, H)

    def step(i):
        cuda_ops.msr_decode_step_split(xs[i % n_pool], state, gamma, w_qkv_s, w_o_s, ret_w, EPS, out=out)

    def barrier():
        if world > 1:
            dist.barrier()

    def max_over_ranks(v):
        if world == 1:
            return v
        t = torch.tensor([v], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    clocks = ClockSampler(local)
    with clocks:
        for i in range(args.warmup):
            step(i)
        torch.cuda.synchronize()
        barrier()
        torch.cuda.synchronize()
        launches0 = _lib.launch_count(local)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for i in range(args.steps):
            step(args.warmup + i)
        e1.record(stream)
        torch.cuda.synchronize()
        launches = _lib.launch_count(local) - launches0
        barrier()
        ms_total = max_over_ranks(e0.elapsed_time(e1))

        # dominant kernel alone (the fp32 state stream), CUDA events on its stream
        qkv = torch.randn(B, 3 * d, generator=g, device=dev)
        o = torch.empty(B, d, device=dev)
        kev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(64)]
        for _ in range(4):
            cuda_ops.retention_step(state, gamma, qkv[:, :d], qkv[:, d:2 * d], qkv[:, 2 * d:], out=o)
        for a, b in kev:
            a.record(stream)
            cuda_ops.retention_step(state, gamma, qkv[:, :d], qkv[:, d:2 * d], qkv[:, 2 * d:], out=o)
            b.record(stream)
        torch.cuda.synchronize()
        kernel_ms = statistics.mean(a.elapsed_time(b) for a, b in kev)

        # end to end through the public API with host buffers
        e2e_ms = run_e2e(args, dev, state, gamma, w_qkv_s, w_o_s, ret_w, cuda_ops, barrier)
        e2e_ms = max_over_ranks(e2e_ms)

    ms_step = ms_total / args.steps
    value = world * B * args.steps / (ms_total / 1e3)
    peaks, peak_kind = load_peaks()
    kbytes = retention_kernel_bytes(B, d, H)
    achieved = kbytes / (kernel_ms / 1e3) / 1e9
    st_b, w_b, a_b = decode_bytes_per_step(B, d, H)
    step_bytes = st_b + w_b + a_b
    line = {
        "metric": METRIC, "value": value, "unit": "tok/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms_step, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic (torch.Generator, seeded, device-resident)",
        "config": {"workload": WORKLOAD, "d_model": d, "num_heads": H, "head_dim": dh, "streams_per_gpu": B,
                   "global_batch": B * world, "parallelism": f"stream-sharded x{world}, no collectives",
                   "l2": "inputs larger than L2 (state 512 MiB per GPU streamed every step)",
                   "eps": EPS},
        "roofline": {"bound": "hbm", "kernel": "retention_step_kernel<256,256>", "achieved": achieved,
                     "peak": peaks["hbm_gbs"], "unit": "GB/s", "frac": achieved / peaks["hbm_gbs"],
                     "peak_source": peak_kind, "traffic": STATE_KERNEL_TRAFFIC,
                     "traffic_source": "ncu dram__bytes_read.sum + dram__bytes_write.sum of one launch, "
                                       "profiles/retention_step_kernel_decode_b256_d2048.md",
                     "kernel_ms": kernel_ms,
                     "algorithmic_bytes_per_launch": kbytes,
                     "step_bytes": step_bytes,
                     "step_frac": step_bytes / (ms_step / 1e3) / 1e9 / peaks["hbm_gbs"]},
        "e2e": {"value": world * B * args.steps / (e2e_ms / 1e3), "unit": "tok/s",
                "h2d_bytes_per_step": B * d * 4, "d2h_bytes_per_step": B * d * 4,
                "ms_per_step": e2e_ms / args.steps},
        "gpu_launches": int(launches),
        "clocks": clocks.summary(),
    }
    if world == 1 and not args.no_prefill:
        line["prefill"] = bench_prefill(dev, args.prefill_passes, peaks)
    if not args.no_longctx and HEADS_LONGCTX % world == 0:
        line["longctx"] = bench_longctx(dev, world, rank, args.longctx_passes, peaks, barrier, max_over_ranks)
    if world == 1 and not args.no_stack:
        line["stack"] = bench_stack(dev, peaks)
    if world == 1 and rank == 0 and not args.no_cpu:
        nthreads = host_threads()
        v, steps, b, el = cpu_decode_sample(args.cpu_seconds, nthreads)
        line["cpu_baseline"] = {"value": v, "unit": "tok/s", "cores": nthreads, "kind": "port",
                                "sample": f"{steps} decode steps x {b} streams (one per thread) in {el:.1f} s, "
                                          "C restatement of gemv_avx2+retention_step_core+rmsnorm_core"}
    if rank == 0:
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return 0


def run_e2e(args, dev, state, gamma, w_qkv_s, w_o_s, ret_w, cuda_ops, barrier):
    """K steps through the public API with host buffers: each step copies its
    x_t from pinned host memory to the device, runs the decode step and
    copies the output back to pinned host memory.  Copies run on their own
    streams, double-buffered, so step t's transfers overlap step t+-1's
    compute; the time spans the first H2D to the last D2H."""
    import torch

    B, d = x_shape = (STREAMS, D_MODEL)
    R = 8
    host_in = [torch.randn(*x_shape).pin_memory() for _ in range(R)]
    host_out = [torch.empty(*x_shape).pin_memory() for _ in range(R)]
    dev_in = [torch.empty(*x_shape, device=dev) for _ in range(2)]
    dev_out = [torch.empty(*x_shape, device=dev) for _ in range(2)]
    s_comp = torch.cuda.current_stream(dev)
    s_h2d = torch.cuda.Stream(dev)
    s_d2h = torch.cuda.Stream(dev)
    ev_in = [torch.cuda.Event() for _ in range(2)]
    ev_comp = [torch.cuda.Event() for _ in range(2)]
    ev_out = [torch.cuda.Event() for _ in range(2)]

    def run(n):
        for t in range(n):
            j = t % 2
            with torch.cuda.stream(s_h2d):
                if t >= 2:
                    s_h2d.wait_event(ev_comp[j])  # dev_in[j] no longer read
                dev_in[j].copy_(host_in[t % R], non_blocking=True)
                ev_in[j].record(s_h2d)
            s_comp.wait_event(ev_in[j])
            if t >= 2:
                s_comp.wait_event(ev_out[j])  # dev_out[j] drained
            cuda_ops.msr_decode_step_split(dev_in[j], state, gamma, w_qkv_s, w_o_s, ret_w, EPS, out=dev_out[j])
            ev_comp[j].record(s_comp)
            with torch.cuda.stream(s_d2h):
                s_d2h.wait_event(ev_comp[j])
                host_out[t % R].copy_(dev_out[j], non_blocking=True)
                ev_out[j].record(s_d2h)
        s_comp.wait_stream(s_d2h)

    run(max(3, args.warmup))
    torch.cuda.synchronize()
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(s_comp)
    s_h2d.wait_stream(s_comp)
    run(args.steps)
    e1.record(s_comp)
    torch.cuda.synchronize()
    barrier()
    return e0.elapsed_time(e1)


# ---------------------------------------------------------------- prefill
PREFILL = dict(B=8, T=4096, d=2048, H=8, C=64)


def prefill_flops(B, T, d, H, C):
    """Algorithmic FLOP of one MSR prefill pass: 4 projections 2*N*d^2 each,
    intra-chunk 4*N*H*C*dh, inter-chunk + state update 4*N*H*dh^2."""
    N, dh = B * T, d // H
    proj = 4 * 2 * N * d * d
    intra = 4 * N * H * C * dh
    inter = 4 * N * H * dh * dh
    return proj, intra, inter


def bench_prefill(dev, passes, peaks):
    import torch

    from aceflow_b200 import _lib, cuda_ops

    c = PREFILL
    B, T, d, H = c["B"], c["T"], c["d"], c["H"]
    g = torch.Generator(device=dev).manual_seed(7)
    x = torch.randn(B, T, d, generator=g, device=dev).bfloat16()
    w_qkv = (0.02 * torch.randn(3 * d, d, generator=g, device=dev)).bfloat16()
    w_o = (0.02 * torch.randn(d, d, generator=g, device=dev)).bfloat16()
    rw = torch.ones(d, device=dev)
    gamma = cuda_ops.gammas(H, dev)
    out = None
    for _ in range(3):
        out, _st = cuda_ops.msr_prefill_bf16(x, w_qkv, w_o, rw, gamma, EPS, want_state=False)
    torch.cuda.synchronize()
    stream = torch.cuda.current_stream(dev)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(passes):
        out, _st = cuda_ops.msr_prefill_bf16(x, w_qkv, w_o, rw, gamma, EPS, want_state=False)
    e1.record(stream)
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / passes
    # the retention core alone (chunkwise kernel), CUDA events on its stream
    qkv = torch.randn(B * T, 3 * d, generator=g, device=dev).bfloat16()
    for _ in range(2):
        cuda_ops.retention_chunkwise_bf16(qkv, B, T, H, gamma, norm_w=rw, want_state=False)
    e2, e3 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e2.record(stream)
    for _ in range(passes):
        cuda_ops.retention_chunkwise_bf16(qkv, B, T, H, gamma, norm_w=rw, want_state=False)
    e3.record(stream)
    torch.cuda.synchronize()
    core_ms = e2.elapsed_time(e3) / passes
    _lib.check_device(dev.index or 0)
    proj, intra, inter = prefill_flops(B, T, d, H, c["C"])
    total = proj + intra + inter
    tfl = total / (ms / 1e3) / 1e12
    core_tfl = (intra + inter) / (core_ms / 1e3) / 1e12
    return {
        "metric": "retention prefill tok/s (B=8,T=4096,d=2048)", "value": B * T / (ms / 1e3), "unit": "tok/s",
        "ms_per_pass": ms, "passes": passes, "dtype": "bf16 (fp32 accumulate)",
        "config": {"workload": "MultiScaleRetention prefill, d_model=2048, 8 heads, B=8, T=4096, chunk 64",
                   "l2": "inputs larger than L2 (x 128 MiB, qkv 384 MiB)"},
        "roofline": {"bound": "tensor", "achieved": tfl, "peak": peaks["bf16_tflops"], "unit": "TFLOP/s",
                     "frac": tfl / peaks["bf16_tflops"], "algorithmic_flop": total},
        "retention_core": {"kernel": "retention_chunkwise_kernel", "ms": core_ms, "achieved": core_tfl,
                           "unit": "TFLOP/s", "frac": core_tfl / peaks["bf16_tflops"],
                           "algorithmic_flop": intra + inter},
    }


# ---------------------------------------------------------------- long context
LONGCTX = dict(B=1, T=65536, d=4096, H=16, C=64)
HEADS_LONGCTX = LONGCTX["H"]


def bench_longctx(dev, world, rank, passes, peaks, barrier, max_over_ranks):
    """Head-sharded prefill of one 65536-token stream (d_model 4096, 16 heads)
    over all ranks: QKV of the rank's heads, chunkwise retention (sequence
    segments), NCCL all-gather of head outputs, output projection of the
    rank's columns.  Total work is fixed, so N GPUs scale it strongly."""
    import torch

    from aceflow_b200 import _lib
    from aceflow_b200.sharded import HeadShardedPrefill, chunkwise_plan

    c = LONGCTX
    B, T, d, H = c["B"], c["T"], c["d"], c["H"]
    g = torch.Generator(device=dev).manual_seed(11)  # same weights and input on every rank
    x = torch.randn(B, T, d, generator=g, device=dev).bfloat16()
    w_qkv = (0.02 * torch.randn(3 * d, d, generator=g, device=dev)).bfloat16()
    w_o = (0.02 * torch.randn(d, d, generator=g, device=dev)).bfloat16()
    rw = torch.ones(d, device=dev)
    sp = HeadShardedPrefill(w_qkv, w_o, rw, H, EPS)
    del w_qkv
    out = torch.empty(B, T, d // world, device=dev)
    for _ in range(2):
        sp(x, out=out)
    torch.cuda.synchronize()
    barrier()
    torch.cuda.synchronize()
    stream = torch.cuda.current_stream(dev)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(passes):
        sp(x, out=out)
    e1.record(stream)
    torch.cuda.synchronize()
    ms = max_over_ranks(e0.elapsed_time(e1) / passes)
    _lib.check_device(dev.index or 0)
    barrier()
    sp.close()
    proj, intra, inter = prefill_flops(B, T, d, H, c["C"])
    total = proj + intra + inter
    per_gpu_tfl = total / world / (ms / 1e3) / 1e12
    nseg, seg_len = chunkwise_plan(torch.cuda.get_device_properties(dev).multi_processor_count, B, T, H // world)
    gather_bytes = (world - 1) * B * T * (d // world) * 2  # bf16 head outputs received per rank
    return {
        "metric": "long-context head-sharded prefill tok/s (B=1,T=65536,d=4096,H=16)",
        "value": B * T / (ms / 1e3), "unit": "tok/s", "ms_per_pass": ms, "passes": passes, "n_gpus": world,
        "scaling": "strong", "dtype": "bf16 (fp32 accumulate)",
        "config": {"workload": "MultiScaleRetention prefill, d_model=4096, 16 heads (head_dim 256), B=1, T=65536, "
                               "chunk 64", "parallelism": f"head-sharded x{world}, {H // world} heads per GPU, "
                                                          "one NCCL all-gather before W_o",
                   "segments": {"nseg": nseg, "seg_len": seg_len},
                   "l2": "inputs larger than L2 (x 512 MiB, qkv per GPU >= 192 MiB)"},
        "roofline": {"bound": "tensor", "achieved": per_gpu_tfl, "peak": peaks["bf16_tflops"], "unit": "TFLOP/s",
                     "per": "GPU", "frac": per_gpu_tfl / peaks["bf16_tflops"], "algorithmic_flop": total,
                     "allgather_bytes_per_rank": gather_bytes},
    }


# ---------------------------------------------------------------- stack
STACK = dict(L=24, d=2048, H=8, f=5632, V=32000, B=64, P=512, n=256)


def bench_stack(dev, peaks):
    import torch

    from aceflow_b200 import _lib
    from aceflow_b200.engine import AceEngine

    c = STACK
    L, d, H, f, V, B, P, n = (c[k] for k in ("L", "d", "H", "f", "V", "B", "P", "n"))
    g = torch.Generator(device=dev).manual_seed(11)
    eng = AceEngine(L, d, H, (0.02 * torch.randn(V, d, generator=g, device=dev)), batch=B,
                    device=str(dev), weight_dtype="bfloat16", eps=1e-6)
    for i in range(L):
        r = lambda *s: 0.02 * torch.randn(*s, generator=g, device=dev)  # noqa: E731
        one = torch.ones(d, device=dev)
        eng.load_layer_weights(i, r(3 * d, d), r(d, d), r(2 * f, d), r(d, f), one, one, one)
    prompts = torch.randint(0, V, (B, P), generator=g, device=dev).cpu().numpy()
    eng.generate_batch(prompts, 4, use_graph=True)  # warm-up (kernels, workspace)
    eng.reset_memory()
    t = {}
    toks = eng.generate_batch(prompts, n, use_graph=True, timing=t)
    _lib.check_device(dev.index or 0)
    params = L * (4 * d * d + 3 * f * d) + V * d
    pre_flop = 2 * params * B * P + L * sum(prefill_flops(B, P, d, H, 64)[1:])
    dec_bytes = 2 * params + 2 * L * B * H * (d // H) ** 2 * 4
    dec_ms = t["decode_ms"] / t["decode_steps"]
    return {
        "metric": "24-layer retention decoder: prefill and greedy decode tok/s",
        "config": {"workload": "24 x [RMSNorm -> MSR -> RMSNorm -> SwiGLU(5632)], d_model=2048, 8 heads, "
                               "vocab 32000 tied, bf16 weights, batch 64, 512-token prompt, 256 greedy steps",
                   "eps": 1e-6},
        "prefill_tok_s": B * P / (t["prefill_ms"] / 1e3), "prefill_ms": t["prefill_ms"],
        "prefill_tflops": pre_flop / (t["prefill_ms"] / 1e3) / 1e12,
        "prefill_frac": pre_flop / (t["prefill_ms"] / 1e3) / 1e12 / peaks["bf16_tflops"],
        "decode_tok_s": B / (dec_ms / 1e3), "decode_ms_per_step": dec_ms,
        "decode_hbm_gbs": dec_bytes / (dec_ms / 1e3) / 1e9,
        "decode_frac": dec_bytes / (dec_ms / 1e3) / 1e9 / peaks["hbm_gbs"],
        "decode_bytes_per_step": dec_bytes, "first_token_ms": t["first_token_ms"],
        "tokens_checksum": int(np.asarray(toks, np.int64).sum()),
    }


def main():
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=1024)
    ap.add_argument("--warmup", type=int, default=16)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline leg")
    ap.add_argument("--no-prefill", action="store_true", help="skip the prefill workload (N=1 only)")
    ap.add_argument("--no-stack", action="store_true", help="skip the 24-layer stack workload (N=1 only)")
    ap.add_argument("--prefill-passes", type=int, default=10)
    ap.add_argument("--no-longctx", action="store_true", help="skip the long-context head-sharded prefill")
    ap.add_argument("--only", choices=["prefill", "longctx", "stack"], default=None,
                    help="run one secondary workload alone and print its object (profiling)")
    ap.add_argument("--longctx-passes", type=int, default=5)
    args = ap.parse_args()
    if args.warmup < 3:
        ap.error("--warmup must be >= 3")
    if args.impl == "reference":
        return run_reference(args)
    return run_ours(args)


if __name__ == "__main__":
    sys.exit(main())
