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
# measured with ncu (dram__bytes_read.sum + dram__bytes_write.sum)
STATE_KERNEL_TRAFFIC = 555.808e6 + 483.676e6
EPS = 1e-6
PEAKS_FALLBACK = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0}


def sustained(achieved, peaks):
    """The fraction of the sustained bf16 peak (a matmul loop of seconds, at
    the 1 kW power cap), the denominator for work timed inside a long step
    (the long-context passes, the stack prefill); {} without that figure."""
    ps = peaks.get("bf16_tflops_sustained")
    return {"peak_sustained": ps, "frac_sustained": achieved / ps} if ps else {}


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


# ---------------------------------------------------------------- checker
def msr_rows_reference(x, w_qkv, w_o, ret_w, num_heads, eps, row_sets, col_range=None, w_g=None):
    """Rows of the MultiScaleRetention forward (aceflow/nn/retention.py:44-66:
    parallel retention, RMSNorm over d_model, W_o) for ONE stream, in float64
    on x's device, used as the parity checker of the large workloads.

    x [T, d] (any float dtype: the values the kernels read), w_qkv [3d, d]
    (rows q | k | v), w_o [d, d], ret_w [d]; row_sets: (r0, r1) ranges of
    output rows; col_range (c0, c1): only those output columns (the W_o rows a
    head-sharded rank owns); w_g [d, d]: the opt-in gated layer instead -
    swish(x W_g^T) * GroupNorm per head (mean 0, variance 1, eps inside the
    square root) replaces the RMSNorm (RetNet's gate, no reference counterpart).  The state before row r0 is formed in one
    product, S = K[:r0]^T diag(gamma^(r0-1-t)) V[:r0], so the cost does not
    grow with the number of chunks.  Returns one [r1 - r0, cols] tensor per set."""
    import torch

    f64 = torch.float64
    T, d = x.shape
    H, dh = num_heads, x.shape[1] // num_heads
    dev = x.device
    Wq, Wk, Wv = (w.to(f64) for w in w_qkv.chunk(3))
    Wo = w_o.to(f64)
    if col_range is not None:
        Wo = Wo[col_range[0]:col_range[1]]
    need = max(r1 for _, r1 in row_sets)
    x64 = x[:need].to(f64)
    K, V = x64 @ Wk.T, x64 @ Wv.T
    rw = ret_w.to(f64)
    outs = []
    for r0, r1 in row_sets:
        q = x64[r0:r1] @ Wq.T
        R = r1 - r0
        i = torch.arange(R, device=dev, dtype=f64)
        dist = i[:, None] - i[None, :]
        o = torch.empty(R, d, dtype=f64, device=dev)
        for h in range(H):
            g = 1.0 - 2.0 ** (-5 - h)
            sl = slice(h * dh, (h + 1) * dh)
            inter = torch.zeros(R, dh, dtype=f64, device=dev)
            if r0 > 0:
                w = g ** (r0 - 1 - torch.arange(r0, device=dev, dtype=f64))
                S = (K[:r0, sl] * w[:, None]).T @ V[:r0, sl]
                inter = (g ** (i + 1))[:, None] * (q[:, sl] @ S)
            D = torch.where(dist >= 0, g ** dist.clamp(min=0), torch.zeros((), dtype=f64, device=dev))
            o[:, sl] = inter + ((q[:, sl] @ K[r0:r1, sl].T) * D) @ V[r0:r1, sl]
        if w_g is None:
            o = o / torch.sqrt((o * o).mean(-1, keepdim=True) + eps) * rw
        else:
            oh = o.view(R, H, dh)
            oh = (oh - oh.mean(-1, keepdim=True)) / torch.sqrt(oh.var(-1, unbiased=False, keepdim=True) + eps)
            gg = x64[r0:r1] @ w_g.to(f64).T
            o = gg / (1.0 + torch.exp(-gg)) * oh.reshape(R, d)
        outs.append(o @ Wo.T)
    return outs


def backward_blocks_reference(qkv, dout, d, heads, T, n=128):
    """float64 gradients of the retention core (o_t = sum_{s<=t}
    gamma^(t-s) (q_t . k_s) v_s, aceflow/nn/retention.py:51-61) for one stream
    of T rows with no initial state, on blocks that need no other rows: dQ of
    rows [0, n) (no earlier rows) and dK, dV of rows [T-n, T) (no later rows),
    for each head in `heads`.  qkv [T, 3d] (q | k | v), dout [T, d], any float
    dtype, head_dim 256.  Returns {(h, "dq" | "dk" | "dv"): [n, 256]}."""
    import torch

    f64 = torch.float64
    dev = qkv.device
    i = torch.arange(n, device=dev, dtype=f64)
    res = {}
    for h in heads:
        gm = 1.0 - 2.0 ** (-5 - h)
        D = torch.where(i[:, None] >= i[None, :], gm ** (i[:, None] - i[None, :]).clamp(min=0),
                        torch.zeros((), dtype=f64, device=dev))  # D[t, s]
        cols = slice(h * 256, (h + 1) * 256)
        for r0, which in ((0, "dq"), (T - n, "dkdv")):
            Q, K, V = (qkv[r0:r0 + n, part * d:(part + 1) * d][:, cols].to(f64) for part in range(3))
            dO = dout[r0:r0 + n, cols].to(f64)
            if which == "dq":
                res[(h, "dq")] = ((dO @ V.T) * D) @ K
            else:
                res[(h, "dk")] = ((dO @ V.T) * D).T @ Q
                res[(h, "dv")] = ((Q @ K.T) * D).T @ dO
    return res


def max_rel_err(got_sets, ref_sets) -> float:
    """max |got - ref| / max |ref| over all sets (the parity metric)."""
    num = max(float((g.double() - r).abs().max()) for g, r in zip(got_sets, ref_sets))
    den = max(float(r.abs().max()) for r in ref_sets)
    return num / max(den, 1e-30)


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


def cpu_prefill_sample(seconds: float, nthreads: int, d: int, H: int, streams: int, piece: int = 8, seed: int = 0):
    """The reference's only CPU prefill, the token-serial recurrence
    (AceEngine.prefill_recurrent, cpu/mod.rs:547-587, per token the whole
    layer as its decode step: gemv_avx2 QKV, retention_step_core,
    rmsnorm_core, gemv_avx2 W_o), in the C restatement (oracle/cpu_ref.c,
    OpenMP over streams), on `min(streams, nthreads)` streams and successive
    `piece`-token slices until `seconds` elapse.  Its cost per token does not
    depend on the position, so tokens/s of this prefix is the rate of the
    whole prompt.  Returns (tok/s, tokens, streams, seconds, threads)."""
    from oracle import cpu_ref

    rng = np.random.default_rng(seed)
    dh = d // H
    B = max(1, min(streams, nthreads))
    w_qkv = (0.02 * rng.standard_normal((3 * d, d))).astype(np.float32)
    w_o = (0.02 * rng.standard_normal((d, d))).astype(np.float32)
    ret_w = np.ones(d, np.float32)
    gamma = np.array([1.0 - 2.0 ** (-5.0 - h) for h in range(H)], np.float32)
    state = np.zeros((B, H, dh, dh), np.float32)
    x = rng.standard_normal((B, piece, d)).astype(np.float32)
    threads = min(nthreads, B)
    cpu_ref.msr_prefill_recurrent(x[:, :1].copy(), state, gamma, w_qkv, w_o, ret_w, EPS, threads)  # warm
    toks, t0 = 0, time.perf_counter()
    while True:
        cpu_ref.msr_prefill_recurrent(x, state, gamma, w_qkv, w_o, ret_w, EPS, threads)
        toks += B * piece
        el = time.perf_counter() - t0
        if el >= seconds:
            break
    return toks / el, toks, B, el, threads


def cpu_stack_sample(seconds: float, nthreads: int, c: dict, sample_layers: int = 2, seed: int = 0):
    """Greedy decode of the decoder stack on the host (AceEngine.
    generate_stream_internal, cpu/mod.rs:708-769, in the C restatement
    oracle/cpu_ref.c: per token every layer's forward_layer_internal and the
    tied LM head), one stream per thread, on a model of `sample_layers`
    layers with the workload's other sizes.  The per-token cost is the
    memory traffic of fp32 weights, state and LM head, so the 24-layer rate is
    the sample's rate times bytes(sample) / bytes(24 layers).  Returns
    (tok/s at the full depth, sample tok/s, streams, seconds, description)."""
    from oracle import cpu_ref

    rng = np.random.default_rng(seed)
    d, H, f, V, L = c["d"], c["H"], c["f"], c["V"], c["L"]
    dh = d // H
    one = np.ones(d, np.float32)
    layers = [dict(w_qkv=(0.02 * rng.standard_normal((3 * d, d))).astype(np.float32),
                   w_o=(0.02 * rng.standard_normal((d, d))).astype(np.float32),
                   w_gate_up=(0.02 * rng.standard_normal((2 * f, d))).astype(np.float32),
                   w_down=(0.02 * rng.standard_normal((d, f))).astype(np.float32),
                   norm1=one, norm2=one, ret_norm=one) for _ in range(sample_layers)]
    emb = (0.02 * rng.standard_normal((V, d))).astype(np.float32)
    B = max(1, min(nthreads, c["B"]))
    prompts = rng.integers(0, V, (B, 1)).astype(np.int32)
    cpu_ref.generate_greedy(layers, emb, prompts, 1, H, 1e-6, nthreads=nthreads)  # warm
    n, el = 2, 0.0
    while True:
        t0 = time.perf_counter()
        cpu_ref.generate_greedy(layers, emb, prompts, n, H, 1e-6, nthreads=nthreads)
        el = time.perf_counter() - t0
        if el >= seconds or n >= 64:
            break
        n *= 2
    sample_rate = B * (n + 1) / el  # prompt token + n generated tokens per stream

    def token_bytes(nl):
        return 4 * (nl * (4 * d * d + 3 * f * d) + V * d) + 2 * 4 * nl * H * dh * dh

    rate = sample_rate * token_bytes(sample_layers) / token_bytes(L)
    desc = (f"{B} streams (one per thread) x {n + 1} tokens of a {sample_layers}-layer model with the workload's "
            f"sizes in {el:.1f} s, scaled to {L} layers by fp32 bytes per token "
            f"({token_bytes(sample_layers) / 1e9:.2f} -> {token_bytes(L) / 1e9:.2f} GB)")
    return rate, sample_rate, B, el, desc


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
            sec = bench_prefill(dev, args.prefill_passes, peaks, 0.0, args.chunk)
        elif args.only == "longctx":
            sec = bench_longctx(dev, world, rank, args.longctx_passes, peaks, barrier1, max1, 0.0,
                                args.longctx_chunk)
        else:
            sec = bench_stack(dev, peaks, steps=args.stack_steps)
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

    def per_rank(v):
        """Every rank's value (for the spread), gathered to all ranks."""
        if world == 1:
            return [v]
        t = torch.tensor([v], dtype=torch.float64, device=dev)
        parts = [torch.empty_like(t) for _ in range(world)]
        dist.all_gather(parts, t)
        return [float(p.item()) for p in parts]

    clocks = ClockSampler(local)
    with clocks:
        for i in range(args.warmup):
            step(i)
        torch.cuda.synchronize()
        # The K timed steps are captured once into a CUDA graph and replayed
        # as one launch: the device runs them back to back, whatever the host
        # (with 8 ranks, 8 Python processes plus NCCL proxy threads) does
        # meanwhile.  The same K steps issued eagerly are timed as well.
        graph = torch.cuda.CUDAGraph()
        cap = torch.cuda.Stream(dev)
        cap.wait_stream(stream)
        launches0 = _lib.launch_count(local)
        with torch.cuda.graph(graph, stream=cap):
            for i in range(args.steps):
                step(args.warmup + i)
        launches = _lib.launch_count(local) - launches0  # this library's kernels in one replay
        stream.wait_stream(cap)
        graph.replay()  # untimed first replay
        torch.cuda.synchronize()
        barrier()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        graph.replay()
        e1.record(stream)
        torch.cuda.synchronize()
        barrier()
        my_ms = e0.elapsed_time(e1)
        ms_all = per_rank(my_ms)
        ms_total = max(ms_all)
        # eager: the same K steps launched one by one from Python
        torch.cuda.synchronize()
        barrier()
        torch.cuda.synchronize()
        e0.record(stream)
        for i in range(args.steps):
            step(args.warmup + i)
        e1.record(stream)
        torch.cuda.synchronize()
        barrier()
        eager_all = per_rank(e0.elapsed_time(e1))
        del graph

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
        e2e_all = per_rank(run_e2e(args, dev, state, gamma, w_qkv_s, w_o_s, ret_w, cuda_ops, barrier))
        e2e_ms = max(e2e_all)

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
                     "traffic_source": "ncu dram__bytes_read.sum + dram__bytes_write.sum of one launch at this workload",
                     "kernel_ms": kernel_ms,
                     "algorithmic_bytes_per_launch": kbytes,
                     "step_bytes": step_bytes,
                     "step_frac": step_bytes / (ms_step / 1e3) / 1e9 / peaks["hbm_gbs"]},
        "e2e": {"value": world * B * args.steps / (e2e_ms / 1e3), "unit": "tok/s",
                "h2d_bytes_per_step": B * d * 4, "d2h_bytes_per_step": B * d * 4,
                "ms_per_step": e2e_ms / args.steps},
        "gpu_launches": int(launches),
        "timing": {"timed_region": "one CUDA-graph replay of the K steps (captured before timing)",
                   "eager_ms_per_step": max(eager_all) / args.steps,
                   "per_rank_ms_per_step": {"graph": [v / args.steps for v in ms_all],
                                            "eager": [v / args.steps for v in eager_all],
                                            "e2e": [v / args.steps for v in e2e_all]}},
        "clocks": clocks.summary(),
    }
    sub_cpu = args.sub_cpu_seconds if (world == 1 and not args.no_cpu) else 0.0
    if world == 1 and not args.no_prefill:
        line["prefill"] = bench_prefill(dev, args.prefill_passes, peaks, sub_cpu, args.chunk)
    if not args.no_longctx and HEADS_LONGCTX % world == 0:
        line["longctx"] = bench_longctx(dev, world, rank, args.longctx_passes, peaks, barrier, max_over_ranks,
                                        sub_cpu, args.longctx_chunk)
    if world == 1 and not args.no_stack:
        line["stack"] = bench_stack(dev, peaks, sub_cpu, steps=args.stack_steps)
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


def _phase_times(dev, fn):
    """Runs fn() once with the library's phase marks on; [(phase, ms)]."""
    from aceflow_b200 import _lib

    idx = dev.index or 0
    _lib.set_option(idx, "phase_marks", 1)
    try:
        fn()
        return [(n, round(ms, 4)) for n, ms in _lib.phase_times(idx)]
    finally:
        _lib.set_option(idx, "phase_marks", 0)


def bench_prefill(dev, passes, peaks, cpu_seconds=0.0, chunk=None):
    """The prefill workload through the reference's module API:
    af.nn.MultiScaleRetention(2048, 8).to("cuda:0") called on a bf16 prompt
    (the tensor-core chunkwise prefill), bf16 output, at the workload's chunk
    length (64) and at 128.  FLOPs are counted by the workload's definition
    (chunk 64) for both, so the two fractions compare time only."""
    import torch

    import aceflow_b200 as af
    from aceflow_b200 import _lib, cuda_ops

    c = PREFILL
    B, T, d, H = c["B"], c["T"], c["d"], c["H"]
    g = torch.Generator(device=dev).manual_seed(7)
    x = torch.randn(B, T, d, generator=g, device=dev).bfloat16()
    ws = [(0.02 * torch.randn(d, d, generator=g, device=dev)).bfloat16() for _ in range(4)]
    m = af.nn.MultiScaleRetention(d, H)
    for name, w in zip(("w_q", "w_k", "w_v", "w_o"), ws):
        setattr(m, name, af.nn.Parameter(af.Tensor(w.float())))
    m.to(str(dev))
    xt = af.Tensor(x, device=str(dev), dtype="bfloat16")
    stream = torch.cuda.current_stream(dev)
    proj, intra, inter = prefill_flops(B, T, d, H, c["C"])
    total = proj + intra + inter
    qkv = torch.randn(B * T, 3 * d, generator=g, device=dev).bfloat16()
    rw = torch.ones(d, device=dev)
    gamma = cuda_ops.gammas(H, dev)
    w_qkv = torch.cat(ws[:3]).contiguous()
    rows = [(0, 128), (T - 128, T)]
    ref = msr_rows_reference(x[0], w_qkv, ws[3], torch.ones(d, device=dev), H, EPS, rows)

    def measure(ck):
        m.prefill_chunk = ck
        out = None
        for _ in range(3):
            out = m(xt)
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(passes):
            out = m(xt)
        e1.record(stream)
        torch.cuda.synchronize()
        ms = e0.elapsed_time(e1) / passes
        phases = _phase_times(dev, lambda: m(xt))
        err = max_rel_err([out.torch[0, r0:r1] for r0, r1 in rows], ref)
        # the retention core alone (chunkwise kernel), CUDA events on its stream
        for _ in range(2):
            cuda_ops.retention_chunkwise_bf16(qkv, B, T, H, gamma, norm_w=rw, want_state=False, chunk=ck)
        e2, e3 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e2.record(stream)
        for _ in range(passes):
            cuda_ops.retention_chunkwise_bf16(qkv, B, T, H, gamma, norm_w=rw, want_state=False, chunk=ck)
        e3.record(stream)
        torch.cuda.synchronize()
        core_ms = e2.elapsed_time(e3) / passes
        _lib.check_device(dev.index or 0)
        tfl = total / (ms / 1e3) / 1e12
        core_tfl = (intra + inter) / (core_ms / 1e3) / 1e12
        kernel = "retention_chunk128_kernel" if ck == 128 else "retention_chunkwise_kernel<0>"
        return {"ms_per_pass": ms, "value": B * T / (ms / 1e3), "max_rel_err": err, "phases_ms": phases,
                "roofline": {"bound": "tensor", "achieved": tfl, "peak": peaks["bf16_tflops"], "unit": "TFLOP/s",
                             "frac": tfl / peaks["bf16_tflops"], "algorithmic_flop": total},
                "retention_core": {"kernel": kernel, "ms": core_ms, "achieved": core_tfl, "unit": "TFLOP/s",
                                   "frac": core_tfl / peaks["bf16_tflops"], "algorithmic_flop": intra + inter}}

    def measure_backward():
        """Backward of the chunkwise core (three retention passes, 128-token
        chunks): dQ, dK, dV for an upstream gradient, no initial state.  FLOPs:
        three cores by the workload's definition.  Checked on stream 0, heads 0
        and H-1: dQ on rows 0-127 (no earlier rows) and dK, dV on rows
        T-128..T-1 (no later rows), in float64."""
        dout = torch.randn(B * T, d, generator=g, device=dev).bfloat16()
        for _ in range(2):
            dq = cuda_ops.retention_chunkwise_backward_bf16(qkv, dout, B, T, H, gamma)[0]
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(passes):
            dq = cuda_ops.retention_chunkwise_backward_bf16(qkv, dout, B, T, H, gamma)[0]
        e1.record(stream)
        torch.cuda.synchronize()
        ms = e0.elapsed_time(e1) / passes
        _lib.check_device(dev.index or 0)
        blocks = backward_blocks_reference(qkv[:T], dout[:T], d, (0, H - 1), T)
        got, ref = [], []
        for (hh, which), rf in blocks.items():
            part = {"dq": 0, "dk": 1, "dv": 2}[which]
            r0 = 0 if which == "dq" else T - 128
            got.append(dq[r0:r0 + 128, part * d + hh * 256:part * d + (hh + 1) * 256])
            ref.append(rf)
        err = max(max_rel_err([gt], [rf]) for gt, rf in zip(got, ref))
        flop = 3 * (intra + inter)
        tfl = flop / (ms / 1e3) / 1e12
        return {"workload": f"backward of the chunkwise core, B={B}, T={T}, {H} heads, 128-token chunks "
                            "(dQ, dK, dV; af_retention_chunkwise_backward_bf16)",
                "ms": ms, "value": B * T / (ms / 1e3), "unit": "tok/s", "max_rel_err": err, "tolerance": 2e-2,
                "parity_rows": "stream 0, heads 0 and 7: dQ rows 0-127, dK and dV rows 3968-4095, against float64",
                "roofline": {"bound": "tensor", "achieved": tfl, "peak": peaks["bf16_tflops"], "unit": "TFLOP/s",
                             "frac": tfl / peaks["bf16_tflops"], "algorithmic_flop": flop}}

    def measure_gated():
        """The opt-in gated layer (swish gate, per-head GroupNorm) over the same
        prompt at chunk 64: five projections and the core."""
        wg = (0.02 * torch.randn(d, d, generator=g, device=dev)).bfloat16()
        out = None
        for _ in range(2):
            out, _ = cuda_ops.msr_gated_prefill_bf16(x, w_qkv, wg, ws[3], None, None, gamma, EPS,
                                                     out_dtype=torch.bfloat16, want_state=False)
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(passes):
            out, _ = cuda_ops.msr_gated_prefill_bf16(x, w_qkv, wg, ws[3], None, None, gamma, EPS,
                                                     out_dtype=torch.bfloat16, want_state=False)
        e1.record(stream)
        torch.cuda.synchronize()
        ms = e0.elapsed_time(e1) / passes
        _lib.check_device(dev.index or 0)
        gref = msr_rows_reference(x[0], w_qkv, ws[3], rw, H, EPS, rows, w_g=wg)
        err = max_rel_err([out[0, r0:r1] for r0, r1 in rows], gref)
        flop = total + 2 * B * T * d * d
        tfl = flop / (ms / 1e3) / 1e12
        return {"workload": f"gated MultiScaleRetention prefill (opt-in; no reference counterpart), B={B}, T={T}, "
                            f"d_model={d}, {H} heads, chunk 64 (af_msr_gated_prefill_bf16)",
                "ms_per_pass": ms, "value": B * T / (ms / 1e3), "unit": "tok/s", "max_rel_err": err,
                "tolerance": 2e-2, "parity_rows": "stream 0, rows 0-127 and 3968-4095, against float64",
                "roofline": {"bound": "tensor", "achieved": tfl, "peak": peaks["bf16_tflops"], "unit": "TFLOP/s",
                             "frac": tfl / peaks["bf16_tflops"], "algorithmic_flop": flop}}

    main = measure(c["C"] if chunk is None else chunk)
    alt = measure(128) if chunk is None else None
    m.prefill_chunk = 64
    res = {
        "metric": "retention prefill tok/s (B=8,T=4096,d=2048)", "value": main["value"], "unit": "tok/s",
        "ms_per_pass": main["ms_per_pass"], "passes": passes, "dtype": "bf16 (fp32 accumulate)",
        "config": {"workload": f"MultiScaleRetention prefill, d_model=2048, 8 heads, B=8, T=4096, "
                               f"chunk {c['C'] if chunk is None else chunk}",
                   "api": "af.nn.MultiScaleRetention(2048, 8).to('cuda') on a bf16 prompt",
                   "l2": "inputs larger than L2 (x 128 MiB, qkv 384 MiB)"},
        "max_rel_err": main["max_rel_err"], "tolerance": 2e-2,
        "parity_rows": "stream 0, rows 0-127 and 3968-4095, against float64",
        "phases_ms": main["phases_ms"], "roofline": main["roofline"], "retention_core": main["retention_core"],
    }
    if alt is not None:
        res["chunk128"] = alt
        res["backward"] = measure_backward()
        res["gated"] = measure_gated()
    if cpu_seconds > 0:
        v, toks, b, el, thr = cpu_prefill_sample(cpu_seconds, host_threads(), d, H, B)
        res["cpu_baseline"] = {"value": v, "unit": "tok/s", "cores": thr, "kind": "port",
                               "sample": f"{toks} tokens ({b} streams x {toks // b}) of the token-serial prefill "
                                         f"(AceEngine.prefill_recurrent, C restatement) in {el:.1f} s"}
    return res


# ---------------------------------------------------------------- long context
LONGCTX = dict(B=1, T=65536, d=4096, H=16, C=128)
HEADS_LONGCTX = LONGCTX["H"]


def bench_longctx(dev, world, rank, passes, peaks, barrier, max_over_ranks, cpu_seconds=0.0, chunk=64):
    """Head-sharded prefill of one 65536-token stream (d_model 4096, 16 heads)
    over all ranks: QKV of the rank's heads, chunkwise retention (sequence
    segments), the exchange of head outputs, output projection.  Two
    exchanges: the all-to-all (each rank owns output rows; 8x fewer bytes
    over NVLink at 8 GPUs than the all-gather), reported as the line's value,
    and the all-gather the workload names (each rank then owns output
    columns), reported beside it.  Total work is fixed, so N GPUs scale it
    strongly.  Rank 0 checks its own output against float64 in both."""
    import torch

    from aceflow_b200 import _lib
    from aceflow_b200.sharded import HeadShardedPrefill, chunkwise_plan, row_range

    c = LONGCTX
    B, T, d, H = c["B"], c["T"], c["d"], c["H"]
    g = torch.Generator(device=dev).manual_seed(11)  # same weights and input on every rank
    x = torch.randn(B, T, d, generator=g, device=dev).bfloat16()
    w_qkv = (0.02 * torch.randn(3 * d, d, generator=g, device=dev)).bfloat16()
    w_o = (0.02 * torch.randn(d, d, generator=g, device=dev)).bfloat16()
    rw = torch.ones(d, device=dev)
    stream = torch.cuda.current_stream(dev)
    check_rows = [(0, 128), (T // 2 - 64, T // 2 + 64), (T - 128, T)]
    proj, intra, inter = prefill_flops(B, T, d, H, chunk)
    total = proj + intra + inter
    res = {}
    for layout in ("columns", "rows"):
        sp = HeadShardedPrefill(w_qkv, w_o, rw, H, EPS, layout=layout, chunk=chunk)
        if layout == "columns":
            out = torch.empty(B, T, d // world, device=dev)
        else:
            out = torch.empty(row_range(B * T, world, rank)[1], d, device=dev)
        for _ in range(2):
            sp(x, out=out)
        torch.cuda.synchronize()
        barrier()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(passes):
            sp(x, out=out)
        e1.record(stream)
        torch.cuda.synchronize()
        ms = max_over_ranks(e0.elapsed_time(e1) / passes)
        barrier()
        phases = _phase_times(dev, lambda: sp(x, out=out))
        _lib.check_device(dev.index or 0)
        barrier()
        sp.close()
        err = None
        if rank == 0:  # rank 0's share of three row blocks against float64
            if layout == "columns":
                dl = d // world
                ref = msr_rows_reference(x[0], w_qkv, w_o, rw, H, EPS, check_rows, col_range=(0, dl))
                got = [out[0, r0:r1] for r0, r1 in check_rows]
            else:
                lo, n = row_range(B * T, world, 0)
                rows0 = [(lo, lo + 128), (lo + n - 128, lo + n)]  # the ends of rank 0's rows
                ref = msr_rows_reference(x[0], w_qkv, w_o, rw, H, EPS, rows0)
                got = [out[r0 - lo:r1 - lo] for r0, r1 in rows0]
            err = max_rel_err(got, ref)
            del ref
        barrier()
        per_gpu_tfl = total / world / (ms / 1e3) / 1e12
        res[layout] = {"ms_per_pass": ms, "value": B * T / (ms / 1e3), "phases_ms_rank0": phases,
                       "max_rel_err_rank0": err, "frac_per_gpu": per_gpu_tfl / peaks["bf16_tflops"],
                       "achieved_per_gpu": per_gpu_tfl}
    nseg, seg_len = chunkwise_plan(torch.cuda.get_device_properties(dev).multi_processor_count, B, T, H // world,
                                   chunk=chunk)
    gather_bytes = (world - 1) * B * T * (d // world) * 2  # bf16 head outputs received per rank
    a2a_bytes = (world - 1) * (-(-B * T // world)) * (d // world) * 2
    rows, col = res["rows"], res["columns"]
    line = {
        "metric": "long-context head-sharded prefill tok/s (B=1,T=65536,d=4096,H=16)",
        "value": rows["value"], "unit": "tok/s", "ms_per_pass": rows["ms_per_pass"], "passes": passes,
        "n_gpus": world, "scaling": "strong", "dtype": "bf16 (fp32 accumulate)",
        "config": {"workload": "MultiScaleRetention prefill, d_model=4096, 16 heads (head_dim 256), B=1, T=65536, "
                               f"chunk {chunk}",
                   "parallelism": f"head-sharded x{world}, {H // world} heads per GPU; NCCL all-to-all of the head "
                                  f"outputs, each rank owns {-(-B * T // world)} output rows and applies the full W_o",
                   "segments": {"nseg": nseg, "seg_len": seg_len},
                   "l2": "inputs larger than L2 (x 512 MiB, qkv per GPU >= 192 MiB)"},
        "max_rel_err": rows["max_rel_err_rank0"], "tolerance": 2e-2,
        "parity_rows": "the first and last 128 of rank 0's own rows against float64",
        "phases_ms_rank0": rows["phases_ms_rank0"],
        "roofline": {"bound": "tensor", "achieved": rows["achieved_per_gpu"], "peak": peaks["bf16_tflops"],
                     "unit": "TFLOP/s", "per": "GPU", "frac": rows["frac_per_gpu"], "algorithmic_flop": total,
                     "alltoall_bytes_per_rank": a2a_bytes, **sustained(rows["achieved_per_gpu"], peaks)},
        "allgather": {"parallelism": f"head-sharded x{world}; one NCCL all-gather of the head outputs before W_o, "
                                     "each rank owns output columns",
                      "bytes_received_per_rank": gather_bytes,
                      "parity_rows": "rank 0's output share of rows 0-127, 32704-32831, 65408-65535 against float64",
                      **col},
    }
    if cpu_seconds > 0 and rank == 0 and world == 1:
        v, toks, b, el, thr = cpu_prefill_sample(cpu_seconds, 1, d, H, B)
        line["cpu_baseline"] = {"value": v, "unit": "tok/s", "cores": thr, "kind": "port",
                                "sample": f"{toks} tokens of the one stream, token-serial (AceEngine.prefill_recurrent, "
                                          f"C restatement; one stream runs on one thread) in {el:.1f} s"}
    return line


# ---------------------------------------------------------------- stack
STACK = dict(L=24, d=2048, H=8, f=5632, V=32000, B=64, P=512, n=256)


def bench_stack(dev, peaks, cpu_seconds=0.0, steps=None):
    import torch

    from aceflow_b200 import _lib
    from aceflow_b200.engine import AceEngine

    c = STACK
    L, d, H, f, V, B, P, n = (c[k] for k in ("L", "d", "H", "f", "V", "B", "P", "n"))
    n = steps or n
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
    res = {
        "metric": "24-layer retention decoder: prefill and greedy decode tok/s",
        "config": {"workload": "24 x [RMSNorm -> MSR -> RMSNorm -> SwiGLU(5632)], d_model=2048, 8 heads, "
                               "vocab 32000 tied, bf16 weights, batch 64, 512-token prompt, 256 greedy steps",
                   "eps": 1e-6},
        "prefill_tok_s": B * P / (t["prefill_ms"] / 1e3), "prefill_ms": t["prefill_ms"],
        "prefill_tflops": pre_flop / (t["prefill_ms"] / 1e3) / 1e12,
        "prefill_frac": pre_flop / (t["prefill_ms"] / 1e3) / 1e12 / peaks["bf16_tflops"],
        "prefill_frac_sustained": sustained(pre_flop / (t["prefill_ms"] / 1e3) / 1e12, peaks).get("frac_sustained"),
        "decode_tok_s": B / (dec_ms / 1e3), "decode_ms_per_step": dec_ms,
        "decode_hbm_gbs": dec_bytes / (dec_ms / 1e3) / 1e9,
        "decode_frac": dec_bytes / (dec_ms / 1e3) / 1e9 / peaks["hbm_gbs"],
        "decode_bytes_per_step": dec_bytes, "first_token_ms": t["first_token_ms"],
        "tokens_checksum": int(np.asarray(toks, np.int64).sum()),
    }
    if cpu_seconds > 0:
        rate, sample_rate, b, el, desc = cpu_stack_sample(cpu_seconds, host_threads(), c)
        res["cpu_baseline"] = {"value": rate, "unit": "tok/s (decode)", "cores": b, "kind": "port",
                               "sample": desc, "sample_value": sample_rate}
    return res


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
    ap.add_argument("--stack-steps", type=int, default=None,
                    help="greedy steps of the stack workload (default: the workload's 256; fewer for profiling)")
    ap.add_argument("--sub-cpu-seconds", type=float, default=4.0,
                    help="seconds of each CPU baseline of the prefill, long-context and stack workloads (N=1)")
    ap.add_argument("--chunk", type=int, default=None,
                    help="chunk length of the prefill workload (default: the workload's 64, and 128 reported beside)")
    ap.add_argument("--longctx-chunk", type=int, default=LONGCTX["C"],
                    help="chunk length of the long-context workload (default: the workload's 128)")
    args = ap.parse_args()
    if args.warmup < 3:
        ap.error("--warmup must be >= 3")
    if args.impl == "reference":
        return run_reference(args)
    return run_ours(args)


if __name__ == "__main__":
    sys.exit(main())
