#!/usr/bin/env python
"""Delta-attention prefill throughput on B200 (the BASELINE.json metric).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference]

Workload (BASELINE.json config 2 at its headline point): one layer of delta
attention with Llama-3.1-8B attention shapes -- 32 query / 8 KV heads,
head_dim 128, N = 131072 tokens, window W = 2048, sink S = 128, stride
gamma = 64, bf16 -- on seeded synthetic post-RoPE q/k/v (N(0,1)*0.5,
RoPE theta 500000).  A step is one prefill of that layer.

Multi-GPU (torchrun, one process per GPU, NCCL only for the barrier and the
max-over-ranks timing): the work is partitioned by (sequence, KV group) unit
(``delta_attention_b200.sharding``); with ``--scaling weak`` (default) the
job holds one sequence per rank, so per-GPU work is fixed.

Printed JSON line (rank 0): ``value`` = tokens/s over the whole job with
inputs resident in HBM (inputs 1.6 GB per GPU > 126 MB L2, so no L2 flush);
``roofline`` for the prefill kernel (analytic FLOPs 4*H*d*(N*(W+S) + (N/gamma)*N/2)
over the live CUDA-event time of its launches, against MEASURED_PEAKS.json);
``e2e`` = the same metric through the reference-facing plug-in
(``DeltaAttention.delta_forward``) with pinned host inputs, host<->device
copies inside the timed region (consecutive steps overlap their upload,
compute and download on three streams); ``cpu_baseline`` = the CPU oracle on a
bounded row sample of the same workload on this host's cores.
``--impl reference`` times that CPU implementation as the reference arm.
"""

from __future__ import annotations

import argparse
import csv
import io
import json
import math
import os
import statistics
import select
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "delta-attn prefill tokens/s/GPU @128K (Llama-3.1-8B shapes); % bf16 TC peak"
FALLBACK_PEAKS = {"bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0, "hbm_gbs": 6650.0}


def parse_args():
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["b200", "reference"], default="b200")
    ap.add_argument("--seq", type=int, default=131072)
    ap.add_argument("--heads", type=int, default=32)
    ap.add_argument("--kv-heads", type=int, default=8)
    ap.add_argument("--head-dim", type=int, default=128)
    ap.add_argument("--window", type=int, default=2048)
    ap.add_argument("--sink", type=int, default=128)
    ap.add_argument("--gamma", type=int, default=64)
    ap.add_argument("--scaling", choices=["weak", "strong"], default="weak")
    ap.add_argument("--split-tiles", type=int, default=0,
                    help="key tiles per split-K chunk of the dense rows (0 = automatic)")
    ap.add_argument("--e2e-steps", type=int, default=10)
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--cpu-seconds", type=float, default=12.0, help="CPU baseline sample budget")
    ap.add_argument("--no-clocks", action="store_true")
    ap.add_argument("--op", choices=["prefill", "decode", "train"], default="prefill",
                    help="decode: HBM throughput of the dense / sparse / one-pass decode kernels; "
                         "train: forward + backward of one layer")
    ap.add_argument("--decode-caches", type=int, default=8,
                    help="distinct KV caches cycled through per decode replay (defeats L2 reuse)")
    return ap.parse_args()


def analytic_flops(H, d, N, W, S, gamma):
    """north_star FLOP count: 4*H*d*(N*(W+S) + (N/gamma)*N/2), split by launch."""
    window = 4.0 * H * d * N * (W + S)
    rows = 4.0 * H * d * (N / gamma) * N / 2.0
    return window + rows, window, rows


def load_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            return json.load(f), "measured"
    return dict(FALLBACK_PEAKS), "fallback"


# ---------------------------------------------------------------------------
# clocks sampler (nvidia-smi during the timed region)
# ---------------------------------------------------------------------------
class ClockSampler:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int, enabled: bool = True):
        self.gpu = gpu_index
        self.enabled = enabled
        self.proc = None
        self.out = ""
        self.pre = ""  # the sampler's first line, taken just before the timed region

    def __enter__(self):
        if self.enabled:
            try:
                self.proc = subprocess.Popen(
                    ["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                     "-lms", "100"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            except OSError:
                self.proc = None
            # nvidia-smi takes a few hundred ms to start: wait for its first
            # sample, so that a short timed region is sampled from its start
            if self.proc is not None:
                ready, _, _ = select.select([self.proc.stdout], [], [], 5.0)
                if ready:
                    self.pre = self.proc.stdout.readline()
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                rest, _ = self.proc.communicate(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
                rest, _ = self.proc.communicate()
            self.out = rest or ""
        return False

    def summary(self):
        rows = [r for r in csv.reader(io.StringIO(self.out)) if len(r) >= 9]
        note = None
        if not rows:
            # a timed region shorter than the sampling interval: report the
            # sample taken as it started
            rows = [r for r in csv.reader(io.StringIO(self.pre)) if len(r) >= 9]
            note = "timed region shorter than the 100 ms sampling interval; sample taken at its start"
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"], "samples": 0}
        sm = [float(r[1]) for r in rows if r[1].strip().replace(".", "").isdigit()]
        mx = [float(r[2]) for r in rows if r[2].strip().replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({n for r in rows for n, v in zip(names, r[5:9]) if v.strip().lower() == "active"})
        out = {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
               "reasons": reasons, "samples": len(rows)}
        if note:
            out["note"] = note
        return out


# ---------------------------------------------------------------------------
# CPU baseline: the oracle on a bounded row sample
# ---------------------------------------------------------------------------
def cpu_sample_inputs(args, r0, R, seed=0):
    """Seeded CPU inputs covering keys [0, r0+R) and query rows [r0, r0+R) of the workload."""
    import torch
    from delta_attention_b200.rope import apply_rope, cos_sin

    H, Hkv, d = args.heads, args.kv_heads, args.head_dim
    n = r0 + R
    g = torch.Generator().manual_seed(seed)
    q = torch.zeros(1, H, n, d)
    q[:, :, r0:] = torch.randn(1, H, R, d, generator=g) * 0.5
    k = torch.randn(1, Hkv, n, d, generator=g) * 0.5
    v = torch.randn(1, Hkv, n, d, generator=g) * 0.5
    cos, sin = cos_sin(torch.arange(n), d, 500000.0)
    q = apply_rope(q, cos, sin).bfloat16()
    k = apply_rope(k, cos, sin).bfloat16()
    return q, k, v.bfloat16()


def cpu_oracle_step(args, q, k, v, r0, R):
    """One bounded CPU step: delta output of rows [r0, r0+R) (sparse rows plus
    their anchors' dense and sparse rows), fp32, via the oracle."""
    import torch
    from oracle import delta_oracle as orc

    rows = torch.arange(r0, r0 + R)
    # the oracle needs the full sequence length for the layout; pad K/V views
    return orc.delta_forward_rows(_PadSeq(q, args.seq), _PadSeq(k, args.seq), _PadSeq(v, args.seq), rows,
                                  args.gamma, args.window, args.sink, dtype=torch.float32)


class _PadSeq:
    """View of a [b, h, n, d] tensor that reports sequence length ``s`` (>= n)
    for layout purposes; only rows < n are ever indexed by the sample."""

    def __init__(self, t, s):
        self.t = t
        self.shape = (t.shape[0], t.shape[1], s, t.shape[3])

    def __getitem__(self, idx):
        return self.t[idx]

    def to(self, *a, **kw):
        return self.t.to(*a, **kw)

    def float(self):
        return self


def cpu_calibration():
    """The committed record (tests/golden/cpu_timing.json, written by
    tests/golden/make_golden.py --timing-only where the reference checkout
    exists) of the reference's own CPU path against the oracle port on one
    host: the port is the CPU baseline timed here, and this says how its speed
    relates to the reference's own code.  None when the record is absent."""
    path = os.path.join(os.path.dirname(os.path.abspath(__file__)), "tests", "golden", "cpu_timing.json")
    try:
        with open(path) as f:
            rec = json.load(f)
    except (OSError, ValueError):
        return None
    return {k: rec[k] for k in ("what", "reference", "host_cpu", "threads", "reference_tokens_per_s",
                                "port_tokens_per_s", "port_over_reference") if k in rec}


def cpu_baseline(args, seconds):
    """Time the oracle on a row sample near N/2 sized to ~``seconds`` of CPU work.
    Returns (tokens/s, threads, description)."""
    import torch

    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    r0 = args.seq // 2
    R = 256
    q, k, v = cpu_sample_inputs(args, r0, 4096)
    t0 = time.perf_counter()
    cpu_oracle_step(args, q, k, v, r0, R)
    t_small = time.perf_counter() - t0
    R = int(max(256, min(4096, R * seconds / max(t_small, 1e-3))) // args.gamma * args.gamma)
    t0 = time.perf_counter()
    cpu_oracle_step(args, q, k, v, r0, R)
    dt = time.perf_counter() - t0
    desc = (f"oracle (torch CPU fp32) rows [{r0}, {r0 + R}) of the N={args.seq} layer, all {args.heads} heads, "
            f"with their {R // args.gamma} anchors' dense and sparse rows; tokens/s = rows / time")
    return R / dt, threads, desc


# ---------------------------------------------------------------------------
# reference arm
# ---------------------------------------------------------------------------
def run_reference(args, rank, world):
    if rank != 0:
        return 0
    import torch

    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    r0 = args.seq // 2
    q, k, v = cpu_sample_inputs(args, r0, 4096)
    budget = max(0.5, min(2.0, 150.0 / max(1, args.steps + args.warmup)))
    t0 = time.perf_counter()
    cpu_oracle_step(args, q, k, v, r0, 128)
    t_small = time.perf_counter() - t0
    R = int(max(args.gamma, min(4096, 128 * budget / max(t_small, 1e-3))) // args.gamma * args.gamma)
    for _ in range(args.warmup):
        cpu_oracle_step(args, q, k, v, r0, R)
    times = []
    for _ in range(args.steps):
        t0 = time.perf_counter()
        cpu_oracle_step(args, q, k, v, r0, R)
        times.append(time.perf_counter() - t0)
    total = sum(times)
    value = R * args.steps / total
    sample = (f"rows [{r0}, {r0 + R}) of the N={args.seq} layer per step (all {args.heads} heads, plus their "
              f"{R // args.gamma} anchors' dense and sparse rows), CPU oracle port fp32")
    line = {
        "metric": METRIC, "impl": "reference", "value": value, "unit": "tokens/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1000.0 * total / args.steps,
        "higher_is_better": True, "scaling": args.scaling, "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (seeded N(0,1)*0.5, RoPE theta 5e5)",
        "config": workload_config(args, world),
        "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": threads, "kind": "port", "sample": sample,
                         "calibration": cpu_calibration()},
        "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


def physical_gpu(local_rank: int) -> str:
    """nvidia-smi id of this process's GPU (honours CUDA_VISIBLE_DEVICES)."""
    vis = os.environ.get("CUDA_VISIBLE_DEVICES")
    if vis:
        ids = [x.strip() for x in vis.split(",") if x.strip()]
        if local_rank < len(ids):
            return ids[local_rank]
    return str(local_rank)


def workload_name(args):
    """The benchmark matrix entry the shapes belong to (config 2: Llama-3.1-8B
    attention, 32/8 heads, W=2048; config 5: Llama-3.1-70B attention, 64/8
    heads, W=4096), else a plain description of the shapes."""
    if (args.heads, args.kv_heads, args.head_dim, args.window, args.sink) == (32, 8, 128, 2048, 128):
        return "config2: single-layer delta-attention prefill, Llama-3.1-8B attention shapes"
    if (args.heads, args.kv_heads, args.head_dim, args.window, args.sink, args.gamma) == (64, 8, 128, 4096, 128, 64):
        return "config5: single-layer delta-attention prefill, Llama-3.1-70B attention shapes"
    return (f"single-layer delta-attention prefill, {args.heads}/{args.kv_heads} heads, d={args.head_dim}, "
            f"W={args.window}, S={args.sink}")


def workload_config(args, world):
    return {
        "workload": workload_name(args),
        "seq_len": args.seq, "n_heads": args.heads, "n_kv_heads": args.kv_heads, "head_dim": args.head_dim,
        "window": args.window, "sink": args.sink, "gamma": args.gamma, "sequences_per_gpu":
            (1 if args.scaling == "weak" else 1.0 / world), "partition": "kv-group units",
        "l2": "inputs 1.6 GB per GPU exceed the 126 MB L2; no flush",
    }


# ---------------------------------------------------------------------------
# decode (bench.py --op decode)
# ---------------------------------------------------------------------------
def run_decode(args, local_rank):
    """HBM throughput of dta_decode at config-2 shapes (one query row per head,
    a KV cache of --seq keys).  Bytes per call are the algorithmic K+V bytes
    read: 2 * Hkv * d * 2 B * keys, with keys = n (dense, and the one-pass
    dense+sparse anchor step) or sink + window (sparse).  Each timed replay is a
    CUDA graph of one call per cache over --decode-caches distinct caches whose
    total size exceeds L2 (the sparse calls additionally see an L2 flush before
    every replay), timed with CUDA events; value = median over --steps replays."""
    import torch

    from delta_attention_b200 import ops

    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    H, Hkv, d, n = args.heads, args.kv_heads, args.head_dim, args.seq
    C = max(1, args.decode_caches)
    gen = torch.Generator(device=dev).manual_seed(7)
    q = (torch.randn(1, H, 1, d, generator=gen, device=dev) * 0.5).bfloat16()
    caches = [((torch.randn(1, Hkv, n, d, generator=gen, device=dev) * 0.5).bfloat16(),
               (torch.randn(1, Hkv, n, d, generator=gen, device=dev) * 0.5).bfloat16()) for _ in range(C)]
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    peaks, peaks_src = load_peaks()
    kw = dict(window=args.window, sink=args.sink, scaling=d ** -0.5)
    sparse_keys = min(n, args.sink + args.window)
    modes = {
        "dense": (dict(want_dense=True, want_sparse=False), n),
        "sparse": (dict(want_dense=False, want_sparse=True), sparse_keys),
        "dense+sparse (anchor step)": (dict(want_dense=True, want_sparse=True), n),
    }
    results = {}
    sampler = ClockSampler(physical_gpu(local_rank), enabled=not args.no_clocks)
    with sampler:
        for name, (flags, keys) in modes.items():
            for _ in range(max(3, args.warmup)):
                for kc, vc in caches:
                    ops.decode(q, kc, vc, **kw, **flags)
            torch.cuda.synchronize()
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g):
                for kc, vc in caches:
                    ops.decode(q, kc, vc, **kw, **flags)
            times = []
            for _ in range(max(1, args.steps)):
                if flags.get("want_dense") is False:
                    flush.zero_()
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                e0.record()
                g.replay()
                e1.record()
                e1.synchronize()
                times.append(e0.elapsed_time(e1) / C)  # ms per call
            del g
            ms = statistics.median(times)
            nbytes = 2 * Hkv * d * 2 * keys
            gbs = nbytes / (ms * 1e-3) / 1e9
            results[name] = {"us_per_call": round(ms * 1e3, 2), "bytes_per_call": nbytes, "GB/s": round(gbs, 1),
                             "frac": round(gbs / peaks["hbm_gbs"], 4)}
    line = {
        "metric": "delta-attn decode HBM GB/s @128K (Llama-3.1-8B shapes, one layer, one token)",
        "op": "decode", "unit": "GB/s", "value": results["dense"]["GB/s"], "higher_is_better": True,
        "n_gpus": 1, "steps": args.steps, "dtype": "bf16", "data": "synthetic",
        "config": {"workload": "config2 decode: 32q/8kv heads, d=128, one query row per head",
                   "n_keys": n, "window": args.window, "sink": args.sink, "caches_per_replay": C,
                   "l2": f"{C} caches x {2 * Hkv * n * d * 2 / 1e6:.0f} MB cycled per replay; sparse replays after an L2 flush"},
        "roofline": {"bound": "hbm", "achieved": results["dense"]["GB/s"], "peak": peaks["hbm_gbs"], "unit": "GB/s",
                     "frac": results["dense"]["frac"], "peak_source": peaks_src,
                     "traffic": None, "traffic_note": "dense key set, ncu at n_keys=131072: 536.9 MB read + "
                                                      "6.3 MB partials written per call (the algorithmic bytes)"},
        "modes": results,
        "clocks": sampler.summary(),
    }
    print(json.dumps(line), flush=True)
    return 0


# ---------------------------------------------------------------------------
# training step of one layer (bench.py --op train)
# ---------------------------------------------------------------------------
def run_train(args, local_rank):
    """Forward + backward of one delta-attention layer through the autograd
    drop-in (``delta_attention_b200.train.delta_forward_train``), the
    reference's per-layer training measurement (Llama-8B dims, gamma 64, sink
    1024 + window 2048 when run with ``--sink 1024``; docs/STATS.md:302-318).
    Roofline: analytic training FLOPs = 3.5 x the forward's north_star count
    (forward 2 products per attended pair, backward 5), over the CUDA-event
    time of a step; the forward and the backward are also timed alone."""
    import torch

    from delta_attention_b200 import train

    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    H, Hkv, d, n = args.heads, args.kv_heads, args.head_dim, args.seq
    gen = torch.Generator(device=dev).manual_seed(0)
    q = (torch.randn(1, H, n, d, generator=gen, device=dev) * 0.5).bfloat16().requires_grad_(True)
    k = (torch.randn(1, Hkv, n, d, generator=gen, device=dev) * 0.5).bfloat16().requires_grad_(True)
    v = (torch.randn(1, Hkv, n, d, generator=gen, device=dev) * 0.5).bfloat16().requires_grad_(True)
    g = torch.randn(1, n, H, d, generator=gen, device=dev).bfloat16()
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    peaks, peaks_src = load_peaks()
    fwd_flops = analytic_flops(H, d, n, args.window, args.sink, args.gamma)[0]
    flops = 3.5 * fwd_flops

    def step():
        q.grad = k.grad = v.grad = None  # gradients are assigned, not accumulated (as after zero_grad)
        out = train.delta_forward_train(q, k, v, args.gamma, args.window, args.sink)
        out.backward(g)
        return out

    for _ in range(max(3, args.warmup)):
        step()
    torch.cuda.synchronize()
    times, t_fwd, t_bwd = [], [], []
    sampler = ClockSampler(physical_gpu(local_rank), enabled=not args.no_clocks)
    with sampler:
        for _ in range(max(1, args.steps)):
            flush.zero_()
            q.grad = k.grad = v.grad = None
            e = [torch.cuda.Event(enable_timing=True) for _ in range(3)]
            e[0].record()
            out = train.delta_forward_train(q, k, v, args.gamma, args.window, args.sink)
            e[1].record()
            out.backward(g)
            e[2].record()
            e[2].synchronize()
            t_fwd.append(e[0].elapsed_time(e[1]))
            t_bwd.append(e[1].elapsed_time(e[2]))
            times.append(e[0].elapsed_time(e[2]))
    ms = statistics.median(times)
    achieved = flops / (ms * 1e-3) / 1e12
    peak = float(peaks.get("bf16_tflops", FALLBACK_PEAKS["bf16_tflops"]))
    G = H // Hkv
    fused = G in (4, 8) and args.gamma >= 8 and args.gamma & (args.gamma - 1) == 0
    line = {
        "metric": "delta-attn training step (forward + backward) of one layer, tokens/s", "op": "train",
        "value": n / (ms * 1e-3), "unit": "tokens/s", "higher_is_better": True, "n_gpus": 1, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms, "dtype": "bf16", "data": "synthetic (seeded N(0,1)*0.5 q/k/v)",
        "config": {"workload": "single-layer delta-attention forward + backward (reference training protocol)",
                   "seq_len": n, "n_heads": H, "n_kv_heads": Hkv, "head_dim": d, "window": args.window,
                   "sink": args.sink, "gamma": args.gamma, "l2": "256 MB flush before every step"},
        "roofline": {"bound": "tensor", "achieved": achieved, "peak": peak, "unit": "TFLOP/s",
                     "frac": achieved / peak, "peak_source": peaks_src, "flops_per_step": flops,
                     "flops_note": "3.5 x 4*H*d*(N*(W+S) + (N/gamma)*N/2)"},
        "phases_ms": {"forward": statistics.median(t_fwd), "backward": statistics.median(t_bwd)},
        # forward: rows + windowed launches (+ the delta kernel when not fused);
        # backward: prep, plan, key-major, two query-major, finalize
        "gpu_launches": ((2 if fused else 3) + 6) * args.steps,
        "clocks": sampler.summary(),
    }
    print(json.dumps(line), flush=True)
    return 0


# ---------------------------------------------------------------------------
# B200 arm
# ---------------------------------------------------------------------------
def run_b200(args, rank, world, local_rank):
    import torch
    import torch.distributed as dist

    from delta_attention_b200 import ops
    from delta_attention_b200._lib import PHASE_ROWS, PHASE_WINDOW
    from delta_attention_b200.sharding import job_for, owned_units

    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    H, Hkv, d, N = args.heads, args.kv_heads, args.head_dim, args.seq
    G = H // Hkv
    n_seqs = job_for(args.scaling, world, Hkv)
    units = owned_units(n_seqs, Hkv, world, rank)
    U = len(units)
    # this rank's units stacked along the batch axis: q [U, G, N, d], k/v [U, 1, N, d]
    gen = torch.Generator(device=dev).manual_seed(1000 + rank)
    q = (torch.randn(U, G, N, d, generator=gen, device=dev, dtype=torch.float32) * 0.5)
    k = (torch.randn(U, 1, N, d, generator=gen, device=dev, dtype=torch.float32) * 0.5)
    v = (torch.randn(U, 1, N, d, generator=gen, device=dev, dtype=torch.float32) * 0.5).bfloat16()
    from delta_attention_b200.rope import apply_rope, cos_sin
    cos, sin = cos_sin(torch.arange(N, device=dev), d, 500000.0)
    q = apply_rope(q, cos, sin).bfloat16()
    k = apply_rope(k, cos, sin).bfloat16()
    del cos, sin
    out = torch.empty(U, N, G, d, dtype=torch.bfloat16, device=dev)
    kw = dict(gamma=args.gamma, window=args.window, sink=args.sink, scaling=d ** -0.5,
              split_tiles=args.split_tiles)
    # one workspace, reused across steps (the kernels never allocate)
    ws = ops.prefill_workspace(U, G, 1, N, d, gamma=args.gamma, window=args.window, sink=args.sink,
                               split_tiles=args.split_tiles, device=dev)

    def step():
        # one call, both launches: the windowed launch may start on SMs the
        # rows launch has finished with (programmatic dependent launch)
        ops.prefill(q, k, v, **kw, workspace=ws, out=out)

    def step_split(evs):
        # diagnostic: the two launches as separate calls, timed apart
        evs[0].record()
        ops.prefill(q, k, v, **kw, workspace=ws, out=out, phases=PHASE_ROWS)
        evs[1].record()
        ops.prefill(q, k, v, **kw, workspace=ws, out=out, phases=PHASE_WINDOW)
        evs[2].record()

    for _ in range(max(args.warmup, 3)):
        step()
    torch.cuda.synchronize()
    ops.check_errors()
    t_start = torch.cuda.Event(enable_timing=True)
    t_end = torch.cuda.Event(enable_timing=True)
    with ClockSampler(physical_gpu(local_rank), enabled=not args.no_clocks) as clk:
        # (the sampler is running before the barrier that starts the timed region)
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        t_start.record()
        for i in range(args.steps):
            step()
        t_end.record()
        torch.cuda.synchronize()
    ops.check_errors()
    if world > 1:
        dist.barrier()
    ms_total = t_start.elapsed_time(t_end)
    # per-launch split (untimed for the headline; a few steps)
    n_split = min(args.steps, 10)
    evs = [[torch.cuda.Event(enable_timing=True) for _ in range(3)] for _ in range(n_split)]
    for i in range(n_split):
        step_split(evs[i])
    torch.cuda.synchronize()
    ops.check_errors()
    ms_rows = sum(e[0].elapsed_time(e[1]) for e in evs) / n_split
    ms_win = sum(e[1].elapsed_time(e[2]) for e in evs) / n_split
    if world > 1:
        t = torch.tensor([ms_total, ms_rows, ms_win], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms_total, ms_rows, ms_win = t.tolist()
    ms_step = ms_total / args.steps
    tokens_per_step_job = N * n_seqs
    value = tokens_per_step_job / (ms_step / 1000.0)

    # roofline of the prefill kernel (both launches are the same kernel function)
    flops_unit, flops_win_unit, flops_rows_unit = analytic_flops(G, d, N, args.window, args.sink, args.gamma)
    flops_rank = flops_unit * U
    peaks, peak_kind = load_peaks()
    peak = float(peaks.get("bf16_tflops", FALLBACK_PEAKS["bf16_tflops"]))
    # both launches are the same kernel function; under the dependent launch
    # they overlap, so the kernel's time per step is the step time
    ms_kernels = ms_step
    achieved = flops_rank / (ms_kernels / 1000.0) / 1e12
    traffic = None
    tpath = os.path.join(ROOT, "profiles", "prefill_traffic.json")
    if os.path.exists(tpath):
        with open(tpath) as f:
            tj = json.load(f)
        same = (tj.get("seq"), tj.get("gamma"), tj.get("window"), tj.get("sink"), tj.get("heads"),
                tj.get("kv_heads"), tj.get("head_dim")) == (N, args.gamma, args.window, args.sink, args.heads,
                                                             args.kv_heads, args.head_dim)
        if same and (world == 1 or args.scaling == "weak"):  # one whole sequence per rank
            traffic = tj.get("bytes_per_step")

    # e2e through the plug-in with pinned host buffers (rank-local units)
    e2e = None
    if not args.no_e2e:
        from delta_attention_b200.attention import DeltaAttention
        from delta_attention_b200.config import Config

        class _ModelCfg:
            pass

        mc = _ModelCfg()
        c = Config(delta_lambda=args.gamma, sliding_window=args.window, sink=args.sink, mode="delta")
        for f_ in ("mode", "delta_lambda", "sliding_window", "sink", "q_block", "log_drift", "stride_policy"):
            setattr(mc, f_, getattr(c, f_))
        mc.num_attention_heads, mc.num_key_value_heads, mc.head_dim = G, 1, d
        plug = DeltaAttention(mc)
        qh, kh, vh = q.cpu().pin_memory(), k.cpu().pin_memory(), v.cpu().pin_memory()
        # Steps are pipelined the way a serving loop overlaps transfers: step i's
        # host->device copies (copy stream), its plug-in call (compute stream)
        # and its device->host read of the output (a second copy stream) each
        # wait only for what they need, with device inputs and host outputs
        # double-buffered, so step i+1's upload runs during step i's compute.
        # Every step still moves its own 1.6 GB in and its output out.
        oh = [torch.empty(U, N, G, d, dtype=torch.bfloat16).pin_memory() for _ in range(2)]
        dbuf = [(torch.empty_like(q), torch.empty_like(k), torch.empty_like(v)) for _ in range(2)]
        s_up, s_comp, s_down = torch.cuda.Stream(), torch.cuda.Stream(), torch.cuda.Stream()
        in_ready = [torch.cuda.Event() for _ in range(2)]
        comp_done = [torch.cuda.Event() for _ in range(2)]
        used = [False, False]

        def e2e_step(i):
            bsl = i & 1
            qd, kd, vd = dbuf[bsl]
            if used[bsl]:
                s_up.wait_event(comp_done[bsl])  # step i-2 has finished reading these inputs
            with torch.cuda.stream(s_up):
                qd.copy_(qh, non_blocking=True)
                kd.copy_(kh, non_blocking=True)
                vd.copy_(vh, non_blocking=True)
                in_ready[bsl].record(s_up)
            s_comp.wait_event(in_ready[bsl])
            with torch.cuda.stream(s_comp):
                o, _ = plug.delta_forward(plug, qd, kd, vd, None, scaling=d ** -0.5)
                comp_done[bsl].record(s_comp)
            s_down.wait_event(comp_done[bsl])
            with torch.cuda.stream(s_down):
                oh[bsl].copy_(o, non_blocking=True)
            o.record_stream(s_down)
            used[bsl] = True

        for i in range(2):
            e2e_step(i)
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        s0, s1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s0.record(s_up)
        for i in range(args.e2e_steps):
            e2e_step(2 + i)
        s1.record(s_down)  # after the last step's output read, which waited for all of its work
        torch.cuda.synchronize()
        ms_e2e = s0.elapsed_time(s1) / args.e2e_steps
        if world > 1:
            t = torch.tensor([ms_e2e], device=dev, dtype=torch.float64)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            ms_e2e = t.item()
        e2e = {"value": tokens_per_step_job / (ms_e2e / 1000.0), "unit": "tokens/s",
               "h2d_bytes_per_step": int(qh.numel() * 2 + kh.numel() * 2 + vh.numel() * 2) * world,
               "d2h_bytes_per_step": int(oh[0].numel() * 2) * world, "ms_per_step": ms_e2e,
               "path": "DeltaAttention.delta_forward (plug-in surface) with pinned host q/k/v and output; "
                       "upload, compute and download of consecutive steps overlap on three streams"}
        del qh, kh, vh, oh, dbuf

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        val, cores, desc = cpu_baseline(args, args.cpu_seconds)
        cpu = {"value": val, "unit": "tokens/s", "cores": cores, "kind": "port", "sample": desc,
               "calibration": cpu_calibration()}

    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
            "warmup": max(args.warmup, 3), "ms_per_step": ms_step, "higher_is_better": True,
            "scaling": args.scaling, "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic (seeded N(0,1)*0.5 q/k/v, RoPE theta 5e5 on q/k)",
            "config": workload_config(args, world),
            "roofline": {"bound": "tensor", "achieved": achieved, "peak": peak, "unit": "TFLOP/s",
                         "frac": achieved / peak, "traffic": traffic, "peak_source": peak_kind,
                         "kernel": "dta::prefill_kernel<128> (rows launch + windowed launch)",
                         "flops_per_step": flops_rank,
                         "frac_of_sustained": achieved / float(peaks.get("bf16_tflops_sustained", 1400.0))},
            "launches": {
                "note": "each launch timed alone (separate calls, no overlap), outside the timed steps",
                "rows": {"ms": ms_rows, "tflops": flops_rows_unit * U / (ms_rows / 1000.0) / 1e12},
                "window": {"ms": ms_win, "tflops": flops_win_unit * U / (ms_win / 1000.0) / 1e12},
            },
            "cpu_baseline": cpu,
            "e2e": e2e,
            # two prefill launches per step, plus the delta kernel unless the
            # windowed launch forms delta itself (4 or 8 heads per KV head,
            # gamma a power of two >= 8)
            "gpu_launches": (2 if (G in (4, 8) and args.gamma >= 8 and args.gamma & (args.gamma - 1) == 0)
                             else 3) * args.steps,
            "clocks": clk.summary(),
        }
        print(json.dumps(line), flush=True)
    return 0


def main():
    args = parse_args()
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if args.gpus != world and world == 1 and args.gpus > 1:
        print(json.dumps({"error": f"--gpus {args.gpus} needs torchrun with {args.gpus} processes"}), flush=True)
        return 2
    if args.impl == "reference":
        return run_reference(args, rank, world)
    if args.op == "decode":
        if world > 1:
            print(json.dumps({"error": "--op decode runs on one GPU"}), flush=True)
            return 2
        return run_decode(args, local_rank)
    if args.op == "train":
        if world > 1:
            print(json.dumps({"error": "--op train runs on one GPU"}), flush=True)
            return 2
        return run_train(args, local_rank)
    if world > 1:
        import datetime

        # NCCL writes its log (version banner, communicator lines) to stdout;
        # rank 0's stdout must hold only the result line, so the log goes to
        # stderr at whatever NCCL_DEBUG level the caller chose
        os.environ.setdefault("NCCL_DEBUG_FILE", "/dev/stderr")
        import torch
        import torch.distributed as dist
        torch.cuda.set_device(local_rank)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device("cuda", local_rank))
    try:
        return run_b200(args, rank, world, local_rank)
    finally:
        if world > 1:
            import torch.distributed as dist
            dist.destroy_process_group()


if __name__ == "__main__":
    sys.exit(main())
