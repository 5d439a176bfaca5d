#!/usr/bin/env python3
"""Benchmark: the ConvRot W4A4 linear at FLUX shapes on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

One step = one pass of the full W4A4 path (fused rotate + A4 quantize, then the
tcgen05 int4 x int4 GEMM with the scale / bias / bf16 epilogue fused) over the
FLUX linear sweep: M in {1536, 4096} x (K, N) in {(3072, 3072), (3072, 9216),
(3072, 12288), (12288, 3072), (15360, 3072), (3072, 21504)}, group 256,
K x packed-N weights (the reference's default ``mpp-w4a4`` layout).  The metric
is whole-job throughput in tera int-ops/s (2 M N K per linear).  One JSON line
is printed by rank 0.

Timing: the step is captured once as a CUDA graph (12 prep + 12 GEMM launches)
and replayed K times between CUDA events on its stream.  The rooflines come
from graphs of the 12 GEMMs alone and the 12 preps alone, timed the same way.
The per-step working set (~1.2 GB) is ~10x the 126 MB L2, and no two
consecutive linears share an operand, so every linear reads cold inputs.
``e2e`` is the same metric through the public API (``ConvRotLinear``) with
host buffers: pinned host -> device copy of each input and device -> host copy
of each output inside the timed region.  ``--impl reference`` times the
reference's eager path (the CPU restatement in ``oracle/torch_cpu.py``) on the
host cores, on a bounded row sample of the same sweep.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))

import numpy as np  # noqa: E402
import torch  # noqa: E402

M_VALUES = (1536, 4096)
KN_PAIRS = ((3072, 3072), (3072, 9216), (3072, 12288), (12288, 3072), (15360, 3072), (3072, 21504))
GROUP = 256
SEED = 20260823
METRIC = "full W4A4 linear TOPS at FLUX shapes vs dense bf16"
UNIT = "TOPS"


def sweep_shapes():
    # all M = 1536 shapes first, then M = 4096: a weight is reused only after
    # five other linears (hundreds of MB) have passed through L2
    return [(m, k, n) for m in M_VALUES for (k, n) in KN_PAIRS]


def total_ops(shapes) -> int:
    return sum(2 * m * k * n for m, k, n in shapes)


# ---------------------------------------------------------------------------
# distributed plumbing


def dist_setup(n_gpus: int):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime

        torch.cuda.set_device(local)
        torch.distributed.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                             device_id=torch.device("cuda", local))
    elif torch.cuda.is_available():
        torch.cuda.set_device(0)
    return rank, world, local


def barrier(world):
    if world > 1:
        torch.distributed.barrier()


def max_over_ranks(value: float, world: int) -> float:
    if world == 1:
        return value
    t = torch.tensor([value], dtype=torch.float64, device="cuda")
    torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
    return float(t.item())


# ---------------------------------------------------------------------------
# clocks


class ClockSampler:
    """nvidia-smi samples (200 ms) of the local GPU during the timed region."""

    QUERY = ("uuid,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, uuid: str):
        self.uuid = uuid.lower().replace("gpu-", "")
        self.proc = None
        self.lines: list[str] = []

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.QUERY}", "--format=csv,noheader,nounits",
                 "-lms", "200"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self._t = threading.Thread(target=self._read, daemon=True)
            self._t.start()
        except OSError:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        rows = []
        for line in self.lines:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9 or parts[0].lower().replace("gpu-", "") != self.uuid:
                continue
            try:
                rows.append(dict(sm=float(parts[1]), max=float(parts[2]), power=float(parts[3]),
                                 hw=parts[5], hw_thermal=parts[6], sw_thermal=parts[7], power_cap=parts[8]))
            except ValueError:
                continue
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"], "samples": 0}
        loaded = [r for r in rows if r["power"] > 200] or rows
        reasons = set()
        for r in loaded:
            for key, name in (("hw", "hw_slowdown"), ("hw_thermal", "hw_thermal_slowdown"),
                              ("sw_thermal", "sw_thermal_slowdown"), ("power_cap", "sw_power_cap")):
                if r[key].lower() in ("active", "1", "yes"):
                    reasons.add(name)
        return {"sm_mhz": statistics.median(r["sm"] for r in loaded), "sm_max_mhz": max(r["max"] for r in rows),
                "reasons": sorted(reasons), "samples": len(loaded), "power_w_max": max(r["power"] for r in rows)}


# ---------------------------------------------------------------------------
# workload construction


def make_linear(k: int, n: int, seed: int, device):
    """A random-init FLUX-like linear: W ~ N(0, 0.02), bias ~ N(0, 0.01) (fp32)."""

    import convrot_mlx_b200 as cr

    g = torch.Generator(device=device).manual_seed(seed)
    w = (torch.randn((n, k), generator=g, device=device, dtype=torch.float32) * 0.02).to(torch.bfloat16)
    bias = torch.randn((n,), generator=g, device=device, dtype=torch.float32) * 0.01
    qnk, ws = cr.quantize_convrot_weight(w, GROUP)
    layer = cr.ConvRotLinear(k, n, group_size=GROUP, backend="mpp-w4a4", device=device)
    layer.qweight = cr.repack_nk_weight_for_mpp(qnk)
    layer.scales = ws
    layer.bias = bias
    return layer, w, qnk


def make_activation(m: int, k: int, seed: int, device):
    """x ~ N(0, 1) with 1% of channels (seeded choice) scaled x20 as outliers."""

    g = torch.Generator(device=device).manual_seed(seed)
    x = torch.randn((m, k), generator=g, device=device, dtype=torch.float32)
    idx = torch.randperm(k, generator=torch.Generator().manual_seed(seed))[: max(1, (k + 99) // 100)]
    x[:, idx.to(device)] *= 20.0
    return x.to(torch.bfloat16)


def measure_int8_peak(device) -> float:
    """Dense int8 tensor throughput of cuBLASLt (torch._int_mm) at 8192^3, best of 10."""

    a = torch.randint(-64, 64, (8192, 8192), dtype=torch.int8, device=device)
    b = torch.randint(-64, 64, (8192, 8192), dtype=torch.int8, device=device)
    bt = b.t()
    for _ in range(3):
        torch._int_mm(a, bt)
    torch.cuda.synchronize()
    best = float("inf")
    for _ in range(10):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        torch._int_mm(a, bt)
        e1.record()
        torch.cuda.synchronize()
        best = min(best, e0.elapsed_time(e1))
    del a, b
    return 2 * 8192**3 / (best * 1e-3) / 1e12


def load_peaks():
    path = ROOT / "MEASURED_PEAKS.json"
    if path.exists():
        d = json.loads(path.read_text())
        return {"hbm_gbs": d.get("hbm_gbs", 6650.0), "bf16_tflops": d.get("bf16_tflops", 1590.0), "source": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "source": "fallback"}


def load_traffic():
    path = ROOT / "profiles" / "traffic.json"
    if path.exists():
        return json.loads(path.read_text())
    return {}


# ---------------------------------------------------------------------------
# our arm


def run_ours(args, rank, world, local):
    import convrot_mlx_b200 as cr
    from convrot_mlx_b200 import _lib, core

    device = torch.device("cuda", local if world > 1 else 0)
    shapes = sweep_shapes()
    peaks = load_peaks()
    int8_peak = measure_int8_peak(device)

    layers, dense_w, xs_dev = {}, {}, []
    for i, (k, n) in enumerate(KN_PAIRS):
        layers[(k, n)], dense_w[(k, n)], _ = make_linear(k, n, SEED + i, device)
    for j, (m, k, n) in enumerate(shapes):
        xs_dev.append(make_activation(m, k, SEED + 100 + j, device))
    torch.cuda.synchronize()

    # preallocated intermediates so the captured step has fixed addresses
    bufs = []
    for (m, k, n), x in zip(shapes, xs_dev):
        bufs.append(dict(codes=torch.empty((m, k), dtype=torch.int8, device=device),
                         xs=torch.empty((m,), dtype=torch.float32, device=device),
                         out=torch.empty((m, n), dtype=torch.bfloat16, device=device)))
    lib = _lib.load()
    stream = torch.cuda.Stream(device=device)

    def enqueue(prep=True, gemm=True):
        s = _lib.stream_of(xs_dev[0])
        for j, ((m, k, n), x) in enumerate(zip(shapes, xs_dev)):
            layer, b = layers[(k, n)], bufs[j]
            if prep:
                _lib.check(lib.convrot_prepare_i8(_lib.ptr(x), _lib.BF16, m, k, GROUP, _lib.ptr(b["codes"]),
                                                  _lib.ptr(b["xs"]), s), "prep")
            if gemm:
                _lib.check(lib.convrot_w4a4_gemm(_lib.ptr(b["codes"]), _lib.ptr(layer.qweight), _lib.LAYOUT_KN,
                                                 _lib.ptr(b["xs"]), _lib.ptr(layer.scales), _lib.ptr(layer.bias),
                                                 _lib.ptr(b["out"]), _lib.BF16, m, n, k, s), "gemm")

    def capture(fn, reps=1):
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=stream):
            for _ in range(reps):
                fn()
        return g

    def replay_ms(g, reps):
        """Run ``g`` ``reps`` times on ``stream`` between two CUDA events."""
        with torch.cuda.stream(stream):
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            for _ in range(reps):
                g.replay()
            e1.record(stream)
        torch.cuda.synchronize()
        return e0.elapsed_time(e1)

    # warm-up (eager), then one graph per kind of pass: the full step (prep +
    # GEMM for all 12 linears), the 12 GEMMs alone, the 12 preps alone
    with torch.cuda.stream(stream):
        for _ in range(max(1, args.warmup)):
            enqueue()
    torch.cuda.synchronize()
    step_graph = capture(enqueue)
    gemm_graph = capture(lambda: enqueue(prep=False))
    prep_graph = capture(lambda: enqueue(gemm=False))
    replay_ms(step_graph, args.warmup)

    # parity spot check of the benchmarked path against the public layer call
    ref = layers[KN_PAIRS[0]](xs_dev[0])
    assert torch.equal(ref, bufs[0]["out"]), "benchmark path and ConvRotLinear disagree"

    # ---- timed region: K steps
    barrier(world)
    torch.cuda.synchronize()
    with ClockSampler(str(torch.cuda.get_device_properties(device).uuid)) as clocks:
        # nvidia-smi samples every 200 ms while the timed region lasts a few ms:
        # untimed replays keep the GPU under the same load for ~0.6 s before
        # and ~0.4 s after it, and the samples of that window are reported
        load_until = time.perf_counter() + 0.6
        while time.perf_counter() < load_until:
            replay_ms(step_graph, 8)
        elapsed_ms = replay_ms(step_graph, args.steps)
        load_until = time.perf_counter() + 0.4
        while time.perf_counter() < load_until:
            replay_ms(step_graph, 8)
    barrier(world)
    elapsed_ms = max_over_ranks(elapsed_ms, world)
    # kernel-kind sweeps for the rooflines: same cold-operand order, events only at the ends
    replay_ms(gemm_graph, 1)
    gemm_sweep_ms = replay_ms(gemm_graph, args.steps) / args.steps
    replay_ms(prep_graph, 1)
    prep_sweep_ms = replay_ms(prep_graph, args.steps) / args.steps
    # isolated per-shape GEMM times (each shape's GEMM replayed back to back)
    per_shape = []
    for j, (m, k, n) in enumerate(shapes):
        b, layer = bufs[j], layers[(k, n)]

        def one(j=j, m=m, k=k, n=n, b=b, layer=layer):
            s = _lib.stream_of(xs_dev[0])
            _lib.check(lib.convrot_w4a4_gemm(_lib.ptr(b["codes"]), _lib.ptr(layer.qweight), _lib.LAYOUT_KN,
                                             _lib.ptr(b["xs"]), _lib.ptr(layer.scales), _lib.ptr(layer.bias),
                                             _lib.ptr(b["out"]), _lib.BF16, m, n, k, s), "gemm")

        g1 = capture(one, reps=3)
        replay_ms(g1, 1)
        us = replay_ms(g1, 2) / 6 * 1e3
        per_shape.append({"m": m, "k": k, "n": n, "gemm_us_isolated": round(us, 2),
                          "gemm_tops_isolated": round(2 * m * k * n / (us * 1e-6) / 1e12, 1)})
        del g1
    ops = total_ops(shapes)
    ms_per_step = elapsed_ms / args.steps
    value = world * ops * args.steps / (elapsed_ms * 1e-3) / 1e12
    # ---- dense bf16 cuBLAS on the same sweep (graph-captured, same L2 conditions)
    outs_dense = [torch.empty((m, n), dtype=torch.bfloat16, device=device) for (m, k, n) in shapes]

    biases_bf16 = {kn: layers[kn].bias.to(torch.bfloat16) for kn in KN_PAIRS}

    def dense_step_addmm():
        for j, ((m, k, n), x) in enumerate(zip(shapes, xs_dev)):
            torch.addmm(biases_bf16[(k, n)], x, dense_w[(k, n)].t(), out=outs_dense[j])

    with torch.cuda.stream(stream):
        for _ in range(max(1, args.warmup)):
            dense_step_addmm()
    torch.cuda.synchronize()
    dgraph = capture(dense_step_addmm)
    replay_ms(dgraph, 1)
    dense_ms = replay_ms(dgraph, args.steps) / args.steps
    dense_tflops = ops / (dense_ms * 1e-3) / 1e12
    del dgraph

    # ---- W4A16 backend (rotate, then the kind::f16 GEMM) on the same sweep and weights
    rot_bufs = [torch.empty((m, k), dtype=torch.bfloat16, device=device) for (m, k, n) in shapes]
    out16 = [torch.empty((m, n), dtype=torch.bfloat16, device=device) for (m, k, n) in shapes]

    def w4a16_step():
        s = _lib.stream_of(xs_dev[0])
        for j, ((m, k, n), x) in enumerate(zip(shapes, xs_dev)):
            layer = layers[(k, n)]
            _lib.check(lib.convrot_rotate(_lib.ptr(x), _lib.BF16, m, k, GROUP, _lib.ptr(rot_bufs[j]), s), "rotate")
            _lib.check(lib.convrot_w4a16_gemm(_lib.ptr(rot_bufs[j]), _lib.BF16, _lib.ptr(layer.qweight), _lib.LAYOUT_KN,
                                              _lib.ptr(layer.scales), _lib.ptr(layer.bias), _lib.ptr(out16[j]),
                                              _lib.BF16, m, n, k, s), "w4a16 gemm")

    with torch.cuda.stream(stream):
        for _ in range(max(1, args.warmup)):
            w4a16_step()
    torch.cuda.synchronize()
    g16 = capture(w4a16_step)
    replay_ms(g16, 1)
    w4a16_ms = replay_ms(g16, args.steps) / args.steps
    del g16, rot_bufs, out16

    # ---- end to end through the public API with host buffers
    e2e = run_e2e(args, shapes, layers, xs_dev, device, world)

    # ---- rooflines
    gemm_tops = ops / (gemm_sweep_ms * 1e-3) / 1e12
    prep_bytes = sum(2 * m * k + m * k + 4 * m for m, k, n in shapes)
    prep_gbs = prep_bytes / (prep_sweep_ms * 1e-3) / 1e9
    traffic = load_traffic()
    bf16_x2 = 2 * peaks["bf16_tflops"]
    roofline = {
        "kernel": "pair_gemm_kernel (tcgen05.mma.cta_group::2 kind::i8, 256x256 pair tiles)", "bound": "tensor",
        "achieved": round(gemm_tops, 1), "peak": round(int8_peak, 1), "unit": "TFLOP/s",
        "frac": round(gemm_tops / int8_peak, 4),
        "peak_source": "dense int8 tensor ops/s of cuBLASLt (torch._int_mm 8192^3, burst) measured in this run; "
                       "MEASURED_PEAKS.json has no int8 entry; nominal 4500",
        "frac_of_2x_measured_bf16": round(gemm_tops / bf16_x2, 4),
        "bf16_x2_peak": round(bf16_x2, 1),
        "ops_note": "int8 tensor ops, 2 M N K per linear; time = the 12 GEMMs of one sweep in a CUDA graph, "
                    "CUDA events on the launching stream, averaged over the K timed sweeps",
        "traffic": traffic.get("gemm_bytes_per_launch"),
    }
    roofline_prep = {
        "kernel": "prep_kernel (fused rotate + A4 quantize, int8 codes)", "bound": "hbm",
        "achieved": round(prep_gbs, 1), "peak": peaks["hbm_gbs"], "unit": "GB/s",
        "frac": round(prep_gbs / peaks["hbm_gbs"], 4), "peak_source": f"MEASURED_PEAKS.json hbm_gbs ({peaks['source']})",
        "bytes_note": "2MK (bf16 in) + MK (int8 codes) + 4M (scales) per launch; time = the 12 preps of one sweep",
        "traffic": traffic.get("prep_bytes_per_launch"),
    }
    cpu = run_cpu_baseline(args, shapes, quick=True) if (rank == 0 and world == 1 and not args.no_cpu) else None
    line = {
        "metric": METRIC, "value": round(value, 2), "unit": UNIT, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(ms_per_step, 4), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "int8 (A4 codes x W4 nibbles, int32 accumulate), bf16 I/O",
        "data": "synthetic, seeded: W ~ N(0, 0.02), bias ~ N(0, 0.01), x ~ N(0, 1) with 1% outlier channels x20",
        "config": {
            "workload": "flux-linear-sweep (BASELINE config 3, W4A4 backend mpp-w4a4)",
            "shapes_mkn": [list(s) for s in shapes], "group_size": GROUP, "weight_layout": "K x packed-N int4",
            "io_dtype": "bf16", "parallelism": f"replicas x{world} (batch data-parallel, no collective)",
            "l2": "per-step working set ~1.2 GB >> 126 MB L2; consecutive linears share no operand",
            "timing": "CUDA graph of one step replayed K times between CUDA events on its stream",
        },
        "gemm_ms_per_sweep": round(gemm_sweep_ms, 4), "prep_ms_per_sweep": round(prep_sweep_ms, 4),
        "dense_bf16": {"value": round(dense_tflops, 1), "unit": "TFLOP/s", "ms_per_step": round(dense_ms, 4),
                       "impl": "torch.addmm bf16 (cuBLAS), same sweep, graph-captured"},
        "speedup_vs_dense_bf16": round(dense_ms / ms_per_step, 3),
        "w4a16": {"value": round(ops / (w4a16_ms * 1e-3) / 1e12, 1), "unit": UNIT, "ms_per_step": round(w4a16_ms, 4),
                  "speedup_vs_dense_bf16": round(dense_ms / w4a16_ms, 3),
                  "impl": "rotate (prep kernel) + W4A16 tcgen05 kind::f16 GEMM, same sweep and weights, graph-captured"},
        "roofline": roofline, "roofline_prep": roofline_prep,
        "e2e": e2e,
        "gpu_launches": 2 * len(shapes) * args.steps,
        "clocks": dict(clocks.summary(), window="nvidia-smi 200 ms samples over ~1 s of step replays enclosing "
                                                  "the timed region"),
        "cpu_baseline": cpu,
        "per_shape": per_shape,
        "device_error": _lib.take_device_error(),
    }
    del step_graph, gemm_graph, prep_graph
    return line


def run_e2e(args, shapes, layers, xs_dev, device, world):
    """Public API end to end: pinned host x -> device, ConvRotLinear, output ->
    pinned host, every step.  A step is a three-stage pipeline over the 12
    linears on three streams (upload j + 1 while computing j while
    downloading j - 1), and consecutive steps overlap the same way.  The K
    timed steps are captured as one CUDA graph (the same calls; the replay
    copies every step's inputs from and outputs to pinned host memory) and
    replayed once -- the reported value, as host-side jitter cannot stretch
    it -- and also run eagerly from Python (``eager_ms_per_step``)."""

    host_x = [x.cpu().pin_memory() for x in xs_dev]
    host_out = [torch.empty((m, n), dtype=torch.bfloat16).pin_memory() for (m, k, n) in shapes]
    h2d = sum(x.numel() * 2 for x in host_x)
    d2h = sum(o.numel() * 2 for o in host_out)
    copy_in, compute, copy_out = (torch.cuda.Stream(device=device) for _ in range(3))

    def steps(n, keep=None):
        # n pipelined steps; steps overlap one another on the three streams.
        # keep (a list): hold every tensor instead of record_stream, so that
        # nothing freed in a graph capture is handed to another stream
        for _ in range(n):
            done_in, done_c = [], []
            for hx in host_x:
                with torch.cuda.stream(copy_in):
                    xd = hx.to(device, non_blocking=True)
                    ev = torch.cuda.Event()
                    ev.record(copy_in)
                done_in.append((xd, ev))
            for j, (m, k, n_) in enumerate(shapes):
                xd, ev = done_in[j]
                with torch.cuda.stream(compute):
                    compute.wait_event(ev)
                    y = layers[(k, n_)](xd)
                    evc = torch.cuda.Event()
                    evc.record(compute)
                done_c.append((y, evc))
                if keep is None:
                    xd.record_stream(compute)
            for j, (y, evc) in enumerate(done_c):
                with torch.cuda.stream(copy_out):
                    copy_out.wait_event(evc)
                    host_out[j].copy_(y, non_blocking=True)
                if keep is None:
                    y.record_stream(copy_out)
            if keep is not None:
                keep.extend(t for t, _ in done_in + done_c)

    def timed(run, n_steps, stream):
        # events on `stream`, max with the wall clock, max over ranks
        torch.cuda.synchronize()
        barrier(world)
        t0 = time.perf_counter()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        run(n_steps)
        torch.cuda.synchronize()
        e1.record(stream)
        torch.cuda.synchronize()
        wall = time.perf_counter() - t0
        return max_over_ranks(max(e0.elapsed_time(e1), wall * 1e3), world)

    steps(max(1, args.warmup))
    eager_ms = timed(steps, args.steps, copy_in)

    # the same K steps captured as one CUDA graph: the three streams fork from
    # the capturing stream once and join it once, so the steps overlap as above
    main = torch.cuda.Stream(device=device)
    g = torch.cuda.CUDAGraph()
    keep = []
    torch.cuda.synchronize()
    with torch.cuda.stream(main):
        with torch.cuda.graph(g, stream=main):
            start = torch.cuda.Event()
            start.record(main)
            for side in (copy_in, compute, copy_out):
                side.wait_event(start)
            steps(args.steps, keep)
            for side in (copy_in, compute, copy_out):
                end = torch.cuda.Event()
                end.record(side)
                main.wait_event(end)
        del keep
        g.replay()  # warm-up: K steps
        dev_ms = timed(lambda n: g.replay(), args.steps, main)
    value = world * total_ops(shapes) * args.steps / (dev_ms * 1e-3) / 1e12
    del g

    # the same bytes with no compute: every upload on one stream, every
    # download (of preallocated device outputs) on another, concurrently
    dev_out = [torch.empty((m, n), dtype=torch.bfloat16, device=device) for (m, k, n) in shapes]
    dev_in = [torch.empty_like(x) for x in xs_dev]

    def copies():
        for hx, dx in zip(host_x, dev_in):
            with torch.cuda.stream(copy_in):
                dx.copy_(hx, non_blocking=True)
        for ho, do in zip(host_out, dev_out):
            with torch.cuda.stream(copy_out):
                ho.copy_(do, non_blocking=True)

    copies()
    torch.cuda.synchronize()
    c0 = time.perf_counter()
    for _ in range(args.steps):
        copies()
    torch.cuda.synchronize()
    copy_ms = (time.perf_counter() - c0) * 1e3 / args.steps
    del dev_out, dev_in
    return {"value": round(value, 2), "unit": UNIT, "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
            "ms_per_step": round(dev_ms / args.steps, 3), "eager_ms_per_step": round(eager_ms / args.steps, 3),
            "copy_only_ms_per_step": round(copy_ms, 3), "frac_of_copy_bound": round(copy_ms / (dev_ms / args.steps), 3),
            "api": "ConvRotLinear.forward (mpp-w4a4) with pinned-host inputs and outputs, copies overlapped on "
                   "three streams; the K timed steps captured as one CUDA graph and replayed once "
                   "(eager_ms_per_step: the same calls made from Python)"}


# ---------------------------------------------------------------------------
# CPU reference (the reference's eager path, restated in torch CPU)


def run_cpu_baseline(args, shapes, quick: bool):
    """Time ``oracle/torch_cpu.linear`` (the reference's ``backend="reference"``
    eager path) on a row sample of every shape and extrapolate linearly in M.
    The weight unpack (per call in the reference) is timed once per shape and
    charged once per linear; prep and matmul scale with the rows."""

    from oracle import torch_cpu as TC

    cores = len(os.sched_getaffinity(0))
    torch.set_num_threads(cores)
    sample_rows = 128
    reps = 1 if quick else 2
    rng = np.random.default_rng(SEED)
    t_total = 0.0
    for (m, k, n) in shapes:
        x = torch.from_numpy(rng.normal(size=(sample_rows, k)).astype(np.float32)).to(torch.bfloat16)
        qnk = torch.from_numpy(rng.integers(0, 256, size=(n, k // 2), dtype=np.uint8))
        ws = torch.full((n,), 0.01)
        b = torch.zeros(n)
        t0 = time.perf_counter()
        wu = TC.unpack(qnk).to(torch.float32)
        t_unpack = time.perf_counter() - t0
        TC.linear(x, qnk, ws, b, GROUP, weight_unpacked=wu)  # warm
        ts = []
        for _ in range(reps):
            t0 = time.perf_counter()
            TC.linear(x, qnk, ws, b, GROUP, weight_unpacked=wu)
            ts.append(time.perf_counter() - t0)
        t_total += t_unpack + min(ts) * (m / sample_rows)
        del wu
    value = total_ops(shapes) / t_total / 1e12
    return {"value": round(value, 5), "unit": UNIT, "cores": cores, "kind": "port",
            "sample": f"{sample_rows} rows of each of the {len(shapes)} sweep linears, timed and scaled linearly "
                      "to full M; weight unpack charged once per linear; torch CPU restatement of the "
                      "reference eager path (prep + reference_w4a4_matmul), bit-exact to the oracle",
            "seconds_per_step_extrapolated": round(t_total, 3)}


def run_reference(args, rank, world):
    if rank != 0:
        return None
    shapes = sweep_shapes()
    for _ in range(args.warmup):
        run_cpu_baseline(args, shapes[:1], quick=True)
    vals = []
    t0 = time.perf_counter()
    for _ in range(args.steps):
        vals.append(run_cpu_baseline(args, shapes, quick=True))
    wall = time.perf_counter() - t0
    v = statistics.median(r["value"] for r in vals)
    cpu = dict(vals[0])
    cpu["value"] = v
    return {
        "metric": METRIC, "value": v, "unit": UNIT, "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(1e3 * total_ops(shapes) / (v * 1e12), 3), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "fp32-held integers, bf16 I/O",
        "data": "synthetic, seeded", "impl": "reference",
        "config": {"workload": "flux-linear-sweep (BASELINE config 3, reference eager path on CPU)",
                   "shapes_mkn": [list(s) for s in shapes], "group_size": GROUP},
        "cpu_baseline": cpu,
        "e2e": {"value": v, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "wall_s": round(wall, 2),
        "note": "MLX is not installable here (Apple-only wheels); the reference's eager contract is timed as its "
                "torch-CPU restatement (oracle/torch_cpu.py), with all host threads",
    }

# ---------------------------------------------------------------------------
# shared timing helper


def graph_ms(fn, reps: int, stream, warm: int = 1) -> float:
    """Capture ``fn`` once as a CUDA graph on ``stream`` and return the mean
    milliseconds of ``reps`` replays between CUDA events on that stream."""

    with torch.cuda.stream(stream):
        fn()
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=stream):
        fn()
    with torch.cuda.stream(stream):
        for _ in range(warm):
            g.replay()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(reps):
            g.replay()
        e1.record(stream)
    torch.cuda.synchronize()
    del g
    return e0.elapsed_time(e1) / reps


# ---------------------------------------------------------------------------
# the fused rotate + A4 quantize alone

C2_M, C2_K = 4096, 3072


def run_c2(args, device):
    """Prep-only throughput at BASELINE config 2 (x bf16 4096 x 3072 ~ N(0, 1)
    with 1% outlier channels x20) for groups 64 and 256, int8 codes out.
    One CUDA graph launches the kernel over 8 distinct inputs (200 MB of
    input, > the 126 MB L2), replayed between CUDA events."""

    from convrot_mlx_b200 import _lib

    lib = _lib.load()
    peaks = load_peaks()
    n_in = 8
    xs = [make_activation(C2_M, C2_K, SEED + 300 + i, device) for i in range(n_in)]
    codes = [torch.empty((C2_M, C2_K), dtype=torch.int8, device=device) for _ in range(n_in)]
    scales = [torch.empty((C2_M,), dtype=torch.float32, device=device) for _ in range(n_in)]
    stream = torch.cuda.Stream(device=device)
    bytes_per_launch = 2 * C2_M * C2_K + C2_M * C2_K + 4 * C2_M
    out = {"shape": [C2_M, C2_K], "bytes_per_launch": bytes_per_launch, "peak_gbs": peaks["hbm_gbs"],
           "timing": "graph of 8 launches on 8 distinct inputs (> L2), CUDA events"}
    for group in (64, 256):
        def launches(group=group):
            s = _lib.stream_of(xs[0])
            for i in range(n_in):
                _lib.check(lib.convrot_prepare_i8(_lib.ptr(xs[i]), _lib.BF16, C2_M, C2_K, group, _lib.ptr(codes[i]),
                                                  _lib.ptr(scales[i]), s), "prep")

        ms = graph_ms(launches, max(3, args.steps), stream) / n_in
        gbs = bytes_per_launch / (ms * 1e-3) / 1e9
        out[f"g{group}"] = {"us_per_launch": round(ms * 1e3, 2), "gbs": round(gbs, 1),
                            "frac": round(gbs / peaks["hbm_gbs"], 4)}
    del xs, codes, scales
    return out


# ---------------------------------------------------------------------------
# few activation rows: the swap-AB GEMM (BASELINE config 1 and the FLUX
# modulation linears at m = batch)

SMALL_M_SHAPES = ((8, 3072, 18432), (8, 3072, 9216), (1, 3072, 18432), (64, 1024, 1024))


def run_small_m(args, device):
    """The W4A4 GEMM at m <= 64, HBM-bound on the packed weights: per shape,
    a CUDA graph of launches over distinct weights (> L2 in total) replayed
    between CUDA events; achieved GB/s = (packed weights + activation codes
    + output) / time against MEASURED_PEAKS.json hbm_gbs.  Beside it the same
    GEMM forced onto the register-fragment GEMV kernel (m <= 8), the
    swap-AB tcgen05 kernel and the CTA-pair kernel, and dense bf16 (cuBLAS)
    on the same shape."""

    from convrot_mlx_b200 import _lib

    lib = _lib.load()
    peaks = load_peaks()
    stream = torch.cuda.Stream(device=device)
    out = []
    for (m, k, n) in SMALL_M_SHAPES:
        w_bytes = k * n // 2
        n_w = max(2, int(300e6 // w_bytes) + 1)
        g = torch.Generator(device=device).manual_seed(m + k + n)
        qs = [torch.randint(0, 256, (k, n // 2), generator=g, device=device, dtype=torch.uint8) for _ in range(n_w)]
        codes = torch.randint(-7, 8, (m, k), generator=g, device=device, dtype=torch.int8)
        xs = torch.rand((m,), generator=g, device=device)
        ws = torch.rand((n,), generator=g, device=device) * 0.01
        bias = torch.randn((n,), generator=g, device=device) * 0.01
        o = torch.empty((m, n), dtype=torch.bfloat16, device=device)

        def launches():
            st = _lib.stream_of(codes)
            for q in qs:
                _lib.check(lib.convrot_w4a4_gemm(_lib.ptr(codes), _lib.ptr(q), _lib.LAYOUT_KN, _lib.ptr(xs), _lib.ptr(ws),
                                                 _lib.ptr(bias), _lib.ptr(o), _lib.BF16, m, n, k, st), "gemm")

        us = graph_ms(launches, max(3, args.steps), stream) / n_w * 1e3
        _lib.check(lib.convrot_set_gemm_route(2), "route")
        pair_us = graph_ms(launches, max(3, args.steps), stream) / n_w * 1e3
        _lib.check(lib.convrot_set_gemm_route(3), "route")
        swap_us = graph_ms(launches, max(3, args.steps), stream) / n_w * 1e3
        gemv_us = None
        if m <= 8:
            _lib.check(lib.convrot_set_gemm_route(4), "route")
            gemv_us = round(graph_ms(launches, max(3, args.steps), stream) / n_w * 1e3, 2)
        _lib.check(lib.convrot_set_gemm_route(0), "route")
        dw = [torch.randn((n, k), generator=g, device=device).to(torch.bfloat16) for _ in range(max(2, n_w // 4))]
        xd = torch.randn((m, k), generator=g, device=device).to(torch.bfloat16)
        bd = bias.to(torch.bfloat16)
        od = torch.empty((m, n), dtype=torch.bfloat16, device=device)

        def dense():
            for wd in dw:
                torch.addmm(bd, xd, wd.t(), out=od)

        dense_us = graph_ms(dense, max(3, args.steps), stream) / len(dw) * 1e3
        algo = w_bytes + m * k + 2 * m * n + 8 * n + 4 * m
        gbs = algo / (us * 1e-6) / 1e9
        out.append({"m": m, "k": k, "n": n, "us": round(us, 2), "gbs": round(gbs, 1),
                    "frac": round(gbs / peaks["hbm_gbs"], 4), "kernel": "gemv" if m <= 8 else "pair",
                    "gemv_kernel_us": gemv_us, "swap_ab_kernel_us": round(swap_us, 2),
                    "pair_kernel_us": round(pair_us, 2),
                    "dense_bf16_us": round(dense_us, 2), "speedup_vs_dense_bf16": round(dense_us / us, 2)})
        del qs, dw
    return {"kernel": "default routing: gemv_kernel (per-warp cp.async rings of packed weights, byte-permuted "
                      "into mma.sync m16n8k32 s8 register fragments, K split over warps and a cluster, DSMEM "
                      "reduction) for m <= 8, else pair_gemm_kernel",
            "bound": "hbm", "peak_gbs": peaks["hbm_gbs"],
            "bytes_note": "packed weights K N / 2 + codes M K + bf16 output 2 M N + scales/bias 8 N + 4 M per launch",
            "shapes": out, "device_error": _lib.take_device_error()}


# ---------------------------------------------------------------------------
# the FLUX DiT, batch 8 split data-parallel (no collective)


def run_dit(args, rank, world, local, gens: int, warm_gens: int):
    """20-step generation latency of the random-init FLUX.1-dev DiT
    (``flux_dit.py``) on 1024 image + 512 text tokens, batch 8 split over the
    ranks with no collective: dense bf16, then with every eligible linear
    swapped for ConvRotLinear (mpp-w4a4, g256) and the modulated norms fused
    into the activation preparation.  One denoise step (forward + Euler
    update) is captured as a CUDA graph; a generation is 20 replays, timed
    with CUDA events, max over ranks."""

    import flux_dit
    from convrot_mlx_b200 import _lib
    from convrot_mlx_b200.adapter import replace_convrot_linears

    device = torch.device("cuda", local if world > 1 else 0)
    total_batch, steps_per_gen = 8, 20
    if total_batch % world:
        raise SystemExit(f"batch {total_batch} does not split over {world} GPUs")
    b = total_batch // world
    model = flux_dit.build_flux_dit(device, SEED)
    flux_dit.build_glue()
    model.fuse_attention_glue = True  # both arms: the q/k norm + rotary + attention layout kernel
    img, txt, y, ids = flux_dit.dit_inputs(b, device, SEED + 7 + rank)
    with torch.no_grad():
        rope = model.rotary(ids)
    guidance = torch.full((b,), 3.5, device=device)
    ts = torch.linspace(1.0, 0.0, steps_per_gen + 1, device=device)
    t_cur, t_next = torch.zeros((b,), device=device), torch.zeros((b,), device=device)
    x = img.clone()

    def denoise_step():
        v = model(x, txt, rope, t_cur, y, guidance)
        x.add_((t_next - t_cur)[:, None, None].to(x.dtype) * v)

    def generation_ms(reps):
        stream = torch.cuda.Stream(device=device)
        with torch.no_grad(), torch.cuda.stream(stream):
            for _ in range(2):
                denoise_step()
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.no_grad(), torch.cuda.graph(graph, stream=stream):
            denoise_step()

        def generation():
            x.copy_(img)
            for i in range(steps_per_gen):
                t_cur.fill_(float(ts[i]))
                t_next.fill_(float(ts[i + 1]))
                graph.replay()

        with torch.cuda.stream(stream):
            for _ in range(max(1, warm_gens)):
                generation()
        torch.cuda.synchronize()
        barrier(world)
        with torch.cuda.stream(stream):
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            for _ in range(reps):
                generation()
            e1.record(stream)
        torch.cuda.synchronize()
        barrier(world)
        ms = max_over_ranks(e0.elapsed_time(e1) / reps, world)
        del graph
        return ms

    dense_ms = generation_ms(gens)
    replaced = replace_convrot_linears(model, backend="mpp-w4a4")
    torch.cuda.empty_cache()
    model.fuse_modulated_norm = False
    unfused_ms = generation_ms(max(1, gens // 2))
    model.fuse_modulated_norm = True
    with ClockSampler(str(torch.cuda.get_device_properties(device).uuid)) as clocks:
        w4_ms = generation_ms(gens)
    linear_ops = flux_dit.linear_ops_per_sample() * total_batch * steps_per_gen
    err = _lib.take_device_error()
    del model
    torch.cuda.empty_cache()
    return {
        "w4a4_ms": round(w4_ms, 2), "dense_bf16_ms": round(dense_ms, 2),
        "speedup_vs_dense_bf16": round(dense_ms / w4_ms, 3), "w4a4_unfused_norm_ms": round(unfused_ms, 2),
        "w4a4_ms_per_denoise_step": round(w4_ms / steps_per_gen, 3), "n_gpus": world, "per_gpu_batch": b,
        "batch": total_batch, "denoise_steps": steps_per_gen, "generations_timed": gens,
        "linears_w4a4": len(replaced), "linear_tops": round(linear_ops / (w4_ms * 1e-3) / 1e12, 1),
        "fused_modulated_norm": True, "attention_glue": "flux_dit_glue.cu (both arms)", "parallelism": f"dp{world} (batch split, no collective)",
        "clocks": clocks.summary(), "device_error": err,
    }


# ---------------------------------------------------------------------------
# video-DiT linears, tensor parallel over the ranks

VIDEO_M = 32760
VIDEO_KN = ((5120, 15360), (5120, 13824), (13824, 5120))


def run_video_tp(args, rank, world, local, steps: int, warmup: int):
    """Large video-DiT linears with the weights N-split over the ranks
    (``ColumnParallelConvRotLinear``, its default ``gather="auto"``): the
    all-gather of the outputs overlaps the GEMM, run in row blocks, by copy
    engine pushes and (from 8 GPUs) epilogue peer stores, then a flag
    barrier.  One step = the three linears on M = 32760 tokens, timed
    eagerly (the barrier epoch advances every call) with CUDA events, max
    over ranks.  Also timed: the layer's other gathers, each rank's GEMMs
    writing only its own shard (compute only), and the same shard GEMMs
    followed by an NCCL all_gather_into_tensor and the permute to (M, N)
    (the library-collective arm).  Parity: every rank compares the
    gathered output of each linear with the single-GPU ConvRotLinear of the
    full weight, bit for bit."""

    import ctypes

    import convrot_mlx_b200 as cr
    from convrot_mlx_b200 import _lib
    from convrot_mlx_b200.tp import ColumnParallelConvRotLinear

    device = torch.device("cuda", local if world > 1 else 0)
    if not torch.distributed.is_initialized():
        # the layer keeps its output in symmetric memory, which needs a process group
        import datetime
        import socket

        with socket.socket() as sock:
            sock.bind(("127.0.0.1", 0))
            port = sock.getsockname()[1]
        torch.distributed.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=0, world_size=1,
                                             timeout=datetime.timedelta(seconds=120), device_id=device)
    layers, fulls, xs = [], [], []
    for i, (k, n) in enumerate(VIDEO_KN):
        full, _, _ = make_linear(k, n, SEED + 50 + i, device)
        layers.append(ColumnParallelConvRotLinear.from_full(full))
        fulls.append(full)
        xs.append(make_activation(VIDEO_M, k, SEED + 60 + i, device))
    torch.cuda.synchronize()
    lib = _lib.load()

    # parity first: the gathered output of every linear against the full layer
    parity = True
    for layer, full, x in zip(layers, fulls, xs):
        got = layer(x)
        want = full(x)
        torch.cuda.synchronize()
        parity &= bool(torch.equal(got.view(torch.int16), want.view(torch.int16)))
        del want
    if world > 1:
        flag = torch.tensor([0 if parity else 1], dtype=torch.int32, device=device)
        torch.distributed.all_reduce(flag, op=torch.distributed.ReduceOp.MAX)
        parity = int(flag.item()) == 0
    del fulls
    torch.cuda.empty_cache()

    def step():
        for layer, x in zip(layers, xs):
            layer(x)

    shards = [torch.empty((VIDEO_M, layer.shard_features), dtype=torch.bfloat16, device=device) for layer in layers]

    def shard_gemms(i):
        layer, x = layers[i], xs[i]
        codes, xsc = cr.metal_fused_prepare_convrot_activation_i8(x, GROUP)
        one = (ctypes.c_void_p * 1)(shards[i].data_ptr())
        _lib.check(lib.convrot_w4a4_gemm_gather(_lib.ptr(codes), _lib.ptr(layer.qweight), layer.layout,
                                                _lib.ptr(xsc), _lib.ptr(layer.scales), _lib.ptr(layer.bias), one, 1,
                                                layer.shard_features, 0, _lib.BF16, VIDEO_M, layer.shard_features,
                                                layer.in_features, _lib.stream_of(x)), "gemm")

    def local_only():
        for i in range(len(layers)):
            shard_gemms(i)

    gathered = [torch.empty((world * VIDEO_M, layer.shard_features), dtype=torch.bfloat16, device=device)
                for layer in layers] if world > 1 else []
    full_out = [torch.empty((VIDEO_M, layer.out_features), dtype=torch.bfloat16, device=device)
                for layer in layers] if world > 1 else []

    def nccl_step():
        for i, layer in enumerate(layers):
            shard_gemms(i)
            torch.distributed.all_gather_into_tensor(gathered[i], shards[i])
            full_out[i].view(VIDEO_M, world, layer.shard_features).copy_(
                gathered[i].view(world, VIDEO_M, layer.shard_features).transpose(0, 1))

    def timed(fn, n):
        for _ in range(warmup):
            fn()
        torch.cuda.synchronize()
        barrier(world)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(n):
            fn()
        e1.record()
        torch.cuda.synchronize()
        barrier(world)
        return max_over_ranks(e0.elapsed_time(e1), world) / n

    with ClockSampler(str(torch.cuda.get_device_properties(device).uuid)) as clocks:
        ms = timed(step, steps)
    local_ms = timed(local_only, steps)
    nccl_ms = timed(nccl_step, steps) if world > 1 else None
    arms = {}  # the other gathers of the same layers (peer stores from the epilogue, copy engines, the split)
    default_epi = layers[0].epilogue_peer_count()
    if world > 1:
        for gather in ("epilogue", "copy-engine", "split"):
            for layer in layers:
                layer.gather = gather
            if layers[0].epilogue_peer_count() != default_epi:
                arms[gather] = round(timed(step, steps), 4)
        for layer in layers:
            layer.gather = "auto"
    ops = sum(2 * VIDEO_M * k * n for k, n in VIDEO_KN)
    out_bytes = sum(VIDEO_M * n * 2 for k, n in VIDEO_KN)
    recv = out_bytes * (world - 1) // world
    exch = ms - local_ms
    line = {
        "tops": round(ops / (ms * 1e-3) / 1e12, 2), "ms_per_step": round(ms, 4), "n_gpus": world,
        "parity_bit_exact": parity, "compute_only_ms": round(local_ms, 4), "exchange_ms": round(exch, 4),
        "received_bytes_per_rank": recv,
        "exchange_gbs_per_rank": round(recv / (ms * 1e-3) / 1e9, 1) if world > 1 else None,
        "gather": (f"auto: 4 row blocks; GEMM epilogue peer stores to {default_epi} peer(s), one strided "
                   f"copy-engine copy per block to each of the other {max(world - 1 - default_epi, 0)}"),
        "other_gather_arms_ms": arms,
        "nccl_allgather_arm_ms": None if nccl_ms is None else round(nccl_ms, 4),
        "nccl_allgather_arm_tops": None if nccl_ms is None else round(ops / (nccl_ms * 1e-3) / 1e12, 2),
        "m": VIDEO_M, "kn": [list(p) for p in VIDEO_KN],
        "parallelism": f"tp{world} (N split; all-gather overlapping the chunked GEMM)",
        "clocks": clocks.summary(), "device_error": _lib.take_device_error(),
    }
    for layer in layers:
        layer._out.clear()
        layer._flags = None
    del layers, xs, shards, gathered, full_out
    torch.cuda.empty_cache()
    return line


def run_case(args):
    """One kernel on one shape, launched ``--case-launches`` times on the
    default stream (eager), for profilers: ``--case gemm`` runs the W4A4 GEMM
    (K x packed-N weights, on the kernel ``--route`` picks), ``--case prep``
    the fused rotate + A4 quantize, ``--case modnorm`` the same fused with a
    modulated LayerNorm; ``--case dit`` runs that many eager denoise steps of
    the W4A4 FLUX DiT (batch 8)."""

    import convrot_mlx_b200 as cr
    from convrot_mlx_b200 import _lib

    device = torch.device("cuda", 0)
    m, k, n = args.m, args.k, args.n
    x = make_activation(m, k, SEED, device)
    if args.case == "prep":
        for _ in range(args.case_launches):
            cr.metal_fused_prepare_convrot_activation_i8(x, args.group)
    elif args.case == "dit":
        # the W4A4 FLUX DiT of the dit entry (batch 8, one GPU, glue kernels and
        # fused preps on): --case-launches eager denoise steps, the last inside
        # an NVTX range "dit_step" (for ncu --nvtx-include "dit_step/")
        import flux_dit
        from convrot_mlx_b200.adapter import replace_convrot_linears

        model = flux_dit.build_flux_dit(device, SEED)
        flux_dit.build_glue()
        model.fuse_attention_glue = True
        replace_convrot_linears(model, backend="mpp-w4a4")
        model.fuse_modulated_norm = True
        img, txt, y, ids = flux_dit.dit_inputs(8, device, SEED + 7)
        with torch.no_grad():
            rope = model.rotary(ids)
            t = torch.full((8,), 0.5, device=device)
            guidance = torch.full((8,), 3.5, device=device)
            for i in range(args.case_launches):
                if i == args.case_launches - 1:
                    torch.cuda.synchronize()
                    torch.cuda.nvtx.range_push("dit_step")
                v = model(img, txt, rope, t, y, guidance)
                img.add_(-0.05 * v)
            torch.cuda.nvtx.range_pop()
        m, k, n = 8, 0, 0
    elif args.case == "modnorm":
        from convrot_mlx_b200.core import modulated_norm_prepare_i8

        g = torch.Generator(device=device).manual_seed(SEED + 1)
        shift, scale = ((torch.randn((1, 1, k), generator=g, device=device) * 0.5).to(torch.bfloat16)
                        for _ in range(2))
        for _ in range(args.case_launches):
            modulated_norm_prepare_i8(x.view(1, m, k), shift, scale, 1e-6, args.group)
    else:
        layer, _, _ = make_linear(k, n, SEED, device)
        codes, xs = cr.metal_fused_prepare_convrot_activation_i8(x, GROUP)
        out = torch.empty((m, n), dtype=torch.bfloat16, device=device)
        lib = _lib.load()
        _lib.check(lib.convrot_set_gemm_route(args.route), "route")
        for _ in range(args.case_launches):
            _lib.check(lib.convrot_w4a4_gemm(_lib.ptr(codes), _lib.ptr(layer.qweight), _lib.LAYOUT_KN, _lib.ptr(xs),
                                             _lib.ptr(layer.scales), _lib.ptr(layer.bias), _lib.ptr(out), _lib.BF16,
                                             m, n, k, _lib.stream_of(x)), "gemm")
    torch.cuda.synchronize()
    err = _lib.take_device_error()
    print(json.dumps({"case": args.case, "m": m, "k": k, "n": n, "launches": args.case_launches, "device_error": err}))
    return 1 if err else 0


def summarize(line):
    """Headline figures at the end of the JSON line (where a tail keeps them)."""

    s = {"value_tops": line["value"], "speedup_vs_dense_bf16": line["speedup_vs_dense_bf16"],
         "dense_bf16_tflops": line["dense_bf16"]["value"], "gemm_frac": line["roofline"]["frac"],
         "gemm_frac_of_2x_bf16": line["roofline"]["frac_of_2x_measured_bf16"],
         "prep_frac": line["roofline_prep"]["frac"], "w4a16_speedup_vs_dense": line["w4a16"]["speedup_vs_dense_bf16"],
         "e2e_tops": line["e2e"]["value"]}
    c2 = line.get("c2_prep")
    if c2:
        s["c2_prep_frac"] = {"g64": c2["g64"]["frac"], "g256": c2["g256"]["frac"]}
    sm = line.get("small_m")
    if sm:
        s["small_m"] = [[x["m"], x["k"], x["n"], x["us"], x["frac"], x["speedup_vs_dense_bf16"]] for x in sm["shapes"]]
    tp = line.get("video_tp")
    if tp:
        s["video_tp"] = {"n_gpus": tp["n_gpus"], "tops": tp["tops"], "ms": tp["ms_per_step"],
                         "parity": tp["parity_bit_exact"], "compute_ms": tp["compute_only_ms"],
                         "exchange_ms": tp["exchange_ms"], "other_gathers_ms": tp["other_gather_arms_ms"],
                         "nccl_arm_ms": tp["nccl_allgather_arm_ms"]}
    dit = line.get("dit")
    if dit:
        s["dit"] = {"n_gpus": dit["n_gpus"], "w4a4_ms": dit["w4a4_ms"], "dense_ms": dit["dense_bf16_ms"],
                    "speedup": dit["speedup_vs_dense_bf16"], "w4a4_unfused_norm_ms": dit["w4a4_unfused_norm_ms"]}
    return s


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=("ours", "reference"), default="ours")
    ap.add_argument("--no-cpu", action="store_true", help="skip the cpu_baseline leg")
    ap.add_argument("--workload", choices=("all", "flux-sweep", "video-tp", "dit", "small-m"), default="all",
                    help="all (default): the config-3 FLUX sweep line with the config-2 prep, config-5 "
                         "tensor-parallel and config-4 DiT entries added; flux-sweep: config 3 alone; video-tp: "
                         "config 5 alone; dit: config 4 alone; small-m: the m <= 64 GEMM entry alone")
    ap.add_argument("--dit-gens", type=int, default=2, help="timed 20-step generations per DiT arm in --workload all")
    ap.add_argument("--case", choices=("gemm", "prep", "modnorm", "dit"), help="run one kernel on one shape (for profilers) and exit")
    ap.add_argument("--m", type=int, default=4096)
    ap.add_argument("--k", type=int, default=3072)
    ap.add_argument("--n", type=int, default=12288)
    ap.add_argument("--group", type=int, default=GROUP)
    ap.add_argument("--case-launches", type=int, default=3)
    ap.add_argument("--route", type=int, default=0, help="--case gemm: convrot_set_gemm_route (0 automatic, "
                    "1 one-CTA, 2 CTA-pair, 3 swap-AB, 4 GEMV)")
    args = ap.parse_args(argv)
    if args.case:
        return run_case(args)
    if args.warmup < 1:
        args.warmup = 1
    if args.impl == "reference":
        rank = int(os.environ.get("RANK", "0"))
        world = int(os.environ.get("WORLD_SIZE", str(args.gpus)))
        line = run_reference(args, rank, world)
        if line is not None:
            print(json.dumps(line), flush=True)
        return 0
    rank, world, local = dist_setup(args.gpus)
    rc = 0
    try:
        device = torch.device("cuda", local if world > 1 else 0)
        if args.workload == "video-tp":
            line = run_video_tp(args, rank, world, local, args.steps, args.warmup)
            rc = 0 if line["parity_bit_exact"] else 1
        elif args.workload == "dit":
            line = run_dit(args, rank, world, local, args.steps, args.warmup)
        elif args.workload == "small-m":
            line = run_small_m(args, device)
        else:
            line = run_ours(args, rank, world, local)
            if args.workload == "all":
                torch.cuda.empty_cache()
                line["c2_prep"] = run_c2(args, device)
                line["small_m"] = run_small_m(args, device)
                line["video_tp"] = run_video_tp(args, rank, world, local, min(args.steps, 10), min(args.warmup, 2))
                line["dit"] = run_dit(args, rank, world, local, args.dit_gens, 1)
                rc = 0 if line["video_tp"]["parity_bit_exact"] else 1
            line["summary"] = summarize(line)
        if rank == 0:
            print(json.dumps(line), flush=True)
    finally:
        if torch.distributed.is_initialized():
            torch.distributed.destroy_process_group()
    return rc


if __name__ == "__main__":
    sys.exit(main())
