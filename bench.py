#!/usr/bin/env python
"""Benchmark: PESQ loss forward + backward on B200, utterance-seconds per second.

Workload (the configuration the headline metric is quoted on): batch 8 x 8 s
at 16 kHz per GPU, speech-like seeded synthetic signals with f0 ~ U[90, 250]
Hz and SNR ~ U[0, 20] dB, forward + backward w.r.t. the degraded signal,
CUDA-graph replayed.  With N GPUs every rank runs its own batch (weak
scaling, batch sharding) and the mean loss is all-reduced over NCCL each
step, the only collective of the path.

Timing: W untimed warm-up steps, then K steps, each bracketed by CUDA events
on the launching stream; the L2 is flushed (a 256 MiB write) between steps
outside the events, because the step's inputs (8 MiB) fit in L2.  The K-step
loop is bracketed by a barrier and synchronize; the reported time is the sum
of the K step times, maximum over ranks.

Also reported: e2e (same metric through the public API, ``PesqLossCuda.graphed``,
with the inputs copied from pinned host memory and the loss read back every
step), eager latency, per-stage kernel times, the roofline of the dominant
kernel and the reference's CPU path (the oracle port, reference dtype mode)
timed on this host.

``--impl reference`` times the reference CPU implementation of the path (the
oracle port in the reference's dtype mode) on this host's cores instead.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "PESQ fwd+bwd utterance-seconds/s per GPU and 1–8 GPU box; 8×8s@16k latency"
UNIT = "utterance-seconds/s"
RATE = 16000
#: per-GPU batch and utterance length of the workloads bench.py can run
WORKLOADS = {"cfg2": (8, 8.0), "cfg5": (512, 3.0)}
BATCH, SECONDS = WORKLOADS["cfg2"]
L2_FLUSH_BYTES = 256 << 20


def parse_args():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["cuda", "reference"], default="cuda")
    ap.add_argument("--cpu-seconds", type=float, default=10.0, help="CPU baseline sample budget")
    ap.add_argument("--skip-configs", action="store_true",
                    help="do not time the other BASELINE configurations (cfg1, cfg3, cfg4, cfg5)")
    ap.add_argument("--workload", choices=sorted(WORKLOADS), default="cfg2",
                    help="cfg2 (8 x 8 s, the headline) or cfg5 (512 x 3 s, larger than L2)")
    ap.add_argument("--skip-cpu", action="store_true", help="leave out the CPU baseline leg")
    ap.add_argument("--op", choices=["iir", "resample", "geometry", "triton-reference"], default=None,
                    help="time only a standalone op on its large case (one JSON line; for profiling)")
    args = ap.parse_args()
    global BATCH, SECONDS
    BATCH, SECONDS = WORKLOADS[args.workload]
    return args


# ---------------------------------------------------------------------------
# helpers
# ---------------------------------------------------------------------------


def dist_env():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return world, rank, local


def measured_peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        with open(path) as fh:
            data = json.load(fh)
        return float(data["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


def profiled_traffic():
    """DRAM bytes per front-kernel launch of the committed ncu summary."""

    path = os.path.join(ROOT, "profiles", "front_kernel_cfg2.txt")
    if not os.path.exists(path):
        return None
    for line in open(path):
        if line.startswith("dram_bytes_per_launch:"):
            return float(line.split(":")[1])
    return None


class ClockSampler:
    """nvidia-smi clock / throttle sampling during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.proc = None
        self.file = tempfile.NamedTemporaryFile(mode="w+", suffix=".csv", delete=False)

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "100"], stdout=self.file, stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None
        time.sleep(0.3)
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        self.file.flush()
        rows = []
        with open(self.file.name) as fh:
            for line in fh:
                parts = [p.strip() for p in line.split(",")]
                if len(parts) >= 9:
                    rows.append(parts)
        os.unlink(self.file.name)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        smax = [float(r[2]) for r in rows if r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[5 + i].lower().startswith("active")})
        return {
            "sm_mhz": statistics.median(sm) if sm else None,
            "sm_max_mhz": max(smax) if smax else None,
            "reasons": reasons,
            "samples": len(rows),
        }


def cpu_reference_step(ref, deg, params):
    """One forward + backward (w.r.t. deg) of the reference CPU path: the
    oracle port in the reference's dtype mode (float32 signal stages, float64
    perceptual chain, as PesqLoss evaluates on the CPU)."""

    import torch

    from oracle import pesq_oracle as O

    d = deg.detach().clone().requires_grad_(True)
    loss = O.forward(ref, d, params, mode="reference")
    (g,) = torch.autograd.grad(loss.sum(), [d])
    return loss, g


def cpu_baseline(budget_s: float):
    import torch

    from oracle import pesq_oracle as O
    from triton_pesq_b200.signals import workload

    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    ref, deg, sr = workload("cfg2", seed=0)
    params = O.OracleParams(factor=1.0, sample_rate=sr)
    cpu_reference_step(ref[:1], deg[:1], params)  # warm-up
    steps, t0 = 0, time.perf_counter()
    while True:
        cpu_reference_step(ref, deg, params)
        steps += 1
        elapsed = time.perf_counter() - t0
        if elapsed >= budget_s and steps >= 2:
            break
    b, secs = WORKLOADS["cfg2"]
    utt_s = steps * b * secs
    return {
        "value": utt_s / elapsed,
        "unit": UNIT,
        "cores": threads,
        "kind": "port",
        "sample": f"{steps} x forward+backward(deg) of the full 8 x 8 s @16 kHz batch, {elapsed:.1f} s, "
                  f"oracle port in the reference dtype mode (float32 signal path, float64 chain)",
    }


# ---------------------------------------------------------------------------
# reference arm
# ---------------------------------------------------------------------------


def run_reference(args):
    world, rank, _ = dist_env()
    if rank != 0:
        return
    import torch

    from oracle import pesq_oracle as O
    from triton_pesq_b200.signals import workload

    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    ref, deg, sr = workload("cfg2", seed=0)
    params = O.OracleParams(factor=1.0, sample_rate=sr)
    # each step is a bounded sample of the workload: 2 of the 8 utterances
    sample = 2
    for _ in range(args.warmup):
        cpu_reference_step(ref[:sample], deg[:sample], params)
    times = []
    for k in range(args.steps):
        lo = (2 * k) % BATCH
        t0 = time.perf_counter()
        cpu_reference_step(ref[lo:lo + sample], deg[lo:lo + sample], params)
        times.append(time.perf_counter() - t0)
    total = sum(times)
    value = args.steps * sample * SECONDS / total
    line = {
        "impl": "reference",
        "metric": METRIC,
        "value": value,
        "unit": UNIT,
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": 1e3 * total / args.steps,
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "f32",
        "data": "synthetic",
        "config": {"workload": "8x8s@16k fwd+bwd(deg)", "sample_per_step": f"{sample} x 8 s utterances",
                   "global_batch": BATCH, "seconds": SECONDS, "sample_rate": RATE},
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": threads, "kind": "port",
                         "sample": f"{sample} of the 8 utterances per step, oracle port in the reference "
                                   "dtype mode (float32 signal path, float64 chain)"},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------------------
# CUDA arm
# ---------------------------------------------------------------------------


def stage_times(model, ref, deg, dev, launches=40):
    """Average device time of every kernel stage, each timed alone with CUDA
    events on the launching stream, inputs rotating over more than L2."""

    import ctypes

    import torch

    from triton_pesq_b200 import _lib

    lib = _lib.library()
    plan = model._plan(dev)
    flags = _lib.GRAD_DEG
    b, n = ref.shape
    nbytes = ctypes.c_size_t()
    _lib.check(lib.pesq_workspace_size(ctypes.c_void_p(plan), b, n, flags, ctypes.byref(nbytes)), "workspace")
    ws = torch.empty(nbytes.value // 4 + 64, dtype=torch.float32, device=dev)
    sets = max(2, (320 << 20) // (2 * ref.numel() * 4))
    refs = [ref.roll(k * 997, dims=1).contiguous() for k in range(sets)]
    degs = [deg.roll(k * 997, dims=1).contiguous() for k in range(sets)]
    outs = [torch.empty(b, device=dev) for _ in range(4)]
    g_loss = torch.ones(b, device=dev)
    g_deg = torch.empty_like(deg)
    stream = torch.cuda.current_stream(dev)
    sp = ctypes.c_void_p(stream.cuda_stream)
    P = ctypes.c_void_p(plan)
    W = ctypes.c_void_p(ws.data_ptr())
    wb = nbytes.value

    def front(i):
        return lib.pesq_forward_front(P, sp, ctypes.c_void_p(refs[i].data_ptr()), n,
                                      ctypes.c_void_p(degs[i].data_ptr()), n, b, n, flags, W, wb)

    def chain_fwd(i):
        return lib.pesq_forward_chain(P, sp, b, n, flags, W, wb, *[ctypes.c_void_p(o.data_ptr()) for o in outs])

    def chain_bwd(i):
        return lib.pesq_backward_chain(P, sp, b, n, flags, W, wb, ctypes.c_void_p(g_loss.data_ptr()), None, None,
                                       None)

    def align(i):
        return lib.pesq_backward_align(P, sp, b, n, flags, W, wb)

    def back(i):
        return lib.pesq_backward_back(P, sp, b, n, flags, W, wb, None, n, ctypes.c_void_p(g_deg.data_ptr()), n)

    # populate the workspace once in order
    for fn in (front, chain_fwd, chain_bwd, align, back):
        _lib.check(fn(0), "stage")
    torch.cuda.synchronize()
    result = {}
    # align runs concurrently with chain_backward inside a step; alone it is
    # timed back to back with itself
    for name, fn in (("front", front), ("chain_forward", chain_fwd), ("chain_backward", chain_bwd),
                     ("align", align), ("back", back)):
        start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda._sleep(20_000_000)  # keep the stream busy while the host enqueues
        start.record(stream)
        for i in range(launches):
            fn(i % sets)
        stop.record(stream)
        torch.cuda.synchronize()
        result[name] = 1e3 * start.elapsed_time(stop) / launches  # microseconds
    return result


def measure_resampler(dev, peak, launches=10):
    """The standalone resampler (ResampleCuda, the reference's TritonResample)
    on 256 rows of 4 s at 44.1 kHz -> 16 kHz (180 MB in, 65 MB out: beyond
    L2), forward and adjoint each timed alone with CUDA events."""

    import torch

    from triton_pesq_b200 import ResampleCuda

    rows, n_in = 256, 4 * 44100
    module = ResampleCuda(44100, 16000).to(dev)
    x = torch.randn(rows, n_in, device=dev)
    handle = module._handle(dev)
    y = torch.ops.pesq_cuda.resample(handle, x)
    n_out = y.shape[1]
    g = torch.randn_like(y)
    stream = torch.cuda.current_stream(dev)

    def timed(fn):
        for _ in range(3):
            fn()
        start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record(stream)
        for _ in range(launches):
            fn()
        stop.record(stream)
        torch.cuda.synchronize()
        return 1e3 * start.elapsed_time(stop) / launches

    fwd_us = timed(lambda: torch.ops.pesq_cuda.resample(handle, x))
    adj_us = timed(lambda: torch.ops.pesq_cuda.resample_adjoint(handle, g, n_in))
    # compulsory traffic: read the input, write the output (and the reverse)
    alg = 4 * rows * (n_in + n_out)
    return {
        "workload": f"{rows} rows x 4 s @44.1 kHz -> 16 kHz, float32, fp64 accumulation",
        "forward_us": fwd_us,
        "adjoint_us": adj_us,
        "forward_gbs": alg / (fwd_us * 1e-6) / 1e9,
        "adjoint_gbs": alg / (adj_us * 1e-6) / 1e9,
        "forward_frac_of_measured_hbm": alg / (fwd_us * 1e-6) / 1e9 / peak,
        "adjoint_frac_of_measured_hbm": alg / (adj_us * 1e-6) / 1e9 / peak,
        "utterance_seconds_per_s_fwd_bwd": rows * 4.0 / ((fwd_us + adj_us) * 1e-6),
    }


def measure_iir(dev, peak, launches=20, large_only=False):
    """The standalone IIR filter (IIRCuda, the reference's TritonIIR) with the
    order 10 PESQ band pass: the reference's own benchmark shapes [8, 16000]
    and [8, 64000] (per call, eager, CUDA events; forward and forward plus
    backward through autograd), and [64, 480000] (123 MB in, 123 MB out:
    beyond L2) for the HBM roofline of the kernel, with the order 2
    pre-emphasis filter beside it."""

    import torch

    from triton_pesq_b200 import IIRCuda
    from triton_pesq_b200.tables import power_filter, pre_filter

    stream = torch.cuda.current_stream(dev)

    def timed(fn, n=launches):
        for _ in range(3):
            fn()
        start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record(stream)
        for _ in range(n):
            fn()
        stop.record(stream)
        torch.cuda.synchronize()
        return 1e3 * start.elapsed_time(stop) / n

    out = {}
    band = IIRCuda(*power_filter()).to(dev)
    for rows, n in (() if large_only else ((8, 16000), (8, 64000))):
        x = torch.randn(rows, n, device=dev)
        out[f"order10_fwd_{rows}x{n}_us"] = timed(lambda: band(x))
        leaf = x.clone().requires_grad_(True)
        g = torch.randn_like(x)
        out[f"order10_fwd_bwd_{rows}x{n}_us"] = timed(
            lambda: torch.autograd.grad(band(leaf), leaf, g))
    large = (((64, 480000), "order10", band), ((64, 480000), "order2", IIRCuda(*pre_filter()).to(dev)),
             ((30720, 1000), "order10", band))
    for (rows, n), label, module in large:
        x = torch.randn(rows, n, device=dev)
        alg = 8.0 * rows * n  # read every sample once, write every output once
        fwd = timed(lambda: module(x))
        handle = module._handle(dev)
        rev = timed(lambda: torch.ops.pesq_cuda.iir(handle, x, module._flags(True)))
        out[f"{label}_{rows}x{n}"] = {
            "forward_us": fwd, "reverse_us": rev,
            "forward_gbs": alg / (fwd * 1e-6) / 1e9, "reverse_gbs": alg / (rev * 1e-6) / 1e9,
            "forward_frac_of_measured_hbm": alg / (fwd * 1e-6) / 1e9 / peak,
            "gsamples_per_s": rows * n / (fwd * 1e-6) / 1e9,
        }
    out["note"] = ("per call, eager (allocation and launch included) for the reference's shapes; "
                   "the reference quotes 83 / 153 us forward and 387 us forward plus backward on a GTX 1080 Ti")
    errors = band.check_errors()
    if errors:
        raise RuntimeError(f"IIR look-back wait gave up (error word {errors})")
    return out


def measure_configs(dev, flush, steps=10):
    """Graph-replayed fwd+bwd (w.r.t. deg) step of the other BASELINE
    configurations on one GPU (L2 flushed before each step): cfg1, cfg3, the
    per-GPU share of cfg4 (8 of its 64 utterances) and cfg5."""

    import torch

    from triton_pesq_b200 import PesqLossCuda
    from triton_pesq_b200.signals import workload

    out = {}
    for name, keep, secs in (("cfg1", 1, 1.0), ("cfg3", 16, 4.0), ("cfg4_per_gpu", 8, 10.0), ("cfg5", 512, 3.0)):
        ref_c, deg_c, sr = workload(name.split("_")[0], seed=0)
        ms = _graphed_step_ms(PesqLossCuda(1.0, sample_rate=sr), ref_c[:keep].to(dev), deg_c[:keep].to(dev), flush,
                              steps)
        out[name] = {"batch": keep, "seconds": secs, "sample_rate": sr, "ms_per_step": ms,
                     "utterance_seconds_per_s": keep * secs / (ms * 1e-3)}
    return out


def _graphed_step_ms(model, ref, deg, flush, steps):
    """Median device time of a graph-replayed fwd+bwd (w.r.t. deg) step, L2
    flushed before each replay."""

    import torch

    deg = deg.detach().requires_grad_(True)

    def step():
        loss = model(ref, deg)
        (g,) = torch.autograd.grad(loss.sum(), [deg])
        return loss, g

    dev = ref.device
    side = torch.cuda.Stream(dev)
    side.wait_stream(torch.cuda.current_stream(dev))
    with torch.cuda.stream(side):
        for _ in range(3):
            step()
    torch.cuda.current_stream(dev).wait_stream(side)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        step()
    torch.cuda.synchronize()
    times = []
    for k in range(steps + 3):
        flush.zero_()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        graph.replay()
        b.record()
        b.synchronize()
        if k >= 3:
            times.append(a.elapsed_time(b))
    del graph
    return statistics.median(times)


def measure_geometries(dev, flush, steps=10):
    """The cfg2 step (8 x 8 s at 16 kHz, fwd+bwd w.r.t. deg, graph replay) with
    other frame geometries of PesqLoss (n_fft, hop_length, win_length): the
    spectrum kernels instead of the fused 512 / 256 transforms."""

    from triton_pesq_b200 import PesqLossCuda
    from triton_pesq_b200.signals import workload

    ref_c, deg_c, sr = workload("cfg2", seed=0)
    ref, deg = ref_c.to(dev), deg_c.to(dev)
    out = {}
    for n_fft, hop, win in ((512, 256, 512), (256, 128, 256), (1024, 512, 1024), (512, 128, 512), (2048, 512, 2048)):
        model = PesqLossCuda(1.0, sample_rate=sr, n_fft=n_fft, hop_length=hop, win_length=win)
        ms = _graphed_step_ms(model, ref, deg, flush, steps)
        out[f"n_fft{n_fft}_hop{hop}"] = {"ms_per_step": ms,
                                         "utterance_seconds_per_s": ref.shape[0] * ref.shape[1] / sr / (ms * 1e-3)}
    return out


def measure_fused(dev, flush, steps=10):
    """The loss inside a caller's mixed-precision training step: the headline
    8 x 8 s fwd+bwd with bfloat16 inputs (graph replay, L2 flushed), and the
    same step on a side stream overlapping a chain of bf16 GEMMs on the
    default stream (a stand-in for the model's backward), against the two
    run back to back."""

    import torch

    from triton_pesq_b200 import PesqLossCuda
    from triton_pesq_b200.signals import workload

    ref_c, deg_c, sr = workload("cfg2", seed=0)
    main = torch.cuda.current_stream(dev)
    side = torch.cuda.Stream(dev)

    def capture(ref, deg):
        model = PesqLossCuda(1.0, sample_rate=sr)

        def step():
            loss = model(ref, deg)
            torch.autograd.grad(loss.sum(), [deg])

        side.wait_stream(main)
        with torch.cuda.stream(side):
            for _ in range(3):
                step()
        main.wait_stream(side)
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            step()
        torch.cuda.synchronize()
        return graph

    def timed(fn):
        times = []
        for k in range(steps + 3):
            flush.zero_()
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record(main)
            fn()
            b.record(main)
            b.synchronize()
            if k >= 3:
                times.append(a.elapsed_time(b))
        return statistics.median(times)

    out = {}
    g16 = capture(ref_c.to(dev, torch.bfloat16), deg_c.to(dev, torch.bfloat16).requires_grad_(True))
    out["bf16_inputs_ms_per_step"] = timed(g16.replay)
    g32 = capture(ref_c.to(dev), deg_c.to(dev).requires_grad_(True))
    out["fp32_inputs_ms_per_step"] = timed(g32.replay)
    a = torch.randn(4096, 4096, device=dev, dtype=torch.bfloat16)

    def gemms():
        c = a
        for _ in range(4):
            c = c @ a

    def both():
        side.wait_stream(main)
        with torch.cuda.stream(side):
            g32.replay()
        gemms()
        main.wait_stream(side)

    out["gemm_chain_ms"] = timed(gemms)
    out["serial_ms"] = out["gemm_chain_ms"] + out["fp32_inputs_ms_per_step"]
    out["overlapped_ms"] = timed(both)
    out["hidden_fraction_of_loss_step"] = (out["serial_ms"] - out["overlapped_ms"]) / out["fp32_inputs_ms_per_step"]
    out["note"] = "gemm chain: 4 bf16 4096^3 products on the default stream; the loss step on a side stream"
    del g16, g32
    return out


def run_cuda(args):
    import torch
    import torch.distributed as dist

    from triton_pesq_b200 import PesqLossCuda
    from triton_pesq_b200.signals import workload

    world, rank, local = dist_env()
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    # libraries print banners (NCCL's version line) on file descriptor 1: send
    # it to stderr until the JSON line, so that stdout carries that line only
    sys.stdout.flush()
    stdout_fd = os.dup(1)
    os.dup2(2, 1)
    if world > 1:
        import datetime

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)

    model = PesqLossCuda(1.0, sample_rate=RATE)
    ref_cpu, deg_cpu, _ = workload(args.workload, seed=rank)
    ref = ref_cpu.to(dev)
    deg = deg_cpu.to(dev)
    flush = torch.empty(L2_FLUSH_BYTES // 4, dtype=torch.float32, device=dev)

    # ---- graph-replayed forward + backward (the headline value)
    deg_p = deg.detach().clone().requires_grad_(True)

    def step():
        loss = model(ref, deg_p)
        (g,) = torch.autograd.grad(loss.sum(), [deg_p])
        return loss, g

    side = torch.cuda.Stream(dev)
    side.wait_stream(torch.cuda.current_stream(dev))
    with torch.cuda.stream(side):
        for _ in range(3):
            step()
    torch.cuda.current_stream(dev).wait_stream(side)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        loss_g, grad_g = step()
    torch.cuda.synchronize()

    # utterances are independent: every rank replays its own shard and no data
    # crosses ranks inside a step (the ranks meet only at the barriers around
    # the timed region and in the max-over-ranks of the timings)
    def replay():
        graph.replay()

    stream = torch.cuda.current_stream(dev)
    for _ in range(args.warmup):
        replay()
        flush.zero_()
    events = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    wall0 = time.perf_counter()
    with ClockSampler(local) as clocks:
        for k in range(args.steps):
            flush.zero_()
            events[k][0].record(stream)
            replay()
            events[k][1].record(stream)
        torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    wall = time.perf_counter() - wall0
    step_ms = [a.elapsed_time(b) for a, b in events]
    total_ms = torch.tensor([sum(step_ms)], device=dev, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(total_ms, op=dist.ReduceOp.MAX)
    total_s = float(total_ms.item()) / 1e3
    utt_per_step = BATCH * SECONDS * world
    value = utt_per_step * args.steps / total_s

    # ---- eager latency (host dispatch included)
    eager = []
    for k in range(max(5, args.steps // 5)):
        flush.zero_()
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        step()
        torch.cuda.synchronize()
        eager.append(time.perf_counter() - t0)

    # ---- end to end through the public API with host buffers
    # Every step copies its inputs from pinned host memory and reads its loss
    # back.  The loop is double buffered as a training input pipeline is: the
    # copy of step k + 1 (on a copy stream, into the second of two graphed
    # input sets) overlaps the compute of step k; a set is overwritten only
    # after the step that used it has finished.  The serial variant (copy,
    # compute, read back, wait) is reported beside it.
    ref_h = ref_cpu.pin_memory()
    deg_h = deg_cpu.pin_memory()
    loss_h = [torch.empty(BATCH, pin_memory=True) for _ in range(2)]
    # (graphed() rebinds the module's forward, as PesqLossTriton.graphed does,
    # so each input set gets its own module instance)
    sets = []
    for _ in range(2):
        ref_d = torch.empty_like(ref)
        deg_d = torch.empty_like(deg).requires_grad_(True)
        with torch.no_grad():
            ref_d.copy_(ref)
            deg_d.copy_(deg)
        sets.append((ref_d, deg_d, PesqLossCuda(1.0, sample_rate=RATE).graphed(ref_d, deg_d)))
    # the reference and the degraded signal are copied on two copy streams
    # (two DMA engines in flight) when `split`, else one after the other
    copy_streams = [torch.cuda.Stream(dev), torch.cuda.Stream(dev)]
    copy_stream = copy_streams[0]
    copied = [[torch.cuda.Event(), torch.cuda.Event()] for _ in range(2)]
    consumed = [torch.cuda.Event() for _ in range(2)]
    split = [True]

    def issue_copy(k):
        ref_d, deg_d, _ = sets[k % 2]
        pairs = ((ref_d, ref_h), (deg_d, deg_h))
        for i, (dst, src) in enumerate(pairs):
            cs = copy_streams[i] if split[0] else copy_stream
            with torch.cuda.stream(cs):
                cs.wait_event(consumed[k % 2])
                with torch.no_grad():
                    dst.copy_(src, non_blocking=True)
                copied[k % 2][i].record(cs)

    def run_step(k):
        ref_d, deg_d, graphed = sets[k % 2]
        stream.wait_event(copied[k % 2][0])
        stream.wait_event(copied[k % 2][1])
        out = graphed(ref_d, deg_d)
        torch.autograd.grad(out.sum(), [deg_d])
        consumed[k % 2].record(stream)
        loss_h[k % 2].copy_(out.detach(), non_blocking=True)

    def pipelined(n):
        start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record(stream)
        for cs in copy_streams:
            cs.wait_event(start)
        issue_copy(0)
        for k in range(n):
            if k + 1 < n:
                issue_copy(k + 1)
            run_step(k)
        stop.record(stream)
        stop.synchronize()
        return start.elapsed_time(stop)

    split[0] = False
    pipelined(4)  # warm-up
    torch.cuda.synchronize()
    one_stream_ms = pipelined(args.steps) / args.steps
    split[0] = True
    pipelined(4)
    torch.cuda.synchronize()
    e2e_total = torch.tensor([pipelined(args.steps)], device=dev, dtype=torch.float64)

    serial_ms = []
    for k in range(max(5, args.steps // 5)):
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        ref_d, deg_d, graphed = sets[0]
        a.record(stream)
        with torch.no_grad():
            ref_d.copy_(ref_h, non_blocking=True)
            deg_d.copy_(deg_h, non_blocking=True)
        out = graphed(ref_d, deg_d)
        torch.autograd.grad(out.sum(), [deg_d])
        loss_h[0].copy_(out.detach(), non_blocking=True)
        b.record(stream)
        b.synchronize()
        serial_ms.append(a.elapsed_time(b))
    if world > 1:
        dist.all_reduce(e2e_total, op=dist.ReduceOp.MAX)
    e2e_ms_total = float(e2e_total.item())
    e2e_value = utt_per_step * args.steps / (e2e_ms_total / 1e3)

    # ---- stage kernels alone, roofline of the dominant one
    stages = stage_times(model, ref, deg, dev)
    dominant = max(stages, key=stages.get)
    peak, peak_kind = measured_peaks()
    # algorithmic bytes per launch: the front kernel must read both input
    # signals (2 x 4 B per utterance sample); the back kernel must write the
    # gradient (4 B); the chain kernels have no compulsory traffic of their own
    alg = {"front": 2 * 4 * BATCH * SECONDS * RATE, "back": 4 * BATCH * SECONDS * RATE,
           "align": 4 * BATCH * SECONDS * RATE, "chain_forward": 0.0, "chain_backward": 0.0}
    front_us = stages["front"]
    achieved = alg["front"] / (front_us * 1e-6) / 1e9
    traffic = profiled_traffic()
    ops = {"resample_44k1_to_16k": measure_resampler(dev, peak), "iir": measure_iir(dev, peak)}
    configs = measure_configs(dev, flush) if not args.skip_configs else None
    fused = measure_fused(dev, flush) if not args.skip_configs else None
    geometries = measure_geometries(dev, flush) if not args.skip_configs else None

    if world > 1:
        graph.reset()
        dist.destroy_process_group()
    if rank != 0:
        return

    line = {
        "metric": METRIC,
        "value": value,
        "unit": UNIT,
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": 1e3 * total_s / args.steps,
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "f32",
        "data": "synthetic",
        "config": {
            "workload": f"{BATCH}x{SECONDS:g}s@16k fwd+bwd(deg), CUDA-graph replay ({args.workload})",
            "global_batch": BATCH * world,
            "seconds": SECONDS,
            "sample_rate": RATE,
            "parallelism": f"dp{world}",
            "l2": "flushed between steps (256 MiB write, outside the step events)",
        },
        "clocks": clocks.summary(),
        "e2e": {
            "value": e2e_value,
            "unit": UNIT,
            "h2d_bytes_per_step": int(ref.numel() * 4 * 2),
            "d2h_bytes_per_step": int(BATCH * 4),
            "api": "PesqLossCuda.graphed (two instances, one per input set), inputs copied from pinned host memory "
                   "every step (reference and degraded signal on two copy streams) overlapping the previous "
                   "step's compute, loss read back every step",
            "ms_per_step": e2e_ms_total / args.steps,
            "one_copy_stream_ms_per_step": one_stream_ms,
            "serial_ms_per_step": statistics.median(serial_ms),
        },
        # front + chain forward, chain adjoint + align + back per step
        "gpu_launches": 5 * args.steps,
        "roofline": {
            "bound": "hbm",
            "kernel": "front",
            "achieved": achieved,
            "peak": peak,
            "peak_source": peak_kind,
            "unit": "GB/s",
            "frac": achieved / peak,
            "traffic": traffic,
            "algorithmic_bytes_per_launch": alg["front"],
            "launch_us": front_us,
        },
        "stages_us": stages,
        "ops": ops,
        "other_configs": configs,
        "in_training_step": fused,
        "frame_geometries": geometries,
        "dominant_stage": dominant,
        "eager_ms_per_step": 1e3 * statistics.median(eager),
        "step_ms_min": min(step_ms),
        "step_ms_median": statistics.median(step_ms),
        "wall_s_timed_loop": wall,
    }
    if not args.skip_cpu:
        line["cpu_baseline"] = cpu_baseline(args.cpu_seconds)
    sys.stdout.flush()
    os.dup2(stdout_fd, 1)
    os.close(stdout_fd)
    print(json.dumps(line), flush=True)


REFERENCE_INSTALL = os.path.join(os.path.dirname(os.path.abspath(__file__)), "baseline", "_ref")


def _import_reference_gpu():
    """``PesqLossTriton`` of the reference installed in baseline/_ref by
    ``pip install --no-index --no-deps --target baseline/_ref <reference>``.
    Two import shims, neither of which changes a computation: ``torchtyping``
    is absent (``TensorType[...]`` becomes ``torch.Tensor``) and the installed
    typeguard 4.x cannot evaluate the reference's string dimensions
    (``typechecked`` becomes the identity)."""

    import types

    import torch

    if not os.path.isdir(os.path.join(REFERENCE_INSTALL, "torch_pesq")):
        raise ImportError("the reference is not installed in baseline/_ref")
    shim = types.ModuleType("torchtyping")

    class _TensorType:
        def __class_getitem__(cls, item):
            return torch.Tensor

    shim.TensorType = _TensorType
    sys.modules.setdefault("torchtyping", shim)
    import typeguard

    typeguard.typechecked = lambda fn: fn
    sys.path.insert(0, REFERENCE_INSTALL)
    from torch_pesq import PesqLossTriton

    return PesqLossTriton


def measure_triton_reference(dev, flush, steps):
    """The reference's own GPU path (``PesqLossTriton``, Triton kernels) on the
    headline workload, timed like this engine: the whole fwd+bwd (w.r.t. deg)
    step captured in one CUDA graph, L2 flushed, CUDA events; plus its own
    ``graphed`` callable and the eager step."""

    import torch

    from triton_pesq_b200 import PesqLossCuda
    from triton_pesq_b200.signals import workload

    PesqLossTriton = _import_reference_gpu()
    out_ops = _measure_reference_ops(dev)
    ref_c, deg_c, sr = workload("cfg2", seed=0)
    ref, deg = ref_c.to(dev), deg_c.to(dev)
    utt_s = ref.shape[0] * ref.shape[1] / sr
    model = PesqLossTriton(1.0, sample_rate=sr).to(dev)
    out = {"workload": "cfg2: 8 x 8 s at 16 kHz, fwd + bwd w.r.t. deg"}

    def timed(fn, n):
        times = []
        for k in range(n + 3):
            flush.zero_()
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record()
            fn()
            b.record()
            b.synchronize()
            if k >= 3:
                times.append(a.elapsed_time(b))
        return statistics.median(times)

    d = deg.detach().requires_grad_(True)

    def eager():
        loss = model(ref, d)
        torch.autograd.grad(loss.sum(), [d])

    out["eager_ms_per_step"] = timed(eager, steps)
    graphed = model.graphed(ref, d)

    def replay():
        loss = graphed(ref, d)
        torch.autograd.grad(loss.sum(), [d])

    out["graphed_callable_ms_per_step"] = timed(replay, steps)
    try:
        out["step_graph_ms_per_step"] = _graphed_step_ms(model, ref, deg, flush, steps)
    except Exception as exc:  # a host synchronisation inside the step breaks the capture
        out["step_graph_ms_per_step"] = None
        out["step_graph_error"] = f"{type(exc).__name__}: {exc}"[:200]
    best = min(v for v in (out["graphed_callable_ms_per_step"], out["step_graph_ms_per_step"]) if v)
    out["utterance_seconds_per_s"] = utt_s / (best * 1e-3)
    # this engine, same workload and timing
    mine = _graphed_step_ms(PesqLossCuda(1.0, sample_rate=sr), ref, deg, flush, steps)
    out["this_engine_ms_per_step"] = mine
    out["speedup"] = best / mine
    # the two agree (float32 reference path vs this engine): relative distance gap
    with torch.no_grad():
        ds_r, da_r = model.raw(ref, deg)
        ds_m, da_m = PesqLossCuda(1.0, sample_rate=sr).raw(ref, deg)
    out["max_rel_diff_d_symm"] = float(((ds_r - ds_m).abs() / ds_m.abs()).max())
    out["max_rel_diff_d_asymm"] = float(((da_r - da_m).abs() / da_m.abs()).max())
    out["ops"] = out_ops
    return out


def _measure_reference_ops(dev, launches=20):
    """The reference's standalone ``TritonIIR`` and ``TritonResample`` and this
    engine's ``IIRCuda`` / ``ResampleCuda`` on the same shapes, each call
    timed the same way (eager, CUDA events over ``launches`` calls after 3
    warm-up calls)."""

    import torch

    from torch_pesq.triton_ops.iir import TritonIIR
    from torch_pesq.triton_ops.resample import TritonResample

    from triton_pesq_b200 import IIRCuda, ResampleCuda
    from triton_pesq_b200.tables import power_filter, pre_filter

    stream = torch.cuda.current_stream(dev)

    def timed(fn):
        for _ in range(3):
            fn()
        start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record(stream)
        for _ in range(launches):
            fn()
        stop.record(stream)
        torch.cuda.synchronize()
        return 1e3 * start.elapsed_time(stop) / launches

    out = {}
    for label, (b, a) in (("order10", power_filter()), ("order2", pre_filter())):
        theirs = TritonIIR(torch.tensor(b, dtype=torch.float32), torch.tensor(a, dtype=torch.float32)).to(dev)
        mine = IIRCuda(b, a).to(dev)
        shapes = ((8, 16000), (8, 64000), (64, 480000), (30720, 1000)) if label == "order10" else ((64, 480000),)
        for rows, n in shapes:
            x = torch.randn(rows, n, device=dev)
            row = {"reference_fwd_us": timed(lambda: theirs(x)), "this_fwd_us": timed(lambda: mine(x))}
            if rows * n <= 512000:
                leaf = x.clone().requires_grad_(True)
                g = torch.randn_like(x)
                row["reference_fwd_bwd_us"] = timed(lambda: torch.autograd.grad(theirs(leaf), leaf, g))
                row["this_fwd_bwd_us"] = timed(lambda: torch.autograd.grad(mine(leaf), leaf, g))
            with torch.no_grad():
                y_t, y_m = theirs(x), mine(x)
                row["max_abs_diff_over_peak"] = float((y_t - y_m).abs().max() / y_m.abs().max())
            row["speedup_fwd"] = row["reference_fwd_us"] / row["this_fwd_us"]
            out[f"iir_{label}_{rows}x{n}"] = row
    theirs = TritonResample(44100, 16000).to(dev)
    mine = ResampleCuda(44100, 16000).to(dev)
    x = torch.randn(256, 4 * 44100, device=dev)
    leaf = x.clone().requires_grad_(True)
    y = mine(x)
    g = torch.randn_like(y)
    row = {"reference_fwd_us": timed(lambda: theirs(x)), "this_fwd_us": timed(lambda: mine(x)),
           "reference_fwd_bwd_us": timed(lambda: torch.autograd.grad(theirs(leaf), leaf, g)),
           "this_fwd_bwd_us": timed(lambda: torch.autograd.grad(mine(leaf), leaf, g))}
    with torch.no_grad():
        row["max_abs_diff_over_peak"] = float((theirs(x) - y).abs().max() / y.abs().max())
    row["speedup_fwd"] = row["reference_fwd_us"] / row["this_fwd_us"]
    row["speedup_fwd_bwd"] = row["reference_fwd_bwd_us"] / row["this_fwd_bwd_us"]
    out["resample_44100_to_16000_256x176400"] = row
    return out


def run_op(args):
    """Only the large case of a standalone op, e.g. as the target of a
    profiler capture; or the reference's own GPU path."""

    import torch

    dev = torch.device("cuda", 0)
    peak, _ = measured_peaks()
    if args.op == "triton-reference":
        flush = torch.empty(L2_FLUSH_BYTES // 4, dtype=torch.float32, device=dev)
        try:
            result = measure_triton_reference(dev, flush, args.steps)
        except ImportError as exc:
            result = {"unavailable": str(exc)}
        print(json.dumps({"op": args.op, "measurements": result}))
        return
    if args.op == "geometry":
        flush = torch.empty(L2_FLUSH_BYTES // 4, dtype=torch.float32, device=dev)
        print(json.dumps({"op": args.op, "measurements": measure_geometries(dev, flush, steps=args.steps)}))
        return
    if args.op == "resample":
        result = measure_resampler(dev, peak, launches=args.steps)
    else:
        result = measure_iir(dev, peak, launches=args.steps, large_only=True)
    print(json.dumps({"op": args.op, "measurements": result}))


def main():
    args = parse_args()
    if args.op is not None:
        run_op(args)
    elif args.impl == "reference":
        run_reference(args)
    else:
        run_cuda(args)


if __name__ == "__main__":
    main()
