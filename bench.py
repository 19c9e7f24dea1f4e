#!/usr/bin/env python
"""Benchmark: PESQ loss forward + backward on B200, utterance-seconds per second.

Workload (the configuration the headline metric is quoted on): batch 8 x 8 s
at 16 kHz per GPU, speech-like seeded synthetic signals with f0 ~ U[90, 250]
Hz and SNR ~ U[0, 20] dB, forward + backward w.r.t. the degraded signal of
the global mean loss, CUDA-graph replayed.  With N GPUs every rank runs its
own batch (weak scaling, batch sharding) and the global mean loss is
all-reduced over NCCL inside the captured step, on a side stream that
overlaps the backward: the only collective of the path.  Beside it the
north star's scaling configuration (512 x 3 s at 16 kHz as one global batch
sharded over the N ranks, strong scaling) and the 64 x 10 s at 48 kHz batch
sharded the same way.

Timing: W untimed warm-up steps, then K steps, each bracketed by CUDA events
on the launching stream; the L2 is flushed (a 256 MiB write) between steps
outside the events, because the step's inputs (8 MiB) fit in L2.  The K-step
loop is bracketed by a barrier and synchronize; the reported time is the sum
of the K step times, maximum over ranks.

Also reported: e2e (same metric through the public API, ``PesqLossCuda.graphed``,
with the inputs copied from pinned host memory and the losses and the
global mean read back every step), eager latency, per-stage kernel times,
the roofline of the dominant kernel and the reference's CPU path (its own
``PesqLoss`` from the offline install in baseline/_ref, with the oracle port
beside it) timed on this host.

``--impl reference`` times the reference CPU implementation of the path (its
``PesqLoss``; the oracle port in the reference's dtype mode where the
reference is not installed) on this host's cores instead.
"""

from __future__ import annotations

import argparse
import gc
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
    ap.add_argument("--op", choices=["iir", "resample", "geometry", "triton-reference", "step"], default=None,
                    help="time only a standalone op on its large case, or (step) the workload's eager "
                         "fwd+bwd W + K times (one JSON line; the target of single-kernel profiler captures)")
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


def profiled_flops():
    """Float64 and float32 FLOPs per front-kernel launch on the headline
    workload, from the ncu instruction counters of the committed summary
    (a fixed count of the workload: DFMA counts two, DADD and DMUL one)."""

    path = os.path.join(ROOT, "profiles", "front_kernel_cfg2.txt")
    out = {}
    if os.path.exists(path):
        for line in open(path):
            for key in ("fp64_flops_per_launch", "fp32_flops_per_launch"):
                if line.startswith(key + ":"):
                    out[key] = float(line.split(":")[1])
    return out if len(out) == 2 else None


def front_compute(flops, launch_us, dev, clocks):
    """The front kernel against its arithmetic pipes: it reads its inputs once
    and is bound by instruction issue and the float64 pipe (the FFTs and the
    pre-emphasis), not by HBM.  Achieved = the profiled FLOPs per launch over
    the live launch time; peaks are nominal, 64 float64 and 128 float32 FMA
    lanes per SM per clock at the sampled maximum SM clock."""

    import torch

    if not flops or not launch_us:
        return None
    mhz = (clocks or {}).get("sm_max_mhz") or 1965.0
    sms = torch.cuda.get_device_properties(dev).multi_processor_count
    peak64 = sms * 64 * 2 * mhz * 1e6 / 1e12
    peak32 = sms * 128 * 2 * mhz * 1e6 / 1e12
    f64 = flops["fp64_flops_per_launch"] / (launch_us * 1e-6) / 1e12
    f32 = flops["fp32_flops_per_launch"] / (launch_us * 1e-6) / 1e12
    return {"fp64_flops_per_launch": flops["fp64_flops_per_launch"], "fp64_tflops": f64,
            "fp64_peak_tflops_nominal": peak64, "fp64_frac": f64 / peak64,
            "fp32_flops_per_launch": flops["fp32_flops_per_launch"], "fp32_tflops": f32,
            "fp32_peak_tflops_nominal": peak32, "fp32_frac": f32 / peak32,
            "source": "ncu sass op counters of profiles/front_kernel_cfg2.txt; nominal peaks"}


def device_identity(index: int):
    """Name and driver version of the GPU (nvidia-smi): step times of the same
    code were seen to differ between boxes with different drivers."""

    try:
        out = subprocess.run(["nvidia-smi", f"--id={index}", "--query-gpu=name,driver_version",
                              "--format=csv,noheader"], capture_output=True, text=True, timeout=20).stdout
        name, driver = [p.strip() for p in out.strip().splitlines()[0].split(",")[:2]]
        return {"name": name, "driver": driver}
    except (OSError, IndexError, ValueError, subprocess.TimeoutExpired):
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


def cpu_port_step(ref, deg, params):
    """One forward + backward (w.r.t. deg) of the oracle port of the reference
    CPU path in the reference's dtype mode (float32 signal stages, float64
    perceptual chain, as PesqLoss evaluates on the CPU)."""

    import torch

    from oracle import pesq_oracle as O

    d = deg.detach().clone().requires_grad_(True)
    loss = O.forward(ref, d, params, mode="reference")
    (g,) = torch.autograd.grad(loss.sum(), [d])
    return loss, g


def reference_cpu_model(sample_rate):
    """The reference's own ``PesqLoss`` (``torch_pesq/loss.py``) from the
    offline install in baseline/_ref, or None when it is not installed."""

    try:
        return _reference_package().PesqLoss(1.0, sample_rate=sample_rate)
    except ImportError:
        return None


def reference_cpu_step(model, ref, deg):
    """One forward + backward (w.r.t. deg) through the reference's
    ``PesqLoss`` on the CPU: its float32 torchaudio signal path and float64
    perceptual chain (``loss.py:300-322``)."""

    import torch

    d = deg.detach().clone().requires_grad_(True)
    loss = model(ref, d)
    (g,) = torch.autograd.grad(loss.sum(), [d])
    return loss, g


def _time_cpu(step, budget_s, min_steps=2):
    steps, t0 = 0, time.perf_counter()
    while True:
        step()
        steps += 1
        elapsed = time.perf_counter() - t0
        if elapsed >= budget_s and steps >= min_steps:
            return steps, elapsed


def cpu_baseline(budget_s: float):
    """The reference's CPU path on this host's cores, on the whole cfg2 batch
    (8 x 8 s at 16 kHz, fwd + bwd w.r.t. deg) for about ``budget_s`` seconds:
    the reference's own ``PesqLoss`` when it is installed (kind "reference"),
    with the oracle port beside it; the port alone otherwise."""

    import torch

    from oracle import pesq_oracle as O
    from triton_pesq_b200.signals import workload

    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    ref, deg, sr = workload("cfg2", seed=0)
    b, secs = WORKLOADS["cfg2"]
    params = O.OracleParams(factor=1.0, sample_rate=sr)
    cpu_port_step(ref[:1], deg[:1], params)  # warm-up
    steps, elapsed = _time_cpu(lambda: cpu_port_step(ref, deg, params), budget_s / 2)
    port = {
        "value": steps * b * secs / elapsed, "unit": UNIT, "cores": threads, "kind": "port",
        "sample": f"{steps} x forward+backward(deg) of the full 8 x 8 s @16 kHz batch, {elapsed:.1f} s, "
                  "oracle port in the reference dtype mode (float32 signal path, float64 chain)",
    }
    model = reference_cpu_model(sr)
    if model is None:
        return port
    reference_cpu_step(model, ref[:1], deg[:1])  # warm-up
    steps, elapsed = _time_cpu(lambda: reference_cpu_step(model, ref, deg), budget_s)
    return {
        "value": steps * b * secs / elapsed, "unit": UNIT, "cores": threads, "kind": "reference",
        "sample": f"{steps} x forward+backward(deg) of the full 8 x 8 s @16 kHz batch, {elapsed:.1f} s, "
                  "the reference's PesqLoss (torch_pesq/loss.py) from baseline/_ref",
        "port": port,
    }


# ---------------------------------------------------------------------------
# reference arm
# ---------------------------------------------------------------------------


def run_reference(args):
    """The reference's CPU implementation of the path on this host: its own
    ``PesqLoss`` forward + backward (w.r.t. deg) on the whole headline batch
    each step, all host threads; the oracle port in the reference's dtype
    mode when the reference is not installed."""

    world, rank, _ = dist_env()
    if rank != 0:
        return
    import torch

    from oracle import pesq_oracle as O
    from triton_pesq_b200.signals import workload

    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    ref, deg, sr = workload("cfg2", seed=0)
    model = reference_cpu_model(sr)
    if model is not None:
        kind = "reference"
        what = "the reference's PesqLoss (torch_pesq/loss.py, offline install in baseline/_ref)"

        def step():
            reference_cpu_step(model, ref, deg)
    else:
        kind = "port"
        what = ("oracle port of PesqLoss in the reference dtype mode (float32 signal path, float64 chain); "
                "the reference is not installed in baseline/_ref")
        params = O.OracleParams(factor=1.0, sample_rate=sr)

        def step():
            cpu_port_step(ref, deg, params)

    for _ in range(args.warmup):
        step()
    times = []
    for _ in range(args.steps):
        t0 = time.perf_counter()
        step()
        times.append(time.perf_counter() - t0)
    total = sum(times)
    value = args.steps * BATCH * SECONDS / total
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
        "config": {"workload": f"{BATCH}x{SECONDS:g}s@16k fwd+bwd(deg)", "global_batch": BATCH, "seconds": SECONDS,
                   "sample_rate": RATE, "sample_per_step": f"the whole batch: {BATCH} x {SECONDS:g} s utterances"},
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": threads, "kind": kind,
                         "sample": f"the whole {BATCH} x {SECONDS:g} s batch per step, {what}"},
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

    from triton_pesq_b200 import IIRCuda, _lib
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
            "tiles": "overlapped" if module.overlap and n > 8448 else ("chained" if n > 8448 else "packed rows"),
        }
        if module.overlap and n > 8448:
            # the same rows with the tiles chained by the look-back instead
            out[f"{label}_{rows}x{n}"]["forward_lookback_us"] = timed(
                lambda: torch.ops.pesq_cuda.iir(handle, x, module._flags(False) | _lib.IIR_CHAINED))
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

    from triton_pesq_b200 import PesqLossCuda, ResampleCuda
    from triton_pesq_b200.signals import workload

    out = {}
    for name, keep, secs in (("cfg1", 1, 1.0), ("cfg3", 16, 4.0), ("cfg4_per_gpu", 8, 10.0), ("cfg5", 512, 3.0)):
        ref_c, deg_c, sr = workload(name.split("_")[0], seed=0, rows=range(keep))
        model = PesqLossCuda(1.0, sample_rate=sr)
        ref, deg = ref_c.to(dev), deg_c.to(dev)
        ms = _graphed_step_ms(model, ref, deg, flush, steps)
        out[name] = {"batch": keep, "seconds": secs, "sample_rate": sr, "ms_per_step": ms,
                     "utterance_seconds_per_s": keep * secs / (ms * 1e-3)}
        if name == "cfg5":
            # the stages of the scaling configuration's whole batch on one GPU
            out[name]["stages_us"] = stage_times(model, ref, deg, dev)
        if sr != 16000:
            # the stages of the resampled step (front and back include the
            # resampler and its adjoint), and the resampler alone on the
            # same rows (2B forward, B gradient rows for the adjoint)
            out[name]["stages_us"] = stage_times(model, ref, deg, dev)
            rs = ResampleCuda(sr, 16000).to(dev)
            handle = rs._handle(dev)
            both = torch.cat([ref, deg])
            y = torch.ops.pesq_cuda.resample(handle, both)
            g = torch.randn_like(y[:keep])
            stream = torch.cuda.current_stream(dev)

            def timed(fn, n=20):
                for _ in range(3):
                    fn()
                a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                a.record(stream)
                for _ in range(n):
                    fn()
                b.record(stream)
                torch.cuda.synchronize()
                return 1e3 * a.elapsed_time(b) / n

            out[name]["resample_us"] = {
                "forward_2B_rows": timed(lambda: torch.ops.pesq_cuda.resample(handle, both)),
                "adjoint_B_rows": timed(lambda: torch.ops.pesq_cuda.resample_adjoint(handle, g, ref.shape[1])),
            }
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


def numa_local_cores(local: int):
    """Pin this process to the host cores NVML names as nearest to its GPU,
    so that the pinned host buffers allocated afterwards land in that NUMA
    node's memory (first touch) and the host-to-device copies of the ranks of
    one box do not cross the socket interconnect.  Changes only this
    process's CPU affinity; returns the cores, or None when NVML cannot say."""

    try:
        import pynvml
        import torch

        props = torch.cuda.get_device_properties(local)
        pynvml.nvmlInit()
        try:
            handle = pynvml.nvmlDeviceGetHandleByPciBusId(
                f"{props.pci_domain_id:08x}:{props.pci_bus_id:02x}:{props.pci_device_id:02x}.0")
            words = pynvml.nvmlDeviceGetCpuAffinity(handle, (os.cpu_count() + 63) // 64)
        finally:
            pynvml.nvmlShutdown()
        cores = {64 * i + b for i, w in enumerate(words) for b in range(64) if (int(w) >> b) & 1}
        cores &= os.sched_getaffinity(0)
        if not cores:
            return None
        os.sched_setaffinity(0, cores)
        return sorted(cores)
    except Exception:
        return None


def capture_step(model, ref, deg, global_batch: int, group=None):
    """One data-parallel fwd+bwd step captured in a CUDA graph.

    Forward of this rank's utterances; the global mean loss (this rank's sum
    and count, all-reduced over NCCL when a process group exists) on a side
    stream that overlaps the backward; the backward of the global mean w.r.t.
    the degraded signals.  Returns ``(graph, (loss, grad, mean))``."""

    import torch

    from triton_pesq_b200.distributed import GlobalMean

    dev = ref.device
    # (a leaf that requires grad is used as it is: its caller refills it in place)
    deg_p = deg if (deg.requires_grad and deg.is_leaf) else deg.detach().clone().requires_grad_(True)
    mean_op = GlobalMean(dev, group)
    side = torch.cuda.Stream(dev)
    # d(global mean)/d(loss_u) = 1 / global batch for every utterance: the
    # upstream gradient autograd forms for loss.sum() / global_batch, passed
    # as the broadcast value it is (the engine takes it as one scalar)
    upstream = torch.full((1,), 1.0 / global_batch, device=dev).expand(ref.shape[0])

    def step():
        main = torch.cuda.current_stream(dev)
        loss, loss_sum = model.forward_sum(ref, deg_p)
        side.wait_stream(main)
        with torch.cuda.stream(side):
            mean = mean_op(loss, loss_sum)
        (g,) = torch.autograd.grad(loss, [deg_p], grad_outputs=upstream)
        main.wait_stream(side)
        return loss, g, mean

    warm = torch.cuda.Stream(dev)
    warm.wait_stream(torch.cuda.current_stream(dev))
    with torch.cuda.stream(warm):
        for _ in range(3):
            step()
    torch.cuda.current_stream(dev).wait_stream(warm)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        out = step()
    torch.cuda.synchronize()
    return graph, out


def timed_replays(graph, steps: int, warmup: int, flush, world: int, clocks=None):
    """Replay a captured step ``warmup`` times untimed, then ``steps`` times,
    each bracketed by CUDA events on the launching stream with the L2 flushed
    before it (outside the events); barrier + synchronize around the timed
    loop.  Returns (per-step ms of this rank, total seconds max over ranks,
    wall seconds of the timed loop)."""

    import torch
    import torch.distributed as dist

    dev = flush.device
    stream = torch.cuda.current_stream(dev)
    for _ in range(warmup):
        flush.zero_()
        graph.replay()
    events = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(steps)]
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    wall0 = time.perf_counter()
    for k in range(steps):
        flush.zero_()
        events[k][0].record(stream)
        graph.replay()
        events[k][1].record(stream)
    torch.cuda.synchronize()
    wall = time.perf_counter() - wall0
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    step_ms = [a.elapsed_time(b) for a, b in events]
    total = torch.tensor([sum(step_ms)], device=dev, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(total, op=dist.ReduceOp.MAX)
    return step_ms, float(total.item()) / 1e3, wall


def measure_sharded(name: str, global_batch: int, steps: int, warmup: int, flush, world: int, rank: int):
    """A BASELINE configuration with a fixed global batch sharded over the
    ranks (strong scaling): rank r evaluates its contiguous slice of the
    utterances, the step (fwd+bwd of the global mean, its all-reduce inside)
    is graph-replayed; time = max over ranks of the summed step times."""

    import torch

    from triton_pesq_b200 import PesqLossCuda
    from triton_pesq_b200.distributed import shard_bounds
    from triton_pesq_b200.signals import WORKLOADS, workload

    dev = flush.device
    lo, hi = shard_bounds(global_batch, rank, world)
    ref_c, deg_c, sr = workload(name, seed=0, rows=range(lo, hi))
    model = PesqLossCuda(1.0, sample_rate=sr)
    graph, _ = capture_step(model, ref_c.to(dev), deg_c.to(dev), global_batch)
    step_ms, total_s, _ = timed_replays(graph, steps, warmup, flush, world)
    del graph
    seconds = WORKLOADS[name][1] / sr
    return {
        "global_batch": global_batch, "per_rank_batch": hi - lo, "seconds": seconds, "sample_rate": sr,
        "scaling": "strong", "steps": steps,
        "ms_per_step": 1e3 * total_s / steps,
        "utterance_seconds_per_s": global_batch * seconds * steps / total_s,
        "step": "graph replay of fwd + bwd(deg) of the global mean loss, NCCL all-reduce of [sum, count] "
                "on a side stream overlapping the backward (none at N = 1)",
    }


def run_cuda(args):
    import torch
    import torch.distributed as dist

    from triton_pesq_b200 import PesqLossCuda
    from triton_pesq_b200.distributed import GlobalMean
    from triton_pesq_b200.signals import workload

    world, rank, local = dist_env()
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    # libraries print banners (NCCL's version line) on file descriptor 1: send
    # it to stderr until the JSON line, so that stdout carries that line only
    sys.stdout.flush()
    stdout_fd = os.dup(1)
    os.dup2(2, 1)
    cores = numa_local_cores(local)
    if world > 1:
        import datetime

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)

    model = PesqLossCuda(1.0, sample_rate=RATE)
    ref_cpu, deg_cpu, _ = workload(args.workload, seed=rank)
    ref = ref_cpu.to(dev)
    deg = deg_cpu.to(dev)
    flush = torch.empty(L2_FLUSH_BYTES // 4, dtype=torch.float32, device=dev)
    global_batch = BATCH * world

    # ---- graph-replayed forward + backward (the headline value): each rank
    # evaluates its own utterances; the global mean loss is all-reduced over
    # NCCL inside the step, overlapping the backward
    graph, (loss_g, grad_g, mean_g) = capture_step(model, ref, deg, global_batch)
    with ClockSampler(local) as clocks:
        step_ms, total_s, wall = timed_replays(graph, args.steps, args.warmup, flush, world)
    clock_summary = clocks.summary()
    utt_per_step = BATCH * SECONDS * world
    value = utt_per_step * args.steps / total_s
    # the all-reduced mean agrees with the losses of every rank
    check = torch.stack([loss_g.detach().double().sum(), torch.tensor(float(BATCH), device=dev, dtype=torch.float64)])
    if world > 1:
        dist.all_reduce(check)
    mean_ok = bool(torch.isclose(mean_g, check[0] / check[1], rtol=1e-12, atol=0).item())

    # ---- eager latency (host dispatch included)
    deg_e = deg.detach().clone().requires_grad_(True)
    eager = []
    for k in range(max(5, args.steps // 5)):
        flush.zero_()
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        out = model(ref, deg_e)
        torch.autograd.grad(out.sum(), [deg_e])
        torch.cuda.synchronize()
        eager.append(time.perf_counter() - t0)

    # ---- end to end through the public API with host buffers
    # Every step copies its inputs from pinned host memory and reads its
    # losses and the global mean back.  The step itself is the captured
    # training step a user builds from the public API (PesqLossCuda.forward_sum,
    # autograd, distributed.GlobalMean; capture_step), on two input sets: the
    # copy of step k + 1 (on copy streams, into the other set) overlaps the
    # compute of step k, and a set is overwritten only after the step that
    # used it has finished.  Beside it: the serial variant (copy, compute,
    # read back, wait), and the same loop through PesqLossCuda.graphed (the
    # reference's graphed API: forward and backward graphs replayed from
    # Python autograd).  With several ranks per box each process first moves
    # to the cores of its GPU's NUMA node (numa_local_cores), so that its
    # pinned buffers are local.
    ref_h = ref_cpu.pin_memory()
    deg_h = deg_cpu.pin_memory()
    loss_h = [torch.empty(BATCH + 1, dtype=torch.float64, pin_memory=True) for _ in range(2)]
    stream = torch.cuda.current_stream(dev)
    sets = []
    for _ in range(2):
        ref_d = ref.clone()
        deg_d = deg.clone().requires_grad_(True)
        g_step, (loss_s, _, mean_s) = capture_step(PesqLossCuda(1.0, sample_rate=RATE), ref_d, deg_d, global_batch)
        result = torch.empty(BATCH + 1, dtype=torch.float64, device=dev)
        sets.append((ref_d, deg_d, g_step, loss_s, mean_s, result))
    copy_streams = [torch.cuda.Stream(dev), torch.cuda.Stream(dev)]
    copied = [[torch.cuda.Event(), torch.cuda.Event()] for _ in range(2)]
    consumed = [torch.cuda.Event() for _ in range(2)]
    split = [True]

    def issue_copy(k):
        ref_d, deg_d = sets[k % 2][:2]
        for i, (dst, src) in enumerate(((ref_d, ref_h), (deg_d, deg_h))):
            cs = copy_streams[i] if split[0] else copy_streams[0]
            with torch.cuda.stream(cs):
                cs.wait_event(consumed[k % 2])
                with torch.no_grad():
                    dst.copy_(src, non_blocking=True)
                copied[k % 2][i].record(cs)

    def run_step(k):
        _, _, g_step, loss_s, mean_s, result = sets[k % 2]
        stream.wait_event(copied[k % 2][0])
        stream.wait_event(copied[k % 2][1])
        g_step.replay()
        consumed[k % 2].record(stream)
        with torch.no_grad():
            result[:BATCH].copy_(loss_s.detach())
            result[BATCH:].copy_(mean_s.reshape(1))
        loss_h[k % 2].copy_(result, non_blocking=True)

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

    if world > 1:
        dist.barrier()
    split[0] = False
    pipelined(4)  # warm-up
    torch.cuda.synchronize()
    one_stream = torch.tensor([pipelined(args.steps)], device=dev, dtype=torch.float64)
    split[0] = True
    pipelined(4)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    e2e_total = torch.tensor([pipelined(args.steps)], device=dev, dtype=torch.float64)

    # host-to-device copy rate of this rank alone (the inputs of one step)
    h2d = []
    for _ in range(5):
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(stream)
        with torch.no_grad():
            sets[0][0].copy_(ref_h, non_blocking=True)
            sets[0][1].copy_(deg_h, non_blocking=True)
        b.record(stream)
        b.synchronize()
        h2d.append(a.elapsed_time(b))
    h2d_gbs = 2 * ref.numel() * 4 / (statistics.median(h2d) * 1e-3) / 1e9
    # the same copies on every rank at once: the box's host-to-device ceiling
    # for this many GPUs (aggregate over the ranks, max-over-ranks time)
    h2d_all = None
    if world > 1:
        dist.barrier()
        torch.cuda.synchronize()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(stream)
        for _ in range(10):
            with torch.no_grad():
                sets[0][0].copy_(ref_h, non_blocking=True)
                sets[0][1].copy_(deg_h, non_blocking=True)
        b.record(stream)
        b.synchronize()
        t_all = torch.tensor([a.elapsed_time(b)], device=dev, dtype=torch.float64)
        dist.all_reduce(t_all, op=dist.ReduceOp.MAX)
        h2d_all = world * 10 * 2 * ref.numel() * 4 / (float(t_all.item()) * 1e-3) / 1e9

    serial_ms = []
    for k in range(max(5, args.steps // 5)):
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        ref_d, deg_d, g_step, loss_s, mean_s, result = sets[0]
        a.record(stream)
        with torch.no_grad():
            ref_d.copy_(ref_h, non_blocking=True)
            deg_d.copy_(deg_h, non_blocking=True)
        g_step.replay()
        with torch.no_grad():
            result[:BATCH].copy_(loss_s.detach())
            result[BATCH:].copy_(mean_s.reshape(1))
        loss_h[0].copy_(result, non_blocking=True)
        b.record(stream)
        b.synchronize()
        serial_ms.append(a.elapsed_time(b))

    # the same loop through the module's graphed callables (forward and
    # backward CUDA graphs of PesqLossCuda.graphed, autograd in Python)
    mod_sets = []
    for _ in range(2):
        ref_d = ref.clone()
        deg_d = deg.clone().requires_grad_(True)
        mod_sets.append((ref_d, deg_d, PesqLossCuda(1.0, sample_rate=RATE).graphed(ref_d, deg_d)))
    side = torch.cuda.Stream(dev)
    mean_op = GlobalMean(dev)
    upstream = torch.full((1,), 1.0 / global_batch, device=dev).expand(BATCH)

    def module_loop(n):
        start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record(stream)
        for k in range(n):
            ref_d, deg_d, graphed = mod_sets[k % 2]
            with torch.no_grad():
                ref_d.copy_(ref_h, non_blocking=True)
                deg_d.copy_(deg_h, non_blocking=True)
            out = graphed(ref_d, deg_d)
            side.wait_stream(stream)
            with torch.cuda.stream(side):
                mean = mean_op(out)
            torch.autograd.grad(out, [deg_d], grad_outputs=upstream)
            stream.wait_stream(side)
            loss_h[k % 2][:BATCH].copy_(out.detach(), non_blocking=True)
            loss_h[k % 2][BATCH:].copy_(mean.reshape(1), non_blocking=True)
        stop.record(stream)
        stop.synchronize()
        return start.elapsed_time(stop)

    module_loop(3)
    module_ms = torch.tensor([module_loop(args.steps)], device=dev, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(e2e_total, op=dist.ReduceOp.MAX)
        dist.all_reduce(one_stream, op=dist.ReduceOp.MAX)
        dist.all_reduce(module_ms, op=dist.ReduceOp.MAX)
    e2e_ms_total = float(e2e_total.item())
    e2e_value = utt_per_step * args.steps / (e2e_ms_total / 1e3)
    one_stream_ms = float(one_stream.item()) / args.steps
    module_ms_per_step = float(module_ms.item()) / args.steps
    del mod_sets

    # ---- the north star's scaling configuration: 512 x 3 s at 16 kHz as one
    # global batch sharded over the ranks, and the 64 x 10 s at 48 kHz batch
    # (half of it at -5 dB SNR) sharded the same way
    sharded = {}
    if not args.skip_configs:
        sharded["cfg5_scaling"] = measure_sharded("cfg5", 512, min(args.steps, 20), args.warmup, flush, world, rank)
        sharded["cfg4_sharded"] = measure_sharded("cfg4", 64, min(args.steps, 10), args.warmup, flush, world, rank)

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
    flops = profiled_flops()
    single = world == 1 and not args.skip_configs
    ops = {"resample_44k1_to_16k": measure_resampler(dev, peak), "iir": measure_iir(dev, peak)} if world == 1 else None
    configs = measure_configs(dev, flush) if single else None
    fused = measure_fused(dev, flush) if single else None
    geometries = measure_geometries(dev, flush) if single else None

    if world > 1:
        # every graph that holds an NCCL call is released before the process
        # group (its teardown waits for them): the headline step, both e2e
        # input sets, and the loop variable that still names one of them
        del graph, sets, g_step
        gc.collect()
        torch.cuda.synchronize()
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
            "workload": f"{BATCH}x{SECONDS:g}s@16k fwd+bwd(deg) of the global mean loss, CUDA-graph replay "
                        f"({args.workload})",
            "global_batch": global_batch,
            "seconds": SECONDS,
            "sample_rate": RATE,
            "parallelism": f"dp{world}",
            "collective": "NCCL all-reduce of the [sum, count] of the losses inside the captured step, on a side "
                          "stream overlapping the backward" if world > 1 else "none (one rank)",
            "l2": "flushed between steps (256 MiB write, outside the step events)",
        },
        "clocks": clock_summary,
        "device": device_identity(local),
        "e2e": {
            "value": e2e_value,
            "unit": UNIT,
            "h2d_bytes_per_step": int(ref.numel() * 4 * 2),
            "d2h_bytes_per_step": int((BATCH + 1) * 8),
            "api": "the captured training step (PesqLossCuda.forward_sum, autograd backward of the global mean, "
                   "distributed.GlobalMean) on two input sets, inputs copied from pinned host memory every step "
                   "(reference and degraded signal on two copy streams) overlapping the previous step's compute, "
                   "losses and global mean read back every step",
            "ms_per_step": e2e_ms_total / args.steps,
            "one_copy_stream_ms_per_step": one_stream_ms,
            "serial_ms_per_step": statistics.median(serial_ms),
            "graphed_module_ms_per_step": module_ms_per_step,
            "h2d_gbs_alone": h2d_gbs,
            "h2d_gbs_all_ranks_aggregate": h2d_all,
            "numa_local_cores": f"{len(cores)} cores" if cores else None,
        },
        # front + chain forward, chain adjoint + align + back per step
        "gpu_launches": 5 * args.steps,
        "mean_allreduce_ok": mean_ok,
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
            "compute": front_compute(flops, front_us, dev, clock_summary),
        },
        "stages_us": stages,
        **sharded,
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


def _reference_package():
    """The reference package ``torch_pesq`` installed in baseline/_ref by
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
    if REFERENCE_INSTALL not in sys.path:
        sys.path.insert(0, REFERENCE_INSTALL)
    import torch_pesq

    return torch_pesq


def _import_reference_gpu():
    """``PesqLossTriton`` of the reference installed in baseline/_ref."""

    return _reference_package().PesqLossTriton


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
    if args.op == "step":
        from triton_pesq_b200 import PesqLossCuda
        from triton_pesq_b200.signals import workload

        ref_c, deg_c, sr = workload(args.workload, seed=0)
        ref, deg = ref_c.to(dev), deg_c.to(dev).requires_grad_(True)
        model = PesqLossCuda(1.0, sample_rate=sr)
        flush = torch.empty(L2_FLUSH_BYTES // 4, dtype=torch.float32, device=dev)
        times = []
        for k in range(args.warmup + args.steps):
            flush.zero_()
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record()
            loss = model(ref, deg)
            torch.autograd.grad(loss.sum(), [deg])
            b.record()
            b.synchronize()
            if k >= args.warmup:
                times.append(a.elapsed_time(b))
        print(json.dumps({"op": "step", "workload": args.workload, "eager_ms_per_step": statistics.median(times)}))
        return
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
