"""Filters, references and tolerances shared by the IIR tests (the structure of
the reference's tests/test_triton_iir.py:1-140).

Every parity test compares the CUDA filter and the float32 ``lfilter`` of
torchaudio (the reference's own oracle) against a float64 ``lfilter`` (the
oracle's restatement, ``oracle.pesq_oracle.lfilter``), and requires the CUDA
filter to be within :data:`TOL` of it and no worse than the float32 oracle,
down to the float32 floor :data:`FLOOR`.  Errors are relative to the peak of
the exact result.
"""

import math

import numpy as np
import torch
from scipy.signal import butter

#: peak relative error bound against float64 (the reference's TOL,
#: test_triton_iir.py:34-39)
TOL = 1e-5
#: float32 floor below which the CUDA filter need not beat the float32 oracle
FLOOR = 3e-6

FILTERS = {
    "order2": (np.array([2.740826, -5.4816519, 2.740826]), np.array([1.0, -1.9444777, 0.94597794])),
    "order10": tuple(np.asarray(c) for c in butter(5, [325, 3250], fs=16000, btype="band")),
}

#: coefficient sets that break naive state space constructions (repeated and
#: zero poles, an unnormalised a[0]); numerator and denominator of equal length
DEGENERATE = {
    "b_longer_than_a": (np.array([1.0, 2.0, 3.0, 4.0, 5.0]), np.array([1.0, -0.5, 0.0, 0.0, 0.0])),
    "double_pole": (np.array([1.0, 0.0, 0.0]), np.array([1.0, -1.0, 0.25])),
    "triple_pole": (np.array([1.0, 0.0, 0.0, 0.0]), np.array([1.0, -2.1, 1.47, -0.343])),
    "unnormalised_a0": (np.array([2.0, 1.0, 0.0]), np.array([4.0, -2.0, 0.5])),
    "single_pole": (np.array([1.0, 0.5]), np.array([1.0, -0.9])),
    "odd_order": tuple(np.asarray(c) for c in butter(3, 3000, fs=16000, btype="low")),
}


def resonator(radius: float, angle: float = 0.3):
    return np.array([1.0, 0.0, 0.0]), np.array([1.0, -2 * radius * np.cos(angle), radius * radius])


def exact(signal: torch.Tensor, b, a) -> torch.Tensor:
    """float64 lfilter on the CPU (the oracle)."""

    from oracle.pesq_oracle import lfilter

    return lfilter(signal.detach().double().cpu(), np.asarray(b, np.float64), np.asarray(a, np.float64))


def exact_vjp(signal: torch.Tensor, upstream: torch.Tensor, b, a) -> torch.Tensor:
    from oracle.pesq_oracle import lfilter

    x = signal.detach().double().cpu().requires_grad_(True)
    y = lfilter(x, np.asarray(b, np.float64), np.asarray(a, np.float64))
    return torch.autograd.grad(y, x, upstream.detach().double().cpu())[0]


def oracle32(signal: torch.Tensor, b, a) -> torch.Tensor:
    """torchaudio's float32 lfilter (the reference's oracle), on the CPU."""

    from torchaudio.functional import lfilter

    b, a = np.asarray(b, np.float64), np.asarray(a, np.float64)
    size = max(b.size, a.size)
    b, a = np.pad(b, (0, size - b.size)), np.pad(a, (0, size - a.size))
    return lfilter(signal.detach().float().cpu(), torch.tensor(a, dtype=torch.float32),
                   torch.tensor(b, dtype=torch.float32), clamp=False)


def oracle32_vjp(signal: torch.Tensor, upstream: torch.Tensor, b, a) -> torch.Tensor:
    from torchaudio.functional import lfilter

    b, a = np.asarray(b, np.float64), np.asarray(a, np.float64)
    size = max(b.size, a.size)
    b, a = np.pad(b, (0, size - b.size)), np.pad(a, (0, size - a.size))
    x = signal.detach().float().cpu().requires_grad_(True)
    y = lfilter(x, torch.tensor(a, dtype=torch.float32), torch.tensor(b, dtype=torch.float32), clamp=False)
    return torch.autograd.grad(y, x, upstream.detach().float().cpu())[0]


def peak_error(value, target) -> float:
    target = target.double().cpu()
    scale = target.abs().max().item()
    if scale == 0.0:
        return value.double().cpu().abs().max().item()
    return (value.double().cpu() - target).abs().max().item() / scale


def check_accuracy(mine, oracle, truth, what=""):
    """Within TOL of float64 and no worse than the float32 oracle (or FLOOR)."""

    ours, theirs = peak_error(mine, truth), peak_error(oracle, truth)
    if not math.isfinite(theirs):
        theirs = math.inf
    assert math.isfinite(ours), f"{what}: {ours}"
    assert ours < TOL, f"{what}: {ours} >= {TOL}"
    assert ours <= max(theirs, FLOOR), f"{what}: {ours} worse than the float32 oracle {theirs}"
    return ours


def noise(*shape, seed=0, scale=1.0, device="cuda"):
    g = torch.Generator(device="cpu").manual_seed(seed)
    return (torch.randn(*shape, generator=g) * scale).to(device)
