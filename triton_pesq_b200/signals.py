"""Seeded synthetic workloads of the benchmark configurations.

There is no public dataset for this path; every input is synthesised from a
seed.  The speech-like model follows the workload description of the
benchmark configurations: a voiced harmonic stack (f0, 30 harmonics of
amplitude 1/k below Nyquist), amplitude-modulated by 0.5 (1 + sin 2 pi 4 t),
plus pink noise 30 dB below it, peak-normalised to 0.3.  Degradations are
white noise at a given SNR and, for the resampling workload, a seeded random
64-tap low pass FIR.
"""

from __future__ import annotations

import math
from typing import Optional, Sequence, Tuple

import torch


def pink_noise(batch: int, n: int, gen: torch.Generator, rows: Optional[Sequence[int]] = None) -> torch.Tensor:
    """Unit-variance 1/f noise by spectral shaping of white noise (the
    ``rows`` of a ``[batch, n]`` draw; all of them by default).  Each row is
    shaped on its own, so a selection equals the same rows of the whole."""

    white = torch.randn(batch, n, generator=gen, dtype=torch.float64)
    if rows is not None:
        white = white[torch.as_tensor([int(r) for r in rows])]
    spec = torch.stack([torch.fft.rfft(w) for w in white])
    f = torch.arange(spec.shape[1], dtype=torch.float64)
    f[0] = 1.0
    spec = spec / f.sqrt()
    pink = torch.stack([torch.fft.irfft(s, n=n) for s in spec])
    return pink / pink.std(dim=1, keepdim=True).clamp_min(1e-30)


def speech_like(
    batch: int,
    n: int,
    sample_rate: int,
    seed: int = 0,
    f0: Optional[Sequence[float]] = None,
    f0_range: Tuple[float, float] = (90.0, 250.0),
    rows: Optional[Sequence[int]] = None,
) -> torch.Tensor:
    """``[batch, n]`` float32 speech-like references (CPU).

    ``rows`` selects utterances of the batch: the result equals
    ``speech_like(batch, ...)[rows]`` bit for bit, but only the selected
    utterances are synthesised (a slice of a large workload is cheap)."""

    gen = torch.Generator().manual_seed(seed)
    rows = list(range(batch)) if rows is None else [int(r) for r in rows]
    t = torch.arange(n, dtype=torch.float64) / sample_rate
    if f0 is None:
        lo, hi = f0_range
        f0 = (lo + (hi - lo) * torch.rand(batch, generator=gen, dtype=torch.float64)).tolist()
    phases = [2 * math.pi * torch.rand(30, generator=gen, dtype=torch.float64) for _ in range(batch)]
    out = torch.zeros(len(rows), n, dtype=torch.float64)
    env = 0.5 * (1.0 + torch.sin(2 * math.pi * 4.0 * t))
    for i, b in enumerate(rows):
        sig = torch.zeros(n, dtype=torch.float64)
        for k in range(1, 31):
            if f0[b] * k >= sample_rate / 2:
                break
            sig += torch.sin(2 * math.pi * f0[b] * k * t + phases[b][k - 1]) / k
        out[i] = sig * env
    voiced_rms = out.pow(2).mean(dim=1, keepdim=True).sqrt()
    out = out + pink_noise(batch, n, gen, rows) * voiced_rms * 10 ** (-30 / 20)
    out = 0.3 * out / out.abs().amax(dim=1, keepdim=True)
    return out.float()


def add_noise(ref: torch.Tensor, snr_db, seed: int = 1, rows: Optional[Sequence[int]] = None,
              batch: Optional[int] = None) -> torch.Tensor:
    """``ref`` plus white Gaussian noise at ``snr_db`` (scalar or per row).

    With ``rows`` (and the full ``batch``), ``ref`` holds those utterances of
    a larger batch, and they receive exactly the noise (and the per-row SNR)
    the full batch would give them."""

    gen = torch.Generator().manual_seed(seed)
    ref64 = ref.double()
    full = ref.shape[0] if rows is None else int(batch)
    idx = torch.arange(full) if rows is None else torch.as_tensor([int(r) for r in rows])
    snr = torch.as_tensor(snr_db, dtype=torch.float64).reshape(-1, 1).expand(full, 1)[idx]
    power = ref64.pow(2).mean(dim=1, keepdim=True)
    noise = torch.randn((full, ref.shape[1]), generator=gen, dtype=torch.float64)[idx]
    return (ref64 + noise * (power / 10 ** (snr / 10)).sqrt()).float()


def lowpass_fir(ref: torch.Tensor, sample_rate: int, cutoff: float = 4000.0, taps: int = 64, seed: int = 2):
    """Convolve every row with a seeded random 64-tap low pass FIR."""

    gen = torch.Generator().manual_seed(seed)
    n = torch.arange(taps, dtype=torch.float64) - (taps - 1) / 2
    fc = cutoff / sample_rate
    sinc = torch.where(n == 0, torch.tensor(2 * fc, dtype=torch.float64), torch.sin(2 * math.pi * fc * n) / (math.pi * n))
    window = torch.hann_window(taps, periodic=False, dtype=torch.float64)
    jitter = 1.0 + 0.2 * (torch.rand(taps, generator=gen, dtype=torch.float64) - 0.5)
    h = sinc * window * jitter
    h = h / h.sum()
    x = ref.double()[:, None, :]
    y = torch.nn.functional.conv1d(torch.nn.functional.pad(x, (taps - 1, 0)), h.flip(0)[None, None, :])
    return y[:, 0, :].float()


#: batch, samples per utterance and sample rate of the named workloads
WORKLOADS = {"cfg1": (1, 16000, 16000), "cfg2": (8, 128000, 16000), "cfg3": (16, 176400, 44100),
             "cfg4": (64, 480000, 48000), "cfg5": (512, 48000, 16000)}


def workload(name: str, seed: int = 0, rows: Optional[Sequence[int]] = None):
    """Inputs of a named benchmark configuration: ``(ref, deg, sample_rate)``.

    * ``"cfg1"``: 1 x 1 s at 16 kHz, f0 = 120 Hz, 10 dB SNR
    * ``"cfg2"``: 8 x 8 s at 16 kHz, f0 ~ U[90, 250], SNR ~ U[0, 20] dB
    * ``"cfg3"``: 16 x 4 s at 44.1 kHz, low-pass FIR + 5 dB noise
    * ``"cfg4"``: 64 x 10 s at 48 kHz, half at -5 dB, half at 25 dB SNR
    * ``"cfg5"``: 512 x 3 s at 16 kHz, SNR ~ U[-5, 30] dB

    ``rows`` selects utterances: the result equals the same rows of the whole
    workload bit for bit, and only those are synthesised.
    """

    if name not in WORKLOADS:
        raise ValueError(f"unknown workload {name!r}")
    batch, n, sr = WORKLOADS[name]
    gen = torch.Generator().manual_seed(seed + 7)
    f0 = [120.0] if name == "cfg1" else None
    ref = speech_like(batch, n, sr, seed, f0=f0, rows=rows)
    if name == "cfg1":
        snr = 10.0
    elif name == "cfg2":
        snr = 20.0 * torch.rand(8, generator=gen, dtype=torch.float64)
    elif name == "cfg3":
        snr = 5.0
    elif name == "cfg4":
        snr = torch.tensor([-5.0] * 32 + [25.0] * 32, dtype=torch.float64)
    else:
        snr = -5.0 + 35.0 * torch.rand(512, generator=gen, dtype=torch.float64)
    clean = lowpass_fir(ref, sr, seed=seed + 2) if name == "cfg3" else ref
    return ref, add_noise(clean, snr, seed + 1, rows=rows, batch=batch), sr
