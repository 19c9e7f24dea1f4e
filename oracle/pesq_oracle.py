"""CPU oracle of the PESQ loss -- TEST INFRASTRUCTURE ONLY.

This module restates, on the CPU, the algorithm of the reference's
``PesqLoss`` (``torch_pesq/loss.py:172-322``) stage by stage, so that the
CUDA engine can be checked against it.  It is imported only by ``tests/``, by
``__graft_entry__.smoke()`` and by the CPU baseline leg of ``bench.py``; the
product path never touches it.

Two evaluation modes:

``float64``
    every stage in double precision with the reference's (float32-rounded)
    constants promoted to double -- the ground truth the north star's 1e-5
    distance / 1e-4 gradient tolerances are quoted against;
``reference``
    the dtype behaviour of ``PesqLoss`` itself: float32 signal stages, and the
    perceptual chain in float64 because the reference's Bark/loudness tables
    are float64 buffers (``bark.py:134-145``, ``loudness.py:52-55``).

Parity pin: ``tests/golden/*.npz`` hold inputs and outputs produced by the
reference code itself (``tests/golden/make_golden.py``), including float64
gradients of ``ref_pipeline`` on a ``.double()`` model; ``tests/test_oracle.py``
checks this module against them.

Third-party algorithms the reference calls and this file restates:
``torchaudio.functional.lfilter`` (zero initial state, ``clamp=False``) via
``scipy.signal.lfilter`` with the exact time-reversed adjoint, and the
torchaudio sinc resampling kernel via ``triton_pesq_b200.tables`` (pinned to
torchaudio 2.11.0's output by ``tests/test_tables.py``).
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Tuple

import numpy as np
import torch
import torch.nn.functional as F

from triton_pesq_b200 import tables as T

__all__ = [
    "OracleParams",
    "lfilter",
    "resample",
    "align_level",
    "preemphasize",
    "stft_bark",
    "chain",
    "raw",
    "forward",
    "mos",
    "epilogue",
]


@dataclass
class OracleParams:
    """Constants of ``PesqLoss(factor, sample_rate)`` (``loss.py:61-108``)."""

    factor: float = 1.0
    sample_rate: int = 16000
    nbarks: int = 49
    n_fft: int = 512
    win_length: int = 512
    hop_length: int = 256

    def __post_init__(self):
        lay = T.bark_layout(self.n_fft // 2, self.nbarks)
        self.fbank = lay.fbank().astype(np.float64)
        self.corr = lay.pow_dens_correction
        self.width_bark = lay.width_bark
        self.total_width = lay.total_width
        self.threshs = T.hearing_thresholds(self.nbarks)
        self.exps = T.loudness_exponents()
        self.pow_b, self.pow_a = T.power_filter()
        self.pre_b, self.pre_a = T.pre_filter()
        self.window = T.centred_window(self.win_length, self.n_fft)
        if self.sample_rate != 16000:
            self.kernel = T.sinc_resample_kernel(self.sample_rate, 16000)
        else:
            self.kernel = None


# ---------------------------------------------------------------------------
# differentiable lfilter (torchaudio.functional.lfilter semantics)
# ---------------------------------------------------------------------------


class _LFilter(torch.autograd.Function):
    """``y = lfilter(b, a, x)`` along the last axis, zero initial conditions.

    The vector-Jacobian product of a causal LTI filter is the same filter run
    backwards in time, which is what the backward pass evaluates.
    """

    @staticmethod
    def forward(ctx, x, b, a):
        from scipy.signal import lfilter as _lf

        ctx.b, ctx.a = b, a
        arr = x.detach().cpu().numpy()
        out = _lf(b.astype(arr.dtype), a.astype(arr.dtype), arr, axis=-1)
        return torch.from_numpy(np.ascontiguousarray(out.astype(arr.dtype)))

    @staticmethod
    def backward(ctx, grad):
        from scipy.signal import lfilter as _lf

        arr = grad.detach().cpu().numpy()[..., ::-1]
        out = _lf(ctx.b.astype(arr.dtype), ctx.a.astype(arr.dtype), arr, axis=-1)
        out = np.ascontiguousarray(out[..., ::-1].astype(arr.dtype))
        return torch.from_numpy(out), None, None


def lfilter(x: torch.Tensor, b: np.ndarray, a: np.ndarray) -> torch.Tensor:
    """Causal IIR filter ``b/a`` with zero initial state, no output clamping
    (``loss.py:127-129`` and ``loss.py:167`` call it with ``clamp=False``)."""

    return _LFilter.apply(x, np.asarray(b, np.float64), np.asarray(a, np.float64))


# ---------------------------------------------------------------------------
# pipeline stages
# ---------------------------------------------------------------------------


def resample(x: torch.Tensor, kern: T.ResampleKernel) -> torch.Tensor:
    """Polyphase sinc resampling of ``[batch, n]`` (torchaudio's
    ``_apply_sinc_resample_kernel``: pad ``(width, width + orig_step)``, strided
    conv1d, interleave phases, cut to ``ceil(new * n / orig)`` in float32)."""

    batch, n = x.shape
    taps = torch.as_tensor(kern.taps, dtype=x.dtype)[:, None, :]
    padded = F.pad(x, (kern.width, kern.width + kern.orig_step))
    out = F.conv1d(padded[:, None], taps, stride=kern.orig_step)
    out = out.transpose(1, 2).reshape(batch, -1)
    return out[:, : T.resample_length(n, kern.orig_step, kern.new_step)]


def align_level(x: torch.Tensor, p: OracleParams) -> torch.Tensor:
    """``loss.py:111-141``: scale so the 325-3250 Hz band power reaches 1e7."""

    filtered = lfilter(x, p.pow_b, p.pow_a)
    power = (filtered**2).sum(dim=1, keepdim=True) / (filtered.shape[1] + T.ALIGN_PAD) / T.ALIGN_DIV
    return x * (T.ALIGN_TARGET / power).sqrt()


def preemphasize(x: torch.Tensor, p: OracleParams) -> torch.Tensor:
    """``loss.py:143-169``: fade 15 samples at either end, then the biquad.

    The two fades are applied one after the other, so for fewer than 30
    samples the overlap receives both weights.
    """

    emp = torch.arange(1, 16, dtype=x.dtype) / 16.0
    x = x.clone()
    x[:, :15] = x[:, :15] * emp
    x[:, -15:] = x[:, -15:] * torch.flip(emp, dims=(0,))
    return lfilter(x, p.pre_b, p.pre_a)


def stft_bark(x: torch.Tensor, p: OracleParams, chain_dtype) -> torch.Tensor:
    """``loss.py:190-203``: pad by ``N % 256``, power STFT (periodic Hann,
    ``center=False``), DC bin zeroed, binary Bark segment sums times the power
    density correction.  Returns ``[batch, frame, band]`` in ``chain_dtype``."""

    x = F.pad(x, (0, x.shape[1] % T.PAD_MODULUS))
    window = torch.as_tensor(p.window, dtype=x.dtype)
    spec = torch.stft(
        x,
        n_fft=p.n_fft,
        hop_length=p.hop_length,
        win_length=p.n_fft,
        window=window,
        center=False,
        normalized=False,
        return_complex=True,
    )
    spec = (spec.real**2 + spec.imag**2).swapaxes(1, 2)
    spec = torch.cat([torch.zeros_like(spec[:, :, :1]), spec[:, :, 1:]], dim=2)
    fbank = torch.as_tensor(p.fbank, dtype=x.dtype)
    bark = torch.einsum("ij,klj->kli", fbank, spec[:, :, :-1])
    return bark.to(chain_dtype) * torch.as_tensor(p.corr, dtype=chain_dtype)


def _total_audible(t: torch.Tensor, thr: torch.Tensor, factor: float) -> torch.Tensor:
    """``loudness.py:72-79``."""

    return (t * (t > thr * factor)).sum(dim=2)


def _loudness(x: torch.Tensor, thr: torch.Tensor, e: torch.Tensor) -> torch.Tensor:
    """Zwicker loudness, ``loudness.py:123-129``."""

    loud = (2.0 * thr) ** e * ((0.5 + 0.5 * x / thr) ** e - 1)
    loud = torch.where(x <= thr, torch.zeros_like(loud), loud)
    return loud * T.SL_16K


def _weighted_norm(t: torch.Tensor, w: torch.Tensor, total: float, p: float) -> torch.Tensor:
    """``bark.py:176-195``, band 0 excluded."""

    return total * (w * t / total ** (1 / p))[:, :, 1:].norm(p, dim=2)


def chain(ref: torch.Tensor, deg: torch.Tensor, p: OracleParams, census: dict = None) -> Tuple[torch.Tensor, torch.Tensor]:
    """Perceptual model from the Bark spectra to both distances,
    ``loss.py:205-268``.

    ``census``, when given a dict, receives per utterance the fraction of the
    values each clamp of the chain acts on (``band_ratio``: bands of the
    band power ratio outside [0.01, 100]; ``frame_ratio``: frames of the
    frame power ratio outside [3e-4, 5]; ``symm_45`` / ``asymm_45``: frames
    whose weighted disturbance exceeds 45) -- the regime of a test input.
    """

    dt = ref.dtype
    thr = torch.as_tensor(p.threshs, dtype=dt)
    e = torch.as_tensor(p.exps, dtype=dt)
    w = torch.as_tensor(p.width_bark, dtype=dt)
    total = torch.as_tensor(p.total_width, dtype=dt)

    silent = _total_audible(ref, thr, 1e2) < 1e7
    keep = (~silent).unsqueeze(2)
    mean_deg = (deg * ((deg > thr * 100.0) * keep)).mean(dim=1)
    mean_ref = (ref * ((ref > thr * 100.0) * keep)).mean(dim=1)

    band_ratio = ((mean_deg + 1000) / (mean_ref + 1000)).unsqueeze(1)
    if census is not None:
        census["band_ratio"] = ((band_ratio < 0.01) | (band_ratio > 100.0)).double().mean(dim=(1, 2))
    band_ratio = band_ratio.clamp(min=0.01, max=100.0)
    equ_ref = band_ratio * ref

    taer = _total_audible(equ_ref, thr, 1.0)
    frame_ratio = (taer + 5e3) / (_total_audible(deg, thr, 1.0) + 5e3)
    frame_ratio = torch.cat([frame_ratio[:, :1], frame_ratio[:, 1:] * 0.8 + frame_ratio[:, :-1] * 0.2], dim=1)
    if census is not None:
        census["frame_ratio"] = ((frame_ratio < 3e-4) | (frame_ratio > 5.0)).double().mean(dim=1)
    frame_ratio = frame_ratio.clamp(min=3e-4, max=5.0)
    equ_deg = frame_ratio.unsqueeze(2) * deg

    deg_loud = _loudness(equ_deg, thr, e)
    ref_loud = _loudness(equ_ref, thr, e)

    deadzone = 0.25 * torch.min(deg_loud, ref_loud)
    dist = deg_loud - ref_loud
    dist = dist.sign() * (dist.abs() - deadzone).clamp(min=0)

    symm = _weighted_norm(dist, w, total, 2).clamp(min=1e-20)

    asym = ((equ_deg + 50.0) / (equ_ref + 50.0)) ** 1.2
    asym = torch.where(asym < 3.0, torch.zeros_like(asym), asym).clamp(max=12.0)
    asymm = _weighted_norm(dist * asym, w, total, 1).clamp(min=1e-20)

    h = ((taer + 1e5) / 1e7) ** 0.04
    if census is not None:
        census["symm_45"] = (symm / h > 45.0).double().mean(dim=1)
        census["asymm_45"] = (asymm / h > 45.0).double().mean(dim=1)
    symm = (symm / h).clamp(max=45.0)
    asymm = (asymm / h).clamp(max=45.0)

    def pool(s):
        win = s.unfold(1, T.PSQM_WINDOW, T.PSQM_STRIDE)  # [batch, windows, 20]
        psqm = (win**6).mean(dim=2) ** (1.0 / 6)
        return psqm.square().mean(dim=1).sqrt()

    return pool(symm), pool(asymm)


def raw(ref: torch.Tensor, deg: torch.Tensor, p: OracleParams, mode: str = "float64", census: dict = None):
    """Symmetric and asymmetric distance, ``loss.py:172-268``.

    ``mode`` is ``"float64"`` (ground truth) or ``"reference"`` (the dtype
    behaviour of ``PesqLoss`` on float32 input); ``census``: see ``chain``.
    """

    if mode == "float64":
        sig_dtype, chain_dtype = torch.float64, torch.float64
    elif mode == "reference":
        sig_dtype, chain_dtype = torch.float32, torch.float64
    else:
        raise ValueError(f"unknown mode {mode!r}")

    ref = torch.atleast_2d(ref).to(sig_dtype)
    deg = torch.atleast_2d(deg).to(sig_dtype)

    peak = torch.max(deg.abs().amax(1, keepdim=True), ref.abs().amax(1, keepdim=True))
    ref, deg = ref / peak, deg / peak

    if p.kernel is not None:
        ref, deg = resample(ref, p.kernel), resample(deg, p.kernel)

    ref, deg = align_level(ref, p), align_level(deg, p)
    ref, deg = preemphasize(ref, p), preemphasize(deg, p)

    ref_bark = stft_bark(ref, p, chain_dtype)
    deg_bark = stft_bark(deg, p, chain_dtype)
    return chain(ref_bark, deg_bark, p, census)


def epilogue(d_symm, d_asymm, factor):
    """MOS compression and loss, ``loss.py:289-297`` and ``loss.py:320-322``."""

    mos_in = 4.5 - 0.1 * d_symm - 0.0309 * d_asymm
    mos = 0.999 + 4 / (1 + torch.exp(-1.3669 * mos_in + 3.8224))
    loss = factor * (0.1 * d_symm + 0.0309 * d_asymm)
    return mos, loss


def forward(ref, deg, p: OracleParams, mode: str = "float64"):
    """``PesqLoss.forward``: ``factor * (0.1 d_symm + 0.0309 d_asymm)``."""

    return epilogue(*raw(ref, deg, p, mode), p.factor)[1]


def mos(ref, deg, p: OracleParams, mode: str = "float64"):
    """``PesqLoss.mos``."""

    return epilogue(*raw(ref, deg, p, mode), p.factor)[0]
