"""The perceptual model's constant-holding submodules of ``PesqLoss``.

``PesqLossTriton`` inherits from ``PesqLoss`` the submodules that hold the
model's constants -- ``fbank`` (``BarkScale``, torch_pesq/bark.py:100-215),
``loudness`` (``Loudness``, torch_pesq/loudness.py:28-129) and ``to_spec``
(torchaudio's ``Spectrogram``, torch_pesq/loss.py:79-87) -- and user code
reads their tensors (``loss.fbank.fbank``, ``loss.loudness.threshs``, ...) or
calls them on spectrograms of its own.  ``PesqLossCuda`` carries the same
three submodules with the same attributes, dtypes and methods.

The loss itself never calls them: its CUDA kernels evaluate the spectrum,
the Bark sums and the loudness model fused (the constants reach the kernels
through the plan).  Their ``forward`` methods are the reference's tensor
expressions, evaluated by torch on whatever device the caller's tensors live
on, for callers that use them directly as the reference's users do.
"""

from __future__ import annotations

import torch
from torch.nn import Parameter

from . import tables as T

__all__ = ["BarkScale", "Loudness", "PowerSpectrogram"]


class BarkScale(torch.nn.Module):
    """Bark filterbank of P.862 (``BarkScale(nfreqs, nbarks)``, bark.py:100-173).

    Attributes (as the reference's, float64 unless noted): ``pow_dens_correction``,
    ``width_hz``, ``width_bark``, ``centre``, ``fbank`` (float32 0/1 matrix
    ``[nbarks, nfreqs]``) and ``total_width`` (0-d, the width of bands 1..).
    """

    def __init__(self, nfreqs: int = 256, nbarks: int = 49):
        super().__init__()
        lay = T.bark_layout(nfreqs, nbarks)
        self.pow_dens_correction = Parameter(torch.tensor(lay.pow_dens_correction), requires_grad=False)
        self.width_hz = Parameter(torch.tensor(lay.width_hz), requires_grad=False)
        self.width_bark = Parameter(torch.tensor(lay.width_bark), requires_grad=False)
        self.centre = Parameter(torch.tensor(lay.centre_hz), requires_grad=False)
        self.fbank = Parameter(torch.from_numpy(lay.fbank()), requires_grad=False)
        self.total_width = self.width_bark[1:].sum()

    def weighted_norm(self, tensor: torch.Tensor, p: float = 2) -> torch.Tensor:
        """``[batch, frame, band]`` -> ``[batch, frame]``: the p-norm over bands
        1.. weighted by the band widths (bark.py:176-195)."""

        total = self.total_width.to(self.width_bark.device)
        return total * (self.width_bark * tensor / total ** (1 / p))[:, :, 1:].norm(p, dim=2)

    def forward(self, tensor: torch.Tensor) -> torch.Tensor:
        """Power spectrogram ``[batch, frame, nfreqs + 1]`` -> Bark spectrogram
        ``[batch, frame, nbarks]`` (the Nyquist bin is dropped, bark.py:198-215)."""

        bark = torch.einsum("ij,klj->kli", self.fbank, tensor[:, :, :-1])
        return bark * self.pow_dens_correction


class Loudness(torch.nn.Module):
    """Zwicker loudness of the Bark spectrogram (``Loudness(nbark)``, loudness.py:28-129).

    Attributes: ``threshs`` (float64 ``[1, 1, nbark]``, the hearing threshold
    per band) and ``exp`` (float32 ``[49]``, the Zwicker exponent per band).
    """

    def __init__(self, nbark: int = 49):
        super().__init__()
        self.threshs = Parameter(torch.tensor(T.hearing_thresholds(nbark))[None, None, :], requires_grad=False)
        self.exp = Parameter(torch.tensor(T.loudness_exponents(), dtype=torch.float32), requires_grad=False)

    def total_audible(self, tensor: torch.Tensor, factor: float = 1.0) -> torch.Tensor:
        """Energy above ``factor`` times the threshold, summed over bands (loudness.py:58-79)."""

        return (tensor * (tensor > self.threshs * factor)).sum(dim=2)

    def time_avg_audible(self, tensor: torch.Tensor, silent: torch.Tensor) -> torch.Tensor:
        """Mean over frames of the energy above 100 times the threshold in the
        non-silent frames (loudness.py:81-105)."""

        mask = (tensor > self.threshs * 100.0) * (~silent.unsqueeze(2))
        return (tensor * mask).mean(dim=1)

    def forward(self, pow_dens: torch.Tensor) -> torch.Tensor:
        """Loudness per band, zero at or below the threshold (loudness.py:107-129)."""

        loud = (2.0 * self.threshs) ** self.exp * ((0.5 + 0.5 * pow_dens / self.threshs) ** self.exp - 1)
        loud = torch.where(pow_dens <= self.threshs, torch.zeros_like(loud), loud)
        return loud * T.SL_16K


class PowerSpectrogram(torch.nn.Module):
    """Power spectrogram of ``PesqLoss.to_spec`` (loss.py:79-87): periodic Hann
    window of ``win_length`` samples centred in ``n_fft``, hop ``hop_length``,
    no centring padding, not normalised, power 2.  ``[..., sample]`` ->
    ``[..., n_fft // 2 + 1, frame]`` as torchaudio's ``Spectrogram``."""

    def __init__(self, win_length: int = 512, n_fft: int = 512, hop_length: int = 256):
        super().__init__()
        self.n_fft = int(n_fft)
        self.win_length = int(win_length)
        self.hop_length = int(hop_length)
        self.power = 2.0
        self.register_buffer("window", torch.tensor(T.hann_window(win_length), dtype=torch.float32))

    def forward(self, waveform: torch.Tensor) -> torch.Tensor:
        shape = waveform.shape
        flat = waveform.reshape(-1, shape[-1])
        spec = torch.stft(flat, n_fft=self.n_fft, hop_length=self.hop_length, win_length=self.win_length,
                          window=self.window.to(flat.dtype), center=False, normalized=False, onesided=True,
                          return_complex=True)
        power = spec.real**2 + spec.imag**2
        return power.reshape(shape[:-1] + power.shape[-2:])


def edge_ramp(signal: torch.Tensor) -> torch.Tensor:
    """The 15-sample fades of the pre-emphasis (loss.py:163-165): the first 15
    samples times k/16 (k = 1..15), then the last 15 times the reversed ramp,
    one product after the other as the reference's two in-place products
    (rows shorter than 30 samples get both in the overlap).  Returns a new
    tensor."""

    out = signal.clone()
    emp = torch.arange(1, 16, device=signal.device, dtype=signal.dtype) / 16.0
    out[..., :15] = out[..., :15] * emp[: out.shape[-1]]
    out[..., -15:] = out[..., -15:] * torch.flip(emp, dims=(0,))[-min(15, out.shape[-1]):]
    return out
