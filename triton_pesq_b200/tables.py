"""Host-side constants and precomputed device tables of the PESQ engine.

Everything in here runs once, on the CPU, in float64, when a
:class:`~triton_pesq_b200.loss.PesqLossCuda` (or one of the standalone ops) is
constructed.  The CUDA kernels only ever see the float32 roundings of these
tables, handed over through the C-ABI ``pesq_plan_create``.

Contents

* the ITU-T P.862 band and loudness tables at 16 kHz, identical in value to
  ``torch_pesq/bark.py:11-78`` and ``torch_pesq/loudness.py:11-25`` of the
  reference (they are the standard's data, not a design choice);
* the reference's parameter derivations on top of them -- band interpolation
  (``bark.py:81-99``), the binary Bark filterbank (``bark.py:147-173``), the
  hearing thresholds and loudness exponents (``loudness.py:52-55``), the
  level-alignment band pass (``loss.py:96-99``) and the pre-emphasis biquad
  (``loss.py:102-108``), both rounded to float32 exactly like the reference's
  ``Parameter(dtype=float32)``;
* a restatement of torchaudio 2.x ``_get_sinc_resample_kernel`` (the
  ``Resample(sample_rate, 16000)`` of ``loss.py:76``), reproducing its dtype
  promotions so that the float32 taps come out identical;
* the constant tables of the chunked IIR scan used by the kernels, see
  :class:`ScanTables`.
"""

from __future__ import annotations

import math
from dataclasses import dataclass, field
from typing import List, Optional, Tuple

import numpy as np
import torch

# ---------------------------------------------------------------------------
# ITU-T P.862 tables, 16 kHz (values as in torch_pesq/bark.py:11-76 and
# torch_pesq/loudness.py:11-21)
# ---------------------------------------------------------------------------

HZ_BINS_PER_BAND = np.array([
    1, 1, 1, 1, 1, 1, 1, 1, 2, 1, 1, 1, 1, 1, 2, 1, 1, 2, 2, 2, 2, 2, 2, 2, 2,
    3, 3, 3, 3, 4, 3, 4, 5, 4, 5, 6, 6, 7, 8, 9, 9, 12, 12, 15, 16, 18, 21, 25, 20,
])
BAND_CENTRE_BARK = np.array([
    0.078672, 0.316341, 0.636559, 0.961246, 1.29045, 1.624217, 1.962597,
    2.305636, 2.653383, 3.005889, 3.363201, 3.725371, 4.092449, 4.464486,
    4.841533, 5.223642, 5.610866, 6.003256, 6.400869, 6.803755, 7.211971,
    7.625571, 8.044611, 8.469146, 8.899232, 9.334927, 9.776288, 10.223374,
    10.676242, 11.134952, 11.599563, 12.070135, 12.546731, 13.029408, 13.518232,
    14.013264, 14.514566, 15.022202, 15.536238, 16.056736, 16.583761, 17.117382,
    17.657663, 18.204674, 18.758478, 19.319147, 19.886751, 20.461355, 21.043034,
])
BAND_CENTRE_HZ = np.array([
    7.867213, 31.634144, 63.655895, 96.124611, 129.044968, 162.421738, 196.259659,
    230.563568, 265.338348, 300.588867, 336.320129, 372.53714, 409.244934, 446.448578,
    484.568604, 526.600586, 570.303833, 619.42334, 672.121643, 728.525696, 785.675964,
    846.835693, 909.69165, 977.063293, 1049.861694, 1129.635986, 1217.257568, 1312.109497,
    1412.501465, 1517.99939, 1628.894165, 1746.194336, 1871.568848, 2008.776123, 2158.979248,
    2326.743164, 2513.787109, 2722.48877, 2952.58667, 3205.835449, 3492.679932, 3820.219238,
    4193.938477, 4619.846191, 5100.437012, 5636.199219, 6234.313477, 6946.734863, 7796.473633,
])
BAND_WIDTH_BARK = np.array([
    0.157344, 0.317994, 0.322441, 0.326934, 0.331474, 0.336061, 0.340697,
    0.345381, 0.350114, 0.354897, 0.359729, 0.364611, 0.369544, 0.374529,
    0.379565, 0.384653, 0.389794, 0.394989, 0.400236, 0.405538, 0.410894,
    0.416306, 0.421773, 0.427297, 0.432877, 0.438514, 0.444209, 0.449962,
    0.455774, 0.461645, 0.467577, 0.473569, 0.479621, 0.485736, 0.491912,
    0.498151, 0.504454, 0.510819, 0.51725, 0.523745, 0.530308, 0.536934,
    0.543629, 0.55039, 0.55722, 0.564119, 0.571085, 0.578125, 0.585232,
])
BAND_WIDTH_HZ = np.array([
    15.734426, 31.799433, 32.244064, 32.693359, 33.147385, 33.60614, 34.069702,
    34.538116, 35.011429, 35.489655, 35.97287, 36.461121, 36.954407, 37.452911,
    40.269653, 42.311859, 45.992554, 51.348511, 55.040527, 56.775208, 58.699402,
    62.445862, 64.820923, 69.195374, 76.745667, 84.016235, 90.825684, 97.931152,
    103.348877, 107.80188, 113.552246, 121.490601, 130.42041, 143.431763, 158.486816,
    176.872803, 198.314697, 219.549561, 240.600098, 268.702393, 306.060059, 349.937012,
    398.686279, 454.713867, 506.841797, 564.86377, 637.26123, 794.717285, 931.068359,
])
POW_DENS_CORRECTION = np.array([
    100.0, 99.999992, 100.0, 100.000008, 100.000008, 100.000015, 99.999992,
    99.999969, 50.000027, 100.0, 99.999969, 100.000015, 99.999947, 100.000061,
    53.047077, 110.000046, 117.991989, 65.0, 68.760147, 69.999931, 71.428818,
    75.000038, 76.843384, 80.968781, 88.646126, 63.864388, 68.15535, 72.547775,
    75.584831, 58.379192, 80.950836, 64.135651, 54.384785, 73.821884, 64.437073,
    59.176456, 65.521278, 61.399822, 58.144047, 57.004543, 64.126297, 54.311001,
    61.114979, 55.077751, 56.849335, 55.628868, 53.137054, 54.985844, 79.546974,
])
ABS_THRESH_POWER = np.array([
    51286152.0, 2454709.5, 70794.59375, 4897.788574, 1174.897705, 389.045166, 104.71286,
    45.70882, 17.782795, 9.772372, 4.897789, 3.090296, 1.905461, 1.258925,
    0.977237, 0.724436, 0.562341, 0.457088, 0.389045, 0.331131, 0.295121,
    0.269153, 0.25704, 0.251189, 0.251189, 0.251189, 0.251189, 0.263027,
    0.288403, 0.30903, 0.338844, 0.371535, 0.398107, 0.436516, 0.467735,
    0.489779, 0.501187, 0.501187, 0.512861, 0.524807, 0.524807, 0.524807,
    0.512861, 0.47863, 0.42658, 0.371535, 0.363078, 0.416869, 0.537032,
])

#: Power density scaling of the 16 kHz filterbank (``bark.py:78``).
SP_16K = 6.910853e-006
#: Zwicker exponent (``loudness.py:24``).
ZWICKER_POWER = 0.23
#: Loudness calibration (``loudness.py:25``).
SL_16K = 1.866055e-001

#: Level alignment target and the two "reference implementation" constants of
#: ``loss.py:132-139``: ``power = sum(f^2) / (N + 5120) / 1.04684``.
ALIGN_TARGET = 1e7
ALIGN_PAD = 5120
ALIGN_DIV = 1.04684

#: Pre-emphasis biquad, ``loss.py:102-108`` (rounded to float32 on use).
PRE_FILTER_B = (2.740826, -5.4816519, 2.740826)
PRE_FILTER_A = (1.0, -1.9444777, 0.94597794)

#: The frames are laid out after padding by ``length % PAD_MODULUS`` zeros
#: (``loss.py:191-192``); the modulus is fixed, independent of the hop.
PAD_MODULUS = 256
#: Frame lengths (n_fft) the CUDA kernels implement: powers of two in this
#: range (512 runs the fused default path, the others the spectrum kernels).
MIN_FFT = 32
MAX_FFT = 4096

#: Overlapping sums of the disturbance, 20 frames with stride 10 (``loss.py:258-266``).
PSQM_WINDOW = 20
PSQM_STRIDE = 10


def as_f32(values) -> np.ndarray:
    """Round to float32 and widen back, i.e. the value a float32 Parameter holds."""

    return np.asarray(values, dtype=np.float64).astype(np.float32).astype(np.float64)


# ---------------------------------------------------------------------------
# band and loudness parametrisation
# ---------------------------------------------------------------------------


def interp_bands(values, nelms_new: int) -> np.ndarray:
    """Linear interpolation of a 49-band table onto ``nelms_new`` bands.

    Same sampling grid as ``bark.py:81-99``: the new band ``i`` sits at
    ``49 * i / nelms_new`` on the old index axis.  For ``nelms_new = 49`` this
    is the identity; beyond 49 bands the grid leaves the table and, like the
    reference, the call fails.
    """

    values = np.asarray(values, dtype=np.float64)
    nelms = values.shape[0]
    grid = np.linspace(0, 49.0, nelms_new, endpoint=False)
    if grid.size and (grid.max() > nelms - 1 or grid.min() < 0):
        raise ValueError(
            f"cannot interpolate a {nelms}-band table onto {nelms_new} bands"
        )
    return np.interp(grid, np.arange(nelms, dtype=np.float64), values)


@dataclass
class BarkLayout:
    """Binary, contiguous Bark filterbank and its per-band constants.

    ``starts[i]``/``ends[i]`` is the half open bin range of band ``i`` over the
    ``nfreqs`` lowest bins (the Nyquist bin is never used, ``bark.py:214``).
    """

    nfreqs: int
    nbarks: int
    starts: np.ndarray
    ends: np.ndarray
    pow_dens_correction: np.ndarray  # float64, includes SP_16K
    width_bark: np.ndarray  # float64
    width_hz: np.ndarray
    centre_hz: np.ndarray
    total_width: float  # sum of width_bark[1:], float64

    def fbank(self) -> np.ndarray:
        """Dense ``[nbarks, nfreqs]`` 0/1 matrix (float32 values)."""

        mat = np.zeros((self.nbarks, self.nfreqs), dtype=np.float32)
        for band in range(self.nbarks):
            mat[band, self.starts[band] : self.ends[band]] = 1.0
        return mat


def bark_layout(nfreqs: int = 256, nbarks: int = 49) -> BarkLayout:
    """Filterbank of ``BarkScale(nfreqs, nbarks)``, ``bark.py:131-173``."""

    corr = interp_bands(POW_DENS_CORRECTION, nbarks) * SP_16K
    width_hz = interp_bands(BAND_WIDTH_HZ, nbarks)
    width_bark = interp_bands(BAND_WIDTH_BARK, nbarks)
    centre = interp_bands(BAND_CENTRE_HZ, nbarks)

    starts = np.zeros(nbarks, dtype=np.int64)
    ends = np.zeros(nbarks, dtype=np.int64)

    if nfreqs == 256 and nbarks == 49:
        edges = np.concatenate([[0], np.cumsum(HZ_BINS_PER_BAND)])
        starts[:] = edges[:-1]
        ends[:] = edges[1:]
    else:
        # every band spans [centre - width/2, centre + width/2) in bins, clipped
        # so that it starts no earlier than where the previous band ended
        prev, bin_width = 0, 8000.0 / nfreqs
        for band in range(nbarks):
            stride = width_hz[band] / bin_width
            centre_bin = centre[band] / bin_width
            lo = max(prev, int(math.floor(centre_bin - stride / 2)))
            hi = min(nfreqs, int(math.ceil(centre_bin + stride / 2)))
            # an empty range (hi <= lo) covers no bin; keep it as [lo, lo)
            starts[band], ends[band] = lo, max(lo, hi)
            prev = hi

    return BarkLayout(
        nfreqs=nfreqs,
        nbarks=nbarks,
        starts=starts,
        ends=ends,
        pow_dens_correction=corr,
        width_bark=width_bark,
        width_hz=width_hz,
        centre_hz=centre,
        total_width=float(width_bark[1:].sum()),
    )


def hearing_thresholds(nbarks: int = 49) -> np.ndarray:
    """Absolute hearing threshold per band (float64), ``loudness.py:52-55``."""

    return interp_bands(ABS_THRESH_POWER, nbarks)


def loudness_exponents() -> np.ndarray:
    """Zwicker exponent per band as the reference's float32 Parameter holds it.

    ``loudness.py:58-61`` evaluates ``(6 / (centre_bark + 2)).clamp(1, 2) ** 0.15
    * 0.23`` on a float32 torch tensor of the 49 tabulated band centres; the
    same torch float32 operations are used here so that every rounding,
    including the one of the power, is identical.
    """

    import torch

    centre = torch.tensor(BAND_CENTRE_BARK.tolist())
    exp = 6 / (centre + 2.0)
    exp = exp.clamp(min=1.0, max=2.0) ** 0.15 * ZWICKER_POWER
    return exp.numpy().astype(np.float64)


def power_filter() -> Tuple[np.ndarray, np.ndarray]:
    """Level-alignment band pass, ``loss.py:96-99``: 5th order Butterworth,
    325-3250 Hz at 16 kHz, stored as float32 coefficients."""

    from scipy.signal import butter

    b, a = butter(5, [325, 3250], fs=16000, btype="band")
    return as_f32(b), as_f32(a)


def pre_filter() -> Tuple[np.ndarray, np.ndarray]:
    """Pre-emphasis biquad, ``loss.py:102-108``, float32 coefficients."""

    return as_f32(PRE_FILTER_B), as_f32(PRE_FILTER_A)


def hann_window(length: int) -> np.ndarray:
    """Periodic Hann window exactly as ``torch.hann_window(length)`` (float32)."""

    import torch

    return torch.hann_window(length, dtype=torch.float32).numpy().astype(np.float64)


def centred_window(win_length: int, n_fft: int) -> np.ndarray:
    """Window zero-padded to ``n_fft`` taps and centred, as ``torch.stft`` does."""

    full = np.zeros(n_fft, dtype=np.float64)
    left = (n_fft - win_length) // 2
    full[left : left + win_length] = hann_window(win_length)
    return full


def frame_count(n: int, n_fft: int = 512, hop: int = 256) -> int:
    """Frames of the padded signal, ``loss.py:191-196`` with ``center=False``."""

    padded = n + n % PAD_MODULUS
    if padded < n_fft:
        return 0
    return 1 + (padded - n_fft) // hop


def psqm_windows(nframes: int) -> int:
    """Number of 20-frame, stride-10 windows of the overlapping sums."""

    if nframes < PSQM_WINDOW:
        return 0
    return (nframes - PSQM_WINDOW) // PSQM_STRIDE + 1


# ---------------------------------------------------------------------------
# sinc resampler (restatement of torchaudio's published kernel design)
# ---------------------------------------------------------------------------


@dataclass
class ResampleKernel:
    """Polyphase sinc kernel of ``torchaudio.transforms.Resample(orig, new)``.

    ``taps[j, k]`` (float32 values) weighs ``x[l * orig_step + k - width]`` for
    output ``l * new_step + j``.  ``first[j]``/``count[j]`` give the nonzero tap
    range of phase ``j``; every other tap rounds to exactly ``0.0f``.
    """

    orig_freq: int
    new_freq: int
    orig_step: int
    new_step: int
    width: int
    taps: np.ndarray  # [new_step, width_total]
    first: np.ndarray
    count: np.ndarray

    @property
    def width_total(self) -> int:
        return int(self.taps.shape[1])


RESAMPLING_METHODS = ("sinc_interp_hann", "sinc_interp_kaiser")
#: default Kaiser window shape of torchaudio's resampler
KAISER_BETA = 14.769656459379492


def sinc_resample_kernel(
    orig_freq: int,
    new_freq: int,
    lowpass_filter_width: int = 6,
    rolloff: float = 0.99,
    resampling_method: str = "sinc_interp_hann",
    beta: Optional[float] = None,
) -> ResampleKernel:
    """Windowed sinc polyphase kernel, float32 taps.

    Restates the published algorithm of torchaudio 2.x
    ``torchaudio.functional.functional._get_sinc_resample_kernel`` (methods
    ``sinc_interp_hann`` and ``sinc_interp_kaiser``), which ``loss.py:76`` uses
    through ``torchaudio.transforms.Resample`` and the reference's
    ``TritonResample`` (``triton_ops/resample.py:442-528``) designs its filter
    bank with.  The phase offsets ``-j / new_step`` are formed in float32 and
    everything after that in float64; the Kaiser window divides by ``i0`` of
    the float32 shape parameter evaluated in float32 -- the dtype promotions of
    that implementation, so the float32 taps agree bit for bit.
    """

    if orig_freq <= 0 or new_freq <= 0:
        raise ValueError("Original and desired frequency have to be positive.")
    if int(orig_freq) != orig_freq or int(new_freq) != new_freq:
        raise ValueError("Frequencies must be integers.")
    if lowpass_filter_width <= 0:
        raise ValueError("Low pass filter width should be positive.")
    if resampling_method not in RESAMPLING_METHODS:
        raise ValueError("Invalid resampling method: {}".format(resampling_method))

    gcd = math.gcd(int(orig_freq), int(new_freq))
    orig = int(orig_freq) // gcd
    new = int(new_freq) // gcd

    base = min(orig, new) * rolloff
    width = math.ceil(lowpass_filter_width * orig / base)

    idx = np.arange(-width, width + orig, dtype=np.float64)[None, :] / orig
    phase = (
        np.arange(0, -new, -1).astype(np.float32) / np.float32(new)
    ).astype(np.float64)[:, None]
    t = (phase + idx) * base
    t = np.clip(t, -lowpass_filter_width, lowpass_filter_width)
    if resampling_method == "sinc_interp_hann":
        window = np.cos(t * math.pi / lowpass_filter_width / 2) ** 2
    else:
        shape = torch.tensor(float(KAISER_BETA if beta is None else beta))  # float32, as torchaudio
        tt = torch.from_numpy(t)
        window = (torch.i0(shape * torch.sqrt(1 - (tt / lowpass_filter_width) ** 2)) / torch.i0(shape)).numpy()
    t = t * math.pi
    scale = base / orig
    with np.errstate(invalid="ignore", divide="ignore"):
        sinc = np.where(t == 0, 1.0, np.sin(t) / t)
    taps = (sinc * (window * scale)).astype(np.float32)

    first = np.zeros(new, dtype=np.int64)
    count = np.zeros(new, dtype=np.int64)
    for j in range(new):
        nz = np.flatnonzero(taps[j] != 0.0)
        if nz.size:
            first[j], count[j] = nz[0], nz[-1] + 1 - nz[0]

    return ResampleKernel(
        orig_freq=int(orig_freq),
        new_freq=int(new_freq),
        orig_step=orig,
        new_step=new,
        width=width,
        taps=taps.astype(np.float64),
        first=first,
        count=count,
    )


def resample_length(n: int, orig_step: int, new_step: int) -> int:
    """Output length of the resampler: ``ceil(new * n / orig)`` evaluated on a
    float32 scalar, as torchaudio's ``torch.ceil(torch.as_tensor(...))`` does."""

    return int(math.ceil(float(np.float32(new_step * n / orig_step))))


# ---------------------------------------------------------------------------
# chunked IIR scan tables
# ---------------------------------------------------------------------------

#: Samples per thread chunk.  33 is coprime with the 32 shared memory banks,
#: so the strided per-thread reads of a linearly staged segment never conflict.
SCAN_CHUNK = 33

#: Chunks of look-back the in-CTA Kogge-Stone scan covers (five doubling
#: levels); the state of any sample depends on the ``SCAN_CHUNK * SCAN_HORIZON``
#: samples before it up to the truncation bound checked in :class:`ScanTables`.
SCAN_LEVELS = 5
SCAN_HORIZON = 1 << SCAN_LEVELS

#: Largest tolerated norm of the dropped state transition ``A^(chunk*horizon)``.
SCAN_TRUNCATION = 1e-11


def _sections(b: np.ndarray, a: np.ndarray) -> np.ndarray:
    """Second order sections (float64) of a transfer function."""

    from scipy.signal import tf2sos

    b = np.atleast_1d(np.asarray(b, dtype=np.float64))
    a = np.atleast_1d(np.asarray(a, dtype=np.float64))
    if a[0] == 0.0:
        raise ValueError("The leading denominator coefficient a[0] must not be zero.")
    if max(b.size, a.size) < 2:
        raise ValueError("The IIR filter needs at least one pole.")
    if max(b.size, a.size) == 2:
        # a first order filter: scipy pads it into a single section itself,
        # keep the call uniform
        pass
    return np.asarray(tf2sos(b, a), dtype=np.float64)


def _section_realisation(sec: np.ndarray):
    """2-state realisation of one section with a well conditioned transition.

    Complex pole pairs become a rotation-scaling block ``[[re, -im], [im, re]]``
    (its powers have norm ``|p|^t``), real poles a diagonal block.  The input
    and read-out vectors are balanced to equal norm.
    """

    b0, b1, b2, a0, a1, a2 = sec / sec[3]
    # strictly proper remainder (beta1 z + beta2) / (z^2 + a1 z + a2)
    beta1 = b1 - a1 * b0
    beta2 = b2 - a2 * b0
    disc = a1 * a1 / 4.0 - a2

    if disc < 0.0:
        re, im = -a1 / 2.0, math.sqrt(-disc)
        trans = np.array([[re, -im], [im, re]])
        # read-out (1, 0): C (zI - A)^-1 g = ((z - re) g1 - im g2) / det
        g1 = beta1
        g2 = -(beta2 + re * g1) / im
        drive = np.array([g1, g2])
        read = np.array([1.0, 0.0])
    else:
        root = math.sqrt(disc)
        p1, p2 = -a1 / 2.0 + root, -a1 / 2.0 - root
        trans = np.diag([p1, p2])
        if p1 != p2:
            r1 = (beta1 * p1 + beta2) / (p1 - p2)
            r2 = (beta1 * p2 + beta2) / (p2 - p1)
            drive = np.array([1.0, 1.0])
            read = np.array([r1, r2])
        else:
            # repeated real pole: a Jordan block
            trans = np.array([[p1, 1.0], [0.0, p1]])
            # C (zI-A)^-1 B with B = (0, 1): (c1 + c2 (z - p)) / (z - p)^2
            drive = np.array([0.0, 1.0])
            read = np.array([beta1 * p1 + beta2, beta1])

    # balance: scale the state so that |drive| == |read|
    nd, nr = np.linalg.norm(drive), np.linalg.norm(read)
    if nd > 0.0 and nr > 0.0:
        alpha = math.sqrt(nr / nd)
        drive = drive * alpha
        read = read / alpha

    return trans, drive, read, float(b0)


def state_space(b, a):
    """Series connection of balanced second order sections.

    Returns ``(A, B, C, D)`` of ``s[n+1] = A s[n] + B x[n]``,
    ``y[n] = C s[n] + D x[n]``.  ``A`` is block lower triangular with the
    section blocks on its diagonal.
    """

    secs = _sections(b, a)
    parts = [_section_realisation(s) for s in secs]
    count = len(parts)
    order = 2 * count

    trans = np.zeros((order, order))
    drive = np.zeros(order)
    read = np.zeros(order)
    feeds = [p[3] for p in parts]

    for k, (tk, dk, _, _) in enumerate(parts):
        rows = slice(2 * k, 2 * k + 2)
        trans[rows, rows] = tk
        # the input of section k is the output of section k-1, which reads
        # every earlier section through the feed-throughs in between
        for j in range(k):
            gain = float(np.prod(feeds[j + 1 : k]))
            trans[rows, 2 * j : 2 * j + 2] = np.outer(dk, parts[j][2]) * gain
        drive[rows] = dk * float(np.prod(feeds[:k]))
    for j in range(count):
        read[2 * j : 2 * j + 2] = parts[j][2] * float(np.prod(feeds[j + 1 :]))

    return trans, drive, read, float(np.prod(feeds))


def direct_impulse_response(b, a, taps: int) -> np.ndarray:
    """First ``taps`` samples of the impulse response from the difference
    equation itself (float64), the ground truth for the realisation."""

    b = np.asarray(b, dtype=np.float64)
    a = np.asarray(a, dtype=np.float64)
    size = max(b.size, a.size)
    num = np.pad(b, (0, size - b.size)) / a[0]
    den = np.pad(a, (0, size - a.size)) / a[0]
    out = np.zeros(taps)
    for n in range(taps):
        acc = num[n] if n < size else 0.0
        for lag in range(1, min(size, n + 1)):
            acc -= den[lag] * out[n - lag]
        out[n] = acc
    return out


@dataclass
class ScanTables:
    """Constants of the chunked scan for one LTI filter (float64 values).

    For a chunk of ``L`` samples that starts in state ``S``:

    * ``y[t] = sum_{k<=t} impulse[t-k] x[k] + carry[t] . S``  (output)
    * ``S_next = power[0] S + sum_k drive[k] x[k]``           (end state)

    and ``power[i] = A^(L * 2^i)`` are the Kogge-Stone doubling steps.
    """

    order: int
    states: int
    chunk: int
    levels: int
    impulse: np.ndarray  # [L]
    carry: np.ndarray  # [L, P]   C A^t
    drive: np.ndarray  # [L, P]   A^(L-1-k) B
    power: np.ndarray  # [levels, P, P]
    truncation: float  # || A^(L * 2^levels) ||_2
    fidelity: float  # realisation vs difference equation, relative
    trans: np.ndarray = field(default=None)  # A
    input: np.ndarray = field(default=None)  # B
    output: np.ndarray = field(default=None)  # C
    feed: float = 0.0  # D
    b: np.ndarray = field(default=None)
    a: np.ndarray = field(default=None)

    @classmethod
    def build(cls, b, a, chunk: int = SCAN_CHUNK, levels: int = SCAN_LEVELS,
              truncation_limit: Optional[float] = SCAN_TRUNCATION) -> "ScanTables":
        b = np.asarray(b, dtype=np.float64)
        a = np.asarray(a, dtype=np.float64)
        trans, drive, read, feed = state_space(b, a)
        order = max(b.size, a.size) - 1
        states = trans.shape[0]

        carry = np.zeros((chunk, states))
        power = np.eye(states)
        for t in range(chunk):
            carry[t] = read @ power
            power = trans @ power
        chunk_power = power  # A^L

        inject = np.zeros((chunk, states))
        acc = np.eye(states)
        for k in range(chunk - 1, -1, -1):
            inject[k] = acc @ drive
            acc = trans @ acc

        impulse = np.zeros(chunk)
        impulse[0] = feed
        impulse[1:] = carry[:-1] @ drive

        truth = direct_impulse_response(b, a, 4 * chunk)
        realised = np.zeros(4 * chunk)
        realised[0] = feed
        vec = drive.copy()
        for n in range(1, 4 * chunk):
            realised[n] = read @ vec
            vec = trans @ vec
        fidelity = float(np.abs(realised - truth).max() / max(np.abs(truth).max(), 1e-300))

        steps = np.zeros((levels, states, states))
        step = chunk_power
        for i in range(levels):
            steps[i] = step
            step = step @ step
        dropped = float(np.linalg.norm(step, 2))

        if truncation_limit is not None and not dropped <= truncation_limit:
            raise RuntimeError(
                f"The filter's state after {chunk << levels} samples still "
                f"carries {dropped:.3g} of its initial value (limit "
                f"{truncation_limit:.1g}); its poles are too close to the unit "
                "circle for the bounded look-back of the chunked scan."
            )
        if not fidelity < 1e-9:
            raise RuntimeError(
                f"The second order section realisation misses the filter's "
                f"impulse response by {fidelity:.3g} relative."
            )

        return cls(order=order, states=states, chunk=chunk, levels=levels,
                   impulse=impulse, carry=carry, drive=inject, power=steps,
                   truncation=dropped, fidelity=fidelity, trans=trans, input=drive,
                   output=read, feed=feed, b=b, a=a)


@dataclass
class PlanConfig:
    """Everything ``PesqLoss(factor, sample_rate, nbarks, win_length, n_fft,
    hop_length)`` derives from its arguments (``loss.py:61-108``), ready for
    ``pesq_plan_create``."""

    factor: float
    sample_rate: int
    nbarks: int
    win_length: int
    n_fft: int
    hop_length: int
    layout: BarkLayout
    thresholds: np.ndarray
    exponents: np.ndarray
    window: np.ndarray
    power_b: np.ndarray
    power_a: np.ndarray
    pre_b: np.ndarray
    pre_a: np.ndarray
    power_scan: ScanTables
    pre_scan: ScanTables
    kernel: Optional[ResampleKernel]
    loudness_sl: float = SL_16K

    @classmethod
    def build(cls, factor: float, sample_rate: int = 48000, nbarks: int = 49,
              win_length: int = 512, n_fft: int = 512, hop_length: int = 256) -> "PlanConfig":
        if nbarks != BAND_CENTRE_BARK.size:
            # loudness.py:58-61 builds one exponent per tabulated band regardless
            # of nbarks, so PesqLoss itself only evaluates with 49 bands
            raise ValueError(
                f"PesqLoss evaluates its loudness model with 49 bands only, got nbarks={nbarks}."
            )
        n_fft, hop_length, win_length = int(n_fft), int(hop_length), int(win_length)
        if n_fft < MIN_FFT or n_fft & (n_fft - 1):
            # the reference's spectral op rejects these too (spectral.py, test_triton_spectral.py:237-255)
            raise ValueError(f"n_fft ({n_fft}) must be a power of two of at least {MIN_FFT}.")
        if n_fft > MAX_FFT:
            raise ValueError(f"n_fft ({n_fft}): the CUDA kernels implement frames of up to {MAX_FFT} samples.")
        if hop_length < 1:
            raise ValueError(f"hop_length ({hop_length}) must be positive.")
        if not 1 <= win_length <= n_fft:
            raise ValueError(f"win_length ({win_length}) must be in [1, n_fft ({n_fft})].")
        layout = bark_layout(n_fft // 2, nbarks)
        power_b, power_a = power_filter()
        pre_b, pre_a = pre_filter()
        return cls(
            factor=float(factor), sample_rate=int(sample_rate), nbarks=nbarks,
            win_length=win_length, n_fft=n_fft, hop_length=hop_length,
            layout=layout, thresholds=hearing_thresholds(nbarks),
            exponents=loudness_exponents(), window=centred_window(win_length, n_fft),
            power_b=power_b, power_a=power_a, pre_b=pre_b, pre_a=pre_a,
            power_scan=ScanTables.build(power_b, power_a),
            pre_scan=ScanTables.build(pre_b, pre_a),
            kernel=None if sample_rate == 16000 else sinc_resample_kernel(sample_rate, 16000),
        )
