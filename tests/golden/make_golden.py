"""Generate the golden fixtures from the reference implementation itself.

Runs only where the reference checkout is present: it imports ``torch_pesq``
from the directory named by the ``REFERENCE_ROOT`` environment variable (the
root of a LarocheC/triton-pesq checkout).  The ``.npz`` files it writes are
committed so that the tests never need the reference at run time.

Two shims make the reference importable with this image's packages:
``torchtyping`` is absent (``TensorType[...]`` is replaced by ``torch.Tensor``)
and the installed typeguard 4.x cannot evaluate the reference's string
dimensions, so ``typeguard.typechecked`` is replaced by the identity.  Neither
changes any computation.

Per case the fixture holds the float32 inputs and

* ``ref32_*``: ``PesqLoss.raw/mos/forward`` and the gradients of
  ``forward(...).sum()`` w.r.t. both inputs, as the reference computes them on
  the CPU (float32 signal path, float64 chain);
* ``f64_*``: ``ref_pipeline`` on ``copy.deepcopy(model).double()`` with float64
  inputs -- the float64 evaluation of the same pipeline -- and its gradients.

``constants.npz`` holds the reference's constant tensors (filterbank,
thresholds, exponents, correction, widths, window, filter coefficients and the
resampling kernels of several rates).

Signals (all seeded): ``speech`` -- a voiced harmonic stack with a broadband
term plus white noise, the regime the loss is used in; ``harmonic`` -- the
harmonic stack alone plus white noise, which pins the asymmetric distance to
its 45.0 clamp in every frame (the saturated regime the reference's own test
signals are built to avoid, ``tests/test_triton_loss.py:60-76``);
``dropout`` -- speech with a 150 ms dropout and a 50 ms burst 18 dB louder in
the degraded signal, which drives the frame power ratio into both of its
clamps; ``fir`` -- speech through a seeded random 64-tap low pass FIR
(4 kHz) plus white noise, the degradation of the 44.1 kHz workload.  ``snr``
may be one value per row.

Usage: ``REFERENCE_ROOT=<checkout> python tests/golden/make_golden.py [case ...]``
from the repository root (all cases and the constants when no case is named).
"""

import copy
import os
import sys
import types

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
def _import_reference():
    root = os.environ.get("REFERENCE_ROOT")
    if not root or not os.path.isdir(os.path.join(root, "torch_pesq")):
        raise SystemExit("set REFERENCE_ROOT to the root of a LarocheC/triton-pesq checkout")
    shim = types.ModuleType("torchtyping")

    class _TensorType:
        def __class_getitem__(cls, item):
            return torch.Tensor

    shim.TensorType = _TensorType
    sys.modules["torchtyping"] = shim
    import typeguard

    typeguard.typechecked = lambda fn: fn
    sys.path.insert(0, root)
    from torch_pesq import PesqLoss
    from torch_pesq.triton_ops.reference import ref_pipeline

    return PesqLoss, ref_pipeline


def speech_pair(batch, n, sr, seed, snr_db, broadband=True):
    """Seeded speech-like reference and a noisy degraded copy (float32);
    ``broadband=False`` leaves out the broadband term (the harmonic stack
    alone)."""

    rng = np.random.default_rng(seed)
    t = np.arange(n) / sr
    ref = np.zeros((batch, n))
    for b in range(batch):
        f0 = rng.uniform(90, 250)
        sig = sum(
            np.sin(2 * np.pi * f0 * k * t + rng.uniform(0, 2 * np.pi)) / k
            for k in range(1, 31)
            if f0 * k < sr / 2
        )
        sig = sig * 0.5 * (1 + np.sin(2 * np.pi * 4 * t))
        if broadband:
            sig = sig + 0.3 * rng.standard_normal(n) * 0.5 * (1 + np.sin(2 * np.pi * 3 * t))
        ref[b] = 0.3 * sig / np.abs(sig).max()
    return ref.astype(np.float32), _noisy(ref, rng, snr_db)


def _noisy(ref, rng, snr_db):
    noise = rng.standard_normal(ref.shape)
    snr = np.broadcast_to(np.asarray(snr_db, np.float64).reshape(-1, 1), (ref.shape[0], 1))
    power = (ref.astype(np.float64) ** 2).mean(axis=1, keepdims=True)
    return (ref + noise * np.sqrt(power / 10 ** (snr / 10))).astype(np.float32)


def dropout_pair(batch, n, sr, seed, snr_db):
    """Speech whose degraded copy loses 150 ms (zeros) and carries a 50 ms
    burst at 8x amplitude."""

    ref, deg = speech_pair(batch, n, sr, seed, snr_db)
    deg = deg.astype(np.float64)
    rng = np.random.default_rng(seed + 100)
    for b in range(batch):
        a = int(rng.uniform(0.2, 0.4) * n)
        deg[b, a : a + int(0.15 * sr)] = 0.0
        c = int(rng.uniform(0.6, 0.8) * n)
        deg[b, c : c + int(0.05 * sr)] *= 8.0
    return ref, deg.astype(np.float32)


def fir_pair(batch, n, sr, seed, snr_db, taps=64, cutoff=4000.0):
    """Speech through a seeded random low pass FIR (windowed sinc with
    +-10 % jitter on the taps), plus white noise."""

    ref, _ = speech_pair(batch, n, sr, seed, snr_db)
    rng = np.random.default_rng(seed + 200)
    k = np.arange(taps) - (taps - 1) / 2
    h = 2 * cutoff / sr * np.sinc(2 * cutoff / sr * k) * np.hanning(taps) * (1 + 0.2 * (rng.uniform(size=taps) - 0.5))
    h = h / h.sum()
    low = np.stack([np.convolve(r.astype(np.float64), h)[:n] for r in ref])
    return ref, _noisy(low, rng, snr_db)


SIGNALS = {"speech": speech_pair, "harmonic": lambda *a: speech_pair(*a, broadband=False),
           "dropout": dropout_pair, "fir": fir_pair}


DEFAULT_GEOMETRY = (512, 256, 512)  # n_fft, hop_length, win_length

CASES = [
    # name, batch, samples, sample_rate, seed, snr_db, factor[, (n_fft, hop_length, win_length)[, signal]]
    ("sr16k_b2_n6000", 2, 6000, 16000, 1, 10.0, 0.5),
    ("sr16k_b1_n8192", 1, 8192, 16000, 2, 3.0, 1.0),
    ("sr16k_b3_n7001", 3, 7001, 16000, 3, 20.0, 1.0),
    ("sr48k_b1_n18000", 1, 18000, 48000, 4, 10.0, 1.0),
    ("sr44k_b1_n16540", 1, 16540, 44100, 5, 10.0, 1.0),
    ("sr8k_b1_n3200", 1, 3200, 8000, 6, 15.0, 1.0),
    # other frame geometries of PesqLoss(..., win_length, n_fft, hop_length)
    ("sr16k_fft256_hop128_b2_n6000", 2, 6000, 16000, 11, 10.0, 1.0, (256, 128, 256)),
    ("sr16k_fft1024_hop512_b1_n20000", 1, 20000, 16000, 12, 5.0, 1.0, (1024, 512, 1024)),
    ("sr16k_fft512_hop200_win400_b1_n9000", 1, 9000, 16000, 13, 15.0, 1.0, (512, 200, 400)),
    ("sr16k_fft512_hop256_win400_b1_n8000", 1, 8000, 16000, 14, 10.0, 1.0, (512, 256, 400)),
    ("sr16k_fft64_hop32_b1_n4000", 1, 4000, 16000, 15, 10.0, 1.0, (64, 32, 64)),
    ("sr16k_fft4096_hop1024_b1_n28000", 1, 28000, 16000, 16, 10.0, 1.0, (4096, 1024, 4096)),
    ("sr16k_fft512_hop600_b1_n16000", 1, 16000, 16000, 17, 10.0, 1.0, (512, 600, 512)),
    ("sr48k_fft256_hop128_b1_n18000", 1, 18000, 48000, 18, 10.0, 1.0, (256, 128, 256)),
    # the clamps of the perceptual chain: saturated asymmetric distance (45.0
    # in every frame), the frame power ratio clamped at both ends, and the
    # degradations of the 44.1 kHz and 48 kHz workloads (a -5 dB row beside a
    # 25 dB row)
    ("sr16k_sat_b2_n16000", 2, 16000, 16000, 21, 10.0, 1.0, DEFAULT_GEOMETRY, "harmonic"),
    ("sr48k_sat_b1_n24000", 1, 24000, 48000, 22, 10.0, 1.0, DEFAULT_GEOMETRY, "harmonic"),
    ("sr16k_clamp_b2_n16000", 2, 16000, 16000, 23, 15.0, 1.0, DEFAULT_GEOMETRY, "dropout"),
    ("sr44k_fir_b1_n22050", 1, 22050, 44100, 24, 5.0, 1.0, DEFAULT_GEOMETRY, "fir"),
    ("sr48k_mix_b2_n24000", 2, 24000, 48000, 25, (-5.0, 25.0), 1.0, DEFAULT_GEOMETRY, "speech"),
]


def main():
    PesqLoss, ref_pipeline = _import_reference()
    torch.manual_seed(0)

    only = set(sys.argv[1:])  # case names to (re)generate; all when empty
    for name, batch, n, sr, seed, snr, factor, *rest in CASES:
        if only and name not in only:
            continue
        n_fft, hop, win = rest[0] if rest else DEFAULT_GEOMETRY
        kind = rest[1] if len(rest) > 1 else "speech"
        model = PesqLoss(factor, sample_rate=sr, n_fft=n_fft, hop_length=hop, win_length=win)
        ref_np, deg_np = SIGNALS[kind](batch, n, sr, seed, snr)
        out = {"ref": ref_np, "deg": deg_np, "factor": np.float64(factor), "sample_rate": np.int64(sr)}
        if rest and rest[0] != DEFAULT_GEOMETRY:
            out.update(n_fft=np.int64(n_fft), hop_length=np.int64(hop), win_length=np.int64(win))

        ref = torch.from_numpy(ref_np).requires_grad_(True)
        deg = torch.from_numpy(deg_np).requires_grad_(True)
        d_symm, d_asymm = model.raw(ref, deg)
        out["ref32_d_symm"] = d_symm.detach().double().numpy()
        out["ref32_d_asymm"] = d_asymm.detach().double().numpy()
        out["ref32_mos"] = model.mos(ref, deg).detach().double().numpy()
        loss = model(ref, deg)
        out["ref32_loss"] = loss.detach().double().numpy()
        g_ref, g_deg = torch.autograd.grad(loss.sum(), [ref, deg])
        out["ref32_grad_ref"] = g_ref.numpy()
        out["ref32_grad_deg"] = g_deg.numpy()

        model64 = copy.deepcopy(model).double()
        ref64 = torch.from_numpy(ref_np).double().requires_grad_(True)
        deg64 = torch.from_numpy(deg_np).double().requires_grad_(True)
        ds, da = ref_pipeline(ref64, deg64, model64)
        out["f64_d_symm"] = ds.detach().numpy()
        out["f64_d_asymm"] = da.detach().numpy()
        loss64 = factor * (0.1 * ds + 0.0309 * da)
        g_ref64, g_deg64 = torch.autograd.grad(loss64.sum(), [ref64, deg64])
        out["f64_grad_ref"] = g_ref64.numpy()
        out["f64_grad_deg"] = g_deg64.numpy()

        np.savez_compressed(os.path.join(HERE, f"{name}.npz"), **out)
        print(name, out["f64_d_symm"], out["f64_d_asymm"], out["ref32_d_symm"])

    if only:
        return
    model = PesqLoss(1.0, sample_rate=16000)
    const = {
        "fbank": model.fbank.fbank.detach().numpy(),
        "pow_dens_correction": model.fbank.pow_dens_correction.detach().numpy(),
        "width_bark": model.fbank.width_bark.detach().numpy(),
        "total_width": np.float64(model.fbank.total_width),
        "threshs": model.loudness.threshs.detach().numpy().reshape(-1),
        "exps": model.loudness.exp.detach().numpy(),
        "window": model.to_spec.window.detach().numpy(),
        "power_filter": model.power_filter.detach().numpy(),
        "pre_filter": model.pre_filter.detach().numpy(),
    }
    for sr in (8000, 22050, 44100, 48000):
        res = PesqLoss(1.0, sample_rate=sr).resampler
        const[f"resample_{sr}_kernel"] = res.kernel.detach().numpy().reshape(res.kernel.shape[0], -1)
        const[f"resample_{sr}_width"] = np.int64(res.width)
    np.savez_compressed(os.path.join(HERE, "constants.npz"), **const)


if __name__ == "__main__":
    main()
