"""Host-side constants against the reference's constant tensors."""

import os

import numpy as np
import pytest

from conftest import GOLDEN
from triton_pesq_b200 import tables as T

CONST = np.load(os.path.join(GOLDEN, "constants.npz"))


def test_filterbank_matches_reference():
    lay = T.bark_layout(256, 49)
    np.testing.assert_array_equal(lay.fbank(), CONST["fbank"])
    # every bin in exactly one band (reference tests/test_fbank.py:5-11)
    assert np.all(lay.fbank().sum(axis=0) == 1.0)
    np.testing.assert_array_equal(lay.fbank().sum(axis=1), T.HZ_BINS_PER_BAND)


def test_band_constants_match_reference():
    lay = T.bark_layout(256, 49)
    np.testing.assert_array_equal(lay.pow_dens_correction, CONST["pow_dens_correction"])
    np.testing.assert_array_equal(lay.width_bark, CONST["width_bark"])
    assert lay.total_width == pytest.approx(float(CONST["total_width"]), rel=1e-15)
    np.testing.assert_array_equal(T.hearing_thresholds(49), CONST["threshs"])
    np.testing.assert_array_equal(T.loudness_exponents().astype(np.float32), CONST["exps"])


def test_filters_and_window_match_reference():
    b, a = T.power_filter()
    np.testing.assert_array_equal(np.stack([b, a]).astype(np.float32), CONST["power_filter"])
    b, a = T.pre_filter()
    np.testing.assert_array_equal(np.stack([b, a]).astype(np.float32), CONST["pre_filter"])
    np.testing.assert_array_equal(T.hann_window(512).astype(np.float32), CONST["window"])


@pytest.mark.parametrize("sr", [8000, 22050, 44100, 48000])
def test_resample_kernel_matches_reference(sr):
    k = T.sinc_resample_kernel(sr, 16000)
    np.testing.assert_array_equal(k.taps.astype(np.float32), CONST[f"resample_{sr}_kernel"])
    assert k.width == int(CONST[f"resample_{sr}_width"])


@pytest.mark.parametrize("orig,new", [(48000, 16000), (44100, 16000), (8000, 16000), (22050, 16000), (32000, 16000)])
def test_resample_kernel_matches_torchaudio(orig, new):
    """Pins the restated sinc design to the installed torchaudio."""

    ta = pytest.importorskip("torchaudio.functional.functional")
    import math

    ref, width = ta._get_sinc_resample_kernel(orig, new, math.gcd(orig, new))
    k = T.sinc_resample_kernel(orig, new)
    np.testing.assert_array_equal(k.taps.astype(np.float32), ref.reshape(ref.shape[0], -1).numpy())
    assert k.width == width


@pytest.mark.parametrize("n", [1, 17, 999, 4001, 16384, 33333, 176400, 480000])
@pytest.mark.parametrize("orig", [8000, 22050, 44100, 48000])
def test_resample_length_matches_torchaudio(orig, n):
    import math

    import torch

    g = math.gcd(orig, 16000)
    want = int(torch.ceil(torch.as_tensor((16000 // g) * n / (orig // g))).long())
    assert T.resample_length(n, orig // g, 16000 // g) == want


@pytest.mark.parametrize("which", ["power", "pre"])
def test_scan_tables_are_exact_and_well_conditioned(which):
    b, a = T.power_filter() if which == "power" else T.pre_filter()
    tab = T.ScanTables.build(b, a)
    assert tab.fidelity < 1e-9
    assert tab.truncation < T.SCAN_TRUNCATION
    # table entries stay O(1): no float32 cancellation at run time
    for arr in (tab.carry, tab.drive, tab.power):
        assert np.abs(arr).max() < 10.0


def test_scan_rejects_poles_on_the_unit_circle():
    with pytest.raises(RuntimeError):
        T.ScanTables.build([1.0, 0.0, 0.0], [1.0, -1.999, 0.9995])


def test_frame_and_window_counts():
    assert T.frame_count(16000) == 62
    assert T.frame_count(128000) == 499
    assert T.frame_count(48000) == 187
    assert T.frame_count(64000) == 249
    assert T.frame_count(160000) == 624
    assert T.psqm_windows(499) == 48


@pytest.mark.parametrize("n_fft", [40, 48, 96, 1000, 16])
def test_rejects_non_power_of_two_n_fft(n_fft):
    """n_fft must be a power of two of at least 32, as for the reference's
    spectral op (test_triton_spectral.py:237-255)."""

    with pytest.raises(ValueError, match="power of two"):
        T.PlanConfig.build(1.0, 16000, n_fft=n_fft, win_length=min(n_fft, 16))


@pytest.mark.parametrize("kw", [dict(n_fft=8192), dict(hop_length=0), dict(win_length=600)])
def test_rejects_other_frame_geometries(kw):
    with pytest.raises(ValueError):
        T.PlanConfig.build(1.0, 16000, **kw)


@pytest.mark.parametrize("n_fft", [32, 64, 128, 256, 1024, 2048, 4096])
def test_bark_bands_segment_every_frame_length(n_fft):
    """The filterbank of every supported n_fft is a sorted, disjoint
    segmentation of the n_fft / 2 bins (test_triton_spectral.py:178-195), as
    the spectrum kernels' band table assumes."""

    lay = T.bark_layout(n_fft // 2, 49)
    prev = 0
    for s, e in zip(lay.starts, lay.ends):
        assert prev <= s <= e <= n_fft // 2
        prev = e
