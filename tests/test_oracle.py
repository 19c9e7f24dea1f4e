"""The CPU oracle against golden vectors produced by the reference itself."""

import glob
import os

import numpy as np
import pytest
import torch

from conftest import GOLDEN, golden_geometry
from oracle import pesq_oracle as O

CASES = sorted(glob.glob(os.path.join(GOLDEN, "sr*.npz")))


def _load(path):
    z = np.load(path)
    p = O.OracleParams(factor=float(z["factor"]), sample_rate=int(z["sample_rate"]), **golden_geometry(z))
    return z, p


@pytest.mark.parametrize("path", CASES, ids=[os.path.basename(c)[:-4] for c in CASES])
def test_float64_oracle_matches_reference_float64(path):
    """Distances within 1e-6 and gradients within 2e-6 (relative to their peak)
    of the reference's own float64 pipeline (``ref_pipeline`` on a ``.double()``
    ``PesqLoss``).  The residual is the conditioning of the order-10 band pass:
    the reference evaluates it as a direct form, this oracle as transposed
    direct form II, both in float64."""

    z, p = _load(path)
    ref = torch.from_numpy(z["ref"]).double().requires_grad_(True)
    deg = torch.from_numpy(z["deg"]).double().requires_grad_(True)
    ds, da = O.raw(ref, deg, p, "float64")
    np.testing.assert_allclose(ds.detach().numpy(), z["f64_d_symm"], rtol=1e-6)
    np.testing.assert_allclose(da.detach().numpy(), z["f64_d_asymm"], rtol=1e-6)
    loss = p.factor * (0.1 * ds + 0.0309 * da)
    g_ref, g_deg = torch.autograd.grad(loss.sum(), [ref, deg])
    for got, want in ((g_ref, z["f64_grad_ref"]), (g_deg, z["f64_grad_deg"])):
        scale = np.abs(want).max()
        assert np.abs(got.numpy() - want).max() / scale < 2e-6


@pytest.mark.parametrize("path", CASES, ids=[os.path.basename(c)[:-4] for c in CASES])
def test_reference_mode_matches_pesqloss_float32(path):
    """The dtype-faithful mode against ``PesqLoss`` on float32 input: the two
    evaluate the level alignment band pass with different float32 recursions,
    whose documented error is up to 4e-3 relative."""

    z, p = _load(path)
    ds, da = O.raw(torch.from_numpy(z["ref"]), torch.from_numpy(z["deg"]), p, "reference")
    np.testing.assert_allclose(ds.numpy(), z["ref32_d_symm"], rtol=4e-3)
    np.testing.assert_allclose(da.numpy(), z["ref32_d_asymm"], rtol=4e-3)
    mos, loss = O.epilogue(ds, da, p.factor)
    np.testing.assert_allclose(mos.numpy(), z["ref32_mos"], rtol=4e-3)
    np.testing.assert_allclose(loss.numpy(), z["ref32_loss"], rtol=4e-3)


def test_loss_is_zero_for_identical_signals():
    """``PesqLoss(ref, ref)`` is (almost) zero (reference tests/test_torch.py:18-27)."""

    z, p = _load(CASES[0])
    ref = torch.from_numpy(z["ref"]).double()
    loss = O.forward(ref, ref, p)
    assert torch.all(loss >= 0.0) and torch.all(loss <= 1e-6)


def test_scale_invariance():
    """Scaling either input leaves the distances unchanged: the peak
    normalisation and the level alignment make the pipeline scale free
    (reference tests/test_triton_elementwise.py:1396-1451)."""

    z, p = _load(CASES[0])
    ref = torch.from_numpy(z["ref"]).double()
    deg = torch.from_numpy(z["deg"]).double()
    ds, da = O.raw(ref, deg, p)
    ds2, da2 = O.raw(ref * 7.5, deg * 0.01, p)
    np.testing.assert_allclose(ds2.numpy(), ds.numpy(), rtol=1e-9)
    np.testing.assert_allclose(da2.numpy(), da.numpy(), rtol=1e-9)


def test_oracle_tolerance_is_not_vacuous():
    """A planted mistake in the oracle (a perturbed pre-emphasis pole) moves
    the distances well outside the parity tolerance of the GPU tests."""

    z, p = _load(CASES[0])
    ref = torch.from_numpy(z["ref"]).double()
    deg = torch.from_numpy(z["deg"]).double()
    good = O.raw(ref, deg, p)
    p.pre_a = p.pre_a.copy()
    p.pre_a[2] *= 1.0 + 1e-4
    bad = O.raw(ref, deg, p)
    moved = max(
        np.abs(b.numpy() - g.numpy()).max() / np.abs(g.numpy()).max() for g, b in zip(good, bad)
    )
    assert moved > 1e-4


SATURATED_CASES = ["sr16k_sat_b2_n16000", "sr48k_sat_b1_n24000"]


@pytest.mark.parametrize("name", SATURATED_CASES)
def test_saturated_fixtures_hit_the_clamp(name):
    """The saturated fixtures really sit at the 45.0 clamp: the reference's
    float32 and float64 asymmetric distances are 45.0, and the oracle finds
    (nearly) every frame clamped -- so comparing them is not comparing two
    unrelated constants by accident, and it is not vacuous either: the
    symmetric distance and the gradients still vary."""

    z, p = _load(os.path.join(GOLDEN, name + ".npz"))
    np.testing.assert_allclose(z["ref32_d_asymm"], 45.0, rtol=1e-6)
    np.testing.assert_allclose(z["f64_d_asymm"], 45.0, rtol=1e-6)
    census = {}
    O.raw(torch.from_numpy(z["ref"]).double(), torch.from_numpy(z["deg"]).double(), p, census=census)
    assert float(census["asymm_45"].min()) > 0.95
    assert np.all(z["f64_d_symm"] < 45.0)
    assert np.abs(z["f64_grad_deg"]).max() > 0


def test_clamp_fixture_hits_every_clamp():
    """The dropout / burst fixture drives the frame power ratio into its
    [3e-4, 5] clamp, the band power ratio into [0.01, 100] and both weighted
    disturbances into the 45.0 clamp in some (not all) frames."""

    z, p = _load(os.path.join(GOLDEN, "sr16k_clamp_b2_n16000.npz"))
    census = {}
    O.raw(torch.from_numpy(z["ref"]).double(), torch.from_numpy(z["deg"]).double(), p, census=census)
    for key in ("frame_ratio", "band_ratio", "symm_45", "asymm_45"):
        assert 0.0 < float(census[key].min()) and float(census[key].max()) < 0.5, key


def test_mixed_snr_fixture_regimes():
    """The 48 kHz -5 dB / 25 dB pair: the -5 dB row clamps far more frames."""

    z, p = _load(os.path.join(GOLDEN, "sr48k_mix_b2_n24000.npz"))
    census = {}
    O.raw(torch.from_numpy(z["ref"]).double(), torch.from_numpy(z["deg"]).double(), p, census=census)
    assert float(census["asymm_45"][0]) > 0.3 > float(census["asymm_45"][1])
