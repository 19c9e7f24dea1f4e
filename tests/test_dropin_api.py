"""The attributes and submodules of PesqLossCuda that PesqLossTriton carries
(its own and those it inherits from PesqLoss), against the reference's
constant tensors (tests/golden/constants.npz, written by the reference)."""

import os

import numpy as np
import pytest
import torch

from conftest import GOLDEN
from triton_pesq_b200 import PesqLossCuda, ResampleCuda
from triton_pesq_b200.model import BarkScale, Loudness, PowerSpectrogram, edge_ramp

CONST = np.load(os.path.join(GOLDEN, "constants.npz"))


def test_submodule_constants_match_reference():
    loss = PesqLossCuda(1.0, sample_rate=16000)
    np.testing.assert_array_equal(loss.fbank.fbank.numpy(), CONST["fbank"])
    assert loss.fbank.fbank.dtype == torch.float32
    np.testing.assert_allclose(loss.fbank.pow_dens_correction.numpy(), CONST["pow_dens_correction"], rtol=1e-15)
    np.testing.assert_allclose(loss.fbank.width_bark.numpy(), CONST["width_bark"], rtol=1e-15)
    assert float(loss.fbank.total_width) == pytest.approx(float(CONST["total_width"]), rel=1e-15)
    np.testing.assert_allclose(loss.loudness.threshs.numpy().reshape(-1), CONST["threshs"], rtol=1e-15)
    assert loss.loudness.threshs.shape == (1, 1, 49)
    np.testing.assert_array_equal(loss.loudness.exp.numpy(), CONST["exps"])
    assert loss.loudness.exp.dtype == torch.float32
    np.testing.assert_array_equal(loss.to_spec.window.numpy(), CONST["window"])
    np.testing.assert_array_equal(loss.power_filter.numpy(), CONST["power_filter"])
    np.testing.assert_array_equal(loss.pre_filter.numpy(), CONST["pre_filter"])


def test_resampler_attributes():
    at16 = PesqLossCuda(1.0, sample_rate=16000)
    assert at16.resample_op is None
    x = torch.randn(2, 100)
    assert at16.resampler(x) is x  # identity at 16 kHz, on any device
    at44 = PesqLossCuda(1.0, sample_rate=44100)
    assert isinstance(at44.resample_op, ResampleCuda) and at44.resample_op is at44.resampler
    np.testing.assert_array_equal(at44.resampler.kernel.numpy(), CONST["resample_44100_kernel"])


def test_submodules_follow_the_reference_semantics_on_cpu():
    """The submodules' own forward methods (torch expressions of bark.py /
    loudness.py / torchaudio's Spectrogram) against the oracle's stages."""

    from oracle import pesq_oracle as O

    p = O.OracleParams(1.0, 16000)
    # float32 signals as the reference's (its fbank is a float32 matrix)
    x = torch.randn(2, 6000, generator=torch.Generator().manual_seed(3))
    spec = PowerSpectrogram()(x)  # [batch, 257, frames]
    want = O.stft_bark(x.double(), p, torch.float64)
    spec = spec.swapaxes(1, 2).clone()
    spec[:, :, 0] = 0.0
    got = BarkScale()(spec)
    assert got.dtype == torch.float64
    np.testing.assert_allclose(got.numpy(), want.numpy(), rtol=1e-4, atol=1e-6 * float(want.abs().max()))
    got = want
    loud = Loudness()
    thr = loud.threshs
    assert torch.equal(loud.total_audible(got, 1.0), O._total_audible(got, thr.reshape(-1), 1.0))
    np.testing.assert_allclose(loud(got).numpy(), O._loudness(got, thr.reshape(-1), loud.exp.double()).numpy(),
                               rtol=1e-12)
    w = BarkScale().width_bark
    np.testing.assert_allclose(BarkScale().weighted_norm(got, 2).numpy(),
                               O._weighted_norm(got, w, float(BarkScale().total_width), 2).numpy(), rtol=1e-12)


def test_edge_ramp_semantics():
    """Head fade then tail fade, one after the other (loss.py:163-165), also
    for rows shorter than 30 samples where the two overlap."""

    x = torch.ones(1, 20)
    got = edge_ramp(x)
    emp = torch.arange(1, 16) / 16.0
    want = torch.ones(1, 20)
    want[:, :15] *= emp
    want[:, -15:] *= torch.flip(emp, dims=(0,))
    assert torch.equal(got, want)
    assert torch.equal(x, torch.ones(1, 20))  # not modified in place


def test_signal_stages_need_a_gpu():
    loss = PesqLossCuda(1.0, sample_rate=16000)
    with pytest.raises(RuntimeError):
        loss.align_level(torch.randn(1, 4000))


def test_native_handles_are_released_after_the_last_reference():
    """A plan / resampler handle lives while its module or an autograd node
    holds its owner, and is released once; a released plan's cached
    workspace offsets go with it (a later plan may reuse the address)."""
    import gc

    from triton_pesq_b200 import _lib
    from triton_pesq_b200 import loss as loss_mod

    released = []
    owner = _lib.Owned(1234, released.append)
    holders = [owner]
    del owner
    gc.collect()
    assert released == []
    holders.clear()
    gc.collect()
    assert released == [1234]

    calls = []
    keys = [(77, 8, 16000, 2), (78, 8, 16000, 2)]
    saved_destroy = _lib.destroy_plan
    try:
        _lib.destroy_plan = calls.append
        for k, key in enumerate(keys):
            loss_mod._SUM_OFFSETS[key] = 256 * (k + 1)
        loss_mod._release_plan(77)
        assert calls == [77]
        assert keys[0] not in loss_mod._SUM_OFFSETS
        assert loss_mod._SUM_OFFSETS[keys[1]] == 512
    finally:
        _lib.destroy_plan = saved_destroy
        loss_mod._SUM_OFFSETS.pop(keys[1], None)

    model = PesqLossCuda(1.0, sample_rate=44100)
    model._plans[0], model._plan_owners[5] = 5, _lib.Owned(5, lambda h: None)
    state = model.__getstate__()
    assert state["_plans"] == {} and state["_plan_owners"] == {}
    rs = ResampleCuda(44100, 16000)
    assert rs.__getstate__()["_owners"] == {}
