"""Standalone resampler: filter bank design (bit for bit against torchaudio,
whose kernel the reference's TritonResample registers,
torch_pesq/triton_ops/resample.py:490-528) and host-side behaviour."""

import math

import numpy as np
import pytest
import torch
import torchaudio.functional.functional as TAF

from triton_pesq_b200 import ResampleCuda
from triton_pesq_b200.tables import resample_length, sinc_resample_kernel

DESIGNS = [
    (44100, 16000, 6, 0.99, "sinc_interp_hann", None),
    (48000, 16000, 6, 0.99, "sinc_interp_hann", None),
    (8000, 16000, 6, 0.99, "sinc_interp_hann", None),
    (22050, 16000, 6, 0.99, "sinc_interp_hann", None),
    (16000, 48000, 6, 0.99, "sinc_interp_hann", None),
    (48000, 16000, 6, 0.99, "sinc_interp_kaiser", None),
    (44100, 16000, 6, 0.99, "sinc_interp_kaiser", 8.555),
    (22050, 8000, 4, 0.9, "sinc_interp_kaiser", None),
    (16000, 44100, 8, 0.95, "sinc_interp_hann", None),
]


@pytest.mark.parametrize("orig,new,lpw,rolloff,method,beta", DESIGNS)
def test_filter_bank_is_torchaudios(orig, new, lpw, rolloff, method, beta):
    gcd = math.gcd(orig, new)
    want, width = TAF._get_sinc_resample_kernel(orig, new, gcd, lpw, rolloff, method, beta)
    got = sinc_resample_kernel(orig, new, lpw, rolloff, method, beta)
    assert got.width == width
    assert np.array_equal(got.taps, want.reshape(got.new_step, -1).numpy().astype(np.float64))
    # the compact phase ranges cover every nonzero tap
    for j in range(got.new_step):
        nz = np.flatnonzero(got.taps[j])
        if nz.size:
            assert got.first[j] == nz[0] and got.count[j] == nz[-1] + 1 - nz[0]


@pytest.mark.parametrize("n", [0, 1, 2, 17, 441, 44100, 176400, 1234567])
def test_output_length_is_torchaudios(n):
    for orig, new in [(441, 160), (3, 1), (1, 2), (160, 441)]:
        want = int(torch.ceil(torch.as_tensor(new * n / orig)).long())
        assert resample_length(n, orig, new) == want


def test_module_attributes_and_identity():
    r = ResampleCuda(44100, 16000)
    assert r.orig_step == 441 and r.new_step == 160 and r.width == 17
    assert tuple(r.kernel.shape) == (160, 475) and r.kernel.dtype == torch.float32
    assert r.output_length(44100) == 16000
    same = ResampleCuda(16000, 16000)
    x = torch.randn(2, 100)  # CPU: no kernel runs when the rates agree
    assert same(x) is x
    assert not hasattr(same, "kernel")


def test_invalid_arguments():
    with pytest.raises(ValueError):
        ResampleCuda(0, 16000)
    with pytest.raises(ValueError):
        ResampleCuda(44100, 16000, resampling_method="linear")
    with pytest.raises(ValueError):
        ResampleCuda(44100, 16000, lowpass_filter_width=0)
    with pytest.raises(RuntimeError):
        ResampleCuda(44100, 16000)(torch.randn(2, 100))
