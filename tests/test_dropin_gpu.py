"""PesqLossCuda's align_level / preemphasize (PesqLossTriton's overrides of
PesqLoss's two signal stages, triton_ops/loss.py:94-102) against the float64
oracle's stages, forward and backward."""

import pytest
import torch

from gpu_helpers import peak_rel_err
from oracle import pesq_oracle as O
from triton_pesq_b200 import PesqLossCuda
from triton_pesq_b200.signals import speech_like

pytestmark = pytest.mark.gpu

#: the IIR filters' parity bound against float64 lfilter (as the reference's
#: TritonIIR tests, tests/test_triton_iir.py:116-135)
IIR_RTOL = 1e-5


@pytest.mark.parametrize("stage", ["align_level", "preemphasize"])
def test_signal_stages_match_float64(cuda_device, stage):
    x = speech_like(3, 20000, 16000, seed=71)
    loss = PesqLossCuda(1.0, sample_rate=16000)
    p = O.OracleParams(1.0, 16000)
    xg = x.to(cuda_device).requires_grad_(True)
    got = getattr(loss, stage)(xg)
    x64 = x.double().requires_grad_(True)
    want = getattr(O, stage)(x64, p)
    assert got.dtype == torch.float32 and got.shape == x.shape
    assert peak_rel_err(got.detach().cpu(), want.detach()) < IIR_RTOL
    g = torch.randn(x.shape, generator=torch.Generator().manual_seed(72))
    (gx,) = torch.autograd.grad(got, [xg], g.to(cuda_device))
    (gx64,) = torch.autograd.grad(want, [x64], g.double())
    assert peak_rel_err(gx.cpu(), gx64) < IIR_RTOL
    # the caller's tensor is left as it was
    assert torch.equal(xg.detach().cpu(), x)


def test_resampler_attribute_on_gpu(cuda_device):
    loss = PesqLossCuda(1.0, sample_rate=48000)
    x = speech_like(2, 9600, 48000, seed=73)
    y = loss.resampler(x.to(cuda_device)).cpu().double()
    want = O.resample(x.double(), O.OracleParams(1.0, 48000).kernel)
    assert peak_rel_err(y, want) < 1e-6
