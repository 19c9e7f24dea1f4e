"""Fusing the loss into a caller's training step: bfloat16 / float16 inputs
with the float32 / float64 internal path, and evaluation on a side stream
overlapping other GPU work (the last of the "next" items of the hot path;
the reference itself accepts float32 only)."""

import pytest
import torch

from triton_pesq_b200 import PesqLossCuda
from triton_pesq_b200.signals import add_noise, speech_like

pytestmark = pytest.mark.gpu


def _eval(model, ref, deg):
    r = ref.detach().clone().requires_grad_(True)
    d = deg.detach().clone().requires_grad_(True)
    loss = model(r, d)
    g_ref, g_deg = torch.autograd.grad(loss.sum(), [r, d])
    ds, da = model.raw(ref, deg)
    return loss.detach(), ds, da, g_ref, g_deg


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("sample_rate,samples", [(16000, 32000), (44100, 66150), (48000, 72000)])
def test_half_inputs_match_float32_of_the_same_values(cuda_device, dtype, sample_rate, samples):
    """Each 16-bit sample is widened exactly, so the whole evaluation is the
    float32 one of the rounded values, bit for bit; the gradients are the
    float32 gradients rounded to the inputs' dtype."""

    ref = speech_like(3, samples, sample_rate, seed=61)
    deg = add_noise(ref, 8.0, seed=62)
    ref_h, deg_h = ref.to(cuda_device, dtype), deg.to(cuda_device, dtype)
    model = PesqLossCuda(0.5, sample_rate=sample_rate)
    loss_h, ds_h, da_h, gr_h, gd_h = _eval(model, ref_h, deg_h)
    loss_f, ds_f, da_f, gr_f, gd_f = _eval(model, ref_h.float(), deg_h.float())
    assert loss_h.dtype == torch.float32 and ds_h.dtype == torch.float32
    assert torch.equal(loss_h, loss_f)
    assert torch.equal(ds_h, ds_f) and torch.equal(da_h, da_f)
    assert gr_h.dtype == dtype and gd_h.dtype == dtype
    assert torch.equal(gr_h, gr_f.to(dtype))
    assert torch.equal(gd_h, gd_f.to(dtype))
    assert torch.isfinite(gd_h.float()).all()


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("n_fft,hop,sample_rate", [(256, 128, 16000), (1024, 400, 44100)])
def test_half_inputs_with_other_frame_geometries(cuda_device, dtype, n_fft, hop, sample_rate):
    """The spectrum kernels' path (general n_fft / hop) reads 16-bit rows the
    same way: bitwise the float32 evaluation of the rounded values."""

    ref = speech_like(2, 2 * sample_rate, sample_rate, seed=65)
    deg = add_noise(ref, 6.0, seed=66)
    ref_h, deg_h = ref.to(cuda_device, dtype), deg.to(cuda_device, dtype)
    model = PesqLossCuda(1.0, sample_rate=sample_rate, n_fft=n_fft, hop_length=hop, win_length=n_fft)
    loss_h, ds_h, da_h, gr_h, gd_h = _eval(model, ref_h, deg_h)
    loss_f, ds_f, da_f, gr_f, gd_f = _eval(model, ref_h.float(), deg_h.float())
    assert torch.equal(loss_h, loss_f)
    assert torch.equal(ds_h, ds_f) and torch.equal(da_h, da_f)
    assert torch.equal(gr_h, gr_f.to(dtype)) and torch.equal(gd_h, gd_f.to(dtype))


def test_half_inputs_strided_and_graphed(cuda_device):
    ref = speech_like(2, 40000, 16000, seed=63)
    deg = add_noise(ref, 5.0, seed=64)
    wide_r = torch.zeros(2, 41000, dtype=torch.bfloat16, device=cuda_device)
    wide_d = torch.zeros_like(wide_r)
    wide_r[:, :40000] = ref.to(cuda_device, torch.bfloat16)
    wide_d[:, :40000] = deg.to(cuda_device, torch.bfloat16)
    model = PesqLossCuda(1.0, sample_rate=16000)
    strided = model(wide_r[:, :40000], wide_d[:, :40000])
    packed = model(wide_r[:, :40000].contiguous(), wide_d[:, :40000].contiguous())
    assert torch.equal(strided, packed)
    r = wide_r[:, :40000].contiguous().requires_grad_(True)
    d = wide_d[:, :40000].contiguous().requires_grad_(True)
    eager = model(r, d)
    eager_g = torch.autograd.grad(eager.sum(), [r, d])
    step = model.graphed(r, d)
    captured = step(r, d)
    captured_g = torch.autograd.grad(captured.sum(), [r, d])
    assert torch.equal(captured, eager)
    for a, b in zip(eager_g, captured_g):
        assert torch.equal(a, b)


def test_mixed_or_unsupported_dtypes_are_rejected(cuda_device):
    model = PesqLossCuda(1.0, sample_rate=16000)
    ref = torch.randn(2, 16000, device=cuda_device)
    with pytest.raises(ValueError):
        model(ref.bfloat16(), ref)
    with pytest.raises(RuntimeError):
        model(ref.double(), ref.double())


def test_side_stream_overlapping_other_work(cuda_device):
    """The loss follows the current stream: evaluated on a side stream while
    the default stream runs matrix products (a stand-in for the model's
    backward), it gives the same bits as on the default stream alone."""

    ref = speech_like(4, 48000, 16000, seed=65).to(cuda_device)
    deg = add_noise(ref.cpu(), 6.0, seed=66).to(cuda_device)
    model = PesqLossCuda(1.0, sample_rate=16000)
    want_loss, _, _, _, want_g = _eval(model, ref, deg)
    a = torch.randn(2048, 2048, device=cuda_device, dtype=torch.bfloat16)
    side = torch.cuda.Stream(cuda_device)
    main = torch.cuda.current_stream(cuda_device)
    for _ in range(3):
        side.wait_stream(main)
        c = a
        for _ in range(8):  # queued on the default stream
            c = (c @ a).tanh()
        with torch.cuda.stream(side):
            d = deg.detach().clone().requires_grad_(True)
            loss = model(ref, d)
            (g,) = torch.autograd.grad(loss.sum(), [d])
        main.wait_stream(side)
        assert torch.equal(loss, want_loss)
        assert torch.equal(g, want_g)
        assert torch.isfinite(c.float()).all()
