"""Standalone resampler on the GPU against torchaudio's own resampling
arithmetic in float64 with the same float32 filter bank (the reference's
TritonResample tests, tests/test_triton_resample.py, compare against
torchaudio.transforms.Resample the same way)."""

import math

import pytest
import torch
import torchaudio
import torchaudio.functional.functional as TAF

from triton_pesq_b200 import ResampleCuda

pytestmark = pytest.mark.gpu

# the usual rates (float64 tensor-core kernels), upsampling, and 96 kHz, whose
# 8-phase tap spans are too long for the tensor-core tiles (staged kernels)
RATES = [(44100, 16000), (48000, 16000), (8000, 16000), (22050, 16000), (16000, 48000), (16000, 44100),
         (24000, 16000), (32000, 16000), (11025, 16000), (16000, 8000), (96000, 16000)]


def _reference64(x, module):
    """torchaudio's polyphase convolution in float64 with the float32 taps."""

    kernel = module.kernel.detach().cpu().double()[:, None, :]
    return TAF._apply_sinc_resample_kernel(x.cpu().double(), module.orig_step, module.new_step, 1, kernel,
                                           module.width)


def _peak_err(got, want):
    got = got.detach().double().cpu()
    return float((got - want).abs().max() / max(want.abs().max(), 1e-30))


@pytest.mark.parametrize("orig,new", RATES)
@pytest.mark.parametrize("method", ["sinc_interp_hann", "sinc_interp_kaiser"])
def test_forward_matches_torchaudio(cuda_device, orig, new, method):
    g = torch.Generator().manual_seed(orig + new)
    x = torch.randn(3, orig // 4 + 37, generator=g)
    module = ResampleCuda(orig, new, resampling_method=method).to(cuda_device)
    y = module(x.to(cuda_device))
    want = _reference64(x, module)
    assert y.shape == want.shape
    # float64 accumulation of float32 products: one float32 rounding of the sum
    assert _peak_err(y, want) < 1e-6
    # and the float32 torchaudio module itself
    ta = torchaudio.transforms.Resample(orig, new, resampling_method=method)(x)
    assert _peak_err(y, ta.double()) < 1e-5


@pytest.mark.parametrize("orig,new", RATES)
def test_adjoint_matches_torchaudio(cuda_device, orig, new):
    """The adjoint (the gradient of the forward) against the gradient of
    torchaudio's float64 convolution with the same taps, at every rate pair."""

    g = torch.Generator().manual_seed(3 * orig + new)
    x = torch.randn(3, orig // 4 + 53, generator=g, dtype=torch.float64)
    module = ResampleCuda(orig, new).to(cuda_device)
    xd = x.float().to(cuda_device).requires_grad_(True)
    y = module(xd)
    gy = torch.randn(y.shape, generator=g, dtype=torch.float64)
    (gx,) = torch.autograd.grad(y, xd, gy.float().to(cuda_device))
    xr = x.clone().requires_grad_(True)
    (want,) = torch.autograd.grad(_reference64(xr, module), xr, gy.float().double())
    assert _peak_err(gx, want) < 1e-6


def test_adjoint_and_double_backward(cuda_device):
    g = torch.Generator().manual_seed(5)
    x = torch.randn(4, 3000, generator=g, dtype=torch.float64)
    module = ResampleCuda(44100, 16000).to(cuda_device)
    xd = x.float().to(cuda_device).requires_grad_(True)
    y = module(xd)
    gy = torch.randn(y.shape, generator=g).to(cuda_device).requires_grad_(True)
    (gx,) = torch.autograd.grad(y, xd, gy, create_graph=True)
    # the gradient of torchaudio's float64 convolution with the same taps
    xr = x.clone().requires_grad_(True)
    (want,) = torch.autograd.grad(_reference64(xr, module), xr, gy.detach().double().cpu())
    assert _peak_err(gx, want) < 1e-6
    # double backward: d<gx, v>/d gy = A v, through the same kernels
    v = torch.randn(x.shape, generator=g).to(cuda_device)
    (ggy,) = torch.autograd.grad((gx * v).sum(), gy)
    torch.testing.assert_close(ggy, module(v), rtol=0, atol=0)


def test_leading_dims_strides_and_large_row_counts(cuda_device):
    module = ResampleCuda(48000, 16000).to(cuda_device)
    x = torch.randn(2, 3, 4800, device=cuda_device)
    y = module(x)
    assert y.shape == (2, 3, 1600)
    torch.testing.assert_close(y[1, 2], module(x[1, 2][None])[0], rtol=0, atol=0)
    wide = torch.randn(4, 9600, device=cuda_device)[:, ::2]  # strided samples
    torch.testing.assert_close(module(wide), module(wide.contiguous()), rtol=0, atol=0)
    many = torch.randn(70000, 30, device=cuda_device)  # more rows than grid y holds
    out = module(many)
    torch.testing.assert_close(out[69999], module(many[69999:])[0], rtol=0, atol=0)
    assert module(torch.empty(0, 100, device=cuda_device)).shape == (0, 34)


def test_short_inputs_and_determinism(cuda_device):
    module = ResampleCuda(44100, 16000).to(cuda_device)
    for n in (1, 5, 16, 17, 100):
        x = torch.randn(2, n)
        y = module(x.to(cuda_device))
        assert _peak_err(y, _reference64(x, module)) < 1e-6
    x = torch.randn(3, 50000, device=cuda_device).requires_grad_(True)
    y1 = module(x)
    g1 = torch.autograd.grad(y1.sum(), x)[0]
    y2 = module(x)
    g2 = torch.autograd.grad(y2.sum(), x)[0]
    assert torch.equal(y1, y2) and torch.equal(g1, g2)


def test_errors(cuda_device):
    module = ResampleCuda(44100, 16000).to(cuda_device)
    with pytest.raises(RuntimeError):
        module(torch.randn(2, 100, device=cuda_device, dtype=torch.float64))
    with pytest.raises(RuntimeError):
        module(torch.randn(2, 100))


def test_cuda_graph_replay(cuda_device):
    """The forward and adjoint kernels captured in a CUDA graph equal eager
    calls bitwise on new inputs."""

    from triton_pesq_b200 import ResampleCuda

    rs = ResampleCuda(44100, 16000)
    handle = rs._handle(cuda_device)
    n_in = 44100
    gen = torch.Generator().manual_seed(3)
    static_x = torch.randn(4, n_in, generator=gen).to(cuda_device)
    static_g = torch.randn(4, rs.output_length(n_in), generator=gen).to(cuda_device)
    torch.ops.pesq_cuda.resample(handle, static_x)
    torch.ops.pesq_cuda.resample_adjoint(handle, static_g, n_in)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        y = torch.ops.pesq_cuda.resample(handle, static_x)
        gx = torch.ops.pesq_cuda.resample_adjoint(handle, static_g, n_in)
    for _ in range(2):
        fx = torch.randn(4, n_in, generator=gen).to(cuda_device)
        fg = torch.randn(4, rs.output_length(n_in), generator=gen).to(cuda_device)
        static_x.copy_(fx)
        static_g.copy_(fg)
        graph.replay()
        torch.cuda.synchronize()
        assert torch.equal(y, torch.ops.pesq_cuda.resample(handle, fx))
        assert torch.equal(gx, torch.ops.pesq_cuda.resample_adjoint(handle, fg, n_in))


@pytest.mark.parametrize("orig", [44100, 48000, 8000])
@pytest.mark.parametrize("samples", [1, 2, 3, 7, 23, 24, 25, 440, 441, 442, 7055, 14112])
def test_short_and_ragged_lengths(cuda_device, orig, samples):
    """Lengths that end inside the first super-frame, on and around a
    super-frame boundary, and on a staged window's edge (partial windows,
    tiles with rows past the row end): forward and adjoint against float64."""

    g = torch.Generator().manual_seed(orig + samples)
    x = torch.randn(2, samples, generator=g, dtype=torch.float64)
    module = ResampleCuda(orig, 16000).to(cuda_device)
    xd = x.float().to(cuda_device).requires_grad_(True)
    y = module(xd)
    want = _reference64(x.float().double(), module)
    assert y.shape == want.shape
    if want.numel() == 0:
        return
    assert _peak_err(y, want) < 1e-6
    gy = torch.randn(y.shape, generator=g, dtype=torch.float64)
    (gx,) = torch.autograd.grad(y, xd, gy.float().to(cuda_device))
    xr = x.float().double().requires_grad_(True)
    (gwant,) = torch.autograd.grad(_reference64(xr, module), xr, gy.float().double())
    assert _peak_err(gx, gwant) < 1e-6
