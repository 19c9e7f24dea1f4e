"""The torch.ops.pesq_cuda custom ops under tracing: their fake (shape)
functions agree with the real ops (torch.library.opcheck), and a
torch.compile'd training step containing PesqLossCuda traces whole
(fullgraph, the aot_eager backend: no code generation) and returns what the
eager step returns, bit for bit."""

import pytest
import torch

from triton_pesq_b200 import IIRCuda, PesqLossCuda, ResampleCuda, _lib
from triton_pesq_b200.signals import add_noise, speech_like
from triton_pesq_b200.tables import pre_filter

pytestmark = pytest.mark.gpu

CHECKS = ("test_schema", "test_faketensor")


def test_opcheck_forward_backward(cuda_device):
    model = PesqLossCuda(1.0, sample_rate=16000)
    plan = model._plan(cuda_device)
    ref = speech_like(2, 16000, 16000, seed=81).to(cuda_device)
    deg = add_noise(ref.cpu(), 5.0, seed=82).to(cuda_device)
    flags = _lib.GRAD_DEG
    torch.library.opcheck(torch.ops.pesq_cuda.forward.default, (plan, ref, deg, flags), test_utils=CHECKS)
    ws = torch.ops.pesq_cuda.forward(plan, ref, deg, flags)[4]
    g = torch.ones(2, device=cuda_device)
    torch.library.opcheck(torch.ops.pesq_cuda.backward.default, (plan, ref, deg, flags, ws, g, None, None, None),
                          test_utils=CHECKS)


def test_opcheck_standalone_ops(cuda_device):
    rs = ResampleCuda(44100, 16000)
    x = torch.randn(3, 4410, device=cuda_device)
    h = rs._handle(cuda_device)
    torch.library.opcheck(torch.ops.pesq_cuda.resample.default, (h, x), test_utils=CHECKS)
    y = torch.ops.pesq_cuda.resample(h, x)
    torch.library.opcheck(torch.ops.pesq_cuda.resample_adjoint.default, (h, torch.randn_like(y), 4410),
                          test_utils=CHECKS)
    iir = IIRCuda(*pre_filter())
    torch.library.opcheck(torch.ops.pesq_cuda.iir.default, (iir._handle(cuda_device), x, 0), test_utils=CHECKS)


def test_compiled_training_step_matches_eager(cuda_device):
    model = PesqLossCuda(1.0, sample_rate=16000)
    ref = speech_like(2, 16000, 16000, seed=83).to(cuda_device)
    deg = add_noise(ref.cpu(), 8.0, seed=84).to(cuda_device)

    def step(r, d):
        loss = model(r, d)
        return loss, loss.mean()

    d_eager = deg.clone().requires_grad_(True)
    loss_e, mean_e = step(ref, d_eager)
    mean_e.backward()
    compiled = torch.compile(step, backend="aot_eager", fullgraph=True)
    d_comp = deg.clone().requires_grad_(True)
    loss_c, mean_c = compiled(ref, d_comp)
    mean_c.backward()  # the backward graph AOTAutograd traced through the fake kernels
    assert torch.equal(loss_c, loss_e)
    assert torch.equal(mean_c, mean_e)
    assert torch.equal(d_comp.grad, d_eager.grad)
