"""Failure detection without a GPU fault: every device-side wait is bounded.

The standalone IIR filter chains the tiles of a long row by a decoupled
look-back, where a tile waits for its predecessor's published state.  With
the poll limit lowered to a handful (pesq_iir_set_spin_limit), tiles whose
predecessor has not published yet give up: the call still returns, the
filter's error word reads nonzero (pesq_iir_check), and the next call with
the normal limit is correct again.  The PESQ plan's own error word (bulk
copies into shared memory that did not land in time) stays clear on normal
calls."""

import ctypes

import pytest
import torch

from triton_pesq_b200 import IIRCuda, PesqLossCuda, _lib
from triton_pesq_b200.signals import add_noise, speech_like
from triton_pesq_b200.tables import power_filter

pytestmark = pytest.mark.gpu


def test_iir_lookback_wait_runs_out_and_recovers(cuda_device):
    iir = IIRCuda(*power_filter())
    # one row of 600 tiles chained by the look-back (this filter's state dies
    # out within a tile's warm-up, so its long rows would otherwise run
    # overlapped tiles that never wait): every tile but the first waits for a
    # predecessor
    iir.force_lookback = True
    x = torch.randn(1, 600 * 8448, device=cuda_device, generator=torch.Generator(cuda_device).manual_seed(5))
    good = iir(x)
    assert iir.check_errors() == 0
    handle = iir._handle(cuda_device)
    lib = _lib.library()
    assert lib.pesq_iir_set_spin_limit(ctypes.c_void_p(handle), 1) == _lib.PESQ_OK
    try:
        iir(x)  # returns (no hang) although waits give up
        torch.cuda.synchronize()
        assert iir.check_errors() != 0
    finally:
        assert lib.pesq_iir_set_spin_limit(ctypes.c_void_p(handle), 1 << 21) == _lib.PESQ_OK
    again = iir(x)
    assert iir.check_errors() == 0  # the word was cleared by the check
    assert torch.equal(again, good)


def test_plan_error_word_clear_after_normal_calls(cuda_device):
    model = PesqLossCuda(1.0, sample_rate=16000)
    ref = speech_like(2, 40000, 16000, seed=3).to(cuda_device)
    deg = add_noise(ref.cpu(), 5.0, seed=4).to(cuda_device).requires_grad_(True)
    loss = model(ref, deg)
    torch.autograd.grad(loss.sum(), [deg])
    plan = model._plan(cuda_device)
    assert _lib.plan_check(plan, torch.cuda.current_stream().cuda_stream) == 0
