"""The allocation-free forward entry point against the regular one.

pesq_forward_noalloc exists for callers that cannot allocate device memory
when they evaluate (real-time audio callbacks, plugins whose host owns the
device memory, code inside a global-mode stream capture): it uses a static
device array as scratch instead of a caller workspace.  This file is collected
last so that a failure here never hides the other GPU tests; it also passes on
its own in a fresh process.
"""

import ctypes

import pytest
import torch

from triton_pesq_b200 import PesqLossCuda, _lib
from triton_pesq_b200.signals import add_noise, speech_like

pytestmark = pytest.mark.gpu


def _ptr(t):
    return ctypes.c_void_p(t.data_ptr())


def _noalloc(lib, plan, ref, deg):
    b, n = ref.shape
    outs = [torch.full((b,), float("nan"), device=ref.device) for _ in range(4)]
    stream = ctypes.c_void_p(torch.cuda.current_stream(ref.device).cuda_stream)
    status = lib.pesq_forward_noalloc(ctypes.c_void_p(plan), stream, _ptr(ref), ref.stride(0), _ptr(deg),
                                      deg.stride(0), b, n, *[_ptr(o) for o in outs])
    return status, outs


@pytest.mark.parametrize("sample_rate,samples", [(16000, 40000), (48000, 60000)])
def test_noalloc_forward_matches_pesq_forward(cuda_device, sample_rate, samples):
    """Same kernels, same inputs, same workspace layout: the outputs are
    bitwise those of pesq_forward with a caller workspace."""

    model = PesqLossCuda(0.5, sample_rate=sample_rate)
    plan = model._plan(cuda_device)
    lib = _lib.library()
    # two calls in a row with different batch sizes, lengths and signals: the
    # second must not see the first call's leftovers in the shared scratch
    for call, (batch, n, snr) in enumerate([(3, samples, 5.0), (2, samples - 7777, 20.0)]):
        ref = speech_like(batch, n, sample_rate, seed=100 + call).to(cuda_device)
        deg = add_noise(ref.cpu(), snr, seed=200 + call).to(cuda_device)
        status, got = _noalloc(lib, plan, ref, deg)
        assert status == _lib.PESQ_OK, _lib.last_error()
        want = torch.ops.pesq_cuda.forward(plan, ref, deg, 0)[:4]
        torch.cuda.synchronize()
        for g, w in zip(got, want):
            assert torch.equal(g, w)


@pytest.mark.parametrize("sample_rate,batch,samples", [(16000, 64, 128000), (48000, 4, 480000)])
def test_documented_capacity(cuda_device, sample_rate, batch, samples):
    """The capacity the header documents: 64 utterances of 8 s at 16 kHz and
    4 of 10 s at 48 kHz fit the 16 MiB array; the 48 kHz batch runs."""

    model = PesqLossCuda(1.0, sample_rate=sample_rate)
    plan = model._plan(cuda_device)
    lib = _lib.library()
    need = ctypes.c_size_t()
    assert lib.pesq_workspace_size(ctypes.c_void_p(plan), batch, samples, 0, ctypes.byref(need)) == _lib.PESQ_OK
    assert need.value <= 16 << 20
    if sample_rate == 48000:
        ref = speech_like(batch, samples, sample_rate, seed=7).to(cuda_device)
        deg = add_noise(ref.cpu(), 10.0, seed=8).to(cuda_device)
        status, got = _noalloc(lib, plan, ref, deg)
        assert status == _lib.PESQ_OK, _lib.last_error()
        want = torch.ops.pesq_cuda.forward(plan, ref, deg, 0)[:4]
        torch.cuda.synchronize()
        for g, w in zip(got, want):
            assert torch.equal(g, w)


def test_noalloc_rejects_batches_beyond_the_static_scratch(cuda_device):
    model = PesqLossCuda(1.0, sample_rate=16000)
    plan = model._plan(cuda_device)
    lib = _lib.library()
    ref = torch.zeros(256, 48000, device=cuda_device)  # needs ~19 MiB of scratch
    status, _ = _noalloc(lib, plan, ref, ref)
    assert status == _lib.PESQ_ERR_WORKSPACE
    assert "16 MiB" in _lib.last_error()
