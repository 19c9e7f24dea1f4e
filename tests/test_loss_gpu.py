"""End-to-end parity of PesqLossCuda on the GPU against the float64 oracle
and the golden vectors of the reference (mirrors the reference's
tests/test_triton_loss.py)."""

import glob
import os

import numpy as np
import pytest
import torch

from conftest import GOLDEN, golden_geometry
from gpu_helpers import F64_RTOL, GRAD_RTOL, oracle_grads, peak_rel_err, rel_err
from triton_pesq_b200 import PesqLossCuda
from triton_pesq_b200.signals import add_noise, speech_like

pytestmark = pytest.mark.gpu

CASES = sorted(glob.glob(os.path.join(GOLDEN, "sr*.npz")))


def _grads(model, ref, deg, which=(True, True)):
    r = ref.detach().clone().requires_grad_(which[0])
    d = deg.detach().clone().requires_grad_(which[1])
    loss = model(r, d)
    inputs = [t for t in (r, d) if t.requires_grad]
    grads = torch.autograd.grad(loss.sum(), inputs)
    return loss, grads


@pytest.mark.parametrize("path", CASES, ids=[os.path.basename(c)[:-4] for c in CASES])
def test_golden_vectors(cuda_device, path):
    """Distances and gradients against the reference's own float64 pipeline
    (default and other frame geometries: n_fft 64..4096, hops shorter and
    longer than the frame, a window shorter than n_fft)."""

    z = np.load(path)
    factor, sr = float(z["factor"]), int(z["sample_rate"])
    model = PesqLossCuda(factor, sample_rate=sr, **golden_geometry(z))
    ref = torch.from_numpy(z["ref"]).to(cuda_device)
    deg = torch.from_numpy(z["deg"]).to(cuda_device)
    ds, da = model.raw(ref, deg)
    assert rel_err(ds.cpu(), z["f64_d_symm"]) < F64_RTOL
    assert rel_err(da.cpu(), z["f64_d_asymm"]) < F64_RTOL
    _, (g_ref, g_deg) = _grads(model, ref, deg)
    assert peak_rel_err(g_ref.cpu(), z["f64_grad_ref"]) < GRAD_RTOL
    assert peak_rel_err(g_deg.cpu(), z["f64_grad_deg"]) < GRAD_RTOL


@pytest.mark.parametrize(
    "batch,samples,sample_rate,snr",
    [(1, 16000, 16000, 10.0), (4, 16000, 16000, 0.0), (3, 20000, 16000, 20.0), (2, 48000, 48000, 10.0),
     (2, 44100, 44100, 5.0), (8, 32000, 16000, 15.0), (2, 24000, 22050, 10.0), (2, 8000, 8000, 10.0)],
)
def test_matches_float64(cuda_device, batch, samples, sample_rate, snr):
    ref = speech_like(batch, samples, sample_rate, seed=batch + samples)
    deg = add_noise(ref, snr, seed=samples)
    ds64, da64, gr64, gd64 = oracle_grads(ref, deg, 1.0, sample_rate)
    model = PesqLossCuda(1.0, sample_rate=sample_rate)
    ref, deg = ref.to(cuda_device), deg.to(cuda_device)
    ds, da = model.raw(ref, deg)
    assert rel_err(ds.cpu(), ds64) < F64_RTOL
    assert rel_err(da.cpu(), da64) < F64_RTOL
    _, (g_ref, g_deg) = _grads(model, ref, deg)
    assert peak_rel_err(g_ref.cpu(), gr64) < GRAD_RTOL
    assert peak_rel_err(g_deg.cpu(), gd64) < GRAD_RTOL


GEOMETRIES = [  # n_fft, hop_length, win_length
    (256, 128, 256), (1024, 256, 1024), (128, 100, 96), (32, 16, 32), (2048, 512, 2048),
    (512, 128, 512), (512, 300, 512), (512, 256, 320), (256, 512, 256),
]
GEOMETRY_CASES = ([g + (3, 20000, 16000) for g in GEOMETRIES] + [g + (2, 33075, 44100) for g in GEOMETRIES] +
                  [(4096, 512, 3000, 2, 20000, 16000), (4096, 1024, 4096, 1, 96000, 48000),
                   # 8 x 8 s at hop 128: T = 999, the chain backward stages its slices
                   # but reads the forward's coefficients from L2
                   (512, 128, 512, 8, 128000, 16000)])


@pytest.mark.parametrize("n_fft,hop,win,batch,samples,sample_rate", GEOMETRY_CASES)
def test_frame_geometries(cuda_device, n_fft, hop, win, batch, samples, sample_rate):
    """PesqLoss(..., win_length, n_fft, hop_length) with the spectrum kernels
    (every geometry but 512 / 256) and the fused path with a shorter window:
    distances and both gradients against the float64 oracle."""

    geometry = dict(n_fft=n_fft, hop_length=hop, win_length=win)
    ref = speech_like(batch, samples, sample_rate, seed=n_fft + hop + batch)
    deg = add_noise(ref, 8.0, seed=win)
    ds64, da64, gr64, gd64 = oracle_grads(ref, deg, 1.0, sample_rate, **geometry)
    model = PesqLossCuda(1.0, sample_rate=sample_rate, **geometry)
    ref, deg = ref.to(cuda_device), deg.to(cuda_device)
    ds, da = model.raw(ref, deg)
    assert rel_err(ds.cpu(), ds64) < F64_RTOL
    assert rel_err(da.cpu(), da64) < F64_RTOL
    _, (g_ref, g_deg) = _grads(model, ref, deg)
    assert peak_rel_err(g_ref.cpu(), gr64) < GRAD_RTOL
    assert peak_rel_err(g_deg.cpu(), gd64) < GRAD_RTOL
    # one-sided gradients agree with the two-sided ones
    _, (g_deg_only,) = _grads(model, ref, deg, which=(False, True))
    assert torch.equal(g_deg_only, g_deg)


def test_frame_geometry_graph_replay_is_bit_exact(cuda_device):
    """The spectrum kernels are deterministic and capturable: a graphed step
    replays bitwise equal to the eager one."""

    ref = speech_like(2, 16000, 16000, seed=5).to(cuda_device).requires_grad_(True)
    deg = add_noise(ref.detach().cpu(), 5.0, seed=6).to(cuda_device).requires_grad_(True)
    model = PesqLossCuda(1.0, sample_rate=16000, n_fft=256, hop_length=128, win_length=256)
    eager = model(ref, deg)
    eager_grads = torch.autograd.grad(eager.sum(), [ref, deg])
    graphed = model.graphed(ref, deg)
    for _ in range(2):
        captured = graphed(ref, deg)
        captured_grads = torch.autograd.grad(captured.sum(), [ref, deg])
        assert torch.equal(captured, eager)
        for want, got in zip(eager_grads, captured_grads):
            assert torch.equal(got, want)


@pytest.mark.parametrize("n_fft", [40, 48, 96, 1000, 16, 8192])
def test_rejects_unsupported_n_fft(n_fft):
    with pytest.raises(ValueError):
        PesqLossCuda(1.0, sample_rate=16000, n_fft=n_fft, win_length=min(n_fft, 16))


def test_outputs_are_consistent(cuda_device):
    ref = speech_like(3, 16000, 16000, seed=3).to(cuda_device)
    deg = add_noise(ref.cpu(), 8.0, seed=4).to(cuda_device)
    model = PesqLossCuda(0.5, sample_rate=16000)
    ds, da = model.raw(ref, deg)
    loss = model(ref, deg)
    mos = model.mos(ref, deg)
    torch.testing.assert_close(loss, 0.5 * (0.1 * ds + 0.0309 * da), rtol=1e-6, atol=1e-7)
    m = 4.5 - 0.1 * ds - 0.0309 * da
    torch.testing.assert_close(mos, 0.999 + 4 / (1 + torch.exp(-1.3669 * m + 3.8224)), rtol=1e-6, atol=1e-6)
    assert torch.all(loss > 0) and torch.all(mos > 1.0) and torch.all(mos < 5.0)


def test_identical_signals(cuda_device):
    ref = speech_like(3, 16000, 16000, seed=11).to(cuda_device)
    loss = PesqLossCuda(1.0, sample_rate=16000)(ref, ref)
    assert torch.all(loss >= 0.0) and torch.all(loss <= 1e-6)


def test_deterministic(cuda_device):
    ref = speech_like(4, 16000, 16000, seed=19).to(cuda_device)
    deg = add_noise(ref.cpu(), 5.0, seed=20).to(cuda_device)
    model = PesqLossCuda(1.0, sample_rate=16000)
    l1, g1 = _grads(model, ref, deg)
    l2, g2 = _grads(model, ref, deg)
    assert torch.equal(l1, l2)
    for a, b in zip(g1, g2):
        assert torch.equal(a, b)


def test_batch_independence(cuda_device):
    ref = speech_like(4, 16000, 16000, seed=23).to(cuda_device)
    deg = add_noise(ref.cpu(), 5.0, seed=24).to(cuda_device)
    model = PesqLossCuda(1.0, sample_rate=16000)
    batched = model(ref, deg)
    single = torch.cat([model(ref[i : i + 1], deg[i : i + 1]) for i in range(4)])
    torch.testing.assert_close(batched, single, rtol=0, atol=0)


def test_non_contiguous_input(cuda_device):
    ref = speech_like(4, 32000, 16000, seed=29).to(cuda_device)
    deg = add_noise(ref.cpu(), 5.0, seed=30).to(cuda_device)
    model = PesqLossCuda(1.0, sample_rate=16000)
    sr, sd = ref[:, ::2], deg[:, ::2]
    assert not sr.is_contiguous()
    torch.testing.assert_close(model(sr, sd), model(sr.contiguous(), sd.contiguous()))
    # strided rows (a column slice) go straight through the row stride
    torch.testing.assert_close(model(ref[:, :20000], deg[:, :20000]),
                               model(ref[:, :20000].contiguous(), deg[:, :20000].contiguous()))


def test_one_dimensional_input(cuda_device):
    ref = speech_like(1, 16000, 16000, seed=31).to(cuda_device)
    deg = add_noise(ref.cpu(), 5.0, seed=32).to(cuda_device)
    model = PesqLossCuda(1.0, sample_rate=16000)
    torch.testing.assert_close(model(ref[0], deg[0]), model(ref, deg))


def test_errors(cuda_device):
    model = PesqLossCuda(1.0, sample_rate=16000)
    ref = torch.randn(2, 16000, device=cuda_device)
    with pytest.raises(ValueError):
        model(ref, torch.randn(2, 15000, device=cuda_device))
    with pytest.raises(ValueError):  # fewer than 20 frames
        model(ref[:, :4000], ref[:, :4000])
    with pytest.raises(RuntimeError):
        model(ref.cpu(), ref.cpu())
    with pytest.raises(RuntimeError):
        model(ref.double(), ref.double())


def test_gradient_only_for_requested_inputs(cuda_device):
    ref = speech_like(2, 16000, 16000, seed=5).to(cuda_device)
    deg = add_noise(ref.cpu(), 5.0, seed=6).to(cuda_device)
    model = PesqLossCuda(1.0, sample_rate=16000)
    _, (g_deg_only,) = _grads(model, ref, deg, (False, True))
    _, (g_ref_only,) = _grads(model, ref, deg, (True, False))
    _, (g_ref, g_deg) = _grads(model, ref, deg)
    assert torch.equal(g_deg_only, g_deg)
    assert torch.equal(g_ref_only, g_ref)


def test_upstream_gradients(cuda_device):
    """Broadcast upstream gradients (sum / mean over the batch, passed as one
    shared value) match the same values given as full arrays, and gradients
    through several outputs add up."""

    ref = speech_like(3, 16000, 16000, seed=45).to(cuda_device)
    deg = add_noise(ref.cpu(), 6.0, seed=46).to(cuda_device).requires_grad_(True)
    model = PesqLossCuda(0.5, sample_rate=16000)
    loss = model(ref, deg)
    (g_sum,) = torch.autograd.grad(loss.sum(), [deg])
    loss = model(ref, deg)
    (g_arr,) = torch.autograd.grad(loss, [deg], grad_outputs=torch.ones(3, device=cuda_device))
    assert torch.equal(g_sum, g_arr)
    loss = model(ref, deg)
    (g_mean,) = torch.autograd.grad(loss.mean(), [deg])
    torch.testing.assert_close(g_mean, g_arr / 3, rtol=1e-5, atol=1e-6 * float(g_arr.abs().max()))
    w = torch.tensor([0.5, -2.0, 1.5], device=cuda_device)
    loss = model(ref, deg)
    (g_w,) = torch.autograd.grad((w * loss).sum(), [deg])
    for i in range(3):
        torch.testing.assert_close(g_w[i], w[i] * g_arr[i], rtol=1e-5, atol=1e-6 * float(g_arr.abs().max()))
    # dL/dmos and dL/dloss together: mos = f(0.1 ds + 0.0309 da) = f(loss / factor)
    ds, da = model.raw(ref, deg.detach())
    m = 4.5 - 0.1 * ds - 0.0309 * da
    dmos_dloss = -4 * 1.3669 * torch.exp(-1.3669 * m + 3.8224) / (1 + torch.exp(-1.3669 * m + 3.8224)) ** 2 / 0.5
    _, _, mos, loss, _ = model._evaluate(ref, deg)  # one call, two differentiated outputs
    (g_both,) = torch.autograd.grad((mos + loss).sum(), [deg])
    want = g_arr * (1.0 + dmos_dloss)[:, None]
    torch.testing.assert_close(g_both, want, rtol=1e-4, atol=1e-4 * float(want.abs().max()))


def test_cuda_graph_is_bit_exact(cuda_device):
    ref = speech_like(2, 16000, 16000, seed=43).to(cuda_device).requires_grad_(True)
    deg = add_noise(ref.detach().cpu(), 5.0, seed=44).to(cuda_device).requires_grad_(True)
    model = PesqLossCuda(1.0, sample_rate=16000)
    eager = model(ref, deg)
    eager_grads = torch.autograd.grad(eager.sum(), [ref, deg])
    graphed = model.graphed(ref, deg)
    captured = graphed(ref, deg)
    captured_grads = torch.autograd.grad(captured.sum(), [ref, deg])
    assert torch.equal(captured, eager)
    for want, got in zip(eager_grads, captured_grads):
        assert torch.equal(got, want)


@pytest.mark.parametrize("sample_rate,seconds", [(48000, 12.0), (16000, 15.0), (16000, 30.0)])
def test_long_signal(cuda_device, sample_rate, seconds):
    n = int(sample_rate * seconds)
    ref = speech_like(1, n, sample_rate, seed=41)
    deg = add_noise(ref, 8.0, seed=42)
    ds64, da64, _, gd64 = oracle_grads(ref, deg, 1.0, sample_rate)
    model = PesqLossCuda(1.0, sample_rate=sample_rate)
    ds, da = model.raw(ref.to(cuda_device), deg.to(cuda_device))
    assert rel_err(ds.cpu(), ds64) < F64_RTOL
    assert rel_err(da.cpu(), da64) < F64_RTOL
    _, (g_deg,) = _grads(model, ref.to(cuda_device), deg.to(cuda_device), (False, True))
    assert peak_rel_err(g_deg.cpu(), gd64) < GRAD_RTOL


def test_batch_beyond_grid_y(cuda_device):
    """33000 utterance pairs (66000 rows, more than a grid dimension y
    holds) at 8 kHz through the resampler: rows on either side of the 65535
    boundary get exactly what they get in a batch of their own (the
    reference folds the batch onto grid x for the same reason,
    triton_ops/resample.py:40-47)."""

    batch, n = 33000, 2700
    gen = torch.Generator(device=cuda_device).manual_seed(91)
    ref = torch.randn(batch, n, device=cuda_device, generator=gen)
    deg = (ref + 0.3 * torch.randn(batch, n, device=cuda_device, generator=gen)).requires_grad_(True)
    model = PesqLossCuda(1.0, sample_rate=8000)
    loss = model(ref, deg)
    (g,) = torch.autograd.grad(loss.sum(), [deg])
    for rows in ([0, 1], [32766, 32767, 32768], [batch - 2, batch - 1]):
        r, d = ref[rows], deg.detach()[rows].clone().requires_grad_(True)
        alone = model(r, d)
        (g_alone,) = torch.autograd.grad(alone.sum(), [d])
        assert torch.equal(alone, loss[rows])
        assert torch.equal(g_alone, g[rows])


@pytest.mark.parametrize("batch", [1, 5, 40])
def test_loss_sum_of_the_chain_kernel(cuda_device, batch):
    """forward_sum's [sum, count] pair (summed by the chain forward's last
    cluster, in a fixed order) against the losses it returns; bitwise the
    same on a repeat call, and inside a CUDA graph replay."""

    ref = speech_like(batch, 8000, 16000, seed=95 + batch).to(cuda_device)
    deg = add_noise(ref.cpu(), 7.0, seed=96).to(cuda_device)
    model = PesqLossCuda(0.5, sample_rate=16000)
    loss, pair = model.forward_sum(ref, deg)
    assert pair.dtype == torch.float64 and pair.shape == (2,)
    assert float(pair[1]) == batch
    assert float(pair[0]) == pytest.approx(float(loss.double().sum()), rel=1e-12)
    loss2, pair2 = model.forward_sum(ref, deg)
    assert torch.equal(pair2, pair) and torch.equal(loss2, loss)
    d = deg.clone().requires_grad_(True)
    static = {}

    def step():
        out, s = model.forward_sum(ref, d)
        static["pair"] = s
        return out

    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        step()
    torch.cuda.current_stream().wait_stream(side)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        step()
    g.replay()
    torch.cuda.synchronize()
    assert torch.equal(static["pair"], pair)


def test_second_device_from_the_autograd_thread(cuda_device):
    """A plan on cuda:1 while cuda:0 is current: the forward and the backward
    (run by autograd's worker thread for that device) use the plan's device,
    and the results equal those of cuda:0 bit for bit (the reference binds
    the context for its autograd thread, triton_ops/iir.py:945-963)."""

    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    ref = speech_like(2, 16000, 16000, seed=97)
    deg = add_noise(ref, 6.0, seed=98)
    model = PesqLossCuda(1.0, sample_rate=16000)
    out = {}
    for index in (0, 1):
        dev = torch.device("cuda", index)
        r, d = ref.to(dev), deg.to(dev).requires_grad_(True)
        with torch.cuda.device(0):  # the current device stays cuda:0
            loss = model(r, d)
            loss.sum().backward()
        out[index] = (loss.detach().cpu(), d.grad.cpu())
    assert torch.equal(out[0][0], out[1][0])
    assert torch.equal(out[0][1], out[1][1])


def test_backward_after_the_module_is_dropped(cuda_device):
    """The autograd graph keeps the plan alive: a module evaluated once and
    dropped (its plan released with it otherwise) still runs its backward,
    and so does a dropped resampler's double backward."""
    import gc

    from triton_pesq_b200 import ResampleCuda

    ref = speech_like(2, 16000, 16000, seed=91).to(cuda_device)
    deg = add_noise(ref.cpu(), 5.0, seed=92).to(cuda_device).requires_grad_(True)
    keep = PesqLossCuda(1.0, sample_rate=16000)
    want = keep(ref, deg)
    (g_want,) = torch.autograd.grad(want.sum(), [deg])
    loss = PesqLossCuda(1.0, sample_rate=16000)(ref, deg)
    gc.collect()
    (g,) = torch.autograd.grad(loss.sum(), [deg])
    assert torch.equal(loss, want)
    assert torch.equal(g, g_want)

    x = torch.randn(2, 4410, device=cuda_device, requires_grad=True)
    rs = ResampleCuda(44100, 16000)
    y_want = rs(x)
    (gx_want,) = torch.autograd.grad(y_want.square().sum(), [x], create_graph=True)
    (ggx_want,) = torch.autograd.grad(gx_want.sum(), [x])
    y = ResampleCuda(44100, 16000)(x)
    gc.collect()
    (gx,) = torch.autograd.grad(y.square().sum(), [x], create_graph=True)
    gc.collect()
    (ggx,) = torch.autograd.grad(gx.sum(), [x])
    assert torch.equal(y, y_want)
    assert torch.equal(gx, gx_want)
    assert torch.equal(ggx, ggx_want)
