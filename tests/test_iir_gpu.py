"""GPU parity of the standalone IIR filter (IIRCuda) against a float64
lfilter, following the reference's tests/test_triton_iir.py case by case:
forward and backward over both PESQ filters and both methods, adversarial and
badly scaled inputs, tiny lengths, tile and batch boundaries, long rows
(chained tiles), filter orders 1-16, other filter families, poles close to the
unit circle, determinism, aliasing, strided inputs, empty inputs, errors."""

import math

import numpy as np
import pytest
import torch
from scipy.signal import butter, cheby1, ellip

from iir_cases import (DEGENERATE, FILTERS, FLOOR, TOL, check_accuracy, exact, exact_vjp, noise, oracle32,
                       oracle32_vjp, peak_error, resonator)
from triton_pesq_b200 import IIRCuda
from triton_pesq_b200 import _lib
from triton_pesq_b200 import iir_design as D

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def modules(cuda_device):
    out = {}
    for name, (b, a) in FILTERS.items():
        for method in ("matmul", "scan"):
            out[(name, method)] = IIRCuda(b, a, chunk_size=128, method=method)
    yield out
    for m in out.values():
        assert m.check_errors() == 0


def _grad(module, signal, upstream):
    leaf = signal.clone().requires_grad_(True)
    return torch.autograd.grad(module(leaf), leaf, upstream)[0]


# ---------------------------------------------------------------------------
# forward parity
# ---------------------------------------------------------------------------


@pytest.mark.parametrize("name", list(FILTERS))
@pytest.mark.parametrize("method", ["matmul", "scan"])
@pytest.mark.parametrize("batch,samples", [(1, 16000), (4, 4097), (3, 100), (2, 129), (17, 1001), (2, 8448),
                                           (2, 8449), (3, 20000), (1, 16896 * 3 + 5)])
def test_forward_parity(modules, name, method, batch, samples):
    b, a = FILTERS[name]
    signal = noise(batch, samples, seed=batch * 1000 + samples)
    check_accuracy(modules[(name, method)](signal), oracle32(signal, b, a), exact(signal, b, a),
                   f"{name}/{method}/{batch}x{samples}")


@pytest.mark.parametrize("name", list(FILTERS))
@pytest.mark.parametrize("kind", ["zeros", "tiny", "huge", "level", "alternating", "impulse", "step", "last"])
def test_forward_adversarial(modules, name, kind):
    b, a = FILTERS[name]
    batch, samples = 2, 3000
    white = noise(batch, samples, seed=7)
    if kind == "zeros":
        signal = torch.zeros(batch, samples, device="cuda")
    elif kind == "tiny":
        signal = white * 1e-25
    elif kind == "huge":
        signal = white * 1e12
    elif kind == "level":
        signal = white * 3000.0
    elif kind == "alternating":
        sign = torch.where(torch.arange(samples, device="cuda") % 2 == 0, 1.0, -1.0).expand(batch, samples)
        signal = (white.abs() + 1.0) * sign
    elif kind == "impulse":
        signal = torch.zeros(batch, samples, device="cuda")
        signal[:, 13] = 1.0
    elif kind == "last":
        signal = torch.zeros(batch, samples, device="cuda")
        signal[:, -1] = 1.0
    else:
        signal = torch.ones(batch, samples, device="cuda")
    out = modules[(name, "matmul")](signal)
    assert torch.isfinite(out).all()
    assert peak_error(out, exact(signal, b, a)) < TOL


@pytest.mark.parametrize("samples", [1, 2, 3, 7, 15, 16, 17, 32, 33, 34, 63, 64, 65, 127, 129, 8447, 8448, 8449])
def test_forward_tiny_and_boundary_lengths(modules, samples):
    b, a = FILTERS["order10"]
    signal = noise(1, samples, seed=samples)
    assert peak_error(modules[("order10", "matmul")](signal), exact(signal, b, a)) < TOL


@pytest.mark.parametrize("batch", [1, 15, 16, 17, 31, 32, 33, 64, 255, 257])
def test_batch_sweep(modules, batch):
    """Rows are packed several to a tile; every row is filtered on its own."""

    b, a = FILTERS["order10"]
    signal = noise(batch, 777, seed=batch)
    out = modules[("order10", "matmul")](signal)
    assert peak_error(out, exact(signal, b, a)) < TOL
    assert (out.abs().amax(dim=1) > 0).all()


@pytest.mark.parametrize("lookback", [False, True])
def test_many_tiles_on_a_single_row(cuda_device, lookback):
    """480000 samples are 57 chained tiles of one row (test_triton_iir.py:916),
    or 65 overlapped ones."""

    b, a = FILTERS["order10"]
    module = IIRCuda(b, a)
    module.force_lookback = lookback
    signal = noise(2, 480000, seed=102)
    out = module(signal)
    assert torch.isfinite(out).all()
    assert peak_error(out, exact(signal, b, a)) < TOL


def test_very_long_row_deep_lookback(modules):
    """One row of 600 tiles: many CTAs in flight, so a tile often finds more
    than a look-back window of predecessors that have only published their
    aggregate; the result must not depend on it."""

    b, a = FILTERS["order2"]
    module = IIRCuda(b, a)
    module.force_lookback = True  # (this filter would run overlapped tiles)
    signal = noise(1, 8448 * 600 + 77, seed=5)
    out = module(signal)
    truth = exact(signal, b, a)
    assert peak_error(out, truth) < TOL
    again = module(signal)
    assert peak_error(again, truth) < TOL
    assert module.check_errors() == 0


def test_batch_beyond_the_grid_y_limit(modules):
    b, a = FILTERS["order2"]
    signal = noise(70000, 64, seed=101)
    out = modules[("order2", "matmul")](signal)
    torch.cuda.synchronize()
    assert torch.isfinite(out).all()
    tail = signal[-200:].contiguous()
    assert peak_error(out[-200:], exact(tail, b, a)) < TOL
    assert (out.abs().amax(dim=1) > 0).all()


# ---------------------------------------------------------------------------
# backward parity
# ---------------------------------------------------------------------------


@pytest.mark.parametrize("name", list(FILTERS))
@pytest.mark.parametrize("method", ["matmul", "scan"])
@pytest.mark.parametrize("batch,samples", [(1, 8000), (3, 2049), (20, 333), (2, 30001)])
def test_backward_parity(modules, name, method, batch, samples):
    b, a = FILTERS[name]
    signal = noise(batch, samples, seed=samples, scale=3000.0)
    upstream = noise(batch, samples, seed=samples + 1)
    mine = _grad(modules[(name, method)], signal, upstream)
    check_accuracy(mine, oracle32_vjp(signal, upstream, b, a), exact_vjp(signal, upstream, b, a),
                   f"{name}/{method}/{batch}x{samples} backward")
    assert (mine != 0).float().mean().item() > 0.99


@pytest.mark.parametrize("samples", [1, 5, 65, 127, 129, 8449])
def test_backward_tiny_lengths(modules, samples):
    b, a = FILTERS["order10"]
    signal = noise(2, samples, seed=samples + 500)
    upstream = noise(2, samples, seed=samples + 900)
    mine = _grad(modules[("order10", "matmul")], signal, upstream)
    assert peak_error(mine, exact_vjp(signal, upstream, b, a)) < TOL


def test_backward_is_the_reversed_filter(modules):
    module = modules[("order10", "matmul")]
    signal = noise(2, 1500, seed=11)
    upstream = noise(2, 1500, seed=12)
    mine = _grad(module, signal, upstream)
    manual = torch.flip(module(torch.flip(upstream, (1,)).contiguous()), (1,))
    # the same kernel on the same (reversed) data: identical bits
    assert torch.equal(mine, manual)


@pytest.mark.parametrize("method", ["matmul", "scan"])
def test_double_backward(modules, method):
    b, a = FILTERS["order10"]
    module = modules[("order10", method)]
    signal = noise(2, 1200, seed=41)
    upstream = noise(2, 1200, seed=42)
    probe = noise(2, 1200, seed=43)
    leaf = signal.clone().requires_grad_(True)
    cotangent = upstream.clone().requires_grad_(True)
    (first,) = torch.autograd.grad(module(leaf), leaf, cotangent, create_graph=True)
    (second,) = torch.autograd.grad((first * probe).sum(), cotangent)
    assert peak_error(second, exact(probe, b, a)) < TOL


def test_backward_through_a_strided_view(modules):
    b, a = FILTERS["order2"]
    leaf = noise(6, 4001, seed=23).requires_grad_(True)
    strided = leaf[1::2, ::3]
    assert not strided.is_contiguous()
    upstream = noise(*strided.shape, seed=24)
    mine = torch.autograd.grad(modules[("order2", "matmul")](strided), leaf, upstream)[0]
    exact_leaf = leaf.detach().double().cpu().requires_grad_(True)
    from oracle.pesq_oracle import lfilter

    want = torch.autograd.grad(lfilter(exact_leaf[1::2, ::3].contiguous(), b, a), exact_leaf,
                               upstream.double().cpu())[0]
    assert peak_error(mine, want) < TOL
    assert torch.equal(mine[0::2], torch.zeros_like(mine[0::2]))
    assert (mine[1::2, ::3] != 0).all()


def test_backward_of_a_zero_signal(modules):
    b, a = FILTERS["order10"]
    signal = torch.zeros(2, 2000, device="cuda")
    upstream = noise(2, 2000, seed=77)
    mine = _grad(modules[("order10", "matmul")], signal, upstream)
    assert torch.isfinite(mine).all()
    assert peak_error(mine, exact_vjp(signal, upstream, b, a)) < TOL


# ---------------------------------------------------------------------------
# determinism, aliasing, plumbing
# ---------------------------------------------------------------------------


def test_determinism(modules):
    module = modules[("order10", "matmul")]
    for shape in ((3, 7777), (2, 40000)):
        signal = noise(*shape, seed=17)
        upstream = noise(*shape, seed=18)
        assert torch.equal(module(signal), module(signal))
        assert torch.equal(_grad(module, signal, upstream), _grad(module, signal, upstream))


def test_interleaved_shapes_do_not_alias(modules):
    b, a = FILTERS["order10"]
    module = modules[("order10", "matmul")]
    first, second, third = noise(2, 1000, seed=31), noise(2, 1000, seed=32), noise(5, 43210, seed=33)
    alone = module(first)
    module(second)
    module(third)
    module(second)
    assert torch.equal(module(first), alone)
    assert peak_error(alone, exact(first, b, a)) < TOL
    assert peak_error(module(third), exact(third, b, a)) < TOL


@pytest.mark.parametrize("method", ["matmul", "scan"])
def test_output_is_fully_written(modules, method):
    module = modules[("order10", method)]
    for shape in ((3, 4001), (2, 30001)):
        signal = noise(*shape, seed=51)
        expected = module(signal).clone()
        torch.cuda.synchronize()
        poison = [torch.full_like(signal, float("nan")) for _ in range(8)]
        del poison
        again = module(signal)
        assert torch.isfinite(again).all()
        assert torch.equal(again, expected)


@pytest.mark.parametrize("samples", [2000, 30000])
def test_nan_does_not_cross_rows(modules, samples):
    """Short rows share a tile: the segmented scan must keep a NaN in its row."""

    module = modules[("order10", "matmul")]
    signal = noise(3, samples, seed=81)
    signal[1, 500] = float("nan")
    out = module(signal)
    assert torch.isfinite(out[0]).all()
    assert torch.isfinite(out[2]).all()
    assert torch.isnan(out[1, 500:]).any()
    assert torch.isfinite(out[1, :500]).all()


def test_non_contiguous_and_no_grad(modules):
    b, a = FILTERS["order2"]
    module = modules[("order2", "matmul")]
    wide = noise(3, 4000, seed=23)
    strided = wide[::2, ::2]
    assert peak_error(module(strided), exact(strided.contiguous(), b, a)) < TOL
    transposed = noise(2500, 4, seed=25).t()
    assert not transposed.is_contiguous()
    assert peak_error(module(transposed), exact(transposed.contiguous(), b, a)) < TOL
    with torch.no_grad():
        out = module(wide.clone().requires_grad_(True))
    assert not out.requires_grad
    assert not module(wide).requires_grad
    assert module(wide.clone().requires_grad_(True)).requires_grad


def test_batch_one_matches_batched(modules):
    module = modules[("order10", "matmul")]
    for samples in (3333, 20000):
        signal = noise(5, samples, seed=29)
        batched = module(signal)
        for row in range(signal.shape[0]):
            single = module(signal[row : row + 1].contiguous())
            assert peak_error(single[0], batched[row]) < FLOOR


def test_empty_inputs(modules):
    module = modules[("order2", "matmul")]
    assert module(torch.zeros(2, 0, device="cuda")).shape == (2, 0)
    assert module(torch.zeros(0, 1000, device="cuda")).shape == (0, 1000)
    leaf = torch.zeros(0, 1000, device="cuda", requires_grad=True)
    out = modules[("order10", "matmul")](leaf)
    grad = torch.autograd.grad(out, leaf, torch.zeros_like(out))[0]
    assert grad.shape == (0, 1000)


def test_rejects_bad_input(modules):
    module = modules[("order2", "matmul")]
    with pytest.raises(RuntimeError):
        module(torch.randn(2, 3, 4, device="cuda"))
    with pytest.raises(RuntimeError):
        module(torch.randn(2, 128, device="cuda", dtype=torch.float64))
    with pytest.raises(RuntimeError):
        module(torch.randn(2, 128))


def test_c_abi_tables_match_the_host_design(cuda_device):
    """The library derives its tables from (A, B, C, D) itself; its largest
    entries and structure agree with the Python scoring."""

    for b, a in list(FILTERS.values()) + list(DEGENERATE.values()):
        m = IIRCuda(b, a)
        handle = m._handle(cuda_device)
        info = _lib.iir_info(handle)
        tabs = m.design.tables()
        assert info.states == m.states and info.kernel_states == tabs.states
        assert bool(info.block_lower) == tabs.lower
        assert info.chunk == D.IIR_CHUNK and info.tile == D.IIR_TILE
        assert info.overlap == tabs.overlap == m.overlap
        assert math.isclose(info.largest32, tabs.largest32, rel_tol=1e-9)
        assert math.isclose(info.largest64, tabs.largest64, rel_tol=1e-9)


def test_scan_and_matmul_agree(modules):
    b, a = FILTERS["order10"]
    signal = noise(3, 2049, seed=161)
    truth = exact(signal, b, a)
    matmul = modules[("order10", "matmul")](signal)
    scan = modules[("order10", "scan")](signal)
    assert peak_error(matmul, truth) < TOL
    assert peak_error(scan, truth) < TOL
    assert peak_error(matmul, scan) < FLOOR


def test_tolerance_is_not_vacuous(modules):
    worst = 0.0
    for name, (b, a) in FILTERS.items():
        for method in ("matmul", "scan"):
            for batch, samples in ((1, 16000), (5, 4097)):
                signal = noise(batch, samples, seed=batch + samples)
                worst = max(worst, peak_error(modules[(name, method)](signal), exact(signal, b, a)))
    assert 0.0 < worst < TOL / 5.0, worst


# ---------------------------------------------------------------------------
# other filters
# ---------------------------------------------------------------------------


@pytest.mark.parametrize("name", list(DEGENERATE))
def test_degenerate_coefficients(cuda_device, name):
    b, a = DEGENERATE[name]
    module = IIRCuda(b, a, chunk_size=128)
    signal = noise(2, 3000, seed=sum(map(ord, name)) % 1000)
    out = module(signal)
    assert torch.isfinite(out).all()
    assert peak_error(out, exact(signal, b, a)) < TOL


def test_high_order_filter_is_not_silently_nan(cuda_device):
    b, a = butter(8, [200, 3800], fs=16000, btype="band")
    module = IIRCuda(b, a, chunk_size=128)
    assert module.states == 16
    signal = noise(2, 4000, seed=91)
    out = module(signal)
    assert torch.isfinite(out).all()
    assert peak_error(out, exact(signal, b, a)) < TOL


@pytest.mark.parametrize("order", [1, 2, 3, 4, 5, 6, 7, 9, 12, 16])
@pytest.mark.parametrize("method", ["matmul", "scan"])
def test_filter_order_sweep(cuda_device, order, method):
    if order == 1:
        b, a = butter(1, 3000, fs=16000)
    elif order % 2:
        b, a = butter(order, 3000, fs=16000, btype="low")
    else:
        b, a = butter(order // 2, [325, 3250], fs=16000, btype="band")
    module = IIRCuda(b, a, chunk_size=256, method=method)
    assert module.order == order
    signal = noise(2, 16000, seed=200 + order)
    upstream = noise(2, 16000, seed=300 + order)
    check_accuracy(module(signal), oracle32(signal, b, a), exact(signal, b, a), f"order{order} forward")
    mine = _grad(module, signal, upstream)
    assert peak_error(mine, exact_vjp(signal, upstream, b, a)) < TOL, f"order{order} backward"


def test_order_sixteen_is_accurate(cuda_device):
    b, a = butter(8, [325, 3250], fs=16000, btype="band")
    module = IIRCuda(b, a, chunk_size=256)
    assert module.states == 16 and module.basis == "cascade"
    signal = noise(2, 16000, seed=113)
    assert peak_error(module(signal), exact(signal, b, a)) < 2e-6


def test_order_twenty_runs(cuda_device):
    """The degraded order 20 band pass warns, and still runs (24-state kernel)."""

    b, a = butter(10, [325, 3250], fs=16000, btype="band")
    with pytest.warns(RuntimeWarning, match="degraded"):
        module = IIRCuda(b, a, chunk_size=128)
    assert module.states == 20 and module.padded == 20
    signal = noise(2, 20000, seed=114)
    err = peak_error(module(signal), exact(signal, b, a))
    assert err < 20 * module.score, (err, module.score)


@pytest.mark.parametrize("name,coeffs", [
    ("bp12", lambda: butter(6, [325, 3250], fs=16000, btype="band")),
    ("bp14", lambda: butter(7, [325, 3250], fs=16000, btype="band")),
    ("cheby1", lambda: cheby1(4, 1, [325, 3250], fs=16000, btype="band")),
    ("ellip", lambda: ellip(4, 1, 60, [325, 3250], fs=16000, btype="band")),
    ("cheby1_hi", lambda: cheby1(6, 1, [325, 3250], fs=16000, btype="band")),
])
def test_other_filter_families(cuda_device, name, coeffs):
    b, a = (np.asarray(c) for c in coeffs())
    module = IIRCuda(b, a, chunk_size=256)
    signal = noise(2, 16000, seed=sum(map(ord, name)) % 997)
    check_accuracy(module(signal), oracle32(signal, b, a), exact(signal, b, a), name)


@pytest.mark.parametrize("radius", [0.99, 0.999, 0.9999])
@pytest.mark.parametrize("samples", [16000, 300000])
def test_poles_close_to_the_unit_circle(cuda_device, radius, samples):
    b, a = resonator(radius)
    module = IIRCuda(b, a, chunk_size=256)
    signal = noise(2, samples, seed=int(radius * 1e4) + samples)
    check_accuracy(module(signal), oracle32(signal, b, a), exact(signal, b, a), f"r={radius} n={samples}")


def test_extreme_pole(cuda_device):
    """Radius 0.99999 over 480000 samples: the reference documents 4.4e-5 here
    (test_triton_iir.py:1073-1096); the float64 tile chaining keeps the CUDA
    filter within the usual tolerance."""

    b, a = resonator(0.99999)
    module = IIRCuda(b, a, chunk_size=256)
    signal = noise(2, 480000, seed=131)
    truth = exact(signal, b, a)
    out = module(signal)
    assert torch.isfinite(out).all()
    ours, theirs = peak_error(out, truth), peak_error(oracle32(signal, b, a), truth)
    assert ours < TOL, ours
    assert ours < theirs / 10.0, (ours, theirs)


@pytest.mark.parametrize("exponent", [-30, -35, -38])
def test_denormal_scale_inputs(cuda_device, exponent):
    b, a = FILTERS["order10"]
    module = IIRCuda(b, a, chunk_size=128)
    unit = noise(2, 2000, seed=141)
    scale = float(10.0**exponent)
    small = module(unit * scale)
    assert torch.isfinite(small).all()
    tolerance = TOL if exponent >= -35 else 1e-5 * 10.0 ** (-35 - exponent)
    assert peak_error(small, exact(unit * scale, b, a)) < tolerance


def test_subnormal_input_does_not_produce_nan(cuda_device):
    b, a = FILTERS["order10"]
    out = IIRCuda(b, a, chunk_size=128)(noise(2, 2000, seed=142) * 1e-42)
    assert torch.isfinite(out).all()


@pytest.mark.parametrize("shape,lookback", [((3, 20000), False), ((3, 20000), True), ((40, 700), False)])
def test_cuda_graph_replay(cuda_device, shape, lookback):
    """Captured in a CUDA graph (chained tiles: the workspace reset is a memset
    node of the graph), replayed on new inputs, bitwise equal to eager calls."""

    module = IIRCuda(*FILTERS["order10"])
    module.force_lookback = lookback
    static = noise(*shape, seed=7)
    module(static)  # plan and kernel set-up outside the capture
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        out = module(static)
    for seed in (8, 9):
        fresh = noise(*shape, seed=seed)
        static.copy_(fresh)
        graph.replay()
        torch.cuda.synchronize()
        assert torch.equal(out, module(fresh))
    assert module.check_errors() == 0


def _spread(order: int, radius: float = 0.85):
    """Order `order` filter with poles of one radius spread over the band and
    zeros on the unit circle beside them (well conditioned in every basis)."""

    th = np.linspace(0.15, 2.9, order // 2)
    poles = np.concatenate([radius * np.exp(1j * th), radius * np.exp(-1j * th)])
    zeros = np.concatenate([np.exp(1j * (th + 0.07)), np.exp(-1j * (th + 0.07))])
    return np.poly(zeros).real / order, np.poly(poles).real


WIDE = {
    "lp20": (lambda: butter(20, 3000, fs=16000), 20),
    "lp23": (lambda: butter(23, 3000, fs=16000), 24),
    "lp24": (lambda: butter(24, 3000, fs=16000), 24),
    "bp22": (lambda: butter(11, [325, 3250], fs=16000, btype="band"), 24),
    "spread20": (lambda: _spread(20), 20),
    "spread24": (lambda: _spread(24), 24),
}


@pytest.mark.parametrize("name,dense", [(name, False) for name in WIDE] +
                         [(name, True) for name in WIDE if name.startswith("spread")])
@pytest.mark.parametrize("method", ["matmul", "scan"])
def test_widest_kernels(cuda_device, name, dense, method):
    """The 20- and 24-state kernel instantiations, block lower (the selected
    cascade) and dense (the same realisation in a random orthonormal basis),
    both output forms, forward and adjoint, chained rows: within a small
    multiple of the error the float32 emulation of the kernel predicts.  The
    high order low passes only have an accurate block lower realisation (any
    dense basis mixes their unbalanced states), so the dense kernels run on
    the well conditioned `spread` filters."""

    import dataclasses
    import warnings

    coeffs, states = WIDE[name]
    b, a = (np.asarray(c) for c in coeffs())
    with warnings.catch_warnings():
        warnings.simplefilter("ignore", RuntimeWarning)
        design = D.design(b, a)
    if dense:
        n = design.trans.shape[0]
        q = np.linalg.qr(np.random.default_rng(n).standard_normal((n, n)))[0]
        design = dataclasses.replace(design, trans=q.T @ design.trans @ q, input=q.T @ design.input,
                                     output=design.output @ q, basis="dense")
    tabs = design.tables()
    assert tabs.states == states and tabs.lower == (not dense)
    bound = max(TOL, 4 * D.emulated_error(tabs, b, a))
    signal = noise(2, 20000, seed=len(name) + states)
    upstream = noise(2, 20000, seed=7 + states)
    flags = _lib.IIR_RERUN if method == "scan" else 0
    handle = _lib.create_iir(design)
    try:
        out = torch.ops.pesq_cuda.iir(handle, signal, flags)
        grad = torch.ops.pesq_cuda.iir(handle, upstream, flags | _lib.IIR_REVERSE)
        assert _lib.iir_check(handle, torch.cuda.current_stream().cuda_stream) == 0
    finally:
        torch.cuda.synchronize()
        _lib.destroy_iir(handle)
    assert peak_error(out, exact(signal, b, a)) < bound
    assert peak_error(grad, exact_vjp(signal, upstream, b, a)) < bound


@pytest.mark.parametrize("method", ["matmul", "scan"])
def test_overlapped_tiles_agree_with_the_lookback(cuda_device, method):
    """Long rows of a filter whose state dies out within a tile's warm-up run
    overlapped tiles (no waits); they agree with the look-back chaining and
    with float64 lfilter, forward and reversed, at lengths that end inside
    the first, a middle and the last warm-up."""

    b, a = FILTERS["order10"]
    module = IIRCuda(b, a, method=method)
    assert module.overlap == 32 * D.IIR_CHUNK  # the overlapped path runs (not vacuous)
    step = D.IIR_TILE - module.overlap
    for n in (D.IIR_TILE + 1, 3 * step + 17, 7 * step + module.overlap - 3):
        x = noise(3, n, seed=n)
        truth = exact(x, b, a)
        for reverse in (False, True):
            module.force_lookback = False
            ovl = module._launch(x, reverse)
            module.force_lookback = True
            chained = module._launch(x, reverse)
            want = exact(x.flip(-1), b, a).flip(-1) if reverse else truth
            assert peak_error(ovl, want) < TOL
            assert peak_error(ovl, chained) < FLOOR
    module.force_lookback = False
