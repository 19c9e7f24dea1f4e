"""Host side of the standalone IIR filter: realisation selection and scoring
(iir_design.py against the reference's iir.py:187-599 and its tests in
test_triton_iir.py:745-885), constructor validation.  No GPU needed."""

import math
import warnings

import numpy as np
import pytest
from scipy.signal import butter, cheby1, ellip

from iir_cases import DEGENERATE, FILTERS
from triton_pesq_b200 import iir_design as D
from triton_pesq_b200.iir import IIRCuda

EXTRA = {
    "resonant": (np.array([1.0, 0.0, 0.0, 0.0, 0.0]),
                 np.poly([0.999 * np.exp(1j * 0.30), 0.999 * np.exp(-1j * 0.30), 0.999 * np.exp(1j * 0.31),
                          0.999 * np.exp(-1j * 0.31)]).real),
    "narrow": tuple(np.asarray(c) for c in butter(3, [0.01, 0.02], btype="band")),
    "cheby1": tuple(np.asarray(c) for c in cheby1(4, 1, [325, 3250], fs=16000, btype="band")),
    "ellip": tuple(np.asarray(c) for c in ellip(4, 1, 60, [325, 3250], fs=16000, btype="band")),
    "bp16": tuple(np.asarray(c) for c in butter(8, [325, 3250], fs=16000, btype="band")),
    "lp24": tuple(np.asarray(c) for c in butter(24, 3000, fs=16000)),
}
ALL = {**FILTERS, **DEGENERATE, **EXTRA}


def test_pesq_filters_pick_the_cascade():
    """The order 10 band pass must not end up in the companion basis, whose
    powers reach 1e4 (iir.py:36-52); both PESQ filters select the cascade."""

    for name in FILTERS:
        d = D.design(*FILTERS[name])
        assert d.basis == "cascade", name
        assert d.score < 1e-6, (name, d.score)
    d = D.design(*FILTERS["order10"])
    assert d.states == 10 and d.order == 10
    assert d.candidates["companion"][0] > 1e-3  # the companion form loses float32
    tabs = d.tables()
    assert tabs.lower and tabs.states == 10
    assert tabs.largest32 < 1e2


@pytest.mark.parametrize("name", list(ALL))
def test_realisation_reproduces_the_difference_equation(name):
    """The selected realisation reproduces the difference equation's impulse
    response in float64 to within its score (the fidelity part of the score
    is exactly this error; for clustered poles, as the narrow band pass, it
    is the root finding of tf2sos that limits it), and the score is small."""

    b, a = ALL[name]
    b, a = D.as_coeffs(b), D.as_coeffs(a)
    truth = D.direct_response(b, a, 2000)
    scale = np.abs(truth).max()
    built = [("companion", D.companion(b, a))]
    comp = built[0][1]
    built.append(("modal", D.modal(*comp)))
    built.append(("cascade", D.cascade(b, a)))
    chosen = D.design(b, a)
    for label, real in built:
        if real is None:
            continue
        got = D.realised_response(*real, 2000)
        err = np.abs(got - truth).max() / scale
        if label == chosen.basis:
            assert err <= chosen.score * (1 + 1e-9), (label, err, chosen.score)
    assert chosen.score < D.ERROR_WARN  # none of these filters is degraded


@pytest.mark.parametrize("name", list(ALL))
def test_conditioning_covers_every_table(name):
    """The scored table entry bounds every float32 table the kernel multiplies
    data with (test_triton_iir.py:768-823); the impulse response, a property
    of the filter rather than of the realisation, is not scored."""

    d = D.design(*ALL[name])
    tabs = d.tables()
    largest = max(np.abs(t).max() for t in (tabs.carry, tabs.drive, tabs.steps, tabs.lanes, tabs.warp_powers,
                                            tabs.trans, tabs.input, tabs.output))
    assert d.entry >= largest * (1.0 - 1e-12)
    assert d.score >= D.emulated_error(tabs, *ALL[name]) * (1.0 - 1e-12)


@pytest.mark.parametrize("name", ["order2", "order10", "lp24", "bp16"])
@pytest.mark.parametrize("samples", [100, D.IIR_TILE, D.IIR_TILE + 4321, 2 * D.IIR_TILE])
def test_emulation_in_float64_is_the_filter(name, samples):
    """The kernel emulation that scores the realisations computes the filter:
    in float64 arithmetic it agrees with the realisation's own recursion to
    rounding, in both output
    forms, over one and two tiles (so its float32 error is rounding alone)."""

    d = D.design(*ALL[name])
    x = np.random.default_rng(samples).standard_normal(samples)
    truth, state = np.empty(samples), np.zeros(d.trans.shape[0])
    for k in range(samples):  # the realisation's own recursion
        truth[k] = d.output @ state + d.feed * x[k]
        state = d.trans @ state + d.input * x[k]
    for y in D.emulate(d.tables(), x, dtype=np.float64):
        assert np.abs(y - truth).max() <= 1e-9 * np.abs(truth).max()


def test_high_order_low_pass_avoids_the_companion_form():
    """The companion form of an order 24 low pass has small table entries
    yet loses every digit in float32; the emulated error sees it and the
    cascade (large entries, seven digits) is taken."""

    d = D.design(*EXTRA["lp24"])
    assert d.basis == "cascade" and d.score < D.ERROR_WARN
    assert d.candidates["companion"][0] > 0.1
    assert d.candidates["companion"][1] < d.candidates["cascade"][1]


@pytest.mark.parametrize("name", list(DEGENERATE))
def test_degenerate_coefficients_have_a_realisation(name):
    """Defective companion matrices have no modal basis; the selection falls
    back instead of raising (test_triton_iir.py:826-840)."""

    d = D.design(*DEGENERATE[name])
    assert d.score < 1e-5
    assert math.isfinite(d.entry)


def test_order_sixteen_picks_the_accurate_realisation():
    """Fidelity counts, not conditioning alone (test_triton_iir.py:1001-1033)."""

    d = D.design(*EXTRA["bp16"])
    assert d.states == 16 and d.basis == "cascade"
    assert d.candidates["modal"][0] > d.candidates["cascade"][0]


def test_unrepresentable_filter_raises():
    b, a = butter(15, [325, 3250], fs=16000, btype="band")
    with pytest.raises(RuntimeError, match="realisation"):
        D.design(b, a)


def test_degraded_filter_warns():
    b, a = butter(10, [325, 3250], fs=16000, btype="band")
    with pytest.warns(RuntimeWarning, match="degraded"):
        D.design(b, a)


def test_kernel_tables_are_consistent():
    """h[t] = C A^(t-1) B, the chunk step is A^33, the lane table its powers,
    the warp powers those of A^(32*33) and the look-back table those of A^8448."""

    d = D.design(*FILTERS["order10"])
    t = d.tables()
    A, B, C = t.trans, t.input, t.output
    step = np.linalg.matrix_power(A, D.IIR_CHUNK)
    np.testing.assert_allclose(t.steps[0], step, rtol=1e-12, atol=1e-15)
    np.testing.assert_allclose(t.steps[3], np.linalg.matrix_power(step, 8), rtol=1e-10, atol=1e-15)
    np.testing.assert_allclose(t.lanes[5], np.linalg.matrix_power(step, 5), rtol=1e-10, atol=1e-15)
    np.testing.assert_allclose(t.warp_powers[1], np.linalg.matrix_power(step, 32), rtol=1e-9, atol=1e-15)
    np.testing.assert_allclose(t.warp_powers[8], t.lookback[1], rtol=1e-9, atol=1e-15)
    np.testing.assert_allclose(t.lookback[1], np.linalg.matrix_power(A, D.IIR_TILE), rtol=1e-8, atol=1e-15)
    for k in (1, 7, 20):
        np.testing.assert_allclose(t.impulse[k], C @ np.linalg.matrix_power(A, k - 1) @ B, rtol=1e-12)
    np.testing.assert_allclose(t.impulse, D.direct_response(*FILTERS["order10"], D.IIR_CHUNK),
                               rtol=1e-9, atol=1e-12 * np.abs(t.impulse).max())


def test_constructor_validation():
    """Bad arguments fail as the reference's do (test_triton_iir.py:717-742)."""

    for bad in (100, 63, 0, -64):
        with pytest.raises(ValueError):
            IIRCuda(*FILTERS["order2"], chunk_size=bad)
    with pytest.raises(ValueError):
        IIRCuda(*FILTERS["order2"], method="magic")
    with pytest.raises(ValueError):
        IIRCuda(np.array([1.0]), np.array([0.0, 1.0]))  # a[0] == 0
    with pytest.raises(ValueError):
        IIRCuda(np.array([1.0]), np.array([1.0]))  # no pole


def test_module_attributes():
    m = IIRCuda(*FILTERS["order10"])
    assert m.candidates == (D.DEFAULT_CHUNK,)
    assert m.method == "matmul"
    assert (m.order, m.states, m.basis, m.padded) == (10, 10, "cascade", 10)
    m = IIRCuda(*DEGENERATE["odd_order"], chunk_size="tune", method="scan")
    assert m.candidates == D.CHUNK_CANDIDATES and m.method == "scan"
    assert m.order == 3 and m.padded == 4
    with warnings.catch_warnings():
        warnings.simplefilter("error")
        IIRCuda(*FILTERS["order2"], chunk_size=128)


def test_overlapped_tiles_only_where_the_state_dies_out():
    """Long rows run overlapped tiles (a 1056-sample warm-up, no waits) when
    ||A^1056|| < 1e-11 in the chosen realisation -- the PESQ filters and the
    usual designs -- and chain their tiles by the look-back for poles close
    to the unit circle."""

    from iir_cases import resonator
    from triton_pesq_b200.tables import power_filter, pre_filter

    for b, a in [power_filter(), pre_filter(), *FILTERS.values(), *DEGENERATE.values()]:
        module = IIRCuda(b, a)
        assert module.overlap == D.IIR_LANES * D.IIR_CHUNK
        assert module.force_lookback is False
    for radius in (0.99, 0.9999):
        tabs = D.design(*resonator(radius)).tables()
        assert tabs.overlap == 0
        assert float(np.abs(tabs.warp_powers[1]).sum(axis=1).max()) >= D.IIR_OVERLAP_TOL
