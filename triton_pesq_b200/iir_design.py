"""Host-side float64 design of the standalone IIR filter.

The reference's ``TritonIIR`` (torch_pesq/triton_ops/iir.py:1266-1482)
evaluates ``lfilter(x, a, b, clamp=False)`` with a chunked parallel scan over a
state space realisation of the difference equation.  Which realisation is used
decides the float32 accuracy, so three are built here and scored
(iir.py:468-599):

``companion``
    the direct form II transposed state (iir.py:187-221);
``modal``
    the real block diagonal form from the eigendecomposition of the companion
    matrix, rebalanced per block (iir.py:290-433);
``cascade``
    the series of second order sections of ``scipy.signal.tf2sos`` stacked into
    one block lower triangular transition (iir.py:224-287).  Each section is
    realised as a balanced rotation-scaling (complex pair) or diagonal (real
    pair) block whose powers have norm ``|p|^t``, which conditions better than
    the per-section companion blocks of the reference.

The score of a realisation is the larger of its float64 *fidelity* (how far its
own impulse response already is from the difference equation's), its
*conditioning* (the largest entry of any table the CUDA kernel multiplies data
with, times the float32 unit round-off), as in iir.py:436-517, and the error of
its recursion run in float32 on seeded white noise (which the reference leaves
to the user: table entries do not see how the recursion amplifies rounding).  The tables are
the ones of the sm_100a kernel (``csrc/iir.cuh``), whose geometry differs from
the reference's Triton tiles: 33-sample thread chunks, a 5 level warp scan, a
lane table, warp powers and a per-tile look-back table.  Selection,
rejection (predicted peak relative error above ``1e5`` round-offs) and the
warning threshold (``1e3`` round-offs) follow iir.py:520-599.
"""

from __future__ import annotations

import math
import warnings
from dataclasses import dataclass
from typing import Optional, Sequence, Tuple, Union

import numpy as np

__all__ = [
    "CHUNK_CANDIDATES",
    "DEFAULT_CHUNK",
    "METHODS",
    "KERNEL_STATES",
    "IIR_CHUNK",
    "IIR_THREADS",
    "IIR_TILE",
    "IIR_LOOKBACK",
    "IIR_OVERLAP_TOL",
    "as_coeffs",
    "companion",
    "modal",
    "cascade",
    "direct_response",
    "realised_response",
    "KernelTables",
    "kernel_tables",
    "emulate",
    "emulated_error",
    "score",
    "IIRDesign",
    "design",
]

#: Chunk lengths the reference accepts (iir.py:150); here they only set the
#: horizon the realisations are scored over.
CHUNK_CANDIDATES = (64, 128, 256, 512)
DEFAULT_CHUNK = 256
METHODS = ("scan", "matmul")

#: Unit round-off of float32 and float64.
FLOAT32_EPS = 2.0**-24
FLOAT64_EPS = 2.0**-53
#: Largest table entry (in float32 round-offs) a realisation may need before it
#: is rejected, and above which it is flagged (iir.py:161-174).
FLOAT32_LIMIT = 1e5
FLOAT32_WARN = 1e3
ERROR_LIMIT = FLOAT32_LIMIT * FLOAT32_EPS
ERROR_WARN = FLOAT32_WARN * FLOAT32_EPS
#: Realisations in the order they are preferred, and the factor within which
#: two predicted errors count as equal.
PREFERENCE = ("cascade", "modal", "companion")
SCORE_TIE = 2.0
#: Realisations with a larger float32 table entry are not used: a product of
#: it with a moderate sample already nears the float32 range.
FLOAT32_MAX_ENTRY = 1e24

#: State counts the CUDA kernel is instantiated for; a realisation is zero
#: padded to the next one.
KERNEL_STATES = (2, 4, 6, 8, 10, 12, 14, 16, 20, 24)

#: Kernel geometry (csrc/iir.cuh): samples per thread chunk, threads per CTA,
#: lanes per warp, warp scan levels, samples per tile, look-back window.
IIR_CHUNK = 33
#: state an overlapped tile may drop after its warm-up of 32 chunks, relative
IIR_OVERLAP_TOL = 1e-11
IIR_THREADS = 256
IIR_LANES = 32
IIR_LEVELS = 5
IIR_WARPS = IIR_THREADS // IIR_LANES
IIR_TILE = IIR_THREADS * IIR_CHUNK
IIR_LOOKBACK = 32
#: Predecessor tiles the look-back reaches (its table of tile powers).
IIR_FAR = 256


def as_coeffs(values: Union[Sequence[float], np.ndarray, "torch.Tensor"]) -> np.ndarray:  # noqa: F821
    """Filter coefficients as a flat float64 array (iir.py:178-184)."""

    if hasattr(values, "detach"):
        values = values.detach().cpu().numpy()
    return np.asarray(values, dtype=np.float64).ravel()


def _normalised(b: np.ndarray, a: np.ndarray) -> Tuple[np.ndarray, np.ndarray]:
    size = max(b.size, a.size)
    b = np.pad(b, (0, size - b.size))
    a = np.pad(a, (0, size - a.size))
    if a[0] == 0.0:
        raise ValueError("The leading denominator coefficient a[0] must not be zero.")
    if size < 2:
        raise ValueError("The CUDA IIR filter needs at least one pole.")
    return b / a[0], a / a[0]


def companion(b: np.ndarray, a: np.ndarray):
    """Direct form II transposed realisation ``(A, B, C, D)`` of ``b / a``.

    The state before sample ``n`` evolves as ``s[n+1] = A s[n] + B x[n]`` and
    ``y[n] = C s[n] + D x[n]`` with ``A[:, 0] = -a[1:]``, ones on the first
    super diagonal, ``B = b[1:] - a[1:] b[0]``, ``C = e_1`` and ``D = b[0]``
    (iir.py:187-221).
    """

    b, a = _normalised(b, a)
    order = a.size - 1
    trans = np.zeros((order, order))
    trans[:, 0] = -a[1:]
    trans[np.arange(order - 1), np.arange(1, order)] = 1.0
    read = np.zeros(order)
    read[0] = 1.0
    return trans, b[1:] - a[1:] * b[0], read, float(b[0])


def modal(trans: np.ndarray, drive: np.ndarray, read: np.ndarray, feed: float):
    """Real block diagonal realisation, ``None`` when it does not exist.

    The basis spans the real invariant subspaces of the eigenvalues of
    ``trans``: one column per real eigenvalue, the real and imaginary parts of
    the eigenvector per conjugate pair (iir.py:290-337).  Complex pairs come
    first so that every 2 x 2 block starts on an even index (the kernel then
    skips the zero blocks); entries outside the diagonal blocks are rounding
    noise of the similarity transform and are dropped.  Each block's input and
    read-out are balanced to equal norm (iir.py:403-433).  A defective matrix
    (repeated poles) has no such basis.
    """

    order = trans.shape[0]
    try:
        values, vectors = np.linalg.eig(trans)
    except np.linalg.LinAlgError:
        return None
    perm = np.argsort(-np.abs(values), kind="stable")
    values, vectors = values[perm], vectors[:, perm]

    used = np.zeros(order, dtype=bool)
    pairs, reals = [], []
    for i in range(order):
        if used[i]:
            continue
        v = values[i]
        if abs(v.imag) <= 1e-13 * max(1.0, abs(v)):
            used[i] = True
            reals.append(vectors[:, i].real.copy())
            continue
        dist = np.where(used, np.inf, np.abs(values - np.conj(v)))
        dist[i] = np.inf
        mate = int(np.argmin(dist))
        if not np.isfinite(dist[mate]):
            return None
        used[i] = used[mate] = True
        pairs.append((vectors[:, i].real.copy(), vectors[:, i].imag.copy()))

    columns, blocks = [], []
    for re_part, im_part in pairs:
        blocks.append((len(columns), 2))
        columns += [re_part, im_part]
    for col in reals:
        blocks.append((len(columns), 1))
        columns.append(col)
    basis = np.stack(columns, axis=1)
    norms = np.linalg.norm(basis, axis=0)
    if not np.all(np.isfinite(basis)) or np.any(norms == 0.0):
        return None
    basis = basis / norms
    try:
        inverse = np.linalg.inv(basis)
    except np.linalg.LinAlgError:
        return None
    if not np.all(np.isfinite(inverse)):
        return None

    full = inverse @ trans @ basis
    state = np.zeros_like(full)
    for start, size in blocks:
        sl = slice(start, start + size)
        state[sl, sl] = full[sl, sl]
    push, tap = inverse @ drive, read @ basis
    for start, size in blocks:
        sl = slice(start, start + size)
        gain, inject = np.linalg.norm(tap[sl]), np.linalg.norm(push[sl])
        if gain > 0.0 and inject > 0.0:
            alpha = math.sqrt(inject / gain)
            tap[sl] *= alpha
            push[sl] /= alpha
    if not (np.all(np.isfinite(state)) and np.all(np.isfinite(push)) and np.all(np.isfinite(tap))):
        return None
    return state, push, tap, feed


def cascade(b: np.ndarray, a: np.ndarray):
    """Series of balanced second order sections (block lower triangular),
    ``None`` when ``tf2sos`` cannot factor the transfer function."""

    from .tables import state_space

    try:
        with warnings.catch_warnings():
            warnings.simplefilter("ignore")
            return state_space(b, a)
    except Exception:
        return None


def direct_response(b: np.ndarray, a: np.ndarray, taps: int) -> np.ndarray:
    """First ``taps`` samples of the impulse response, straight from the
    difference equation in float64 (iir.py:379-400)."""

    from .tables import direct_impulse_response

    return direct_impulse_response(b, a, taps)


def realised_response(trans, drive, read, feed, taps: int) -> np.ndarray:
    """Impulse response ``h[0] = D``, ``h[t] = C A^(t-1) B`` of a realisation."""

    out = np.zeros(taps)
    out[0] = feed
    vec = np.array(drive, dtype=np.float64)
    for t in range(1, taps):
        out[t] = read @ vec
        vec = trans @ vec
    return out


def _kernel_states(states: int) -> int:
    for p in KERNEL_STATES:
        if p >= states:
            return p
    raise RuntimeError(
        f"The realisation of this filter has {states} states; the CUDA IIR kernel handles at most "
        f"{KERNEL_STATES[-1]}. Split the filter into second order sections and chain several filters."
    )


def _block_lower(trans: np.ndarray) -> bool:
    """All entries above the 2 x 2 block diagonal are exactly zero."""

    p = trans.shape[0]
    for i in range(p):
        for j in range(p):
            if (j >> 1) > (i >> 1) and trans[i, j] != 0.0:
                return False
    return True



@dataclass
class KernelTables:
    """The constants of the CUDA kernel for one realisation (float64 values,
    zero padded to ``states`` = the kernel's state count).

    For a thread chunk of ``L`` samples starting in state ``S``:
    ``y[t] = sum_k impulse[t-k] x[k] + carry[t] . S`` and the end state is
    ``A^L S + sum_k drive[k] x[k]``; ``steps[i] = A^(L 2^i)`` drive the warp
    scan, ``lanes[l] = A^(L l)`` carry a warp's start state to its lanes,
    ``warp_powers[k] = A^(32 L k)`` (k = 0..8) give every warp its start state
    from the totals of the warps before it, and ``lookback[k] = A^(k T)``
    (``T`` samples per tile, float64) chains the tiles of a row.
    """

    order: int
    realised_states: int
    states: int
    lower: bool
    impulse: np.ndarray  # [L]
    carry: np.ndarray  # [L, P]
    drive: np.ndarray  # [L, P]
    steps: np.ndarray  # [levels, P, P]
    lanes: np.ndarray  # [32, P, P]
    warp_powers: np.ndarray  # [9, P, P]
    lookback: np.ndarray  # [257, P, P]
    trans: np.ndarray
    input: np.ndarray
    output: np.ndarray
    feed: float

    @property
    def largest32(self) -> float:
        """Largest entry of the float32 tables (the impulse response, a property
        of the filter rather than the realisation, excluded as iir.py:768-823)."""

        return float(max(np.abs(t).max() for t in (self.carry, self.drive, self.steps, self.lanes,
                                                   self.warp_powers, self.trans, self.input, self.output)))

    @property
    def largest64(self) -> float:
        """Largest entry of the float64 tables (tile chaining)."""

        return float(np.abs(self.lookback).max())

    @property
    def overlap(self) -> int:
        """Warm-up samples of the overlapped tiles long rows run (one warp's
        chunks, ``32 L``) when the state dies out within them --
        ``||A^(32 L)||`` (max row sum) below ``IIR_OVERLAP_TOL`` -- else 0 (the
        tiles are chained by the look-back)."""

        norm = float(np.abs(self.warp_powers[1]).sum(axis=1).max())
        return IIR_LANES * IIR_CHUNK if np.isfinite(norm) and norm < IIR_OVERLAP_TOL else 0


def kernel_tables(trans, drive, read, feed, order: Optional[int] = None) -> KernelTables:
    """Tables of the CUDA kernel for the realisation ``(A, B, C, D)``."""

    realised = trans.shape[0]
    p = _kernel_states(realised)
    A = np.zeros((p, p))
    A[:realised, :realised] = trans
    B = np.zeros(p)
    B[:realised] = drive
    C = np.zeros(p)
    C[:realised] = read
    L = IIR_CHUNK

    carry = np.zeros((L, p))
    power = np.eye(p)
    for t in range(L):
        carry[t] = C @ power
        power = A @ power
    chunk_step = power  # A^L
    drive_tab = np.zeros((L, p))
    acc = np.eye(p)
    for k in range(L - 1, -1, -1):
        drive_tab[k] = acc @ B
        acc = A @ acc
    impulse = np.zeros(L)
    impulse[0] = feed
    impulse[1:] = carry[:-1] @ B

    steps = np.zeros((IIR_LEVELS, p, p))
    step = chunk_step
    for i in range(IIR_LEVELS):
        steps[i] = step
        step = step @ step
    lanes = np.zeros((IIR_LANES, p, p))
    cur = np.eye(p)
    for l in range(IIR_LANES):
        lanes[l] = cur
        cur = chunk_step @ cur
    warp_step = cur  # A^(32 L)
    warp_powers = np.zeros((IIR_WARPS + 1, p, p))
    cur = np.eye(p)
    for k in range(IIR_WARPS + 1):
        warp_powers[k] = cur
        cur = warp_step @ cur
    tile_step = warp_powers[IIR_WARPS]  # A^T
    lookback = np.zeros((IIR_FAR + 1, p, p))
    cur = np.eye(p)
    with np.errstate(over="ignore", invalid="ignore"):
        for k in range(IIR_FAR + 1):
            lookback[k] = cur
            cur = tile_step @ cur

    return KernelTables(order=order if order is not None else realised, realised_states=realised, states=p,
                        lower=_block_lower(A), impulse=impulse, carry=carry, drive=drive_tab, steps=steps,
                        lanes=lanes, warp_powers=warp_powers, lookback=lookback, trans=A, input=B, output=C,
                        feed=float(feed))


def emulate(tabs: KernelTables, x: np.ndarray, dtype=np.float32) -> Tuple[np.ndarray, np.ndarray]:
    """The CUDA kernel's float32 arithmetic (``dtype``) on one row of up to two tiles,
    step by step as csrc/iir.cuh (scan_kernel) runs it: chunk end states from
    zero, the warp's doubling scan, the warp start states from the warp
    totals, the second tile's start state (float64 look-back, rounded to
    float32), the chunk start states from the lane table, and the outputs in
    the impulse form and in the re-run form.  Returns both output rows."""

    f = dtype
    p, L, T = tabs.states, IIR_CHUNK, IIR_TILE
    h, G, W = tabs.impulse.astype(f), tabs.carry.astype(f), tabs.drive.astype(f)
    M, A = tabs.steps.astype(f), tabs.trans.astype(f)
    Bv, C, D = tabs.input.astype(f), tabs.output.astype(f), f(tabs.feed)
    lanes, wpow = tabs.lanes.astype(f), tabs.warp_powers.astype(f)
    n = x.size
    tiles = -(-n // T)
    if tiles > 2:
        raise ValueError("emulate() covers one or two tiles")
    xp = np.zeros(tiles * T, f)
    xp[:n] = x
    chunks = xp.reshape(tiles, IIR_WARPS, IIR_LANES, L)
    # 1. chunk end states from zero
    e = chunks @ W
    # 2. doubling scan within each warp
    lane = np.arange(IIR_LANES)[None, None, :, None]
    for lv in range(IIR_LEVELS):
        d = 1 << lv
        pv = np.zeros_like(e)
        pv[:, :, d:] = e[:, :, :-d]
        e = np.where(lane >= d, e + pv @ M[lv].T, e)
    ex = np.zeros_like(e)
    ex[:, :, 1:] = e[:, :, :-1]
    tot = e[:, :, -1]  # [tiles, warps, p]
    # 3. warp start states (tile-local), the tile aggregate, the start state
    # of the second tile
    xw = np.zeros((tiles, IIR_WARPS, p), f)
    for w in range(IIR_WARPS):
        for v in range(w):
            xw[:, w] += tot[:, v] @ wpow[w - 1 - v].T
    if tiles == 2:
        agg = np.zeros(p, f)
        for v in range(IIR_WARPS):
            agg += wpow[IIR_WARPS - 1 - v] @ tot[0, v]
        start = agg.astype(f)  # the first tile's inclusive state: its aggregate
        xw[1] += np.einsum("wij,j->wi", wpow[:IIR_WARPS], start).astype(f)
    # 4. chunk start states; the row's first chunk starts from zero
    s = ex + np.einsum("lij,twj->twli", lanes, xw).astype(f)
    s[0, 0, 0] = 0.0
    s = s.reshape(-1, p)
    xc = chunks.reshape(-1, L)
    # 5. outputs
    zero = np.stack([xc[:, :t + 1] @ h[t::-1] for t in range(L)], axis=1)
    impulse_form = zero + s @ G.T
    rerun = np.empty_like(xc)
    st = s.copy()
    for t in range(L):
        rerun[:, t] = st @ C + D * xc[:, t]
        st = st @ A.T + np.outer(xc[:, t], Bv)
    return impulse_form.reshape(-1)[:n], rerun.reshape(-1)[:n]


def emulated_error(tabs: KernelTables, b: np.ndarray, a: np.ndarray) -> float:
    """Peak relative error of the kernel's float32 arithmetic (both output
    forms) on two tiles of seeded white noise, against a float64 lfilter of
    the coefficients.

    The reference predicts the error from the largest table entry alone
    (iir.py:468-517) and documents that this underestimates it by up to two
    orders of magnitude.  Table entries bound the rounding of one product, not
    how the state magnitudes amplify it: the companion form of an order 24
    low pass has entries below 1e4 and returns noise, while its cascade has
    entries near 1e7 and keeps seven digits.  Running the arithmetic itself
    measures both."""

    from scipy.signal import lfilter

    x = np.random.default_rng(0).standard_normal(2 * IIR_TILE).astype(np.float32)
    truth = lfilter(np.asarray(b, np.float64), np.asarray(a, np.float64), x.astype(np.float64))
    scale = float(np.abs(truth).max())
    if not (math.isfinite(scale) and scale > 0.0):
        return math.inf
    with np.errstate(over="ignore", invalid="ignore"):
        worst = max(float(np.abs(y.astype(np.float64) - truth).max()) for y in emulate(tabs, x))
    err = worst / scale
    return err if math.isfinite(err) else math.inf


def score(trans, drive, read, feed, reference: np.ndarray, scale: float, b=None, a=None) -> Tuple[float, float]:
    """Predicted peak relative error of a realisation and its largest float32
    table entry: the larger of the float64 fidelity of its impulse response
    and the conditioning of its float64 tables (iir.py:468-517) and, given the
    coefficients, the error of the kernel's own float32 arithmetic
    (emulated_error; without them, the reference's estimate from the largest
    float32 table entry)."""

    with np.errstate(over="ignore", invalid="ignore"):
        response = realised_response(trans, drive, read, feed, reference.size)
        fidelity = float(np.abs(response - reference).max() / scale)
        if not math.isfinite(fidelity):
            return math.inf, math.inf
        tabs = kernel_tables(trans, drive, read, feed)
        entry32, entry64 = tabs.largest32, tabs.largest64
    if not (math.isfinite(entry32) and math.isfinite(entry64)) or entry32 > FLOAT32_MAX_ENTRY:
        return math.inf, math.inf
    predicted = max(fidelity, entry64 * FLOAT64_EPS)
    if b is None:
        return max(predicted, entry32 * FLOAT32_EPS), entry32
    return max(predicted, emulated_error(tabs, b, a)), entry32


@dataclass
class IIRDesign:
    """The selected realisation of a filter."""

    basis: str
    order: int
    trans: np.ndarray
    input: np.ndarray
    output: np.ndarray
    feed: float
    score: float
    entry: float
    candidates: dict  # name -> (score, entry)

    @property
    def states(self) -> int:
        return self.trans.shape[0]

    def tables(self) -> KernelTables:
        return kernel_tables(self.trans, self.input, self.output, self.feed, self.order)


def design(b, a, taps: int = DEFAULT_CHUNK, stacklevel: int = 3) -> IIRDesign:
    """Most accurate realisation of ``b / a`` for the CUDA kernel.

    Scored over ``max(taps, 32 * 33)`` samples of the impulse response.  Raises
    ``RuntimeError`` when no realisation is expected to keep two significant
    float32 digits, warns (``RuntimeWarning``) when accuracy is degraded, as
    iir.py:520-599.
    """

    b, a = as_coeffs(b), as_coeffs(a)
    trans, drive, read, feed = companion(b, a)  # validates a[0] and the order
    order = trans.shape[0]
    horizon = max(int(taps), IIR_LANES * IIR_CHUNK)
    reference = direct_response(b, a, horizon)
    scale = max(float(np.abs(reference).max()), 1e-30)

    candidates = [("companion", trans, drive, read, feed)]
    m = modal(trans, drive, read, feed)
    if m is not None:
        candidates.append(("modal",) + tuple(m))
    c = cascade(b, a)
    if c is not None:
        candidates.append(("cascade",) + tuple(c))

    scores = {}
    for name, A, B, C, D in candidates:
        scores[name] = (math.inf, math.inf) if A.shape[0] > KERNEL_STATES[-1] else \
            score(A, B, C, D, reference, scale, b, a)
    # the emulated errors of two good realisations differ by rounding noise:
    # take the first in the order cascade, modal, companion (the block lower
    # ones skip the zero blocks of their tables) within SCORE_TIE of the best
    lowest = min(s for s, _ in scores.values())
    best, best_score, best_entry = None, math.inf, math.inf
    for name, A, B, C, D in sorted(candidates, key=lambda c: PREFERENCE.index(c[0])):
        s, e = scores[name]
        if math.isfinite(s) and s <= SCORE_TIE * lowest:
            best, best_score, best_entry = (name, A, B, C, D), s, e
            break

    if best is None or not math.isfinite(best_score):
        if order > KERNEL_STATES[-1]:
            _kernel_states(order)  # raises with the state count
        raise RuntimeError("Could not build a numerically valid state space realisation for the given "
                           "coefficients.")
    name, A, B, C, D = best
    if best_score > ERROR_LIMIT:
        raise RuntimeError(
            f"The best state space realisation of this filter (`{name}`, order {order}) is expected to "
            f"reach a peak relative error of only {best_score:.3g} in float32 (largest table entry "
            f"{best_entry:.3g}), so the result would carry no significant digits. Split the filter into "
            f"second order sections and chain several filters instead.")
    if best_score > ERROR_WARN:
        warnings.warn(
            f"The state space realisation of this filter (`{name}`, order {order}) has a largest table "
            f"entry of {best_entry:.3g}; float32 accuracy will be degraded to a peak relative error of "
            f"about {best_score:.3g}.", RuntimeWarning, stacklevel=stacklevel)
    return IIRDesign(basis=name, order=order, trans=A, input=B, output=C, feed=float(D), score=best_score,
                     entry=best_entry, candidates=scores)
