"""Parity of PesqLossCuda on the benchmark workloads themselves and against
the reference's own float32 ``PesqLoss``.

* The inputs the benchmark times (``signals.workload``: cfg2 whole, cfg3
  whole, four rows of cfg4 -- two at -5 dB SNR, where the asymmetric
  distance runs into its 45.0 clamp, and two at 25 dB -- and a 32-utterance
  slice of cfg5) against the float64 oracle: 1e-5 relative on the
  distances, 1e-4 of the peak on both gradients.
* Every golden fixture against the outputs of the reference's float32
  ``PesqLoss`` stored in it (``ref32_*``): within the reference's documented
  float32 ``lfilter`` error -- at most 4e-3 relative on the distances, the
  loss and the MOS (``README.md:89-92``, ``docs/triton.md:165-168``), and
  1e-6 where a distance is saturated at the 45.0 clamp
  (``torch_pesq/loss.py:252-255``); gradients within 1.5e-2 of their peak,
  the documented backward error of that float32 ``lfilter``
  (``triton_ops/iir.py:77-82``), or -- where the reference's own float32
  gradient is further than that from float64 -- no further from it than
  float64 is.  That happens on the saturated fixtures: their harmonic
  references have no energy between the partials, and there the reference's
  float32 gradient w.r.t. the reference signal is 25-35 % of its peak away
  from the float64 one (0.3-6 % w.r.t. the degraded signal), while this
  engine stays within 1e-4 of float64 (``test_golden_vectors``).
"""

import glob
import os

import numpy as np
import pytest
import torch

from conftest import GOLDEN, golden_geometry
from gpu_helpers import F64_RTOL, GRAD_RTOL, oracle_grads, peak_rel_err, rel_err
from oracle import pesq_oracle as O
from triton_pesq_b200 import PesqLossCuda
from triton_pesq_b200.signals import workload

pytestmark = pytest.mark.gpu

#: the reference's float32 PesqLoss against float64 (documented bounds)
REF32_RTOL = 4e-3
REF32_SATURATED_RTOL = 1e-6
REF32_GRAD_RTOL = 1.5e-2
SATURATED = 45.0

WORKLOAD_CASES = [
    ("cfg2", None),
    ("cfg3", None),
    ("cfg4", [0, 1, 32, 33]),
    ("cfg5", list(range(32))),
]


def _both_grads(model, ref, deg):
    r = ref.detach().clone().requires_grad_(True)
    d = deg.detach().clone().requires_grad_(True)
    loss = model(r, d)
    g_ref, g_deg = torch.autograd.grad(loss.sum(), [r, d])
    return loss, g_ref, g_deg


@pytest.mark.parametrize("name,rows", WORKLOAD_CASES, ids=[c[0] for c in WORKLOAD_CASES])
def test_benchmark_workloads_match_float64(cuda_device, name, rows):
    ref, deg, sr = workload(name, seed=0, rows=rows)
    ds64, da64, gr64, gd64 = oracle_grads(ref, deg, 1.0, sr)
    model = PesqLossCuda(1.0, sample_rate=sr)
    ds, da = model.raw(ref.to(cuda_device), deg.to(cuda_device))
    assert rel_err(ds.cpu(), ds64) < F64_RTOL
    assert rel_err(da.cpu(), da64) < F64_RTOL
    _, g_ref, g_deg = _both_grads(model, ref.to(cuda_device), deg.to(cuda_device))
    assert peak_rel_err(g_ref.cpu(), gr64) < GRAD_RTOL
    assert peak_rel_err(g_deg.cpu(), gd64) < GRAD_RTOL
    if name == "cfg4":
        # the -5 dB rows are in the clamp-saturated regime the bench includes:
        # a good part of their frames sit at the 45.0 clamp, so the check
        # above covers the clamped frames and not only the free ones
        census = {}
        O.raw(ref.double(), deg.double(), O.OracleParams(1.0, sr), census=census)
        assert float(census["asymm_45"][:2].min()) > 0.2
        assert float(census["asymm_45"][2:].max()) < float(census["asymm_45"][:2].min())


CASES = sorted(glob.glob(os.path.join(GOLDEN, "sr*.npz")))


@pytest.mark.parametrize("path", CASES, ids=[os.path.basename(c)[:-4] for c in CASES])
def test_matches_reference_float32(cuda_device, path):
    z = np.load(path)
    factor, sr = float(z["factor"]), int(z["sample_rate"])
    model = PesqLossCuda(factor, sample_rate=sr, **golden_geometry(z))
    ref = torch.from_numpy(z["ref"]).to(cuda_device)
    deg = torch.from_numpy(z["deg"]).to(cuda_device)
    ds, da = (t.cpu().double().numpy() for t in model.raw(ref, deg))
    for got, want in ((ds, z["ref32_d_symm"]), (da, z["ref32_d_asymm"])):
        assert rel_err(got, want) < REF32_RTOL
        saturated = want >= SATURATED
        if saturated.any():
            assert rel_err(got[saturated], want[saturated]) < REF32_SATURATED_RTOL
    assert rel_err(model.mos(ref, deg).cpu(), z["ref32_mos"]) < REF32_RTOL
    loss, g_ref, g_deg = _both_grads(model, ref, deg)
    assert rel_err(loss.detach().cpu(), z["ref32_loss"]) < REF32_RTOL
    for got, key in ((g_ref, "grad_ref"), (g_deg, "grad_deg")):
        ref32_err = peak_rel_err(z["ref32_" + key], z["f64_" + key])
        assert peak_rel_err(got.cpu(), z["ref32_" + key]) < max(REF32_GRAD_RTOL, ref32_err + GRAD_RTOL)


def test_saturated_fixtures_are_covered():
    """The saturated fixtures are among the cases above (the glob would
    silently drop a renamed file)."""

    names = {os.path.basename(c) for c in CASES}
    assert {"sr16k_sat_b2_n16000.npz", "sr48k_sat_b1_n24000.npz", "sr16k_clamp_b2_n16000.npz"} <= names


@pytest.mark.parametrize("name,batch,segments", [("cfg5", 160, 4), ("cfg4", 40, 11)])
def test_half_size_front_ctas_on_a_large_batch(cuda_device, name, batch, segments):
    """A batch whose front kernel would need more than one wave of one
    512-thread CTA per SM runs half-size CTAs (two per SM, 27-frame
    segments; at 48 kHz behind the resampler, with the float residual of the
    resampled rows): its utterances match float64 and the same utterances
    evaluated in a batch of their own."""

    sms = torch.cuda.get_device_properties(cuda_device).multi_processor_count
    assert 2 * batch * segments > sms  # (the half-size path runs)
    ref, deg, sr = workload(name, seed=0, rows=range(batch))
    model = PesqLossCuda(1.0, sample_rate=sr)
    loss, g_ref, g_deg = _both_grads(model, ref.to(cuda_device), deg.to(cuda_device))
    few = [0, 1, batch // 2 - 3, batch - 1]
    alone, a_ref, a_deg = _both_grads(model, ref[few].to(cuda_device), deg[few].to(cuda_device))
    assert rel_err(loss[few].detach().cpu(), alone.detach().cpu()) < 1e-6
    assert peak_rel_err(g_deg[few].cpu(), a_deg.cpu()) < 1e-5
    assert peak_rel_err(g_ref[few].cpu(), a_ref.cpu()) < 1e-5
    check = few[:2] if name == "cfg4" else few  # (10-s rows at 48 kHz: two of them in float64)
    ds64, da64, gr64, gd64 = oracle_grads(ref[check], deg[check], 1.0, sr)
    ds, da = model.raw(ref.to(cuda_device), deg.to(cuda_device))
    assert rel_err(ds[check].cpu(), ds64) < F64_RTOL
    assert rel_err(da[check].cpu(), da64) < F64_RTOL
    assert peak_rel_err(g_ref[check].cpu(), gr64) < GRAD_RTOL
    assert peak_rel_err(g_deg[check].cpu(), gd64) < GRAD_RTOL


def test_chain_cluster_size_leaves_results_unchanged(cuda_device):
    """The plan sizes the chain clusters from the batch (8 utterances of 3 s:
    6 CTAs each; 16: 4 each) while the front and back kernels keep the same
    segments (half-size front CTAs, 27-frame segments, in both): the
    utterances of the smaller batch come out the same bit for bit inside the
    larger one."""

    ref, deg, sr = workload("cfg5", seed=0, rows=range(16))
    model = PesqLossCuda(1.0, sample_rate=sr)
    sms = torch.cuda.get_device_properties(cuda_device).multi_processor_count
    assert 2 * 16 * 7 <= 2 * sms  # (both batches: one wave of half-size front CTAs)
    big = _both_grads(model, ref.to(cuda_device), deg.to(cuda_device))
    small = _both_grads(model, ref[:8].to(cuda_device), deg[:8].to(cuda_device))
    for b, s in zip(big, small):
        assert torch.equal(b[:8], s)


def test_full_and_half_size_front_ctas_agree(cuda_device):
    """8 utterances of 8 s are the one shape class that keeps full-size front
    CTAs (144 of them fit one wave, their 304 half-size ones would not); a
    ninth utterance moves the batch to half-size CTAs (19 segments of 27
    frames per row instead of 9 of 56).  The eight utterances agree across
    the two layouts within 1e-6 (the segments' warm-up boundaries differ)."""

    ref, deg, sr = workload("cfg2", seed=0)
    model = PesqLossCuda(1.0, sample_rate=sr)
    full = _both_grads(model, ref.to(cuda_device), deg.to(cuda_device))
    ref9, deg9 = torch.cat([ref, ref[:1]]), torch.cat([deg, deg[:1]])
    half = _both_grads(model, ref9.to(cuda_device), deg9.to(cuda_device))
    assert rel_err(half[0][:8].detach().cpu(), full[0].detach().cpu()) < 1e-6
    assert peak_rel_err(half[1][:8].cpu(), full[1].cpu()) < 1e-5
    assert peak_rel_err(half[2][:8].cpu(), full[2].cpu()) < 1e-5
