"""The seeded workload generator: a row selection reproduces the same rows
of the whole workload bit for bit (the GPU parity tests check slices of the
large benchmark workloads through it)."""

import pytest
import torch

from triton_pesq_b200.signals import WORKLOADS, workload


@pytest.mark.parametrize("name,rows", [("cfg1", [0]), ("cfg2", [1, 5]), ("cfg3", [0, 7, 15])])
def test_row_selection_matches_whole_workload(name, rows):
    ref, deg, sr = workload(name, seed=0)
    ref_s, deg_s, sr_s = workload(name, seed=0, rows=rows)
    assert sr == sr_s == WORKLOADS[name][2]
    assert ref.shape == WORKLOADS[name][:2]
    assert torch.equal(ref[rows], ref_s)
    assert torch.equal(deg[rows], deg_s)


def test_cfg4_snr_halves():
    """cfg4: the first 32 utterances at -5 dB SNR, the last 32 at 25 dB."""

    ref, deg, _ = workload("cfg4", seed=0, rows=[0, 63])
    noise = (deg - ref).double().pow(2).mean(dim=1)
    snr = 10 * torch.log10(ref.double().pow(2).mean(dim=1) / noise)
    assert abs(float(snr[0]) + 5.0) < 0.1 and abs(float(snr[1]) - 25.0) < 0.1


def test_unknown_workload():
    with pytest.raises(ValueError):
        workload("cfg9")
