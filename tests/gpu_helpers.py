"""Shared helpers of the GPU parity tests."""

import numpy as np
import torch

from oracle import pesq_oracle as O

#: Distances of the CUDA engine against the float64 evaluation of the same
#: pipeline (north star: 1e-5 relative); gradients relative to their peak
#: (north star: 1e-4).
F64_RTOL = 1e-5
GRAD_RTOL = 1e-4


def oracle_grads(ref, deg, factor, sample_rate, **geometry):
    """float64 distances and gradients of ``factor*(0.1 ds + 0.0309 da)``
    (``geometry``: n_fft / hop_length / win_length of ``PesqLoss``)."""

    p = O.OracleParams(factor=factor, sample_rate=sample_rate, **geometry)
    r = ref.detach().cpu().double().requires_grad_(True)
    d = deg.detach().cpu().double().requires_grad_(True)
    ds, da = O.raw(r, d, p, "float64")
    loss = factor * (0.1 * ds + 0.0309 * da)
    g_ref, g_deg = torch.autograd.grad(loss.sum(), [r, d])
    return ds.detach().numpy(), da.detach().numpy(), g_ref.numpy(), g_deg.numpy()


def rel_err(got, want):
    got = np.asarray(got, dtype=np.float64)
    want = np.asarray(want, dtype=np.float64)
    return float((np.abs(got - want) / np.maximum(np.abs(want), 1e-12)).max())


def peak_rel_err(got, want):
    got = np.asarray(got, dtype=np.float64)
    want = np.asarray(want, dtype=np.float64)
    return float(np.abs(got - want).max() / max(np.abs(want).max(), 1e-30))
