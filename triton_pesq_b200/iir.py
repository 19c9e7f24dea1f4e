"""``IIRCuda``: the causal IIR filter as a standalone op on sm_100a kernels.

Drop-in for the reference's ``TritonIIR`` (torch_pesq/triton_ops/iir.py:
1266-1482): the same constructor (``b_coeffs``, ``a_coeffs``, ``chunk_size``,
``method``), the same semantics -- ``torchaudio.functional.lfilter(x, a, b,
clamp=False)`` with zero initial state along the last axis of a
``[batch, sample]`` float32 tensor -- the same realisation selection
(``basis`` is ``"cascade"``, ``"modal"`` or ``"companion"``, scored by
:mod:`triton_pesq_b200.iir_design`), the same errors and warnings for filters
float32 cannot represent, and an autograd backward that is the same filter run
back to front, itself differentiable (iir.py:1232-1263).

What differs is the evaluation: one kernel launch per call, a chunked scan
whose tiles are chained by a decoupled look-back in float64, so the carry
across a long signal is exact and no sequential pass over the chunks remains
(csrc/iir.cuh).  ``chunk_size`` is validated as the reference validates it and
sets the horizon the realisations are scored over, but the kernel's own
geometry (33-sample thread chunks, 8448-sample tiles) is fixed; ``"tune"`` has
nothing to benchmark and records the shapes it saw.  ``method="scan"`` re-runs
the recursion inside each chunk, ``"matmul"`` (the default, as ``"auto"``)
multiplies by the chunk's impulse response.  Offsets are 64-bit: there is no
``2**31`` element limit.
"""

from __future__ import annotations

import math
import weakref
from typing import Dict, Optional, Union

import numpy as np
import torch

from . import _lib
from .iir_design import CHUNK_CANDIDATES, DEFAULT_CHUNK, METHODS, as_coeffs, design

__all__ = ["IIRCuda", "CHUNK_CANDIDATES", "DEFAULT_CHUNK", "METHODS"]


def _release(handles: Dict[int, int]) -> None:
    for handle in handles.values():
        try:
            _lib.destroy_iir(handle)
        except Exception:  # interpreter shutdown
            pass
    handles.clear()


class _IIRFunction(torch.autograd.Function):
    """y = T x (``reverse=False``) or J T J x; the vector-Jacobian product of
    one is the other, so the backward flips the direction and stays
    differentiable (iir.py:1232-1263)."""

    @staticmethod
    def forward(ctx, signal, module, reverse):
        ctx.module, ctx.reverse = module, reverse
        return module._launch(signal, reverse)

    @staticmethod
    def backward(ctx, grad):
        if not ctx.needs_input_grad[0]:
            return None, None, None
        reverse = not ctx.reverse
        if torch.is_grad_enabled() and grad.requires_grad:
            return _IIRFunction.apply(grad, ctx.module, reverse), None, None
        return ctx.module._launch(grad, reverse), None, None


class IIRCuda(torch.nn.Module):
    """Causal IIR filter with zero initial conditions, evaluated on the GPU.

    Parameters
    ----------
    b_coeffs, a_coeffs
        Numerator and denominator of the difference equation; everything is
        normalised by ``a_coeffs[0]``.  No gradient flows into them.
    chunk_size : Optional[Union[int, str]]
        A positive multiple of 64, ``None`` (256) or ``"tune"``: the horizon
        the realisations are scored over (the longest candidate).
    method : str
        ``"matmul"``, ``"scan"`` or ``"auto"`` (``"matmul"``).

    Attributes
    ----------
    order : int
        Number of poles of the difference equation
    states : int
        State count of the selected realisation
    basis : str
        ``"cascade"``, ``"modal"`` or ``"companion"``
    padded : int
        State count of the kernel instantiation (the realisation zero padded)
    feed : float
        Direct feed-through ``D``
    overlap : int
        Warm-up samples of the overlapped tiles rows longer than one tile run
        (each tile re-runs that much of the row before it from zero state, no
        waits between tiles), or 0 when the filter's state does not die out
        within them and the tiles are chained by the look-back
    force_lookback : bool
        Chain the tiles of long rows by the look-back even where overlapped
        tiles would do (False by default)
    """

    def __init__(self, b_coeffs, a_coeffs, chunk_size: Optional[Union[int, str]] = None, method: str = "auto"):
        super().__init__()
        if method == "auto":
            method = "matmul"
        if method not in METHODS:
            raise ValueError(f"Unknown method `{method}`, pick one of {METHODS}.")
        self.method = method
        if chunk_size == "tune":
            candidates = list(CHUNK_CANDIDATES)
        elif chunk_size is None:
            candidates = [DEFAULT_CHUNK]
        else:
            chunk_size = int(chunk_size)
            if chunk_size < 64 or chunk_size % 64 != 0:
                raise ValueError("`chunk_size` has to be a positive multiple of 64.")
            candidates = [chunk_size]
        self.candidates = tuple(candidates)
        self._tuned: Dict[tuple, int] = {}

        numerator, denominator = as_coeffs(b_coeffs), as_coeffs(a_coeffs)
        self.design = design(numerator, denominator, max(candidates), stacklevel=3)
        self.order = max(numerator.size, denominator.size) - 1
        self.states = self.design.states
        self.basis = self.design.basis
        self.overlap = self.design.tables().overlap
        self.force_lookback = False
        self.feed = self.design.feed
        self.padded = self.design.tables().states
        self.score = self.design.score
        for name, value in (("trans", self.design.trans), ("drive", self.design.input),
                            ("read", self.design.output)):
            self.register_buffer(f"_{name}", torch.as_tensor(np.ascontiguousarray(value), dtype=torch.float64),
                                 persistent=False)
        self._handles: Dict[int, int] = {}
        self._finalizer = weakref.finalize(self, _release, self._handles)
        _lib.load_ops()

    def _handle(self, device: torch.device) -> int:
        index = device.index if device.index is not None else torch.cuda.current_device()
        handle = self._handles.get(index)
        if handle is None:
            with torch.cuda.device(index):
                handle = _lib.create_iir(self.design)
            self._handles[index] = handle
        return handle

    def _flags(self, reverse: bool) -> int:
        return ((_lib.IIR_REVERSE if reverse else 0) | (_lib.IIR_RERUN if self.method == "scan" else 0)
                | (_lib.IIR_CHAINED if self.force_lookback else 0))

    def _launch(self, signal: torch.Tensor, reverse: bool) -> torch.Tensor:
        return torch.ops.pesq_cuda.iir(self._handle(signal.device), signal, self._flags(reverse))

    def check_errors(self) -> int:
        """Synchronise and return the error word of every device's filter (nonzero
        if a tile of an earlier call gave up waiting for its predecessor)."""

        failed = 0
        for index, handle in self._handles.items():
            with torch.cuda.device(index):
                failed |= _lib.iir_check(handle, torch.cuda.current_stream().cuda_stream)
        return failed

    def forward(self, signal: torch.Tensor) -> torch.Tensor:
        """Filter a batch of time signals ``[batch, sample]``."""

        if not isinstance(signal, torch.Tensor):
            raise TypeError("`signal` must be a torch.Tensor")
        if not signal.is_cuda:
            raise RuntimeError("The CUDA IIR filter needs `signal` to live on a GPU.")
        if signal.dtype != torch.float32:
            raise RuntimeError(f"The CUDA IIR filter only supports float32, `signal` is {signal.dtype}.")
        if signal.dim() != 2:
            raise RuntimeError(f"The CUDA IIR filter needs a [batch, sample] tensor, got {tuple(signal.shape)}.")
        if signal.shape[1] == 0:
            return signal.clone()
        if len(self.candidates) > 1:
            self._tuned.setdefault(tuple(signal.shape), max(self.candidates))
        if not (torch.is_grad_enabled() and signal.requires_grad):
            return self._launch(signal, False)
        return _IIRFunction.apply(signal, self, False)

    def extra_repr(self) -> str:
        return f"order={self.order}, basis={self.basis}, states={self.states}, method={self.method}"
