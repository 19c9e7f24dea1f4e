"""``PesqLossCuda``: the PESQ loss on hand-written sm_100a kernels.

Drop-in for the reference's ``PesqLossTriton`` (torch_pesq/triton_ops/loss.py:18-215):
same constructor arguments, ``raw`` / ``mos`` / ``forward`` / ``graphed`` and
an autograd backward w.r.t. either input.  Every evaluation goes through the
C ABI of ``libpesq_cuda.so`` (via the ``torch.ops.pesq_cuda`` custom ops);
there is no Triton, no CPU path and no fallback.

Pipeline per call at 16 kHz (plus the resampler and its adjoint at other
rates): front (level-alignment power, pre-emphasis, STFT -> Bark) and chain
forward (silent frames, equalisation, loudness, disturbance, pooling,
MOS/loss); in the backward the chain adjoint, the align kernel
(H^T H x of the level-alignment band pass, overlapping the chain adjoint) and
the back end (spectral adjoint, reverse pre-emphasis, alignment term).
"""

from __future__ import annotations

from typing import Dict, Tuple

import numpy as np
import torch

from . import _lib
from .model import BarkScale, Loudness, PowerSpectrogram, edge_ramp
from .resample import ResampleCuda
from .tables import ALIGN_DIV, ALIGN_PAD, ALIGN_TARGET, PlanConfig

__all__ = ["PesqLossCuda"]


# (plan handle, batch, samples, flags) -> byte offset of the loss sum pair;
# a plan's entries go when the plan is released (a later plan may reuse the
# address)
_SUM_OFFSETS: Dict[tuple, int] = {}


def _release_plan(handle: int) -> None:
    for key in [k for k in _SUM_OFFSETS if k[0] == handle]:
        del _SUM_OFFSETS[key]
    _lib.destroy_plan(handle)


def _loss_sum_view(ws: torch.Tensor, plan: int, ref: torch.Tensor, flags: int) -> torch.Tensor:
    """The [loss sum, batch] float64 pair the chain forward leaves in the workspace."""

    key = (plan, ref.shape[0], ref.shape[1], flags)
    off = _SUM_OFFSETS.get(key)
    if off is None:
        off = _SUM_OFFSETS[key] = _lib.loss_sum_offset(plan, ref.shape[0], ref.shape[1], flags)
    return ws[off // 4 : off // 4 + 4].view(torch.float64)


class _PesqFunction(torch.autograd.Function):
    """(ref, deg) -> (d_symm, d_asymm, mos, loss, loss_sum), one forward launch
    sequence; ``loss_sum`` is the float64 pair [sum of the batch's losses,
    batch] (not differentiable).

    The backward takes the upstream gradient of the four per-utterance outputs
    at once (the epilogue adjoint runs inside the chain adjoint kernel) and
    returns the gradients of the inputs that asked for one.
    """

    @staticmethod
    def forward(ctx, ref, deg, plan, owner):
        flags = (_lib.GRAD_REF if ctx.needs_input_grad[0] else 0) | (
            _lib.GRAD_DEG if ctx.needs_input_grad[1] else 0
        )
        d_symm, d_asymm, mos, loss, ws = torch.ops.pesq_cuda.forward(plan, ref, deg, flags)
        in_flag = (_lib.INPUT_BF16 if ref.dtype == torch.bfloat16 else
                   _lib.INPUT_F16 if ref.dtype == torch.float16 else 0)
        if ref.shape[0] > 0:
            loss_sum = _loss_sum_view(ws, plan, ref, flags | in_flag)
        else:
            loss_sum = torch.zeros(2, dtype=torch.float64, device=ref.device)
        ctx.mark_non_differentiable(loss_sum)
        # outputs nobody differentiates get no (zero-filled) gradient
        ctx.set_materialize_grads(False)
        ctx.plan = plan
        # the plan's owner (None while tracing) lives as long as this node
        ctx.owner = owner
        ctx.flags = flags
        if flags:
            # the workspace is neither an input nor an output; saving such an
            # intermediate is fine for a once-differentiable backward
            ctx.save_for_backward(ref, deg, ws)
        return d_symm, d_asymm, mos, loss, loss_sum

    @staticmethod
    @torch.autograd.function.once_differentiable
    def backward(ctx, g_dsymm, g_dasymm, g_mos, g_loss, g_sum):
        ref, deg, ws = ctx.saved_tensors

        # broadcast gradients (of a sum or mean over the batch) are passed on
        # as one shared value, without materialising them
        def prep(g):
            return None if g is None else g.float()

        g_ref, g_deg = torch.ops.pesq_cuda.backward(
            ctx.plan, ref, deg, ctx.flags, ws,
            prep(g_loss), prep(g_mos), prep(g_dsymm), prep(g_dasymm),
        )
        return (
            g_ref if ctx.flags & _lib.GRAD_REF else None,
            g_deg if ctx.flags & _lib.GRAD_DEG else None,
            None,
            None,
        )


def _check_signal(t: torch.Tensor, name: str) -> torch.Tensor:
    if not isinstance(t, torch.Tensor):
        raise TypeError(f"`{name}` must be a torch.Tensor")
    if not t.is_cuda:
        raise RuntimeError(f"The CUDA PESQ backend needs `{name}` to live on a GPU.")
    if t.dtype not in _INPUT_DTYPES:
        raise RuntimeError(
            f"The CUDA PESQ backend supports float32 (and bfloat16 / float16 inputs), `{name}` is {t.dtype}.")
    return t


#: input dtypes: float32 as the reference, plus bfloat16 / float16 for callers
#: training in mixed precision (each sample is widened to float as the first
#: kernel reads it; the whole path then runs as for float32 inputs of the same
#: values; losses are float32, gradients come back in the inputs' dtype)
_INPUT_DTYPES = (torch.float32, torch.bfloat16, torch.float16)


class PesqLossCuda(torch.nn.Module):
    """Perceptual Evaluation of Speech Quality on B200 CUDA kernels.

    Same interface as ``PesqLossTriton(factor, sample_rate, nbarks, win_length,
    n_fft, hop_length)`` (triton_ops/loss.py:60-92); the perceptual model and
    every constant are those of ``PesqLoss`` (torch_pesq/loss.py:61-108).

    Inputs are float32 CUDA tensors ``[batch, sample]`` (``[sample]`` is promoted
    to a batch of one); rows may have any stride.  Gradients flow to whichever
    input requires one.  bfloat16 / float16 inputs are accepted too (both of
    the same dtype): they are widened to float as they are read and evaluated
    exactly as float32 inputs of the same values; the outputs are float32 and
    the gradients come back in the inputs' dtype.  Every launch goes to the
    current stream, so a caller overlaps the loss with other work (e.g. the
    model's backward) by evaluating it under ``torch.cuda.stream``.

    Attributes
    ----------
    factor : float
        Scaling of the loss
    source_sample_rate : int
        Input sampling rate; other rates than 16 kHz are resampled first
    power_filter, pre_filter : torch.nn.Parameter
        The float32 filter coefficients of the level alignment band pass and
        the pre-emphasis, as in ``PesqLoss`` (no gradient)
    config : PlanConfig
        The host float64 tables the plans are built from
    resampler : ResampleCuda
        Resampler to 16 kHz (returns its input at 16 kHz), as ``PesqLoss.resampler``
    resample_op : ResampleCuda or None
        The same, None at 16 kHz, as ``PesqLossTriton.resample_op``
    power_iir, pre_iir : IIRCuda
        The level alignment band pass and the pre-emphasis as standalone
        filters (built on first use), as ``PesqLossTriton.power_iir`` /
        ``pre_iir``; used by ``align_level`` / ``preemphasize``
    to_spec, fbank, loudness : torch.nn.Module
        The constant-holding submodules ``PesqLossTriton`` inherits from
        ``PesqLoss`` (power spectrogram, Bark filterbank, loudness model; see
        :mod:`triton_pesq_b200.model`).  The loss itself evaluates them fused
        in its kernels and never calls them.
    """

    def __init__(
        self,
        factor: float,
        sample_rate: int = 48000,
        nbarks: int = 49,
        win_length: int = 512,
        n_fft: int = 512,
        hop_length: int = 256,
    ):
        super().__init__()
        self.factor = float(factor)
        self.source_sample_rate = int(sample_rate)
        self.config = PlanConfig.build(factor, sample_rate, nbarks, win_length, n_fft, hop_length)
        self.power_filter = torch.nn.Parameter(
            torch.tensor(np.stack([self.config.power_b, self.config.power_a]), dtype=torch.float32),
            requires_grad=False,
        )
        self.pre_filter = torch.nn.Parameter(
            torch.tensor(np.stack([self.config.pre_b, self.config.pre_a]), dtype=torch.float32),
            requires_grad=False,
        )
        # device index -> plan handle, and handle -> its owner (_lib.Owned)
        self._plans: Dict[int, int] = {}
        self._plan_owners: Dict[int, _lib.Owned] = {}
        self.resampler = ResampleCuda(self.source_sample_rate, 16000)
        self.resample_op = None if self.source_sample_rate == 16000 else self.resampler
        self.to_spec = PowerSpectrogram(win_length, n_fft, hop_length)
        self.fbank = BarkScale(n_fft // 2, nbarks)
        self.loudness = Loudness(nbarks)
        _lib.load_ops()

    # ------------------------------------------------------------------
    # the two signal stages of PesqLoss as standalone methods
    # ------------------------------------------------------------------

    def _filter(self, name: str, coeffs: torch.nn.Parameter):
        module = self._modules.get(name)
        if module is None:
            from .iir import IIRCuda

            module = IIRCuda(coeffs[0].detach().cpu().double().numpy(), coeffs[1].detach().cpu().double().numpy())
            self.add_module(name, module)
        return module

    @property
    def power_iir(self):
        """The order-10 level alignment band pass as an ``IIRCuda`` filter."""

        return self._filter("_power_iir", self.power_filter)

    @property
    def pre_iir(self):
        """The pre-emphasis biquad as an ``IIRCuda`` filter."""

        return self._filter("_pre_iir", self.pre_filter)

    def align_level(self, signal: torch.Tensor) -> torch.Tensor:
        """Scale each row so that its 325-3250 Hz band power is 1e7
        (``PesqLoss.align_level``, loss.py:111-141; ``PesqLossTriton``
        evaluates it with its IIR and a scaling kernel, triton_ops/loss.py:94-97).
        ``[batch, sample]`` float32 CUDA rows in, the scaled rows out,
        differentiable w.r.t. the signal.  The band power is summed in float64."""

        filtered = self.power_iir(signal)
        power = filtered.double().pow(2).sum(dim=-1, keepdim=True) / (filtered.shape[-1] + ALIGN_PAD) / ALIGN_DIV
        return signal * (ALIGN_TARGET / power).sqrt().to(signal.dtype)

    def preemphasize(self, signal: torch.Tensor) -> torch.Tensor:
        """The 15-sample edge fades, then the pre-emphasis biquad
        (``PesqLoss.preemphasize``, loss.py:143-169; triton_ops/loss.py:99-102).
        Unlike the reference's version the input is not modified in place."""

        return self.pre_iir(edge_ramp(signal))

    # ------------------------------------------------------------------
    # plans
    # ------------------------------------------------------------------

    def _plan(self, device: torch.device) -> int:
        index = device.index if device.index is not None else torch.cuda.current_device()
        plan = self._plans.get(index)
        if plan is None:
            with torch.cuda.device(index):
                plan = _lib.create_plan(self.config)
            self._plan_owners[plan] = _lib.Owned(plan, _release_plan)
            self._plans[index] = plan
        return plan

    def __getstate__(self):
        state = self.__dict__.copy()
        state["_plans"] = {}
        state["_plan_owners"] = {}
        return state

    # ------------------------------------------------------------------
    # evaluation
    # ------------------------------------------------------------------

    def _evaluate(self, ref: torch.Tensor, deg: torch.Tensor):
        deg, ref = torch.atleast_2d(deg), torch.atleast_2d(ref)
        if ref.shape != deg.shape:
            raise ValueError(
                "Reference and degraded signal must have the same shape, "
                f"got {tuple(ref.shape)} and {tuple(deg.shape)}."
            )
        _check_signal(ref, "ref")
        _check_signal(deg, "deg")
        if ref.dim() != 2:
            raise ValueError(f"expected [batch, sample] signals, got {tuple(ref.shape)}")
        if ref.device != deg.device:
            raise RuntimeError("ref and deg must live on the same device")
        if ref.stride(-1) != 1:
            ref = ref.contiguous()
        if deg.stride(-1) != 1:
            deg = deg.contiguous()
        plan = self._plan(ref.device)
        # eager autograd nodes keep the plan alive (a traced graph holds the
        # handle as a constant and its caller the module)
        owner = None if torch.compiler.is_compiling() else self._plan_owners[plan]
        return _PesqFunction.apply(ref, deg, plan, owner)

    def raw(self, ref: torch.Tensor, deg: torch.Tensor) -> Tuple[torch.Tensor, torch.Tensor]:
        """Symmetric and asymmetric distance, both ``[batch]`` (loss.py:172-268)."""

        d_symm, d_asymm = self._evaluate(ref, deg)[:2]
        return d_symm, d_asymm

    def mos(self, ref: torch.Tensor, deg: torch.Tensor) -> torch.Tensor:
        """Mean opinion score in (1.08, 4.999) (loss.py:271-297)."""

        return self._evaluate(ref, deg)[2]

    def forward(self, ref: torch.Tensor, deg: torch.Tensor) -> torch.Tensor:
        """Loss ``factor * (0.1 d_symm + 0.0309 d_asymm)`` (loss.py:300-322)."""

        return self._evaluate(ref, deg)[3]

    def forward_sum(self, ref: torch.Tensor, deg: torch.Tensor) -> Tuple[torch.Tensor, torch.Tensor]:
        """``forward`` plus the float64 pair [sum of the batch's losses, batch],
        summed by the chain kernel itself (no extra launch): the numerator and
        denominator of the global mean a data-parallel step all-reduces
        (``distributed.GlobalMean``).  The pair is not differentiable."""

        out = self._evaluate(ref, deg)
        return out[3], out[4]

    def graphed(self, ref: torch.Tensor, deg: torch.Tensor):
        """Capture forward (and backward) in a CUDA graph for one input shape.

        Mirrors ``PesqLossTriton.graphed`` (triton_ops/loss.py:149-201): the
        returned callable replaces ``self.__call__`` for inputs of this shape
        and these ``requires_grad`` flags and is bit exact w.r.t. eager
        evaluation.  The plan is built and every kernel configured before the
        capture, which then only records launches.
        """

        sample = tuple(t.detach().clone().requires_grad_(t.requires_grad) for t in (ref, deg))
        self._plan(sample[0].device)
        stream = torch.cuda.Stream()
        stream.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(stream):
            out = self(*sample)
            if out.requires_grad:
                torch.autograd.grad(out.sum(), [t for t in sample if t.requires_grad])
        torch.cuda.current_stream().wait_stream(stream)
        torch.cuda.synchronize()
        return torch.cuda.make_graphed_callables(self, sample)

    def extra_repr(self) -> str:
        return f"factor={self.factor}, sample_rate={self.source_sample_rate}"
