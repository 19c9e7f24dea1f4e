"""``ResampleCuda``: the polyphase sinc resampler as a standalone op.

Drop-in for the reference's ``TritonResample``
(torch_pesq/triton_ops/resample.py:442-574): same constructor arguments
(``orig_freq``, ``new_freq``, ``lowpass_filter_width``, ``rolloff``,
``resampling_method``, ``beta``), numerically ``torchaudio.transforms.Resample``
with the same arguments (float32 taps designed on the host, identical bit for
bit; accumulated in float64 on the GPU), a ``kernel`` buffer of shape
``[new_step, width_total]``, an autograd backward through the adjoint kernel
and a double backward (the adjoint is itself differentiable, its derivative is
the forward again, as resample.py:386-419).  ``orig_freq == new_freq`` returns
the input unchanged without a kernel, on any device.
"""

from __future__ import annotations

import math
from typing import Dict, Optional

import torch

from . import _lib
from .tables import sinc_resample_kernel

__all__ = ["ResampleCuda"]


class _ResampleAdjoint(torch.autograd.Function):
    """gx = A^T gy, differentiable: its derivative w.r.t. gy is A."""

    @staticmethod
    def forward(ctx, grad_out, handle, n_in, owner):
        ctx.handle = handle
        ctx.owner = owner  # keeps the resampler alive while this node may run
        return torch.ops.pesq_cuda.resample_adjoint(handle, grad_out, n_in)

    @staticmethod
    def backward(ctx, grad_grad_x):
        if not ctx.needs_input_grad[0]:
            return None, None, None, None
        return torch.ops.pesq_cuda.resample(ctx.handle, grad_grad_x), None, None, None


class _ResampleFunction(torch.autograd.Function):
    """y = A x over the rows of x."""

    @staticmethod
    def forward(ctx, waveform, handle, owner):
        ctx.handle = handle
        ctx.owner = owner  # keeps the resampler alive while this node may run
        ctx.n_in = waveform.shape[1]
        return torch.ops.pesq_cuda.resample(handle, waveform)

    @staticmethod
    def backward(ctx, grad_out):
        if not ctx.needs_input_grad[0]:
            return None, None, None
        return _ResampleAdjoint.apply(grad_out, ctx.handle, ctx.n_in, ctx.owner), None, None


class ResampleCuda(torch.nn.Module):
    """Resample a signal from one frequency to another on sm_100a kernels.

    Parameters
    ----------
    orig_freq : int
        Sampling rate of the input signal
    new_freq : int
        Sampling rate of the output signal
    lowpass_filter_width : int
        Number of zero crossings kept in the sinc kernel
    rolloff : float
        Cut-off of the anti-aliasing filter as a fraction of the Nyquist rate
    resampling_method : str
        ``"sinc_interp_hann"`` or ``"sinc_interp_kaiser"``
    beta : Optional[float]
        Shape parameter of the Kaiser window

    Attributes
    ----------
    kernel : torch.Tensor
        Filter bank ``[new_step, width_total]`` (float32), only when the rates differ
    width : int
        Number of samples the input is zero padded with on the left
    """

    def __init__(
        self,
        orig_freq: int = 16000,
        new_freq: int = 16000,
        lowpass_filter_width: int = 6,
        rolloff: float = 0.99,
        resampling_method: str = "sinc_interp_hann",
        beta: Optional[float] = None,
    ):
        super().__init__()
        if orig_freq <= 0 or new_freq <= 0:
            raise ValueError("Original and desired frequency have to be positive.")
        self.orig_freq = orig_freq
        self.new_freq = new_freq
        self.gcd = math.gcd(int(orig_freq), int(new_freq))
        self.lowpass_filter_width = lowpass_filter_width
        self.rolloff = rolloff
        self.resampling_method = resampling_method
        self.beta = beta
        self.orig_step = int(orig_freq) // self.gcd
        self.new_step = int(new_freq) // self.gcd
        # device index -> resampler handle, and handle -> its owner (_lib.Owned)
        self._handles: Dict[int, int] = {}
        self._owners: Dict[int, _lib.Owned] = {}
        if self.orig_freq != self.new_freq:
            self.design = sinc_resample_kernel(
                orig_freq, new_freq, lowpass_filter_width, rolloff, resampling_method, beta
            )
            self.width = self.design.width
            self.register_buffer("kernel", torch.tensor(self.design.taps, dtype=torch.float32))
            _lib.load_ops()
        else:
            self.design = None
            self.width = 0

    def _handle(self, device: torch.device) -> int:
        index = device.index if device.index is not None else torch.cuda.current_device()
        handle = self._handles.get(index)
        if handle is None:
            with torch.cuda.device(index):
                handle = _lib.create_resampler(self.design)
            self._owners[handle] = _lib.Owned(handle, _lib.destroy_resampler)
            self._handles[index] = handle
        return handle

    def __getstate__(self):
        state = self.__dict__.copy()
        state["_handles"] = {}
        state["_owners"] = {}
        return state

    def output_length(self, samples: int) -> int:
        """Number of output samples for ``samples`` input samples."""

        if self.orig_freq == self.new_freq:
            return samples
        from .tables import resample_length

        return resample_length(samples, self.orig_step, self.new_step)

    def forward(self, waveform: torch.Tensor) -> torch.Tensor:
        """Resample a batch of time signals ``[..., sample]`` -> ``[..., resampled]``."""

        if self.orig_freq == self.new_freq:
            return waveform
        if not isinstance(waveform, torch.Tensor):
            raise TypeError("`waveform` must be a torch.Tensor")
        if not waveform.is_cuda:
            raise RuntimeError("The CUDA resampler needs `waveform` to live on a GPU.")
        if waveform.dtype != torch.float32:
            raise RuntimeError(f"The CUDA resampler only supports float32, `waveform` is {waveform.dtype}.")
        if waveform.dim() == 0:
            raise ValueError("`waveform` needs a sample dimension")
        shape = waveform.shape
        rows = math.prod(shape[:-1])
        packed = waveform.reshape(rows, shape[-1])
        handle = self._handle(waveform.device)
        # eager autograd nodes keep the resampler alive (a traced graph holds
        # the handle as a constant and its caller the module)
        owner = None if torch.compiler.is_compiling() else self._owners[handle]
        out = _ResampleFunction.apply(packed, handle, owner)
        return out.reshape(shape[:-1] + out.shape[-1:])

    def extra_repr(self) -> str:
        return f"orig_freq={self.orig_freq}, new_freq={self.new_freq}"
