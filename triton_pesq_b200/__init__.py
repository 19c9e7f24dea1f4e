"""B200-native PESQ loss engine.

``PesqLossCuda`` is a drop-in for the reference's ``PesqLossTriton``
(torch_pesq/triton_ops/loss.py) evaluated by hand-written sm_100a kernels
through the C ABI of ``libpesq_cuda.so`` (``include/pesq_cuda.h``);
``ResampleCuda`` is the reference's ``TritonResample`` (its polyphase sinc
resampler as a standalone op) and ``IIRCuda`` its ``TritonIIR`` (the causal
IIR filter as a standalone op) on the same library.
"""

from .iir import IIRCuda
from .loss import PesqLossCuda
from .resample import ResampleCuda

__all__ = ["PesqLossCuda", "ResampleCuda", "IIRCuda"]
