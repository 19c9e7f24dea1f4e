"""B200-native PESQ loss engine.

``PesqLossCuda`` is a drop-in for the reference's ``PesqLossTriton``
(torch_pesq/triton_ops/loss.py) evaluated by hand-written sm_100a kernels
through the C ABI of ``libpesq_cuda.so`` (``include/pesq_cuda.h``).
"""

from .loss import PesqLossCuda

__all__ = ["PesqLossCuda"]
