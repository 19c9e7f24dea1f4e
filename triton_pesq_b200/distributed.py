"""Data parallelism of the PESQ loss: batch sharding and the scalar mean.

Utterances are scored independently, so a batch splits into contiguous
per-rank slices and every rank evaluates its own slice; per-sample gradients
stay on their rank.  The only collective is the all-reduce of the scalar mean
loss (a sum and a count, 16 bytes over NCCL on NVLink), which the training
loop needs for logging.  Nothing here touches another GPU's memory.
"""

from __future__ import annotations

from typing import Optional, Tuple

import torch
import torch.distributed as dist


def shard_bounds(batch: int, rank: int, world: int) -> Tuple[int, int]:
    """Half-open slice of a batch owned by ``rank``: contiguous, sizes differ by at most one."""

    if world <= 0 or not 0 <= rank < world:
        raise ValueError(f"invalid rank {rank} of {world}")
    base, extra = divmod(int(batch), int(world))
    lo = rank * base + min(rank, extra)
    return lo, lo + base + (1 if rank < extra else 0)


def _group_info(group) -> Tuple[int, int]:
    if dist.is_available() and dist.is_initialized():
        return dist.get_rank(group), dist.get_world_size(group)
    return 0, 1


def shard(ref: torch.Tensor, deg: torch.Tensor, group=None) -> Tuple[torch.Tensor, torch.Tensor]:
    """This rank's slice of a global ``[batch, sample]`` pair."""

    rank, world = _group_info(group)
    lo, hi = shard_bounds(ref.shape[0], rank, world)
    return ref[lo:hi], deg[lo:hi]


def mean_loss(local: torch.Tensor, group=None, async_op: bool = False):
    """Global mean of per-utterance losses spread over the ranks.

    ``local`` is this rank's ``[b]`` loss vector (any ``b``, also 0).  The sum
    and the count are reduced together, so uneven shards average correctly.
    Returns the mean as a 0-d tensor (and the work handle when ``async_op``).
    """

    buf = torch.stack([local.detach().double().sum(), torch.tensor(float(local.numel()), dtype=torch.float64,
                                                                    device=local.device)])
    work = None
    if dist.is_available() and dist.is_initialized():
        work = dist.all_reduce(buf, group=group, async_op=async_op)
    if async_op:
        return buf, work
    return buf[0] / buf[1].clamp_min(1.0)


class GlobalMean:
    """The global mean loss of a data-parallel step, capturable in a CUDA graph.

    ``mean_loss`` builds its ``[sum, count]`` message from a host value, which
    a CUDA graph cannot record.  This keeps the message in a persistent
    float64 device buffer instead: every call writes this rank's sum and count
    into it on the current stream, all-reduces it over the process group (an
    NCCL all-reduce of 16 bytes; nothing when no group is initialised) and
    returns the mean as a 0-d device tensor.  The loss gradient does not
    depend on it, so a caller runs it under ``torch.cuda.stream(side)`` and
    joins that stream after the backward: the collective then overlaps the
    backward kernels, in eager mode and inside a captured step alike.  All
    ranks must call it the same number of times, in the same order.
    """

    def __init__(self, device, group=None):
        self.group = group
        self.buf = torch.zeros(2, dtype=torch.float64, device=device)

    def __call__(self, local: torch.Tensor, loss_sum: Optional[torch.Tensor] = None) -> torch.Tensor:
        """``local``: this rank's ``[b]`` losses; ``loss_sum``: their float64
        ``[sum, count]`` pair when the loss module produced it already
        (``PesqLossCuda.forward_sum``: summed inside its chain kernel, so no
        reduction kernel runs here)."""

        if loss_sum is not None:
            self.buf.copy_(loss_sum)
        else:
            self.buf[0] = local.detach().sum(dtype=torch.float64)
            self.buf[1].fill_(float(local.numel()))
        if dist.is_available() and dist.is_initialized():
            dist.all_reduce(self.buf, group=self.group)
        return self.buf[0] / self.buf[1]


class ShardedPesqLoss(torch.nn.Module):
    """Evaluate a PESQ loss module on this rank's slice of a global batch.

    ``forward(ref, deg)`` takes the *global* batch, scores this rank's slice
    and returns ``(local_losses, global_mean)``: the local per-utterance losses
    (differentiable, for the backward of this rank's inputs) and the detached
    global mean for logging.
    """

    def __init__(self, loss: torch.nn.Module, group=None):
        super().__init__()
        self.loss = loss
        self.group = group

    def forward(self, ref: torch.Tensor, deg: torch.Tensor):
        r, d = shard(ref, deg, self.group)
        if hasattr(self.loss, "forward_sum"):
            local, pair = self.loss.forward_sum(r, d)
            buf = pair.detach().clone()
            if dist.is_available() and dist.is_initialized():
                dist.all_reduce(buf, group=self.group)
            return local, buf[0] / buf[1].clamp_min(1.0)
        local = self.loss(r, d)
        return local, mean_loss(local, self.group)
