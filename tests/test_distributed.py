"""Batch sharding and the scalar mean all-reduce on world-size-2 gloo ranks (CPU)."""

import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from triton_pesq_b200.distributed import ShardedPesqLoss, mean_loss, shard_bounds


@pytest.mark.parametrize("batch,world", [(8, 2), (7, 2), (1, 2), (0, 2), (512, 8), (5, 3)])
def test_shards_cover_the_batch_once(batch, world):
    seen = []
    for rank in range(world):
        lo, hi = shard_bounds(batch, rank, world)
        assert 0 <= lo <= hi <= batch
        seen.extend(range(lo, hi))
    assert seen == list(range(batch))
    sizes = [shard_bounds(batch, r, world)[1] - shard_bounds(batch, r, world)[0] for r in range(world)]
    assert max(sizes) - min(sizes) <= 1


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


class _OracleLoss(torch.nn.Module):
    """CPU stand-in for the CUDA loss: the float64 oracle (tests only)."""

    def __init__(self):
        super().__init__()
        from oracle import pesq_oracle as O

        self.O = O
        self.p = O.OracleParams(factor=1.0, sample_rate=16000)

    def forward(self, ref, deg):
        return self.O.forward(ref, deg, self.p)


def _worker(rank, world, port, batch, out):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from triton_pesq_b200.signals import add_noise, speech_like

        ref = speech_like(batch, 8000, 16000, seed=5).double()
        deg = add_noise(ref.float(), 5.0, seed=6).double()
        model = ShardedPesqLoss(_OracleLoss())
        d = deg.clone().requires_grad_(True)
        local, mean = model(ref, d)
        local.sum().backward()
        lo, hi = shard_bounds(batch, rank, world)
        # gradients land only on this rank's rows
        assert torch.all(d.grad[:lo] == 0) and torch.all(d.grad[hi:] == 0)
        out[rank] = (float(mean), local.detach().tolist())
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("batch", [3, 4])
def test_global_mean_over_two_gloo_ranks(batch):
    world = 2
    manager = mp.Manager()
    out = manager.dict()
    mp.spawn(_worker, args=(world, _free_port(), batch, out), nprocs=world, join=True)
    from oracle import pesq_oracle as O
    from triton_pesq_b200.signals import add_noise, speech_like

    ref = speech_like(batch, 8000, 16000, seed=5).double()
    deg = add_noise(ref.float(), 5.0, seed=6).double()
    want = O.forward(ref, deg, O.OracleParams(factor=1.0, sample_rate=16000))
    got_all = out[0][1] + out[1][1]
    assert torch.allclose(torch.tensor(got_all, dtype=torch.float64), want, rtol=1e-12, atol=0)
    for rank in range(world):
        assert out[rank][0] == pytest.approx(float(want.mean()), rel=1e-12)


def test_mean_loss_without_process_group():
    assert float(mean_loss(torch.tensor([1.0, 3.0]))) == 2.0
    assert float(mean_loss(torch.zeros(0))) == 0.0
