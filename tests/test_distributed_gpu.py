"""Data parallelism on two GPUs over NCCL (skipped with fewer than two).

``ShardedPesqLoss(PesqLossCuda)`` on two ranks gives every utterance the
loss and the gradient one GPU gives it when it evaluates the whole batch
(bitwise: utterances are independent and each runs the same kernels), and
both ranks the same global mean; ``GlobalMean`` inside a captured step
(forward, the mean's all-reduce on a side stream, backward) replays to the
same values as the eager step.
"""

import os
import socket

import pytest
import torch

pytestmark = pytest.mark.gpu

BATCH, SAMPLES = 6, 16000


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _inputs():
    from triton_pesq_b200.signals import add_noise, speech_like

    ref = speech_like(BATCH, SAMPLES, 16000, seed=61)
    return ref, add_noise(ref, [0.0, 5.0, 10.0, 15.0, 20.0, -5.0], seed=62)


def _worker(rank, world, port, out):
    import datetime

    import torch.distributed as dist

    from triton_pesq_b200 import PesqLossCuda
    from triton_pesq_b200.distributed import GlobalMean, ShardedPesqLoss, shard_bounds

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dev = torch.device("cuda", rank)
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=dev)
    graph = None
    try:
        ref_c, deg_c = _inputs()
        ref, deg = ref_c.to(dev), deg_c.to(dev).requires_grad_(True)
        model = PesqLossCuda(1.0, sample_rate=16000)
        local, mean = ShardedPesqLoss(model)(ref, deg)
        (grad,) = torch.autograd.grad(local.sum(), [deg])
        lo, hi = shard_bounds(BATCH, rank, world)
        untouched = torch.cat([grad[:lo], grad[hi:]])
        # the same step captured: forward, the mean on a side stream, backward
        r, d = ref[lo:hi], deg_c[lo:hi].to(dev).requires_grad_(True)
        mean_op = GlobalMean(dev)
        side = torch.cuda.Stream(dev)

        def step():
            main = torch.cuda.current_stream(dev)
            loss = model(r, d)
            side.wait_stream(main)
            with torch.cuda.stream(side):
                m = mean_op(loss)
            (g,) = torch.autograd.grad(loss.sum(), [d])
            main.wait_stream(side)
            return loss, g, m

        warm = torch.cuda.Stream(dev)
        warm.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(warm):
            for _ in range(2):
                step()
        torch.cuda.current_stream(dev).wait_stream(warm)
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            g_loss, g_grad, g_mean = step()
        replays = []
        for _ in range(2):
            graph.replay()
            torch.cuda.synchronize()
            replays.append((g_loss.detach().cpu(), g_grad.detach().cpu(), float(g_mean)))
        out[rank] = {
            "local": local.detach().cpu(), "grad": grad[lo:hi].detach().cpu(), "mean": float(mean),
            "untouched_zero": bool(torch.all(untouched == 0)), "replays": replays,
        }
    finally:
        del graph
        dist.destroy_process_group()


def test_sharded_loss_on_two_gpus():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    import torch.multiprocessing as mp

    from triton_pesq_b200 import PesqLossCuda

    world = 2
    manager = mp.Manager()
    out = manager.dict()
    mp.spawn(_worker, args=(world, _free_port(), out), nprocs=world, join=True)

    ref_c, deg_c = _inputs()
    dev = torch.device("cuda", 0)
    deg = deg_c.to(dev).requires_grad_(True)
    whole = PesqLossCuda(1.0, sample_rate=16000)(ref_c.to(dev), deg)
    (grad,) = torch.autograd.grad(whole.sum(), [deg])
    whole, grad = whole.detach().cpu(), grad.cpu()
    mean = float(whole.double().mean())
    got = torch.cat([out[r]["local"] for r in range(world)])
    assert torch.equal(got, whole)
    assert torch.equal(torch.cat([out[r]["grad"] for r in range(world)]), grad)
    for r in range(world):
        assert out[r]["untouched_zero"]
        assert out[r]["mean"] == pytest.approx(mean, rel=1e-12)
        lo = 0 if r == 0 else BATCH // 2
        for loss, g, m in out[r]["replays"]:
            assert torch.equal(loss, whole[lo:lo + BATCH // 2])
            assert torch.equal(g, grad[lo:lo + BATCH // 2])
            assert m == pytest.approx(mean, rel=1e-12)
