"""The collectives of the head-sharded C head on CPU (gloo, two ranks): the head gather's
forward concatenates the ranks' slices and its backward returns each rank its own slice with
no communication; the gradient share of the inputs is summed over the ranks."""
import os
import socket

import torch
import torch.multiprocessing as mp


def _worker(rank, world, port, out):
    import torch.distributed as dist
    from sca2_b200 import tp
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world)
    try:
        torch.manual_seed(100 + rank)
        x = torch.randn(2, 3, 2, 4, requires_grad=True)          # this rank's 2 heads
        y = tp._GatherHeads.apply(x, None, world, rank)          # (2, 3, 2 * world, 4)
        w = torch.arange(y.numel(), dtype=torch.float32).view_as(y)  # the same on every rank
        (y * w).sum().backward()
        z = torch.full((3,), float(rank + 1), requires_grad=True)
        (tp._ShareGrad.apply(z, None) * (rank + 1)).sum().backward()
        out[rank] = (x.detach(), y.detach(), x.grad, z.grad)
    finally:
        dist.destroy_process_group()


def test_head_gather_and_gradient_share():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    out = mp.Manager().dict()
    mp.spawn(_worker, args=(2, port, out), nprocs=2, join=True)
    xs = [out[r][0] for r in range(2)]
    full = torch.cat(xs, 2)
    w = torch.arange(full.numel(), dtype=torch.float32).view_as(full)
    for r in range(2):
        assert torch.equal(out[r][1], full)
        assert torch.equal(out[r][2], w[:, :, 2 * r:2 * r + 2])   # own slice of the full gradient
        assert torch.equal(out[r][3], torch.full((3,), 3.0))      # 1 + 2 summed over the ranks
