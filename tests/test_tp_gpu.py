"""The head-sharded GatedLayer on two GPUs (NCCL, skipped below two GPUs) against the same
layer unsharded on each rank: output, new state, input gradient, every parameter gradient
(after summing the sharded ones over the ranks) and decode steps, fp32 at 1e-4."""
import copy
import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

from tests._util import TOL_F32, relerr

pytestmark = pytest.mark.gpu


def _worker(rank, world, port, out):
    import datetime
    import torch.distributed as dist
    from sca2_b200 import layers, tp
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=120))
    try:
        torch.manual_seed(0)  # the same weights and inputs on every rank
        cfg = layers.LayerCfg(d=64, Mc=64, Md=4, G=8, ff=96, freq="rope", theta_scale=0.3, max_len=512, dv=64,
                              c_heads=4, c_decay=True, conv=3)
        ref = layers.GatedLayer(cfg).cuda()
        x = torch.randn(1, 150, 64, device="cuda")
        dy = torch.randn(1, 150, 64, device="cuda")
        xs = torch.randn(1, 3, 64, device="cuda")
        sh = tp.shard_layer(copy.deepcopy(ref), None)
        res = {}
        for name, lay in (("ref", ref), ("tp", sh)):
            xx = x.clone().requires_grad_(True)
            y, st = lay.prefill(xx)
            (y * dy).sum().backward()
            if name == "tp":
                tp.reduce_sharded_grads(lay)
            with torch.no_grad():
                ys = []
                for t in range(xs.shape[1]):
                    yt, st = lay.step(xs[:, t], st)
                    ys.append(yt)
            res[name] = dict(y=y.detach().cpu(), dx=xx.grad.cpu(), ys=torch.stack(ys, 1).cpu(),
                             sr=st["c"]["sr"].cpu(), grads={n: p.grad.cpu() for n, p in lay.named_parameters()})
        Hr = 4 // world
        res["tp"]["sr_full"] = res["ref"]["sr"][:, rank * Hr:(rank + 1) * Hr]
        out[rank] = res
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_head_sharded_layer_two_gpus():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    out = mp.Manager().dict()
    mp.spawn(_worker, args=(2, port, out), nprocs=2, join=True)
    for r in range(2):
        a, b = out[r]["tp"], out[r]["ref"]
        assert relerr(a["y"], b["y"]) < TOL_F32 and relerr(a["dx"], b["dx"]) < TOL_F32, r
        assert relerr(a["ys"], b["ys"]) < TOL_F32, r
        assert relerr(a["sr"], a["sr_full"]) < TOL_F32, r      # this rank's heads' decode state
        for n, g in b["grads"].items():
            assert relerr(a["grads"][n], g) < TOL_F32, (r, n)
