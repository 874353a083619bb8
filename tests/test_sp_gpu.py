"""Sequence-parallel prefill on the GPU: sub-slab splitting on one GPU, and two NCCL ranks
(skipped below two GPUs), against the plain scan of the whole sequence and the oracle."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

from oracle import scan as ora
from tests._util import TOL_BF16_ABS, TOL_BF16_COS, TOL_F32, cosine, cuda, relerr, rms_np, seeded_phase_inputs

pytestmark = pytest.mark.gpu


def _bf16r(x):
    return torch.tensor(x).bfloat16().double().numpy()


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_sp_split_one_gpu(dtype):
    from sca2_b200 import ops
    from sca2_b200.sp import sp_phase_prefill
    B, T, H, Mh, V = 1, 2048, 4, 32, 64
    d = seeded_phase_inputs(B, T, H, Mh, V, seed=21, g=True, S0=True)
    if dtype == torch.bfloat16:
        d["v"] = _bf16r(d["v"])
    t = {k: cuda(d[k]) for k in ("phw", "phq", "beta", "g", "lam", "wr", "wi", "S0")}
    v = cuda(d["v"], dtype)
    o, S = sp_phase_prefill(t["phw"], t["phq"], v, t["beta"], t["g"], t["lam"], t["wr"], t["wi"], t["S0"], split=8)
    with torch.no_grad():
        o1, S1 = ops.phase_scan(t["phw"], t["phq"], v, t["beta"], t["g"], t["lam"], t["wr"], t["wi"], t["S0"])
    ro, rS = ora.phase_forward(d["phw"].astype(np.float64), d["phq"].astype(np.float64), d["v"], d["beta"], d["g"],
                               d["lam"], d["wr"], d["wi"], d["S0"], chunked=True, C=64)
    if dtype == torch.float32:
        assert relerr(o, ro) < TOL_F32 and relerr(S, rS) < TOL_F32
    else:
        u, ru = rms_np(o.double().cpu().numpy().reshape(B, T, H, -1)), rms_np(ro.reshape(B, T, H, -1))
        assert np.abs(u - ru).max() < TOL_BF16_ABS and cosine(u, ru) > TOL_BF16_COS
        assert relerr(S, rS) < TOL_BF16_ABS
    assert relerr(o.float(), o1.float()) < 3e-2  # same kernels, different split points


def _worker(rank, world, port, d, out):
    import datetime
    import torch.distributed as dist
    from sca2_b200.sp import sp_phase_prefill
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=120))
    try:
        T = d["phw"].shape[1] // world
        dev = torch.device("cuda", rank)
        sl = lambda x, dt=torch.float32: None if x is None else torch.tensor(x[:, rank * T:(rank + 1) * T]).to(dev, dt)
        t = lambda x: None if x is None else torch.tensor(x).to(dev, torch.float32)
        o, S = sp_phase_prefill(sl(d["phw"]), sl(d["phq"]), sl(d["v"], torch.bfloat16), sl(d["beta"]), sl(d["g"]),
                                t(d["lam"]), t(d["wr"]), t(d["wi"]), t(d["S0"]))
        torch.cuda.synchronize()
        out[rank] = (o.float().cpu().numpy(), S.cpu().numpy())
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_sp_two_gpus():
    B, T, H, Mh, V = 1, 4096, 4, 32, 64
    d = seeded_phase_inputs(B, T, H, Mh, V, seed=22, S0=True)
    d["v"] = _bf16r(d["v"])
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    out = mp.Manager().dict()
    mp.spawn(_worker, args=(2, port, d, out), nprocs=2, join=True)
    o = np.concatenate([out[0][0], out[1][0]], 1)
    ro, rS = ora.phase_forward(d["phw"].astype(np.float64), d["phq"].astype(np.float64), d["v"], d["beta"], None,
                               d["lam"], d["wr"], d["wi"], d["S0"], chunked=True, C=64)
    u, ru = rms_np(o.reshape(B, T, H, -1)), rms_np(ro.reshape(B, T, H, -1))
    assert np.abs(u - ru).max() < TOL_BF16_ABS and cosine(u, ru) > TOL_BF16_COS
    for r in range(2):
        assert relerr(out[r][1], rS) < TOL_BF16_ABS
