"""Host logic of the sequence-parallel prefill on CPU: two gloo ranks, each holding half of
a sequence split into sub-slabs, with a float64 token-loop scan standing in for the CUDA
kernel; the combined outputs and final state must equal the oracle's scan of the whole
sequence."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

from oracle import scan as ora
from tests._util import seeded_phase_inputs


def _token_scan(phw, phq, v, beta, g, lam, wr, wi, S0):
    """Phase-coded delta scan, one token at a time (float64, CPU)."""
    B, T, H, Mh = phw.shape
    K, V = 2 * Mh, v.shape[-1]
    k = torch.cat([torch.cos(phw), torch.sin(phw)], -1)                       # (B,T,H,K)
    cq, sq = torch.cos(phq), torch.sin(phq)
    c1, c2 = wr * cq + wi * sq, wr * sq - wi * cq
    Qre, Qim = torch.cat([c1, c2], -1), torch.cat([-c2, c1], -1)
    lamf = torch.cat([lam, lam], -1) if lam is not None else torch.zeros(H, K, dtype=phw.dtype)
    S = S0.clone()
    o = torch.zeros(B, T, H, 2, V, dtype=phw.dtype)
    for t in range(T):
        gam = torch.exp(-lamf)[None, :, :, None] * (torch.exp(g[:, t])[:, :, None, None] if g is not None else 1.0)
        S = gam * S
        kt = k[:, t]
        e = v[:, t] - (beta[:, t, :, None] if beta is not None else 0.0) * torch.einsum("bhk,bhkv->bhv", kt, S) / Mh
        S = S + kt[..., None] * e[:, :, None, :]
        o[:, t, :, 0] = torch.einsum("bhk,bhkv->bhv", Qre[:, t], S) / Mh
        o[:, t, :, 1] = torch.einsum("bhk,bhkv->bhv", Qim[:, t], S) / Mh
    return o, S


def _worker(rank, world, port, d, out):
    import torch.distributed as dist
    from sca2_b200.sp import sp_phase_prefill
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=__import__("datetime").timedelta(seconds=60))
    try:
        T = d["phw"].shape[1] // world
        sl = lambda x: None if x is None else torch.tensor(x[:, rank * T:(rank + 1) * T])
        t = lambda x: None if x is None else torch.tensor(x)
        o, S = sp_phase_prefill(sl(d["phw"]), sl(d["phq"]), sl(d["v"]), sl(d["beta"]), sl(d["g"]), t(d["lam"]),
                                t(d["wr"]), t(d["wi"]), t(d["S0"]), split=2, scan=_token_scan, state_dtype=torch.float64)
        out[rank] = (o.numpy(), S.numpy())
    finally:
        dist.destroy_process_group()


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


@pytest.mark.parametrize("gates", [dict(beta=True, g=False, lam=True), dict(beta=True, g=True, lam=True)])
def test_sp_prefill_two_ranks(gates):
    B, T, H, Mh, V = 1, 256, 2, 4, 8
    d = seeded_phase_inputs(B, T, H, Mh, V, seed=5, S0=True, **gates)
    d = {k: (x.astype(np.float64) if isinstance(x, np.ndarray) else x) for k, x in d.items()}
    out = mp.Manager().dict()
    mp.spawn(_worker, args=(2, _free_port(), d, out), nprocs=2, join=True)
    o = np.concatenate([out[0][0], out[1][0]], 1)
    ro, rS = ora.phase_forward(d["phw"], d["phq"], d["v"], d["beta"], d["g"], d["lam"], d["wr"], d["wi"], d["S0"])
    assert np.abs(o - ro).max() < 1e-9 * max(1.0, np.abs(ro).max())
    for r in range(2):
        assert np.abs(out[r][1] - rS).max() < 1e-9 * max(1.0, np.abs(rS).max())
