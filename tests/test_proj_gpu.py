"""Projected phases (the fused phase prologue): the scan fed by K(h), K(z), theta, omega and
the position, with the phases formed inside the kernels, against the same scan fed by the
phases computed in torch with the reference's expression K(x) theta + p omega.  Same kernels
underneath, so outputs agree to rounding; gradients of the projections and of theta come
from the fused backward pass instead of autograd."""
import pytest
import torch

from tests._util import relerr

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("kdt,gates", [(torch.bfloat16, "beta_lam"), (torch.float32, "g"), (torch.bfloat16, "none")])
def test_proj_matches_torch_phases(kdt, gates):
    from sca2_b200 import ops
    g0 = torch.Generator(device="cuda").manual_seed(3)
    rn = lambda *s: torch.randn(*s, device="cuda", generator=g0)
    B, T, H, Mh, V = 2, 203, 4, 32, 128
    kh0, kz0 = rn(B, T, H, Mh).to(kdt), rn(B, T, H, Mh).to(kdt)
    theta0 = 0.5 * rn(H, Mh)
    omega = torch.pi * 1e4 ** (-torch.arange(Mh, device="cuda") / (Mh - 1)).repeat(H, 1)
    pos = torch.tensor(37.0, device="cuda")
    v0 = rn(B, T, H, V).bfloat16()
    beta = torch.sigmoid(rn(B, T, H)) if gates == "beta_lam" else None
    lam = 0.05 * torch.rand(H, Mh, device="cuda", generator=g0) if gates == "beta_lam" else None
    g = -0.1 * torch.rand(B, T, H, device="cuda", generator=g0) if gates == "g" else None
    wr, wi = 1 + 0.3 * rn(H, Mh), 0.3 * rn(H, Mh)
    S0 = 0.1 * rn(B, H, 2 * Mh, V)
    do = rn(B, T, H, 2, V).bfloat16()
    res = []
    for fused in (True, False):
        kh, kz, th, v = (x.clone().requires_grad_(True) for x in (kh0, kz0, theta0, v0))
        if fused:
            assert ops._proj_ok(kh, v)
            o, S = ops.phase_scan_proj(kh, kz, th, omega, pos, v, beta, g, lam, wr, wi, S0)
        else:
            p = (torch.arange(T, device="cuda", dtype=torch.float32) + pos)[:, None, None]
            o, S = ops.phase_scan(kh.float() * th + p * omega, kz.float() * th + p * omega, v, beta, g, lam, wr, wi,
                                  S0)
        ((o.float() * do.float()).sum() + S.sum()).backward()
        res.append([o.float(), S, kh.grad.float(), kz.grad.float(), th.grad, v.grad.float()])
    names = ["o", "S", "dkh", "dkz", "dtheta", "dv"]
    for n, a, b in zip(names, *res):
        assert relerr(a, b) < (1e-5 if n in ("o", "S", "dv") else 2e-3), n
