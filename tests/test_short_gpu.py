"""Short head on the GPU: the window-read kernels against the oracle (forward, new ring
buffer, every gradient incl. the state's, windows L = 1..32, ragged T, T shorter than the
window, decode T = 1, value widths across slices) and the drop-in heads against the
reference fixtures (lapa ShortHead, sca2 CHeadShort).  fp32 bar: 1e-4 relative."""
import numpy as np
import pytest
import torch

from oracle import short as so
from tests._util import TOL_F32, cuda, relerr
from tests.golden import fixtures as fx

pytestmark = pytest.mark.gpu

CASES = [  # B, T, L, dv, pos, with_state
    (2, 45, 8, 6, 5, True), (2, 5, 16, 8, 13, True), (1, 1, 16, 64, 1000003, True),
    (3, 200, 16, 64, 0, False), (2, 130, 32, 130, 7, True), (1, 70, 1, 5, 3, False),
    (2, 64, 4, 3, 2, True), (1, 97, 16, 200, 11, True), (2, 33, 32, 16, 0, True),
]


def _inputs(case, seed):
    B, T, L, dv, pos, with_state = case
    rng = np.random.default_rng(seed)
    n = L - 1
    x = dict(kh=rng.standard_normal((B, T, L)), kz=rng.standard_normal((B, T, L)),
             v=rng.standard_normal((B, T, dv)), theta=0.5 * rng.standard_normal(L),
             omega=np.arange(L) * 2 * np.pi / L, wr=1 + 0.3 * rng.standard_normal(L), wi=0.3 * rng.standard_normal(L))
    if with_state:
        ph = rng.standard_normal((B, n, L))
        x.update(c0=np.cos(ph), s0=np.sin(ph), e0=rng.standard_normal((B, n, dv)))
    else:
        x.update(c0=None, s0=None, e0=None)
    dO = rng.standard_normal((B, T, 2 * dv))
    dn = (rng.standard_normal((B, n, L)), rng.standard_normal((B, n, L)), rng.standard_normal((B, n, dv)))
    return x, pos, dO, dn


@pytest.mark.parametrize("case", CASES)
def test_short_vs_oracle(case):
    from sca2_b200 import ops
    x, pos, dO, dn = _inputs(case, sum(case[:4]))
    omega32 = x["omega"].astype(np.float32).astype(np.float64)  # the kernel's fp32 grid
    t = {k: (cuda(v, torch.float32, k != "omega") if v is not None else None) for k, v in x.items()}
    st = (t["c0"], t["s0"], t["e0"]) if t["c0"] is not None else None
    o, (c1, s1, e1) = ops.short_read(t["kh"], t["kz"], t["v"], t["theta"], t["omega"], t["wr"], t["wi"], st,
                                     torch.tensor(pos, device="cuda"))
    ((o * cuda(dO)).sum() + (c1 * cuda(dn[0])).sum() + (s1 * cuda(dn[1])).sum() + (e1 * cuda(dn[2])).sum()).backward()
    ro, rnew = so.short_forward(x["kh"], x["kz"], x["v"], x["theta"], omega32, x["wr"], x["wi"], x["c0"], x["s0"],
                                x["e0"], pos)
    g = so.short_backward(x["kh"], x["kz"], x["v"], x["theta"], omega32, x["wr"], x["wi"], x["c0"], x["s0"],
                          x["e0"], pos, dO, dn)
    assert relerr(o, ro) < TOL_F32
    for a, b in zip((c1, s1, e1), rnew):
        if b.size:
            assert relerr(a, b) < TOL_F32
    for k in ("kh", "kz", "v", "theta", "wr", "wi"):
        assert relerr(t[k].grad, g[k]) < TOL_F32, k
    if st is not None and case[2] > 1:
        for k in ("c0", "s0", "e0"):
            assert relerr(t[k].grad, g[k]) < TOL_F32, k


def test_short_long_sequence():
    """B=1, T=4096, L=16, dv=64 against the oracle (many CTAs, every chunk boundary)."""
    from sca2_b200 import ops
    x, pos, dO, dn = _inputs((1, 4096, 16, 64, 3, True), 9)
    omega32 = x["omega"].astype(np.float32).astype(np.float64)
    t = {k: (cuda(v, torch.float32, k != "omega") if v is not None else None) for k, v in x.items()}
    o, _ = ops.short_read(t["kh"], t["kz"], t["v"], t["theta"], t["omega"], t["wr"], t["wi"],
                          (t["c0"], t["s0"], t["e0"]), torch.tensor(pos, device="cuda"))
    (o * cuda(dO)).sum().backward()
    ro, _ = so.short_forward(x["kh"], x["kz"], x["v"], x["theta"], omega32, x["wr"], x["wi"], x["c0"], x["s0"],
                             x["e0"], pos)
    g = so.short_backward(x["kh"], x["kz"], x["v"], x["theta"], omega32, x["wr"], x["wi"], x["c0"], x["s0"],
                          x["e0"], pos, dO)
    assert relerr(o, ro) < TOL_F32
    for k in ("kh", "kz", "v", "theta", "wr", "wi", "c0", "e0"):
        assert relerr(t[k].grad, g[k]) < TOL_F32, k


def test_short_identity_tap():
    """theta = 0, w = 1: the Dirichlet comb is an exact tap at lag 0, o_t = [v_t | 0]
    (sca2/arch_short.py self-test), to fp32 rounding of the comb."""
    from sca2_b200 import ops
    B, T, L, dv = 2, 50, 16, 8
    kh, kz, v = torch.randn(B, T, L, device="cuda"), torch.randn(B, T, L, device="cuda"), torch.randn(B, T, dv, device="cuda")
    omega = (torch.arange(L, dtype=torch.float64) * (2 * np.pi / L)).float().cuda()
    o, _ = ops.short_read(kh, kz, v, torch.zeros(L, device="cuda"), omega, torch.ones(L, device="cuda"),
                          torch.zeros(L, device="cuda"))
    assert (o[..., :dv] - v).abs().max().item() < 1e-5 and o[..., dv:].abs().max().item() < 1e-5


@pytest.mark.parametrize("name,cls", [("head_short_lapa.npz", "ShortHead"), ("head_short_sca2.npz", "CHeadShort")])
def test_short_head_vs_reference(name, cls):
    from sca2_b200 import heads
    f = fx.load(name)
    B, T, d, L, dv, T2, steps = (int(x) for x in f["meta"])
    head = (heads.ShortHead(heads.LaplaceConfig(d=d, L=L, dv=dv)) if cls == "ShortHead"
            else heads.CHeadShort(d, L, dv)).cuda()
    head.load_state_dict({k[3:]: torch.tensor(f[k]).float() for k in f if k.startswith("sd_")}, strict=True)
    z, h = cuda(f["z"], torch.float32, True), cuda(f["h"], torch.float32, True)
    c0, s0, e0 = (cuda(f[k], torch.float32, True) for k in ("c0", "s0", "e0"))
    st = {"c": c0, "s": s0, "e": e0, "pos": torch.tensor(int(f["pos0"]), device="cuda")}
    u, st1 = head.prefill(z, h, st)
    ((u * cuda(f["dU"])).sum() + (st1["c"] * cuda(f["dc1"])).sum() + (st1["s"] * cuda(f["ds1"])).sum()
     + (st1["e"] * cuda(f["de1"])).sum()).backward()
    assert relerr(u, f["u"]) < TOL_F32
    for k in ("c", "s", "e"):
        assert relerr(st1[k], f[k + "1"]) < TOL_F32, k
    assert relerr(z.grad, f["d_z"]) < TOL_F32 and relerr(h.grad, f["d_h"]) < TOL_F32
    assert relerr(c0.grad, f["d_c0"]) < TOL_F32 and relerr(s0.grad, f["d_s0"]) < TOL_F32
    assert relerr(e0.grad, f["d_e0"]) < TOL_F32
    for n, p in head.named_parameters():
        assert relerr(p.grad, f["g_" + n]) < TOL_F32, n
    with torch.no_grad():
        st = {k: v.detach() for k, v in st1.items()}
        u2, st = head.prefill(cuda(f["z2"]), cuda(f["h2"]), st)
        assert relerr(u2, f["u2"]) < TOL_F32
        for k in ("c", "s", "e"):
            assert relerr(st[k], f[k + "2"]) < TOL_F32, k
        for t in range(steps):
            ut, st = head.step(cuda(f["zs"][:, t]), cuda(f["hs"][:, t]), st)
            assert relerr(ut, f["us"][:, t]) < TOL_F32
        assert relerr(st["c"], f["cs"]) < TOL_F32 and relerr(st["e"], f["es"]) < TOL_F32
        assert int(st["pos"]) == int(f["pos_end"])


def test_short_empty_and_unsupported():
    from sca2_b200 import _lib, ops
    L, dv, B = 8, 4, 2
    z = lambda *s: torch.zeros(*s, device="cuda")
    st = (torch.randn(B, L - 1, L, device="cuda"), torch.randn(B, L - 1, L, device="cuda"), torch.randn(B, L - 1, dv, device="cuda"))
    o, new = ops.short_read(z(B, 0, L), z(B, 0, L), z(B, 0, dv), z(L), z(L), z(L), z(L), st)
    assert o.shape == (B, 0, 2 * dv) and all(torch.equal(a, b) for a, b in zip(new, st))
    with pytest.raises(_lib.Sca2Error):  # window beyond 32
        ops.short_read(z(1, 3, 40), z(1, 3, 40), z(1, 3, 4), z(40), z(40), z(40), z(40))
