"""D-head diagonal scan on the GPU: kernel against the oracle (forward, backward, full and
separable read, M = 1..32, ragged checkpoint blocks) and the drop-in D heads against the
reference fixtures (output, state, every gradient, decode steps).  fp32 bar: 1e-4 relative."""
import numpy as np
import pytest
import torch

from oracle import dscan as dor
from tests._util import TOL_F32, cuda, relerr
from tests.golden import fixtures as fx

pytestmark = pytest.mark.gpu

CASES = [  # B, T, M, G, V, sep  (T > 64: 16-token blocks in parallel; otherwise one pass)
    (2, 45, 4, 4, 32, False), (2, 37, 8, 4, 16, True), (1, 100, 16, 8, 64, True),
    (3, 16, 1, 1, 32, False), (2, 5, 32, 16, 32, False), (2, 33, 2, 2, 32, True),
    (2, 203, 4, 4, 32, False), (2, 150, 32, 16, 32, True), (1, 1001, 16, 8, 64, True),
    (2, 65, 8, 2, 64, False), (1, 80, 1, 1, 32, True),
]


@pytest.mark.parametrize("blocks", [True, False])
@pytest.mark.parametrize("case", CASES)
def test_dscan_vs_oracle(case, blocks):
    from sca2_b200 import ops
    B, T, M, G, V, sep = case
    rng = np.random.default_rng(B * T + M)
    a_re, a_im = 0.6 * rng.standard_normal((B, T, M, G)), 0.6 * rng.standard_normal((B, T, M, G))
    v = rng.standard_normal((B, T, V))
    cs = (B, T, M) if sep else (B, T, M, V)
    c_re, c_im = rng.standard_normal(cs), rng.standard_normal(cs)
    S0 = (0.3 * rng.standard_normal((B, M, V)), 0.3 * rng.standard_normal((B, M, V)))
    dab = rng.standard_normal((B, T, 2, V))
    dS = (rng.standard_normal((B, M, V)), rng.standard_normal((B, M, V)))
    t = [cuda(x, torch.float32, True) for x in (a_re, a_im, v, c_re, c_im, S0[0], S0[1])]
    ab, (sr, si) = ops.dscan(t[0], t[1], t[2], t[3], t[4], (t[5], t[6]), sep=sep, blocks=blocks)
    ((ab * cuda(dab)).sum() + (sr * cuda(dS[0])).sum() + (si * cuda(dS[1])).sum()).backward()
    rab, (rsr, rsi) = dor.dscan_forward(a_re, a_im, v, c_re, c_im, S0, sep=sep)
    g = dor.dscan_backward(a_re, a_im, v, c_re, c_im, S0, dab, dS, sep=sep)
    assert relerr(ab, rab) < TOL_F32 and relerr(sr, rsr) < TOL_F32 and relerr(si, rsi) < TOL_F32
    for k, n in enumerate(("a_re", "a_im", "v", "c_re", "c_im")):
        assert relerr(t[k].grad, g[n]) < TOL_F32, n
    assert relerr(t[5].grad, g["S0"][0]) < TOL_F32 and relerr(t[6].grad, g["S0"][1]) < TOL_F32


@pytest.mark.parametrize("name,cls", [("head_dref.npz", "DHeadRef"), ("head_dsepq.npz", "DHeadSepQ"),
                                      ("head_dpolar.npz", "DHeadSepQPolar")])
def test_dhead_vs_reference(name, cls):
    from sca2_b200 import heads
    f = fx.load(name)
    B, T, d, M, G, dv, gated = (int(x) for x in f["meta"])
    head = getattr(heads, cls)(d, M, G, dv=dv, gated_read=bool(gated)).cuda()
    head.load_state_dict({k[3:]: torch.tensor(f[k]) for k in f if k.startswith("sd_")}, strict=True)
    z, h = cuda(f["z"], torch.float32, True), cuda(f["h"], torch.float32, True)
    u, st = head.prefill(z, h, {"sr": cuda(f["sr0"]), "si": cuda(f["si0"])})
    (u * cuda(f["dU"])).sum().backward()
    assert relerr(u, f["u"]) < TOL_F32
    assert relerr(st["sr"], f["sr"]) < TOL_F32 and relerr(st["si"], f["si"]) < TOL_F32
    assert relerr(z.grad, f["d_z"]) < TOL_F32 and relerr(h.grad, f["d_h"]) < TOL_F32
    for n, p in head.named_parameters():
        assert relerr(p.grad, f["g_" + n]) < TOL_F32, n
    st = {"sr": cuda(f["sr"]), "si": cuda(f["si"])}
    with torch.no_grad():
        for t in range(f["zs"].shape[1]):
            ut, st = head.step(cuda(f["zs"][:, t]), cuda(f["hs"][:, t]), st)
            assert relerr(ut, f["us"][:, t]) < TOL_F32
    assert relerr(st["sr"], f["srs"]) < TOL_F32 and relerr(st["si"], f["sis"]) < TOL_F32


def test_dscan_empty_and_unsupported():
    from sca2_b200 import _lib, ops
    z = lambda *s: torch.zeros(*s, device="cuda")
    S0 = (torch.randn(2, 4, 32, device="cuda"), torch.randn(2, 4, 32, device="cuda"))
    ab, (sr, si) = ops.dscan(z(2, 0, 4, 4), z(2, 0, 4, 4), z(2, 0, 32), z(2, 0, 4, 32), z(2, 0, 4, 32), S0)
    assert ab.shape == (2, 0, 2, 32) and torch.equal(sr, S0[0]) and torch.equal(si, S0[1])
    with pytest.raises(_lib.Sca2Error):  # M not a power of two
        ops.dscan(z(1, 3, 3, 1), z(1, 3, 3, 1), z(1, 3, 32), z(1, 3, 3, 32), z(1, 3, 3, 32))
    with pytest.raises(_lib.Sca2Error):  # 4 channels per group < 32 / M = 8
        ops.dscan(z(1, 3, 4, 8), z(1, 3, 4, 8), z(1, 3, 32), z(1, 3, 4, 32), z(1, 3, 4, 32))


@pytest.mark.parametrize("sep", [True, False])
def test_dscan_blocks_long_sequence(sep):
    """The block-parallel form against the sequential one on a long sequence (no oracle at
    this size): read, final state and every gradient agree to fp32 rounding."""
    from sca2_b200 import ops
    B, T, M, G, V = 2, 4096, 16, 8, 64
    g = torch.Generator(device="cuda").manual_seed(5)
    rn = lambda *sh: torch.randn(*sh, device="cuda", generator=g)
    mag = torch.exp(-torch.nn.functional.softplus(rn(B, T, M, G)))
    ph = rn(B, T, M, G)
    cs = (B, T, M) if sep else (B, T, M, V)
    base = [mag * torch.cos(ph), mag * torch.sin(ph), rn(B, T, V), rn(*cs), rn(*cs), rn(B, M, V), rn(B, M, V)]
    dab, dS = rn(B, T, 2, V), (rn(B, M, V), rn(B, M, V))
    res = []
    for blocks in (True, False):
        t = [x.clone().requires_grad_(True) for x in base]
        ab, (sr, si) = ops.dscan(*t[:5], (t[5], t[6]), sep=sep, blocks=blocks)
        ((ab * dab).sum() + (sr * dS[0]).sum() + (si * dS[1]).sum()).backward()
        res.append([ab.detach(), sr.detach(), si.detach()] + [x.grad for x in t])
    for a, b in zip(*res):
        assert relerr(a, b) < TOL_F32
