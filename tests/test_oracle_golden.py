"""Pin the CPU oracle to the golden fixtures made from the reference's own modules.

The oracle (oracle/scan.py) is the checker every GPU parity test uses, so it is checked
here first, in float64, against outputs and autograd gradients of the unmodified
reference heads (lapa.layer.LongHead, sca2.arch_cdelta.CHeadDelta,
sca2.arch_damp.CHeadDeltaDamp, sca2.arch_gatedc.CHeadGated) and of fla's naive GDN.
"""
import numpy as np
import pytest

from oracle import scan as ora
from tests.golden import fixtures as fx

TOL = 1e-10  # float64 vs float64 (the reference's own fp64 tolerance, sca2/iso.py:24)
TOL_FLA = 2e-5  # fla's naive GDN casts every input to float32 internally (naive.py:42,100)


def _rel(a, b):
    return float(np.abs(np.asarray(a) - np.asarray(b)).max() / max(np.abs(b).max(), 1e-30))


def _check_phase(inp, out, chunked, C=16):
    o, S = ora.phase_forward(inp["phw"], inp["phq"], inp["v"], inp["beta"], inp["g"],
                             inp["lam"], inp["wr"], inp["wi"], inp["S0"], chunked=chunked, C=C)
    assert _rel(o, out["o"]) < TOL
    assert _rel(S, out["S"]) < TOL
    if "grads" not in out:
        return None
    gr = ora.phase_backward(inp["phw"], inp["phq"], inp["v"], inp["beta"], inp["g"],
                            inp["lam"], inp["wr"], inp["wi"], inp["S0"], out["dO"], out["dS"],
                            chunked=chunked, C=C)
    ref = out["grads"]
    for n in ("phw", "phq", "v", "wr", "wi", "S0"):
        assert _rel(gr[n], ref[n]) < TOL, n
    return gr


@pytest.mark.parametrize("chunked", [False, True])
@pytest.mark.parametrize("name", ["scan_longhead.npz", "scan_longhead_chunkpath.npz"])
def test_longhead(name, chunked):
    inp, out = fx.longhead(name)
    gr = _check_phase(inp, out, chunked)
    b = inp["beta"]
    assert _rel(gr["beta"] * b * (1 - b), out["grads"]["blogit"]) < TOL
    dlam_raw = gr["lam"] * out["lam_raw_sig"] * out["lam_mask"]
    assert _rel(dlam_raw, out["grads"]["lam_raw"]) < TOL


@pytest.mark.parametrize("chunked", [False, True])
@pytest.mark.parametrize("damp", [False, True])
def test_cdelta(damp, chunked):
    inp, out = fx.cdelta(damp)
    gr = _check_phase(inp, out, chunked)
    b = inp["beta"]
    assert _rel(gr["beta"] * b * (1 - b), out["grads"]["blogit"]) < TOL
    if damp:
        assert _rel(gr["lam"] * out["lam_raw_sig"], out["grads"]["lam_raw"]) < TOL


@pytest.mark.parametrize("chunked", [False, True])
def test_gated(chunked):
    inp, out = fx.gated()
    gr = _check_phase(inp, out, chunked)
    dxg = gr["g"] * -(1.0 / (1.0 + np.exp(-out["xg"])))   # g = -softplus(xg)
    assert _rel(dxg, out["grads"]["xg"]) < TOL


def test_longhead_step():
    inp, out = fx.longhead_step()
    o, S = ora.phase_forward(inp["phw"], inp["phq"], inp["v"], inp["beta"], None, inp["lam"],
                             inp["wr"], inp["wi"], inp["S0"])
    assert _rel(o, out["o"]) < TOL
    assert _rel(S, out["S"]) < TOL


@pytest.mark.parametrize("chunked", [False, True])
def test_gdn_fla(chunked):
    f = fx.gdn()
    o, S = ora.gdn_forward(f["q"], f["k"], f["v"], f["g"], f["beta"], S0=f["S0"], chunked=chunked,
                           C=16)
    assert _rel(o, f["o"]) < TOL_FLA and _rel(o, f["o_rec"]) < TOL_FLA
    assert _rel(S, f["S"]) < TOL_FLA and _rel(S, f["S_rec"]) < TOL_FLA
    gr = ora.gdn_backward(f["q"], f["k"], f["v"], f["g"], f["beta"], f["dO"], S0=f["S0"],
                          dS_final=f["dS"], chunked=chunked, C=16)
    for n in ("q", "k", "v", "g", "beta", "S0"):
        assert _rel(gr[n], f["d_" + n]) < TOL_FLA, n


def test_chunk_invariance():
    """The closed form does not depend on the chunk size (sca2/test_chunk_invariance.py:37)."""
    inp, out = fx.longhead()
    ref, _ = ora.phase_forward(inp["phw"], inp["phq"], inp["v"], inp["beta"], None, inp["lam"],
                               inp["wr"], inp["wi"], inp["S0"])
    for C in (1, 7, 16, 64):
        o, _ = ora.phase_forward(inp["phw"], inp["phq"], inp["v"], inp["beta"], None, inp["lam"],
                                 inp["wr"], inp["wi"], inp["S0"], chunked=True, C=C)
        assert _rel(o, ref) < TOL


# ---- D heads ---------------------------------------------------------------------------------
@pytest.mark.parametrize("name,kind", [("head_dref.npz", "ref"), ("head_dsepq.npz", "sepq"),
                                       ("head_dpolar.npz", "polar")])
def test_dhead_oracle_vs_reference(name, kind):
    """The numpy D-head scan (with the heads' projections) reproduces the reference heads:
    prefill output, new state and decode steps."""
    from oracle import dscan as dor
    f = fx.load(name)
    B, T, d, M, G, dv, _ = (int(x) for x in f["meta"])
    sd = {k[3:]: f[k] for k in f if k.startswith("sd_")}
    u, (sr, si) = dor.d_head(kind, sd, f["z"], f["h"], (f["sr0"], f["si0"]), M, G, dv)
    assert np.abs(u - f["u"]).max() < 1e-9 and np.abs(sr - f["sr"]).max() < 1e-9
    assert np.abs(si - f["si"]).max() < 1e-9
    S = (f["sr"], f["si"])
    for t in range(f["zs"].shape[1]):
        ut, S = dor.d_head(kind, sd, f["zs"][:, t:t + 1], f["hs"][:, t:t + 1], S, M, G, dv)
        assert np.abs(ut[:, 0] - f["us"][:, t]).max() < 1e-9
    assert np.abs(S[0] - f["srs"]).max() < 1e-9 and np.abs(S[1] - f["sis"]).max() < 1e-9


@pytest.mark.parametrize("sep", [False, True])
def test_dscan_oracle_backward_finite_difference(sep):
    """The oracle's adjoint against central differences of its forward."""
    from oracle import dscan as dor
    rng = np.random.default_rng(3 + sep)
    B, T, M, G, V = 2, 7, 4, 2, 8
    a_re, a_im = 0.6 * rng.standard_normal((B, T, M, G)), 0.6 * rng.standard_normal((B, T, M, G))
    v = rng.standard_normal((B, T, V))
    cs = (B, T, M) if sep else (B, T, M, V)
    c_re, c_im = rng.standard_normal(cs), rng.standard_normal(cs)
    S0 = (rng.standard_normal((B, M, V)), rng.standard_normal((B, M, V)))
    dab = rng.standard_normal((B, T, 2, V))
    dS = (rng.standard_normal((B, M, V)), rng.standard_normal((B, M, V)))
    g = dor.dscan_backward(a_re, a_im, v, c_re, c_im, S0, dab, dS, sep=sep)

    def loss(a_re, a_im, v, c_re, c_im, s0r, s0i):
        ab, S = dor.dscan_forward(a_re, a_im, v, c_re, c_im, (s0r, s0i), sep=sep)
        return (ab * dab).sum() + (S[0] * dS[0]).sum() + (S[1] * dS[1]).sum()
    args = [a_re, a_im, v, c_re, c_im, S0[0], S0[1]]
    names = ["a_re", "a_im", "v", "c_re", "c_im", "s0r", "s0i"]
    for k, n in enumerate(names):
        x = args[k]
        idx = tuple(rng.integers(0, s) for s in x.shape)
        e = 1e-6
        xp, xm = x.copy(), x.copy()
        xp[idx] += e
        xm[idx] -= e
        fd = (loss(*[xp if i == k else args[i] for i in range(7)]) -
              loss(*[xm if i == k else args[i] for i in range(7)])) / (2 * e)
        an = g["S0"][0][idx] if n == "s0r" else g["S0"][1][idx] if n == "s0i" else g[n][idx]
        assert abs(fd - an) < 1e-6 * max(1.0, abs(fd)), (n, fd, an)


# ---- short heads -----------------------------------------------------------------------------
def _rms_bwd(o, du, eps=1e-6):
    r = 1.0 / np.sqrt((o * o).mean(-1, keepdims=True) + eps)
    return r * du - o * r ** 3 * (o * du).mean(-1, keepdims=True)


@pytest.mark.parametrize("name", ["head_short_lapa.npz", "head_short_sca2.npz"])
def test_short_oracle_vs_reference(name):
    """The numpy window read (with the heads' projections and RMS) reproduces the reference
    short heads: prefill output, new ring buffer, every gradient (hand-written adjoint plus
    the projections' chain rule), a second prefill shorter than the window and decode steps."""
    from oracle import short as so
    f = fx.load(name)
    B, T, d, L, dv, T2, steps = (int(x) for x in f["meta"])
    sd = {k[3:]: f[k] for k in f if k.startswith("sd_")}
    pos0 = int(f["pos0"])
    st = {"c": f["c0"], "s": f["s0"], "e": f["e0"]}
    u, st1 = so.short_head(sd, f["z"], f["h"], st, pos0)
    assert np.abs(u - f["u"]).max() < 1e-9
    for k in ("c", "s", "e"):
        assert np.abs(st1[k] - f[k + "1"]).max() < 1e-9
    # gradients: rms, the window read's adjoint, then the projections
    K, V = sd["K.weight"], sd["V.weight"]
    kh, kz, v = f["h"] @ K.T, f["z"] @ K.T, f["z"] @ V.T
    o, _ = so.short_forward(kh, kz, v, sd["theta"], sd["omega"], sd["wr"], sd["wi"], f["c0"], f["s0"], f["e0"], pos0)
    g = so.short_backward(kh, kz, v, sd["theta"], sd["omega"], sd["wr"], sd["wi"], f["c0"], f["s0"], f["e0"], pos0,
                          _rms_bwd(o, f["dU"]), (f["dc1"], f["ds1"], f["de1"]))
    close = lambda a, b: np.abs(a - b).max() < 1e-9 * max(1.0, np.abs(b).max())
    assert close(g["kh"] @ K, f["d_h"])
    assert close(g["kz"] @ K + g["v"] @ V, f["d_z"])
    dK = np.einsum("btl,btd->ld", g["kh"], f["h"]) + np.einsum("btl,btd->ld", g["kz"], f["z"])
    assert close(dK, f["g_K.weight"]) and close(np.einsum("btj,btd->jd", g["v"], f["z"]), f["g_V.weight"])
    for n in ("theta", "wr", "wi"):
        assert close(g[n], f["g_" + n]), n
    assert close(g["c0"], f["d_c0"]) and close(g["s0"], f["d_s0"]) and close(g["e0"], f["d_e0"])
    u2, st2 = so.short_head(sd, f["z2"], f["h2"], st1, pos0 + T)
    assert np.abs(u2 - f["u2"]).max() < 1e-9
    for k in ("c", "s", "e"):
        assert np.abs(st2[k] - f[k + "2"]).max() < 1e-9
    st, pos = st2, pos0 + T + T2
    for t in range(steps):
        ut, st = so.short_head(sd, f["zs"][:, t:t + 1], f["hs"][:, t:t + 1], st, pos)
        pos += 1
        assert np.abs(ut[:, 0] - f["us"][:, t]).max() < 1e-9
    assert np.abs(st["c"] - f["cs"]).max() < 1e-9 and np.abs(st["e"] - f["es"]).max() < 1e-9
    assert pos == int(f["pos_end"])
