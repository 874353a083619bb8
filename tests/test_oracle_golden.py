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
