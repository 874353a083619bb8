"""Load the golden fixtures (made by make_golden.py from the reference's own modules) into
the scan's code-space inputs: per-token tensors (B,T,H,...), per-head (H,...), state
(B,H,2Mh,V) = [sr ; si], raw read o (B,T,H,2,V)."""
from __future__ import annotations

import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))


def load(name):
    with np.load(os.path.join(HERE, name)) as f:
        return {k: f[k] for k in f.files}


def _single_head(f, with_beta=True, with_lam=False):
    """Single-head fixtures (LongHead, CHeadDelta, CHeadDeltaDamp): add an H=1 axis."""
    B, T, M = f["phw"].shape
    dv = f["v"].shape[-1]
    inp = dict(
        phw=f["phw"][:, :, None], phq=f["phq"][:, :, None], v=f["v"][:, :, None],
        beta=f["beta"][:, :, None] if with_beta else None, g=None,
        lam=f["lam"][None] if with_lam else None,
        wr=f["wr"][None], wi=f["wi"][None],
        S0=np.concatenate([f["sr0"], f["si0"]], 1)[:, None],
    )
    out = dict(o=f["o"].reshape(B, T, 1, 2, dv),
               S=np.concatenate([f["sr"], f["si"]], 1)[:, None])
    if "dO" in f:
        out["dO"] = f["dO"].reshape(B, T, 1, 2, dv)
        out["dS"] = np.concatenate([f["dsr"], f["dsi"]], 1)[:, None]
        grads = dict(phw=f["d_phw"][:, :, None], phq=f["d_phq"][:, :, None],
                     v=f["d_v"][:, :, None], wr=f["d_wr"][None], wi=f["d_wi"][None],
                     S0=np.concatenate([f["d_sr0"], f["d_si0"]], 1)[:, None])
        if with_beta:
            grads["blogit"] = f["d_blogit"][:, :, None]
        if with_lam:
            grads["lam_raw"] = f["d_lam_raw"][None]
        out["grads"] = grads
    return inp, out


def longhead(name="scan_longhead.npz"):
    f = load(name)
    inp, out = _single_head(f, with_beta=True, with_lam=True)
    out["lam_mask"] = f["lam_mask"][None]
    out["lam_raw_sig"] = f["lam_raw_sig"][None]
    out["chunk"] = int(f["meta"][4])
    return inp, out


def longhead_step():
    f = load("step_longhead.npz")
    inp, out = _single_head(f, with_beta=True, with_lam=True)
    return inp, out


def cdelta(damp=False):
    f = load("scan_cdelta_damp.npz" if damp else "scan_cdelta.npz")
    inp, out = _single_head(f, with_beta=True, with_lam=damp)
    if damp:
        out["lam_raw_sig"] = f["lam_raw_sig"][None]
    out["chunk"] = int(f["meta"][4])
    return inp, out


def gated():
    """CHeadGated: H heads, scalar decay g = -softplus(xg), additive write.  Its read-out
    u is laid out [re of all heads | im of all heads] (sca2/arch_gatedc.py:155-156)."""
    f = load("scan_gated.npz")
    B, T, H, Mh, dvh, ctx = (int(x) for x in f["meta"])
    sp = lambda x: x.reshape(B, T, H, -1)
    inp = dict(phw=sp(f["phw"]), phq=sp(f["phq"]), v=sp(f["v"]), beta=None, g=f["g"], lam=None,
               wr=f["wr"].reshape(H, Mh), wi=f["wi"].reshape(H, Mh),
               S0=np.concatenate([f["sr0"], f["si0"]], 2))
    u2o = lambda u: u.reshape(B, T, 2, H, dvh).transpose(0, 1, 3, 2, 4)
    grads = dict(phw=sp(f["d_phw"]), phq=sp(f["d_phq"]), v=sp(f["d_v"]), xg=f["d_xg"],
                 wr=f["d_wr"].reshape(H, Mh), wi=f["d_wi"].reshape(H, Mh),
                 S0=np.concatenate([f["d_sr0"], f["d_si0"]], 2))
    out = dict(o=u2o(f["u"]), S=np.concatenate([f["sr"], f["si"]], 2), dO=u2o(f["dU"]),
               dS=np.concatenate([f["dsr"], f["dsi"]], 2), grads=grads, xg=f["xg"], chunk=ctx)
    return inp, out


def gdn():
    return load("gdn_fla.npz")
