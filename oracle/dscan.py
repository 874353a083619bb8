"""CPU oracle of the D-head diagonal scan (test infrastructure only: tests, smoke and the
bench's CPU baseline may call it; the product path never does).

Restates, in numpy float64 token loops:
  * the recurrence of DHeadRef.prefill / step (sca2/ref.py:239-275) and of DHeadSepQ's
    plain prefill / step (sca2/arch_sepq.py:110-178, same recurrence in chunked closed form):
        s_t[m, j] = a_t[m, g(j)] s_{t-1}[m, j] + v_t[j]      (complex s and a, real v)
  * the read contracted over m (ref.py:252-256 with c = q / |q|; arch_sepq.py:100-104 with
    c = alpha over m):  A = mean_m (sr cr + si ci),  Bv = mean_m (si cr - sr ci)
  * its adjoint (reverse sweep) for every input;
  * the heads' projections and epilogues on top (tanh / sqrt 2 cartesian gate
    ref.py:244-245, log-polar gate arch_sepq.py:275-278, query normalisations
    ref.py:252-255 and arch_sepq.py:93-98, separable output arch_sepq.py:100-104,
    RMS and the gated read-out ref.py:29-50).
Pinned in tests/test_oracle_golden.py against fixtures made by the reference's own heads.
"""
from __future__ import annotations

import numpy as np


def dscan_forward(a_re, a_im, v, c_re, c_im, S0=None, sep=False):
    """a (B,T,M,G), v (B,T,V), c (B,T,M,V) or (B,T,M) with sep; S0 = (sr, si) (B,M,V).
    Returns ab (B,T,2,V) and (sr, si)."""
    B, T, M, G = a_re.shape
    V = v.shape[-1]
    gs = V // G
    sr = np.zeros((B, M, V)) if S0 is None else np.array(S0[0], np.float64)
    si = np.zeros((B, M, V)) if S0 is None else np.array(S0[1], np.float64)
    ab = np.zeros((B, T, 2, V))
    for t in range(T):
        ar = np.repeat(a_re[:, t], gs, axis=-1)           # (B,M,V)
        ai = np.repeat(a_im[:, t], gs, axis=-1)
        sr, si = ar * sr - ai * si + v[:, t, None, :], ar * si + ai * sr
        cr = c_re[:, t, :, None] if sep else c_re[:, t]
        ci = c_im[:, t, :, None] if sep else c_im[:, t]
        ab[:, t, 0] = (sr * cr + si * ci).mean(1)
        ab[:, t, 1] = (si * cr - sr * ci).mean(1)
    return ab, (sr, si)


def dscan_backward(a_re, a_im, v, c_re, c_im, S0, dab, dS=None, sep=False):
    """Adjoint of dscan_forward: gradients of sum(ab * dab) + sum(S * dS) for every input."""
    B, T, M, G = a_re.shape
    V = v.shape[-1]
    gs = V // G
    sr = np.zeros((B, M, V)) if S0 is None else np.array(S0[0], np.float64)
    si = np.zeros((B, M, V)) if S0 is None else np.array(S0[1], np.float64)
    hist = []
    for t in range(T):
        hist.append((sr, si))
        ar = np.repeat(a_re[:, t], gs, axis=-1)
        ai = np.repeat(a_im[:, t], gs, axis=-1)
        sr, si = ar * sr - ai * si + v[:, t, None, :], ar * si + ai * sr
    dsr = np.zeros((B, M, V)) if dS is None else np.array(dS[0], np.float64)
    dsi = np.zeros((B, M, V)) if dS is None else np.array(dS[1], np.float64)
    da_re, da_im = np.zeros_like(a_re), np.zeros_like(a_im)
    dv = np.zeros_like(v)
    dc_re, dc_im = np.zeros_like(c_re), np.zeros_like(c_im)
    for t in range(T - 1, -1, -1):
        pr, pi = hist[t]
        ar = np.repeat(a_re[:, t], gs, axis=-1)
        ai = np.repeat(a_im[:, t], gs, axis=-1)
        s_r = ar * pr - ai * pi + v[:, t, None, :]
        s_i = ar * pi + ai * pr
        gA = dab[:, t, 0][:, None, :] / M
        gB = dab[:, t, 1][:, None, :] / M
        cr = c_re[:, t, :, None] if sep else c_re[:, t]
        ci = c_im[:, t, :, None] if sep else c_im[:, t]
        dsr = dsr + gA * cr - gB * ci
        dsi = dsi + gA * ci + gB * cr
        er, ei = gA * s_r + gB * s_i, gA * s_i - gB * s_r
        if sep:
            dc_re[:, t] = er.sum(-1)
            dc_im[:, t] = ei.sum(-1)
        else:
            dc_re[:, t] = er
            dc_im[:, t] = ei
        dv[:, t] = dsr.sum(1)
        da_re[:, t] = (dsr * pr + dsi * pi).reshape(B, M, G, gs).sum(-1)
        da_im[:, t] = (-dsr * pi + dsi * pr).reshape(B, M, G, gs).sum(-1)
        dsr, dsi = ar * dsr + ai * dsi, -ai * dsr + ar * dsi
    return dict(a_re=da_re, a_im=da_im, v=dv, c_re=dc_re, c_im=dc_im, S0=(dsr, dsi))


# ---- heads on top of the scan (numpy, float64) ---------------------------------------------
def _lin(sd, name, x):
    y = x @ sd[name + ".weight"].T
    b = sd.get(name + ".bias")
    return y if b is None else y + b


def _rms(u, eps=1e-6):
    return u / np.sqrt((u * u).mean(-1, keepdims=True) + eps)


def _softplus(x):
    return np.logaddexp(0.0, x)


def d_head(kind, sd, z, h, S0, M, G, dv):
    """u (B,T,2dv) and the new state of a D head ("ref" | "sepq" | "polar") with the
    reference's parameters `sd` (state_dict arrays) on inputs z, h (B,T,d)."""
    B, T, _ = z.shape
    gr, gi = _lin(sd, "gr", h).reshape(B, T, M, G), _lin(sd, "gi", h).reshape(B, T, M, G)
    if kind == "polar":
        mag = np.exp(-_softplus(gr))
        a_re, a_im = mag * np.cos(gi), mag * np.sin(gi)
    else:
        a_re, a_im = np.tanh(gr) / np.sqrt(2.0), np.tanh(gi) / np.sqrt(2.0)
    v = _lin(sd, "V", z)
    if kind == "ref":
        qr, qi = _lin(sd, "qr", z).reshape(B, T, M, dv), _lin(sd, "qi", z).reshape(B, T, M, dv)
        qn = np.sqrt(qr * qr + qi * qi + 1e-6)
        ab, S = dscan_forward(a_re, a_im, v, qr / qn, qi / qn, S0)
        return _rms(ab.reshape(B, T, 2 * dv)), S
    ar, ai = _lin(sd, "qa_r", z), _lin(sd, "qa_i", z)
    br, bi = _lin(sd, "qb_r", z), _lin(sd, "qb_i", z)
    an = 1.0 / np.sqrt(ar * ar + ai * ai + 1e-6)
    bn = 1.0 / np.sqrt(br * br + bi * bi + 1e-6)
    ab, S = dscan_forward(a_re, a_im, v, ar * an, ai * an, S0, sep=True)
    A, Bv = ab[:, :, 0], ab[:, :, 1]
    br, bi = br * bn, bi * bn
    u = _rms(np.concatenate([br * A + bi * Bv, br * Bv - bi * A], -1))
    if "rgate.weight" in sd:
        gz = _lin(sd, "rgate", z)
        u = u * gz / (1.0 + np.exp(-gz))
    return u, S
