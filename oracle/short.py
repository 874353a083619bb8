"""CPU oracle of the short head's windowed read (test infrastructure only: tests, smoke and the
bench's CPU baseline may call it; the product path never does).

Restates, in numpy float64 token loops, the exact L-tap window read of
  * lapa.layer.ShortHead (lapa/layer.py:418-545: _phase :444-448, _read :450-469, prefill
    :471-486, _banded :488-522, step :524-545) and
  * sca2.arch_short.CHeadShort (sca2/arch_short.py:45-158, same read; output through
    _gated_out, sca2/ref.py:33-50):

    phi_t = K(h_t) theta + ((pos + t) mod L) omega      (write phase, L modes)
    psi_t = K(z_t) theta + ((pos + t) mod L) omega      (read phase)
    kappa(t, s) = (1/L) sum_m w_m exp(i (phi_s - psi_t)),   w = wr + i wi
    o_t = [ sum_s Re kappa(t,s) e_s  |  sum_s Im kappa(t,s) e_s ]   over s = t-L+1 .. t

with the L-1 previous writes (cos phi, sin phi, value) buffered in the state and prepended
to the call's own writes (the "extended" sequence: query t reads extended indices t .. t+L-1).
The read side is folded as in the reference (c1 = wr cq + wi sq, c2 = wr sq - wi cq), and
short_backward is the hand-written adjoint of that folded form.
Pinned in tests/test_oracle_golden.py against fixtures made by the reference's own heads.
"""
from __future__ import annotations

import numpy as np


def _extended(kh, kz, v, theta, omega, wr, wi, c0, s0, e0, pos):
    B, T, L = kh.shape
    dv = v.shape[-1]
    n = L - 1
    p = ((int(pos) + np.arange(T)) % L).astype(np.float64)
    phi = kh * theta + p[None, :, None] * omega
    psi = kz * theta + p[None, :, None] * omega
    c0 = np.ones((B, n, L)) if c0 is None else np.asarray(c0, np.float64)
    s0 = np.zeros((B, n, L)) if s0 is None else np.asarray(s0, np.float64)
    e0 = np.zeros((B, n, dv)) if e0 is None else np.asarray(e0, np.float64)
    cw = np.concatenate([c0, np.cos(phi)], 1)
    sw = np.concatenate([s0, np.sin(phi)], 1)
    e = np.concatenate([e0, v], 1)
    cq, sq = np.cos(psi), np.sin(psi)
    c1, c2 = wr * cq + wi * sq, wr * sq - wi * cq
    return phi, psi, cw, sw, e, cq, sq, c1, c2


def short_forward(kh, kz, v, theta, omega, wr, wi, c0=None, s0=None, e0=None, pos=0):
    """kh, kz (B,T,L) = K(h), K(z); v (B,T,dv); theta, omega, wr, wi (L); state c0, s0 (B,L-1,L),
    e0 (B,L-1,dv) or None (the reference's init_state: c = 1, s = 0, e = 0).
    Returns o (B,T,2dv) and the new state (c, s, e) = the last L-1 extended writes."""
    B, T, L = kh.shape
    dv = v.shape[-1]
    n = L - 1
    _, _, cw, sw, e, _, _, c1, c2 = _extended(kh, kz, v, theta, omega, wr, wi, c0, s0, e0, pos)
    o = np.zeros((B, T, 2 * dv))
    for t in range(T):
        w = slice(t, t + L)
        kre = (cw[:, w] * c1[:, t, None] + sw[:, w] * c2[:, t, None]).sum(-1) / L   # (B, L)
        kim = (sw[:, w] * c1[:, t, None] - cw[:, w] * c2[:, t, None]).sum(-1) / L
        o[:, t, :dv] = (kre[:, :, None] * e[:, w]).sum(1)
        o[:, t, dv:] = (kim[:, :, None] * e[:, w]).sum(1)
    N = T + n
    return o, (cw[:, N - n:], sw[:, N - n:], e[:, N - n:])


def short_backward(kh, kz, v, theta, omega, wr, wi, c0, s0, e0, pos, dO, dnew=None):
    """Adjoint of short_forward: gradients of sum(o * dO) + sum(new_state * dnew) for kh, kz,
    v, theta, wr, wi and the incoming state."""
    B, T, L = kh.shape
    dv = v.shape[-1]
    n = L - 1
    phi, psi, cw, sw, e, cq, sq, c1, c2 = _extended(kh, kz, v, theta, omega, wr, wi, c0, s0, e0, pos)
    dcw, dsw, de = np.zeros_like(cw), np.zeros_like(sw), np.zeros_like(e)
    dc1, dc2 = np.zeros_like(c1), np.zeros_like(c2)
    for t in range(T):
        w = slice(t, t + L)
        kre = (cw[:, w] * c1[:, t, None] + sw[:, w] * c2[:, t, None]).sum(-1) / L
        kim = (sw[:, w] * c1[:, t, None] - cw[:, w] * c2[:, t, None]).sum(-1) / L
        dre, dim = dO[:, t, :dv], dO[:, t, dv:]
        dkre = (dre[:, None, :] * e[:, w]).sum(-1)                               # (B, L)
        dkim = (dim[:, None, :] * e[:, w]).sum(-1)
        de[:, w] += kre[:, :, None] * dre[:, None, :] + kim[:, :, None] * dim[:, None, :]
        dc1[:, t] = (dkre[:, :, None] * cw[:, w] + dkim[:, :, None] * sw[:, w]).sum(1) / L
        dc2[:, t] = (dkre[:, :, None] * sw[:, w] - dkim[:, :, None] * cw[:, w]).sum(1) / L
        dcw[:, w] += (dkre[:, :, None] * c1[:, t, None, :] - dkim[:, :, None] * c2[:, t, None, :]) / L
        dsw[:, w] += (dkre[:, :, None] * c2[:, t, None, :] + dkim[:, :, None] * c1[:, t, None, :]) / L
    if dnew is not None:
        N = T + n
        dcw[:, N - n:] += dnew[0]
        dsw[:, N - n:] += dnew[1]
        de[:, N - n:] += dnew[2]
    dwr = (dc1 * cq + dc2 * sq).sum((0, 1))
    dwi = (dc1 * sq - dc2 * cq).sum((0, 1))
    dcq, dsq = dc1 * wr - dc2 * wi, dc1 * wi + dc2 * wr
    dpsi = -sq * dcq + cq * dsq
    dphi = -sw[:, n:] * dcw[:, n:] + cw[:, n:] * dsw[:, n:]
    return dict(kh=dphi * theta, kz=dpsi * theta, v=de[:, n:], theta=(dphi * kh + dpsi * kz).sum((0, 1)),
                wr=dwr, wi=dwi, c0=dcw[:, :n], s0=dsw[:, :n], e0=de[:, :n])


def _rms(u, eps=1e-6):
    return u / np.sqrt((u * u).mean(-1, keepdims=True) + eps)


def short_head(sd, z, h, state=None, pos=0):
    """u (B,T,2dv) = rms(o) and the new state of a short head with the reference's
    parameters `sd` (K.weight, V.weight, theta, wr, wi, omega) on inputs z, h (B,T,d)."""
    K, V = sd["K.weight"], sd["V.weight"]
    st = state or {}
    o, new = short_forward(h @ K.T, z @ K.T, z @ V.T, sd["theta"], sd["omega"], sd["wr"], sd["wi"],
                           st.get("c"), st.get("s"), st.get("e"), pos)
    return _rms(o), {"c": new[0], "s": new[1], "e": new[2], "pos": pos + z.shape[1]}
