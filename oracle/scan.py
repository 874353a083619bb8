"""CPU oracle for the SCA2 / Laplace-attention decayed-state scan (numpy, test infrastructure).

This module is the CHECKER, never the product: only tests, the smoke check and the
CPU-baseline leg of the benchmark import it. It restates, in plain numpy, the
recurrence that every C-head / long-head variant of the reference computes:

    S~_t = diag(gamma_t) S_{t-1}          gamma_t[m] = exp(g_t) * exp(-lam[m])
    e_t  = v_t - beta_t * (k_t^T S~_t) / kappa
    S_t  = S~_t + k_t e_t^T
    o_t  = Q_t^T S_t / kappa              (R read columns)

Reference sources restated here (paths relative to the reference project):
  * lapa/layer.py:387-412       LongHead.step (damp, read back, delta write, read)
  * lapa/layer.py:298-366       LongHead._batched (chunk closed form, scaled codes,
                                Gram + unit-lower triangular solve, state loop)
  * sca2/arch_damp.py:225-245   CHeadDeltaDamp.step; :288-301 complex token loop
  * sca2/arch_cdelta.py:186-206 CHeadDelta.step (beta, no decay)
  * sca2/arch_gatedc.py:171-193 CHeadGated.step (scalar decay exp(g_t), no beta)
  * sca2/ref.py:192-203         CHeadRef.step (additive, no decay)
  * fla 0.5.1 ops/gated_delta_rule/naive.py naive_recurrent_gated_delta_rule, as called
    at lapa/benchmarks/baselines.py:142-144 (write-gated form e = beta (v - k^T S~),
    i.e. v pre-scaled by beta, kappa = 1, R = 1, q pre-scaled by 1/sqrt(K))

Three forms are provided, all vectorised over (batch, head):
  forward_tokens / backward_tokens   token loop (float64); the backward is the
                                     adjoint recurrence, pinned against the
                                     reference's own autograd by the golden tests
  forward_chunked / backward_chunked chunk closed form with the same algebra as the
                                     CUDA kernels (decay factorised into scaled
                                     codes, scalar decay as a C x C mask)
plus the two code-space mappings used by the heads: phase codes (phase_*) and the
GDN form (gdn_*).
"""
from __future__ import annotations

import numpy as np

__all__ = [
    "forward_tokens", "backward_tokens", "forward_chunked", "backward_chunked",
    "phase_codes", "phase_grads", "phase_forward", "phase_backward",
    "gdn_forward", "gdn_backward", "to_phase_output", "from_phase_output",
]


# ----------------------------------------------------------------------------------
#  token loop (float64)
# ----------------------------------------------------------------------------------
def _gamma(g, lam, t, B, H, K, dt):
    """Per-channel decay of step t: (B,H,K)."""
    gam = np.ones((B, H, K), dtype=dt)
    if lam is not None:
        gam = gam * np.exp(-lam)[None]
    if g is not None:
        gam = gam * np.exp(g[:, t])[:, :, None]
    return gam


def forward_tokens(k, Q, v, beta=None, g=None, lam=None, kappa=1.0, S0=None,
                   return_states=False):
    """Token-by-token scan.

    k (B,T,H,K), Q (B,T,H,K,R), v (B,T,H,V), beta (B,T,H) or None (additive write),
    g (B,T,H) or None (no scalar decay), lam (H,K) or None (no per-channel decay),
    S0 (B,H,K,V) or None.  Returns o (B,T,H,R,V) and the final state (B,H,K,V).
    Follows lapa/layer.py:387-412 with the decay of sca2/arch_gatedc.py:182-184.
    """
    dt = np.float64
    k, Q, v = (np.asarray(x, dt) for x in (k, Q, v))
    B, T, H, K = k.shape
    V, R = v.shape[-1], Q.shape[-1]
    S = np.zeros((B, H, K, V), dt) if S0 is None else np.array(S0, dt)
    o = np.zeros((B, T, H, R, V), dt)
    states = [S.copy()]
    for t in range(T):
        St = _gamma(g, lam, t, B, H, K, dt)[..., None] * S
        if beta is not None:
            r = np.einsum("bhk,bhkv->bhv", k[:, t], St) / kappa
            e = v[:, t] - beta[:, t][..., None] * r
        else:
            e = v[:, t]
        S = St + k[:, t][..., None] * e[:, :, None, :]
        o[:, t] = np.einsum("bhkr,bhkv->bhrv", Q[:, t], S) / kappa
        if return_states:
            states.append(S.copy())
    if return_states:
        return o, S, states
    return o, S


def backward_tokens(k, Q, v, beta, g, lam, kappa, S0, do, dS_final=None):
    """Adjoint of forward_tokens (reverse-time recurrence).

    dS~_t = (I - beta_t k_t k_t^T / kappa) dS_t,  dS_{t-1} = diag(gamma_t) dS~_t.
    Returns dict of gradients: k, Q, v, beta, g, lam, S0 (None where the input was None).
    """
    dt = np.float64
    k, Q, v, do = (np.asarray(x, dt) for x in (k, Q, v, do))
    B, T, H, K = k.shape
    V = v.shape[-1]
    _, _, states = forward_tokens(k, Q, v, beta, g, lam, kappa, S0, return_states=True)
    dk = np.zeros_like(k)
    dQ = np.zeros_like(Q)
    dv = np.zeros_like(v)
    dbeta = None if beta is None else np.zeros((B, T, H), dt)
    dg = None if g is None else np.zeros((B, T, H), dt)
    dlam = None if lam is None else np.zeros((H, K), dt)
    dS = np.zeros((B, H, K, V), dt) if dS_final is None else np.array(dS_final, dt)
    for t in range(T - 1, -1, -1):
        Sprev, St_ = states[t], states[t + 1]
        gam = _gamma(g, lam, t, B, H, K, dt)
        St = gam[..., None] * Sprev
        if beta is not None:
            r = np.einsum("bhk,bhkv->bhv", k[:, t], St) / kappa
            e = v[:, t] - beta[:, t][..., None] * r
        else:
            e = v[:, t]
        dtot = dS + np.einsum("bhkr,bhrv->bhkv", Q[:, t], do[:, t]) / kappa
        dQ[:, t] = np.einsum("bhkv,bhrv->bhkr", St_, do[:, t]) / kappa
        dk[:, t] = np.einsum("bhkv,bhv->bhk", dtot, e)
        de = np.einsum("bhkv,bhk->bhv", dtot, k[:, t])
        dSt = dtot.copy()
        dv[:, t] = de
        if beta is not None:
            dbeta[:, t] = -(de * r).sum(-1)
            dr = -beta[:, t][..., None] * de
            dSt += k[:, t][..., None] * dr[:, :, None, :] / kappa
            dk[:, t] += np.einsum("bhkv,bhv->bhk", St, dr) / kappa
        dlog = (dSt * St).sum(-1)          # d/d(log gamma) (B,H,K)
        if g is not None:
            dg[:, t] = dlog.sum(-1)
        if lam is not None:
            dlam -= dlog.sum(0)
        dS = gam[..., None] * dSt
    return {"k": dk, "Q": dQ, "v": dv, "beta": dbeta, "g": dg, "lam": dlam, "S0": dS}


# ----------------------------------------------------------------------------------
#  chunk closed form (the CUDA kernels' algebra)
# ----------------------------------------------------------------------------------
def _chunk_pieces(k, Q, v, beta, g, lam, kappa, c0, Cl, dt):
    """Chunk-local operands for tokens [c0, c0+Cl): all (B,H,...) with chunk axis 2."""
    B, T, H, K = k.shape
    kc = np.ascontiguousarray(k[:, c0:c0 + Cl].transpose(0, 2, 1, 3)).astype(dt)   # (B,H,C,K)
    Qc = np.ascontiguousarray(Q[:, c0:c0 + Cl].transpose(0, 2, 1, 3, 4)).astype(dt)  # (B,H,C,K,R)
    vc = np.ascontiguousarray(v[:, c0:c0 + Cl].transpose(0, 2, 1, 3)).astype(dt)   # (B,H,C,V)
    i = np.arange(Cl, dtype=dt)
    if g is not None:
        Gc = np.cumsum(g[:, c0:c0 + Cl].transpose(0, 2, 1).astype(dt), -1)         # (B,H,C)
    else:
        Gc = np.zeros((B, H, Cl), dt)
    if lam is not None:
        lm = lam.astype(dt)
        ell = np.exp(-lm[:, None, :] * i[None, :, None])                          # (H,C,K)
        ellinv = np.exp(lm[:, None, :] * i[None, :, None])
        d1 = np.exp(-lm)                                                           # (H,K)
        dCl = np.exp(-lm * Cl)
        dCm1 = np.exp(-lm * (Cl - 1))
    else:
        ell = ellinv = np.ones((H, Cl, K), dt)
        d1 = dCl = dCm1 = np.ones((H, K), dt)
    bc = None if beta is None else beta[:, c0:c0 + Cl].transpose(0, 2, 1).astype(dt)  # (B,H,C)
    diff = Gc[..., :, None] - Gc[..., None, :]
    low_incl = np.tril(np.ones((Cl, Cl), bool))
    Dg = np.where(low_incl, np.exp(np.minimum(diff, 0.0)), 0.0)                    # (B,H,C,C)
    a = np.exp(Gc)
    w = np.exp(Gc[..., -1:] - Gc)
    kr = kc * ell[None]
    kw = kc * ellinv[None]
    qr = Qc * ell[None][..., None]
    return dict(kc=kc, Qc=Qc, vc=vc, bc=bc, Gc=Gc, Dg=Dg, a=a, w=w, kr=kr, kw=kw, qr=qr,
                d1=d1, dCl=dCl, dCm1=dCm1, ell=ell, ellinv=ellinv, i=i)


def _unit_lower_solve(Lstrict, Y):
    """Solve (I + Lstrict) E = Y by forward substitution; Lstrict (...,C,C) strictly lower."""
    E = np.array(Y, copy=True)
    C = Y.shape[-2]
    for r in range(1, C):
        E[..., r, :] -= np.einsum("...j,...jv->...v", Lstrict[..., r, :r], E[..., :r, :])
    return E


def _unit_upper_solve_T(Lstrict, dE):
    """Solve (I + Lstrict)^T dY = dE by backward substitution."""
    dY = np.array(dE, copy=True)
    C = dE.shape[-2]
    for r in range(C - 2, -1, -1):
        dY[..., r, :] -= np.einsum("...j,...jv->...v", Lstrict[..., r + 1:, r], dY[..., r + 1:, :])
    return dY


def _chunk_fwd(p, S, kappa):
    """One chunk of the closed form given the incoming state S (B,H,K,V)."""
    S0p = p["d1"][None, :, :, None] * S
    strict = np.tril(np.ones(p["Dg"].shape[-2:], bool), -1)
    KK = np.einsum("bhik,bhjk->bhij", p["kr"], p["kw"]) / kappa
    Graw = np.where(strict, KK * p["Dg"], 0.0)
    KS = np.einsum("bhik,bhkv->bhiv", p["kr"], S0p) / kappa
    R0 = p["a"][..., None] * KS
    if p["bc"] is not None:
        Y = p["vc"] - p["bc"][..., None] * R0
        E = _unit_lower_solve(p["bc"][..., None] * Graw, Y)
    else:
        Y = p["vc"]
        E = Y.copy()
    QK = np.einsum("bhikr,bhjk->bhrij", p["qr"], p["kw"]) / kappa
    P = QK * p["Dg"][:, :, None]
    QS = np.einsum("bhikr,bhkv->bhriv", p["qr"], S0p) / kappa
    O = p["a"][:, :, None, :, None] * QS + np.einsum("bhrij,bhjv->bhriv", P, E)
    aC = p["a"][..., -1]
    Snew = (aC[..., None, None] * p["dCl"][None, :, :, None] * S
            + p["dCm1"][None, :, :, None]
            * np.einsum("bhjk,bhjv->bhkv", p["kw"], p["w"][..., None] * E))
    return O, Snew, dict(S0p=S0p, KK=KK, Graw=Graw, KS=KS, R0=R0, Y=Y, E=E, QK=QK, P=P, QS=QS)


def forward_chunked(k, Q, v, beta=None, g=None, lam=None, kappa=1.0, S0=None, C=64,
                    dtype=np.float64, return_chunk_states=False):
    """Chunk closed form (lapa/layer.py:298-366 generalised with the scalar decay mask of
    sca2/arch_gatedc.py:136-139).  Same signature/returns as forward_tokens."""
    B, T, H, K = k.shape
    V, R = v.shape[-1], Q.shape[-1]
    S = np.zeros((B, H, K, V), dtype) if S0 is None else np.array(S0, dtype)
    o = np.zeros((B, T, H, R, V), dtype)
    chunk_states = []
    for c0 in range(0, T, C):
        Cl = min(C, T - c0)
        p = _chunk_pieces(k, Q, v, beta, g, lam, kappa, c0, Cl, dtype)
        chunk_states.append(S.copy())
        O, S, _ = _chunk_fwd(p, S, kappa)
        o[:, c0:c0 + Cl] = O.transpose(0, 3, 1, 2, 4)
    if return_chunk_states:
        return o, S, chunk_states
    return o, S


def backward_chunked(k, Q, v, beta, g, lam, kappa, S0, do, dS_final=None, C=64,
                     dtype=np.float64):
    """Chunk closed form of backward_tokens: a reverse scan of the adjoint state over
    chunk boundaries, then every per-token gradient of a chunk from (S0, dS_C) at once.
    This is the algebra the CUDA backward kernels implement."""
    B, T, H, K = k.shape
    V, R = v.shape[-1], Q.shape[-1]
    _, _, cstates = forward_chunked(k, Q, v, beta, g, lam, kappa, S0, C, dtype, True)
    dk = np.zeros((B, T, H, K), dtype)
    dQ = np.zeros((B, T, H, K, R), dtype)
    dv = np.zeros((B, T, H, V), dtype)
    dbeta = None if beta is None else np.zeros((B, T, H), dtype)
    dg = None if g is None else np.zeros((B, T, H), dtype)
    dlam = None if lam is None else np.zeros((H, K), dtype)
    dS = np.zeros((B, H, K, V), dtype) if dS_final is None else np.array(dS_final, dtype)
    starts = list(range(0, T, C))
    for ci in range(len(starts) - 1, -1, -1):
        c0 = starts[ci]
        Cl = min(C, T - c0)
        p = _chunk_pieces(k, Q, v, beta, g, lam, kappa, c0, Cl, dtype)
        S = cstates[ci]
        _, _, f = _chunk_fwd(p, S, kappa)
        doc = do[:, c0:c0 + Cl].transpose(0, 2, 3, 1, 4).astype(dtype)           # (B,H,R,C,V)
        strict = np.tril(np.ones((Cl, Cl), bool), -1)
        E, S0p, a, w, Dg = f["E"], f["S0p"], p["a"], p["w"], p["Dg"]
        aC = a[..., -1]
        # ---- state-carry terms
        dSc = p["dCm1"][None, :, :, None] * dS                                    # (B,H,K,V)
        KWdS = np.einsum("bhjk,bhkv->bhjv", p["kw"], dSc)                          # (B,H,C,V)
        dE = w[..., None] * KWdS
        dE += np.einsum("bhrij,bhriv->bhjv", f["P"], doc)
        # ---- delta solve
        if p["bc"] is not None:
            Lst = p["bc"][..., None] * f["Graw"]
            dY = _unit_upper_solve_T(Lst, dE)
            dL = -np.einsum("bhiv,bhjv->bhij", dY, E)
            dL = np.where(strict, dL, 0.0)
            dbeta_c = (dL * f["Graw"]).sum(-1) - (dY * f["R0"]).sum(-1)
            dR0 = -p["bc"][..., None] * dY
            dGm = p["bc"][..., None] * dL                                          # wrt Graw
        else:
            dY = dE
            dR0 = np.zeros_like(dY)
            dGm = np.zeros(Dg.shape, dtype)
        dvc = dY
        # ---- output terms
        dP = np.einsum("bhriv,bhjv->bhrij", doc, E)
        dP = np.where(np.tril(np.ones((Cl, Cl), bool))[None, None, None], dP, 0.0)
        dQK = dP * Dg[:, :, None]                                                  # wrt QK (already /kappa)
        dKK = dGm * Dg                                                             # wrt KK (already /kappa)
        # d(qr) (B,H,C,K,R)
        dqr = (np.einsum("bhrij,bhjk->bhikr", dQK, p["kw"]) / kappa
               + np.einsum("bhi,bhriv,bhkv->bhikr", a, doc, S0p) / kappa)
        dkr = (np.einsum("bhij,bhjk->bhik", dKK, p["kw"]) / kappa
               + np.einsum("bhi,bhiv,bhkv->bhik", a, dR0, S0p) / kappa)
        dkw = (np.einsum("bhij,bhik->bhjk", dKK, p["kr"]) / kappa
               + np.einsum("bhrij,bhikr->bhjk", dQK, p["qr"]) / kappa
               + w[..., None] * np.einsum("bhjv,bhkv->bhjk", E, dSc))
        dS0p = (np.einsum("bhikr,bhi,bhriv->bhkv", p["qr"], a, doc) / kappa
                + np.einsum("bhik,bhi,bhiv->bhkv", p["kr"], a, dR0) / kappa)
        # ---- decay gradients
        if g is not None:
            dDg = (dGm * f["KK"] + (dP * f["QK"]).sum(2))                       # wrt Dg entries
            dDg = np.where(np.tril(np.ones((Cl, Cl), bool)), dDg, 0.0) * Dg
            da = ((doc * f["QS"]).sum((2, 4)) + (dR0 * f["KS"]).sum(-1)) * a
            dw = (E * KWdS).sum(-1) * w
            daC = (p["dCl"][None, :, :, None] * S * dS).sum((2, 3)) * aC
            dGc = dDg.sum(-1) - dDg.sum(-2) + da - dw
            dGc[..., -1] += dw.sum(-1) + daC
            dg[:, c0:c0 + Cl] = np.cumsum(dGc[..., ::-1], -1)[..., ::-1].transpose(0, 2, 1)
        if lam is not None:
            i = p["i"]
            dl = (-(i[None, None, :, None] * (dkr * p["kr"])).sum(2)
                  - (i[None, None, :, None, None] * (dqr * p["qr"])).sum((2, 4))
                  + (i[None, None, :, None] * (dkw * p["kw"])).sum(2)
                  - (dS0p * S0p).sum(-1)
                  - Cl * (aC[..., None, None] * p["dCl"][None, :, :, None] * S * dS).sum(-1)
                  - (Cl - 1) * ((dSc * np.einsum("bhjk,bhjv->bhkv", p["kw"], w[..., None] * E)).sum(-1)))
            dlam += dl.sum(0)
        dk[:, c0:c0 + Cl] = (dkr * p["ell"][None] + dkw * p["ellinv"][None]).transpose(0, 2, 1, 3)
        dQ[:, c0:c0 + Cl] = (dqr * p["ell"][None][..., None]).transpose(0, 2, 1, 3, 4)
        dv[:, c0:c0 + Cl] = dvc.transpose(0, 2, 1, 3)
        if beta is not None:
            dbeta[:, c0:c0 + Cl] = dbeta_c.transpose(0, 2, 1)
        # ---- adjoint state to the previous chunk
        dS = aC[..., None, None] * p["dCl"][None, :, :, None] * dS + p["d1"][None, :, :, None] * dS0p
    return {"k": dk, "Q": dQ, "v": dv, "beta": dbeta, "g": dg, "lam": dlam, "S0": dS}


# ----------------------------------------------------------------------------------
#  phase-code mapping (LongHead / CHeadDelta(Damp) / CHeadGated / CHeadRef)
# ----------------------------------------------------------------------------------
def phase_codes(phw, phq, wr, wi):
    """Write phases phi (B,T,H,Mh), read phases psi (B,T,H,Mh), spectral read weights
    wr, wi (H,Mh) -> k (B,T,H,2Mh) and Q (B,T,H,2Mh,2).

    k = [cos phi ; sin phi] (lapa/layer.py:394, ||k||^2 = Mh exactly).
    Read columns: o_re = c1.sr + c2.si, o_im = c1.si - c2.sr with
    c1 = wr cos psi + wi sin psi, c2 = wr sin psi - wi cos psi (lapa/layer.py:403-411).
    """
    cw, sw = np.cos(phw), np.sin(phw)
    cq, sq = np.cos(phq), np.sin(phq)
    c1 = wr * cq + wi * sq
    c2 = wr * sq - wi * cq
    k = np.concatenate([cw, sw], -1)
    Qre = np.concatenate([c1, c2], -1)
    Qim = np.concatenate([-c2, c1], -1)
    return k, np.stack([Qre, Qim], -1)


def phase_grads(dk, dQ, phw, phq, wr, wi):
    """Chain rule from code-space gradients back to (phi, psi, wr, wi)."""
    Mh = phw.shape[-1]
    cw, sw = np.cos(phw), np.sin(phw)
    cq, sq = np.cos(phq), np.sin(phq)
    dphw = -sw * dk[..., :Mh] + cw * dk[..., Mh:]
    dc1 = dQ[..., :Mh, 0] + dQ[..., Mh:, 1]
    dc2 = dQ[..., Mh:, 0] - dQ[..., :Mh, 1]
    dwr = (dc1 * cq + dc2 * sq).sum((0, 1))
    dwi = (dc1 * sq - dc2 * cq).sum((0, 1))
    dcq = dc1 * wr - dc2 * wi
    dsq = dc1 * wi + dc2 * wr
    dphq = -sq * dcq + cq * dsq
    return dphw, dphq, dwr, dwi


def to_phase_output(o):
    """(B,T,H,2,V) kernel layout -> (B,T,H,2V) [re | im] per head."""
    B, T, H, R, V = o.shape
    return o.reshape(B, T, H, R * V)


def from_phase_output(u):
    B, T, H, RV = u.shape
    return u.reshape(B, T, H, 2, RV // 2)


def _lam_full(lam):
    return None if lam is None else np.concatenate([lam, lam], -1)


def phase_forward(phw, phq, v, beta, g, lam, wr, wi, S0=None, chunked=False, C=64):
    """Phase-coded head scan.  lam (H,Mh) per mode; S0 (B,H,2Mh,V) = [sr ; si].
    Returns o (B,T,H,2,V), S (B,H,2Mh,V)."""
    Mh = phw.shape[-1]
    k, Q = phase_codes(phw, phq, wr, wi)
    if chunked:
        return forward_chunked(k, Q, v, beta, g, _lam_full(lam), float(Mh), S0, C)
    return forward_tokens(k, Q, v, beta, g, _lam_full(lam), float(Mh), S0)


def phase_backward(phw, phq, v, beta, g, lam, wr, wi, S0, do, dS_final=None, chunked=False, C=64):
    Mh = phw.shape[-1]
    k, Q = phase_codes(phw, phq, wr, wi)
    if chunked:
        gr = backward_chunked(k, Q, v, beta, g, _lam_full(lam), float(Mh), S0, do, dS_final, C)
    else:
        gr = backward_tokens(k, Q, v, beta, g, _lam_full(lam), float(Mh), S0, do, dS_final)
    dphw, dphq, dwr, dwi = phase_grads(gr["k"], gr["Q"], phw, phq, wr, wi)
    dlam = None if gr["lam"] is None else gr["lam"][:, :Mh] + gr["lam"][:, Mh:]
    return {"phw": dphw, "phq": dphq, "v": gr["v"], "beta": gr["beta"], "g": gr["g"],
            "lam": dlam, "wr": dwr, "wi": dwi, "S0": gr["S0"]}


# ----------------------------------------------------------------------------------
#  GDN form (fla naive_recurrent_gated_delta_rule semantics)
# ----------------------------------------------------------------------------------
def gdn_forward(q, k, v, g, beta, scale=None, S0=None, chunked=False, C=64):
    """q,k (B,T,H,K), v (B,T,H,V), g,beta (B,T,H).  e = beta (v - k^T S~): the erase form
    with v' = beta v, kappa = 1, Q = scale q.  Returns o (B,T,H,V), S (B,H,K,V)."""
    K = k.shape[-1]
    scale = K ** -0.5 if scale is None else scale
    Q = (scale * np.asarray(q, np.float64))[..., None]
    vb = np.asarray(v, np.float64) * beta[..., None]
    f = forward_chunked if chunked else forward_tokens
    kw = dict(C=C) if chunked else {}
    o, S = f(k, Q, vb, beta, g, None, 1.0, S0, **kw)
    return o[:, :, :, 0], S


def gdn_backward(q, k, v, g, beta, do, scale=None, S0=None, dS_final=None, chunked=False, C=64):
    K = k.shape[-1]
    scale = K ** -0.5 if scale is None else scale
    Q = (scale * np.asarray(q, np.float64))[..., None]
    vb = np.asarray(v, np.float64) * beta[..., None]
    if chunked:
        gr = backward_chunked(k, Q, vb, beta, g, None, 1.0, S0, do[:, :, :, None], dS_final, C)
    else:
        gr = backward_tokens(k, Q, vb, beta, g, None, 1.0, S0, do[:, :, :, None], dS_final)
    dbeta = gr["beta"] + (gr["v"] * v).sum(-1)
    return {"q": scale * gr["Q"][..., 0], "k": gr["k"], "v": gr["v"] * beta[..., None],
            "g": gr["g"], "beta": dbeta, "S0": gr["S0"]}
