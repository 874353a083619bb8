"""Generate the golden fixtures in this folder from the reference's own modules.

Run in a container where the reference project is importable (read-only is fine):

    PYTHONDONTWRITEBYTECODE=1 python tests/golden/make_golden.py /path/to/reference

Every fixture is produced by running an UNMODIFIED reference head in float64 with
torch autograd; nothing of this repository's CUDA path is involved.  Two kinds:

kernel-level ("scan_*.npz")
    The scan's own inputs (write phase phi, read phase psi, value v, erase gate beta,
    scalar log-decay g, per-mode decay lam, read weights wr/wi, incoming state) are
    fed to the reference head through an exact encoding: K = [I 0 0], V = [0 I 0],
    theta = 1 and omega = 0 make K(x) theta + p omega = x[..., :M], so the head's
    phases ARE the first M features of z (read) and h (write); the remaining features
    carry v and the gate logits.  The RMS read-out is switched off (rms_read=False,
    rscale = 1, or lapa.layer._rms -> identity) so the raw read o is recorded.
    Gradients come from autograd of  sum(o * dO) + sum(S_final * dS_final).

head-level ("head_*.npz")
    A reference head with ordinary random weights (rope grid, theta != 0) is run on
    random z, h and a random incoming state; the fixture stores its state_dict, the
    inputs, the RMS'd output u, the new state and every parameter / input gradient.
    These pin the drop-in head classes (projections + scan + epilogue).  head_d*.npz are
    the D heads (DHeadRef, DHeadSepQ, DHeadSepQPolar), with decode steps after the prefill;
    head_short_*.npz the short heads (lapa ShortHead, sca2 CHeadShort): prefill with state
    gradients, a second prefill shorter than the window, decode steps.

layer-level ("layer_*.npz", "lm_lapa.npz")
    Whole reference layers (SCA2Layer, GatedLayer, LaplaceAttention) with random weights:
    output, new state, every gradient, decode steps; and a 2-layer LaplaceLM: logits,
    cross-entropy gradients and a greedy generation.

gdn_fla.npz
    fla 0.5.1 naive_chunk_gated_delta_rule / naive_recurrent_gated_delta_rule
    (the GDN baseline as called at lapa/benchmarks/baselines.py:111-120,142-144).
"""
from __future__ import annotations

import math
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))


def _np(t):
    return None if t is None else t.detach().cpu().double().numpy()


def _save(name, **arrays):
    path = os.path.join(HERE, name)
    np.savez_compressed(path, **{k: v for k, v in arrays.items() if v is not None})
    print("wrote", path, sum(v.size for v in arrays.values() if v is not None), "values")


def _encode(lin, col0, n, d):
    """Make an nn.Linear select features [col0, col0+n) of its input exactly."""
    w = torch.zeros(lin.weight.shape, dtype=torch.float64)
    w[torch.arange(n), col0 + torch.arange(n)] = 1.0
    with torch.no_grad():
        lin.weight.copy_(w)
        if lin.bias is not None:
            lin.bias.zero_()


# --------------------------------------------------------------------------------------
#  kernel-level fixtures
# --------------------------------------------------------------------------------------
def longhead_scan(gen, B=2, T=45, M=12, dv=5, chunk=16, path="batched"):
    """lapa.layer.LongHead: per-mode lam + delta beta (lapa/layer.py:170-412)."""
    import lapa.layer as LL
    d = M + dv + 1
    cfg = LL.LaplaceConfig(d=d, M=M, dv=dv, L=16, chunk=chunk, persist=0.5, theta_scale=0.02,
                           long_path=path)
    head = LL.LongHead(cfg).double()
    _encode(head.K, 0, M, d)
    _encode(head.V, M, dv, d)
    with torch.no_grad():
        head.bproj.weight.zero_()
        head.bproj.weight[0, d - 1] = 1.0
        head.bproj.bias.zero_()
        head.theta.fill_(1.0)
        head.omega.zero_()
        head.wr.copy_(torch.randn(M, generator=gen, dtype=torch.float64) * 0.5 + 1.0)
        head.wi.copy_(torch.randn(M, generator=gen, dtype=torch.float64) * 0.5)
        lam = torch.rand(M, generator=gen, dtype=torch.float64) * 0.055 + 0.003
        head.lam_raw.copy_(torch.log(torch.expm1(lam)))
    phw = torch.randn(B, T, M, generator=gen, dtype=torch.float64) * 2.0
    phq = torch.randn(B, T, M, generator=gen, dtype=torch.float64) * 2.0
    v = torch.randn(B, T, dv, generator=gen, dtype=torch.float64)
    blog = torch.randn(B, T, 1, generator=gen, dtype=torch.float64)
    z = torch.cat([phq, v, blog], -1).requires_grad_(True)
    h = torch.cat([phw, torch.zeros(B, T, dv + 1, dtype=torch.float64)], -1).requires_grad_(True)
    sr0 = (torch.randn(B, M, dv, generator=gen, dtype=torch.float64) * 0.3).requires_grad_(True)
    si0 = (torch.randn(B, M, dv, generator=gen, dtype=torch.float64) * 0.3).requires_grad_(True)
    st = {"sr": sr0, "si": si0, "pos": torch.zeros((), dtype=torch.float64)}
    rms = LL._rms
    LL._rms = lambda u, eps=1e-6: u
    try:
        o, st1 = head.prefill(z, h, st)
    finally:
        LL._rms = rms
    dO = torch.randn(o.shape, generator=gen, dtype=torch.float64)
    dsr = torch.randn(B, M, dv, generator=gen, dtype=torch.float64)
    dsi = torch.randn(B, M, dv, generator=gen, dtype=torch.float64)
    ((o * dO).sum() + (st1["sr"] * dsr).sum() + (st1["si"] * dsi).sum()).backward()
    lam_eff = head.lam().detach()
    mask = head.lam_mask.detach()
    sig = torch.sigmoid(head.lam_raw.detach())
    # d lam_raw = d lam * sigmoid(lam_raw) * mask (softplus below the clamp)
    return dict(
        phw=_np(phw), phq=_np(phq), v=_np(v), beta=_np(torch.sigmoid(blog[..., 0])),
        lam=_np(lam_eff), lam_mask=_np(mask), lam_raw_sig=_np(sig),
        wr=_np(head.wr), wi=_np(head.wi), sr0=_np(sr0), si0=_np(si0),
        o=_np(o), sr=_np(st1["sr"]), si=_np(st1["si"]), dO=_np(dO), dsr=_np(dsr), dsi=_np(dsi),
        d_phq=_np(z.grad[..., :M]), d_v=_np(z.grad[..., M:M + dv]),
        d_blogit=_np(z.grad[..., -1]), d_phw=_np(h.grad[..., :M]),
        d_wr=_np(head.wr.grad), d_wi=_np(head.wi.grad), d_lam_raw=_np(head.lam_raw.grad),
        d_sr0=_np(sr0.grad), d_si0=_np(si0.grad),
        meta=np.array([B, T, M, dv, chunk]),
    )


def longhead_step(gen, B=3, T=6, M=12, dv=5):
    """lapa.layer.LongHead.step token by token (lapa/layer.py:387-412)."""
    import lapa.layer as LL
    d = M + dv + 1
    cfg = LL.LaplaceConfig(d=d, M=M, dv=dv, L=16, chunk=16, persist=0.5)
    head = LL.LongHead(cfg).double()
    _encode(head.K, 0, M, d)
    _encode(head.V, M, dv, d)
    with torch.no_grad():
        head.bproj.weight.zero_()
        head.bproj.weight[0, d - 1] = 1.0
        head.bproj.bias.zero_()
        head.theta.fill_(1.0)
        head.omega.zero_()
        head.wr.copy_(torch.randn(M, generator=gen, dtype=torch.float64) * 0.5 + 1.0)
        head.wi.copy_(torch.randn(M, generator=gen, dtype=torch.float64) * 0.5)
        lam = torch.rand(M, generator=gen, dtype=torch.float64) * 0.055 + 0.003
        head.lam_raw.copy_(torch.log(torch.expm1(lam)))
    phw = torch.randn(B, T, M, generator=gen, dtype=torch.float64) * 2.0
    phq = torch.randn(B, T, M, generator=gen, dtype=torch.float64) * 2.0
    v = torch.randn(B, T, dv, generator=gen, dtype=torch.float64)
    blog = torch.randn(B, T, 1, generator=gen, dtype=torch.float64)
    sr0 = torch.randn(B, M, dv, generator=gen, dtype=torch.float64) * 0.3
    si0 = torch.randn(B, M, dv, generator=gen, dtype=torch.float64) * 0.3
    st = {"sr": sr0, "si": si0, "pos": torch.zeros((), dtype=torch.float64)}
    rms = LL._rms
    LL._rms = lambda u, eps=1e-6: u
    outs = []
    try:
        with torch.no_grad():
            for t in range(T):
                z = torch.cat([phq[:, t], v[:, t], blog[:, t]], -1)
                h = torch.cat([phw[:, t], torch.zeros(B, dv + 1, dtype=torch.float64)], -1)
                u, st = head.step(z, h, st)
                outs.append(u)
    finally:
        LL._rms = rms
    return dict(phw=_np(phw), phq=_np(phq), v=_np(v), beta=_np(torch.sigmoid(blog[..., 0])),
                lam=_np(head.lam()), wr=_np(head.wr), wi=_np(head.wi), sr0=_np(sr0), si0=_np(si0),
                o=_np(torch.stack(outs, 1)), sr=_np(st["sr"]), si=_np(st["si"]),
                meta=np.array([B, T, M, dv]))


def gated_scan(gen, B=2, T=45, H=2, Mh=6, dvh=4, ctx=16):
    """sca2.arch_gatedc.CHeadGated, heads + data-dependent scalar decay, additive write
    (sca2/arch_gatedc.py:58-193).  g = -exp(A_log) softplus(a(z) + dt_bias) with A_log = 0,
    dt_bias = 0, so g = -softplus(x_g) for the encoded feature x_g."""
    from sca2.arch_gatedc import CHeadGated
    M, dv = H * Mh, H * dvh
    d = M + dv + H
    head = CHeadGated(d, M, freq="rope", theta_scale=0.02, max_len=64, dv=dv, heads=H,
                      decay=True).double()
    head.CTX = ctx
    _encode(head.K, 0, M, d)
    _encode(head.V, M, dv, d)
    _encode(head.a, M + dv, H, d)
    with torch.no_grad():
        head.theta.fill_(1.0)
        head.omega.zero_()
        head.A_log.zero_()
        head.dt_bias.zero_()
        head.wr.copy_(torch.randn(M, generator=gen, dtype=torch.float64) * 0.5 + 1.0)
        head.wi.copy_(torch.randn(M, generator=gen, dtype=torch.float64) * 0.5)
    head.rms_read = False
    head.rscale = torch.ones(2 * dv, dtype=torch.float64)
    phw = torch.randn(B, T, M, generator=gen, dtype=torch.float64) * 2.0
    phq = torch.randn(B, T, M, generator=gen, dtype=torch.float64) * 2.0
    v = torch.randn(B, T, dv, generator=gen, dtype=torch.float64)
    xg = torch.randn(B, T, H, generator=gen, dtype=torch.float64) - 1.0
    z = torch.cat([phq, v, xg], -1).requires_grad_(True)
    h = torch.cat([phw, torch.zeros(B, T, dv + H, dtype=torch.float64)], -1).requires_grad_(True)
    sr0 = (torch.randn(B, H, Mh, dvh, generator=gen, dtype=torch.float64) * 0.3).requires_grad_(True)
    si0 = (torch.randn(B, H, Mh, dvh, generator=gen, dtype=torch.float64) * 0.3).requires_grad_(True)
    st = {"sr": sr0, "si": si0, "pos": torch.zeros((), dtype=torch.float64), "empty": False}
    u, st1 = head.prefill(z, h, st)
    dU = torch.randn(u.shape, generator=gen, dtype=torch.float64)
    dsr = torch.randn(sr0.shape, generator=gen, dtype=torch.float64)
    dsi = torch.randn(si0.shape, generator=gen, dtype=torch.float64)
    ((u * dU).sum() + (st1["sr"] * dsr).sum() + (st1["si"] * dsi).sum()).backward()
    g = -torch.nn.functional.softplus(xg)
    return dict(
        phw=_np(phw), phq=_np(phq), v=_np(v), g=_np(g), xg=_np(xg), wr=_np(head.wr), wi=_np(head.wi),
        sr0=_np(sr0), si0=_np(si0), u=_np(u), sr=_np(st1["sr"]), si=_np(st1["si"]),
        dU=_np(dU), dsr=_np(dsr), dsi=_np(dsi),
        d_phq=_np(z.grad[..., :M]), d_v=_np(z.grad[..., M:M + dv]), d_xg=_np(z.grad[..., M + dv:]),
        d_phw=_np(h.grad[..., :M]), d_wr=_np(head.wr.grad), d_wi=_np(head.wi.grad),
        d_sr0=_np(sr0.grad), d_si0=_np(si0.grad), meta=np.array([B, T, H, Mh, dvh, ctx]),
    )


def cdelta_scan(gen, B=2, T=45, M=10, dv=6, ctx=16, damp=False):
    """sca2.arch_cdelta.CHeadDelta (beta, no decay) or sca2.arch_damp.CHeadDeltaDamp
    (per-mode lam), both through their own prefill (sca2/arch_cdelta.py:92-206,
    sca2/arch_damp.py:43-245)."""
    from sca2.arch_cdelta import CHeadDelta
    from sca2.arch_damp import CHeadDeltaDamp
    d = M + dv + 1
    cls = CHeadDeltaDamp if damp else CHeadDelta
    head = cls(d, M, freq="rope", theta_scale=0.3, dv=dv, max_len=T).double()
    head.CTX = ctx
    _encode(head.K, 0, M, d)
    _encode(head.V, M, dv, d)
    with torch.no_grad():
        head.bproj.weight.zero_()
        head.bproj.weight[0, d - 1] = 1.0
        head.bproj.bias.zero_()
        head.theta.fill_(1.0)
        head.omega.zero_()
        head.wr.copy_(torch.randn(M, generator=gen, dtype=torch.float64) * 0.5 + 1.0)
        head.wi.copy_(torch.randn(M, generator=gen, dtype=torch.float64) * 0.5)
        if damp:
            lam = torch.rand(M, generator=gen, dtype=torch.float64) * 0.1 + 0.003
            head.lam_raw.copy_(torch.log(torch.expm1(lam)))
    head.rms_read = False
    head.rscale = torch.ones(2 * dv, dtype=torch.float64)
    phw = torch.randn(B, T, M, generator=gen, dtype=torch.float64) * 2.0
    phq = torch.randn(B, T, M, generator=gen, dtype=torch.float64) * 2.0
    v = torch.randn(B, T, dv, generator=gen, dtype=torch.float64)
    blog = torch.randn(B, T, 1, generator=gen, dtype=torch.float64)
    z = torch.cat([phq, v, blog], -1).requires_grad_(True)
    h = torch.cat([phw, torch.zeros(B, T, dv + 1, dtype=torch.float64)], -1).requires_grad_(True)
    sr0 = (torch.randn(B, M, dv, generator=gen, dtype=torch.float64) * 0.3).requires_grad_(True)
    si0 = (torch.randn(B, M, dv, generator=gen, dtype=torch.float64) * 0.3).requires_grad_(True)
    st = {"sr": sr0, "si": si0, "pos": torch.zeros((), dtype=torch.float64), "empty": False}
    o, st1 = head.prefill(z, h, st)
    dO = torch.randn(o.shape, generator=gen, dtype=torch.float64)
    dsr = torch.randn(sr0.shape, generator=gen, dtype=torch.float64)
    dsi = torch.randn(si0.shape, generator=gen, dtype=torch.float64)
    ((o * dO).sum() + (st1["sr"] * dsr).sum() + (st1["si"] * dsi).sum()).backward()
    out = dict(
        phw=_np(phw), phq=_np(phq), v=_np(v), beta=_np(torch.sigmoid(blog[..., 0])),
        wr=_np(head.wr), wi=_np(head.wi), sr0=_np(sr0), si0=_np(si0),
        o=_np(o), sr=_np(st1["sr"]), si=_np(st1["si"]), dO=_np(dO), dsr=_np(dsr), dsi=_np(dsi),
        d_phq=_np(z.grad[..., :M]), d_v=_np(z.grad[..., M:M + dv]),
        d_blogit=_np(z.grad[..., -1]), d_phw=_np(h.grad[..., :M]),
        d_wr=_np(head.wr.grad), d_wi=_np(head.wi.grad),
        d_sr0=_np(sr0.grad), d_si0=_np(si0.grad), meta=np.array([B, T, M, dv, ctx]),
    )
    if damp:
        out.update(lam=_np(head.lam()), lam_raw_sig=_np(torch.sigmoid(head.lam_raw.detach())),
                   d_lam_raw=_np(head.lam_raw.grad))
    return out


def gdn_fla(gen, B=2, T=45, H=2, K=8, V=6, chunk=16):
    """fla naive gated delta rule, chunked and recurrent (third-party arithmetic of the GDN
    baseline; called at lapa/benchmarks/baselines.py:111-120,142-144)."""
    from fla.ops.gated_delta_rule.naive import (naive_chunk_gated_delta_rule,
                                                naive_recurrent_gated_delta_rule)
    f64 = torch.float64
    q = torch.nn.functional.normalize(torch.randn(B, T, H, K, generator=gen, dtype=f64), dim=-1)
    k = torch.nn.functional.normalize(torch.randn(B, T, H, K, generator=gen, dtype=f64), dim=-1)
    v = torch.randn(B, T, H, V, generator=gen, dtype=f64)
    g = -torch.nn.functional.softplus(torch.randn(B, T, H, generator=gen, dtype=f64))
    beta = torch.sigmoid(torch.randn(B, T, H, generator=gen, dtype=f64))
    S0 = torch.randn(B, H, K, V, generator=gen, dtype=f64) * 0.3
    leaves = [x.clone().requires_grad_(True) for x in (q, k, v, g, beta, S0)]
    qq, kk, vv, gg, bb, ss = leaves
    o, S = naive_chunk_gated_delta_rule(qq, kk, vv, gg, bb, chunk_size=chunk, initial_state=ss,
                                        output_final_state=True)
    o, S = o.double(), S.double()
    dO = torch.randn(o.shape, generator=gen, dtype=f64)
    dS = torch.randn(S.shape, generator=gen, dtype=f64)
    ((o * dO).sum() + (S * dS).sum()).backward()
    with torch.no_grad():
        o_rec, S_rec = naive_recurrent_gated_delta_rule(q, k, v, beta, g, initial_state=S0,
                                                        output_final_state=True)
    return dict(q=_np(q), k=_np(k), v=_np(v), g=_np(g), beta=_np(beta), S0=_np(S0),
                o=_np(o), S=_np(S), o_rec=_np(o_rec), S_rec=_np(S_rec), dO=_np(dO), dS=_np(dS),
                d_q=_np(qq.grad), d_k=_np(kk.grad), d_v=_np(vv.grad), d_g=_np(gg.grad),
                d_beta=_np(bb.grad), d_S0=_np(ss.grad), meta=np.array([B, T, H, K, V, chunk]))


# --------------------------------------------------------------------------------------
#  head-level fixtures
# --------------------------------------------------------------------------------------
def head_longhead(gen, B=2, T=45, d=24, M=12, dv=6, chunk=16):
    """lapa.layer.LongHead with ordinary random weights: u = rms(o), the new state, and all
    gradients of sum(u * dU) + sum(S * dS)."""
    import lapa.layer as LL
    torch.manual_seed(int(torch.randint(0, 2**31 - 1, (1,), generator=gen)))
    cfg = LL.LaplaceConfig(d=d, M=M, dv=dv, L=16, chunk=chunk, persist=0.5, theta_scale=0.3)
    head = LL.LongHead(cfg).double()
    with torch.no_grad():
        head.wi.copy_(torch.randn(M, generator=gen, dtype=torch.float64) * 0.3)
        head.bproj.weight.copy_(torch.randn(1, d, generator=gen, dtype=torch.float64) * 0.3)
    z = torch.randn(B, T, d, generator=gen, dtype=torch.float64).requires_grad_(True)
    h = torch.randn(B, T, d, generator=gen, dtype=torch.float64).requires_grad_(True)
    sr0 = torch.randn(B, M, dv, generator=gen, dtype=torch.float64) * 0.3
    si0 = torch.randn(B, M, dv, generator=gen, dtype=torch.float64) * 0.3
    pos0 = 7.0
    st = {"sr": sr0, "si": si0, "pos": torch.tensor(pos0, dtype=torch.float64)}
    u, st1 = head.prefill(z, h, st)
    dU = torch.randn(u.shape, generator=gen, dtype=torch.float64)
    (u * dU).sum().backward()
    sd = {k: _np(v) for k, v in head.state_dict().items()}
    grads = {"g_" + n: _np(p.grad) for n, p in head.named_parameters() if p.grad is not None}
    return dict(z=_np(z), h=_np(h), sr0=_np(sr0), si0=_np(si0), pos0=np.array(pos0),
                u=_np(u), sr=_np(st1["sr"]), si=_np(st1["si"]), dU=_np(dU),
                d_z=_np(z.grad), d_h=_np(h.grad),
                meta=np.array([B, T, d, M, dv, chunk]),
                **{"sd_" + k: v for k, v in sd.items()}, **grads)


def head_gated(gen, B=2, T=45, d=24, H=2, Mh=6, dvh=4, ctx=16):
    """sca2.arch_gatedc.CHeadGated (heads=2, decay) with random weights and RMS read-out."""
    from sca2.arch_gatedc import CHeadGated
    torch.manual_seed(int(torch.randint(0, 2**31 - 1, (1,), generator=gen)))
    M, dv = H * Mh, H * dvh
    head = CHeadGated(d, M, freq="rope", theta_scale=0.3, max_len=64, dv=dv, heads=H,
                      decay=True).double()
    head.CTX = ctx
    with torch.no_grad():
        head.wi.copy_(torch.randn(M, generator=gen, dtype=torch.float64) * 0.3)
    z = torch.randn(B, T, d, generator=gen, dtype=torch.float64).requires_grad_(True)
    h = torch.randn(B, T, d, generator=gen, dtype=torch.float64).requires_grad_(True)
    sr0 = torch.randn(B, H, Mh, dvh, generator=gen, dtype=torch.float64) * 0.3
    si0 = torch.randn(B, H, Mh, dvh, generator=gen, dtype=torch.float64) * 0.3
    pos0 = 5.0
    st = {"sr": sr0, "si": si0, "pos": torch.tensor(pos0, dtype=torch.float64), "empty": False}
    u, st1 = head.prefill(z, h, st)
    dU = torch.randn(u.shape, generator=gen, dtype=torch.float64)
    (u * dU).sum().backward()
    sd = {k: _np(v) for k, v in head.state_dict().items()}
    grads = {"g_" + n: _np(p.grad) for n, p in head.named_parameters() if p.grad is not None}
    return dict(z=_np(z), h=_np(h), sr0=_np(sr0), si0=_np(si0), pos0=np.array(pos0),
                u=_np(u), sr=_np(st1["sr"]), si=_np(st1["si"]), dU=_np(dU),
                d_z=_np(z.grad), d_h=_np(h.grad),
                meta=np.array([B, T, d, H, Mh, dvh, ctx]),
                **{"sd_" + k: v for k, v in sd.items()}, **grads)


def head_d(gen, kind, B=2, T=45, d=24, M=4, G=4, dv=32, steps=3):
    """A reference D head (DHeadRef, DHeadSepQ or DHeadSepQPolar; sca2/ref.py:209-275,
    sca2/arch_sepq.py:46-290) with random weights: prefill on random z, h and a random
    incoming state, the RMS'd output u, the new state, every parameter / input gradient of
    sum(u * dU), then `steps` decode steps continuing from the prefill's state."""
    from sca2.ref import DHeadRef
    from sca2.arch_sepq import DHeadSepQ, DHeadSepQPolar
    torch.manual_seed(int(torch.randint(0, 2**31 - 1, (1,), generator=gen)))
    cls = {"ref": DHeadRef, "sepq": DHeadSepQ, "polar": DHeadSepQPolar}[kind]
    gated = kind != "ref"
    head = cls(d, M, G, dv=dv, gated_read=gated).double()
    z = torch.randn(B, T, d, generator=gen, dtype=torch.float64).requires_grad_(True)
    h = torch.randn(B, T, d, generator=gen, dtype=torch.float64).requires_grad_(True)
    sr0 = torch.randn(B, M, dv, generator=gen, dtype=torch.float64) * 0.3
    si0 = torch.randn(B, M, dv, generator=gen, dtype=torch.float64) * 0.3
    u, st1 = head.prefill(z, h, {"sr": sr0, "si": si0})
    dU = torch.randn(u.shape, generator=gen, dtype=torch.float64)
    (u * dU).sum().backward()
    sd = {k: _np(v) for k, v in head.state_dict().items()}
    grads = {"g_" + n: _np(p.grad) for n, p in head.named_parameters() if p.grad is not None}
    zs = torch.randn(B, steps, d, generator=gen, dtype=torch.float64)
    hs = torch.randn(B, steps, d, generator=gen, dtype=torch.float64)
    st = {"sr": st1["sr"].detach(), "si": st1["si"].detach()}
    us = []
    with torch.no_grad():
        for t in range(steps):
            ut, st = head.step(zs[:, t], hs[:, t], st)
            us.append(ut)
    return dict(z=_np(z), h=_np(h), sr0=_np(sr0), si0=_np(si0), u=_np(u), sr=_np(st1["sr"]),
                si=_np(st1["si"]), dU=_np(dU), d_z=_np(z.grad), d_h=_np(h.grad),
                zs=_np(zs), hs=_np(hs), us=_np(torch.stack(us, 1)), srs=_np(st["sr"]), sis=_np(st["si"]),
                meta=np.array([B, T, d, M, G, dv, int(gated)]),
                **{"sd_" + k: v for k, v in sd.items()}, **grads)


def head_short(gen, kind, B=2, T=45, d=24, L=8, dv=6, T2=3, steps=3, pos0=5):
    """The short head's exact L-tap window read: lapa.layer.ShortHead (kind "lapa",
    lapa/layer.py:418-545) or sca2.arch_short.CHeadShort (kind "sca2", sca2/arch_short.py:45-158),
    random weights (wr, wi perturbed off the identity tap), a random incoming ring buffer
    (cos / sin of random phases, random values) at position pos0.  Records the prefill's u and
    new state with every gradient of sum(u * dU) + sum(new state * dNew) (state gradients
    included), then a second prefill of T2 < L-1 tokens (the new buffer mixes old and new
    writes) and `steps` decode steps, forward only."""
    torch.manual_seed(int(torch.randint(0, 2**31 - 1, (1,), generator=gen)))
    if kind == "lapa":
        import lapa.layer as LL
        head = LL.ShortHead(LL.LaplaceConfig(d=d, L=L, dv=dv, theta_scale=0.5)).double()
    else:
        from sca2.arch_short import CHeadShort
        head = CHeadShort(d, L, dv, theta_scale=0.5).double()
    with torch.no_grad():
        head.wr.add_(0.3 * torch.randn(L, generator=gen, dtype=torch.float64))
        head.wi.add_(0.3 * torch.randn(L, generator=gen, dtype=torch.float64))
    n = L - 1
    z = torch.randn(B, T, d, generator=gen, dtype=torch.float64).requires_grad_(True)
    h = torch.randn(B, T, d, generator=gen, dtype=torch.float64).requires_grad_(True)
    ph0 = torch.randn(B, n, L, generator=gen, dtype=torch.float64)
    c0 = ph0.cos().requires_grad_(True)
    s0 = ph0.sin().requires_grad_(True)
    e0 = torch.randn(B, n, dv, generator=gen, dtype=torch.float64).requires_grad_(True)
    st = {"c": c0, "s": s0, "e": e0, "pos": torch.tensor(pos0, dtype=torch.long)}
    u, st1 = head.prefill(z, h, st)
    dU = torch.randn(u.shape, generator=gen, dtype=torch.float64)
    dc = torch.randn(B, n, L, generator=gen, dtype=torch.float64)
    ds = torch.randn(B, n, L, generator=gen, dtype=torch.float64)
    de = torch.randn(B, n, dv, generator=gen, dtype=torch.float64)
    ((u * dU).sum() + (st1["c"] * dc).sum() + (st1["s"] * ds).sum() + (st1["e"] * de).sum()).backward()
    sd = {k: _np(v) for k, v in head.state_dict().items()}
    grads = {"g_" + nm: _np(p.grad) for nm, p in head.named_parameters() if p.grad is not None}
    st1 = {k: v.detach() for k, v in st1.items()}
    z2 = torch.randn(B, T2, d, generator=gen, dtype=torch.float64)
    h2 = torch.randn(B, T2, d, generator=gen, dtype=torch.float64)
    zs = torch.randn(B, steps, d, generator=gen, dtype=torch.float64)
    hs = torch.randn(B, steps, d, generator=gen, dtype=torch.float64)
    us = []
    with torch.no_grad():
        u2, st2 = head.prefill(z2, h2, st1)
        st = st2
        for t in range(steps):
            ut, st = head.step(zs[:, t], hs[:, t], st)
            us.append(ut)
    return dict(z=_np(z), h=_np(h), c0=_np(c0), s0=_np(s0), e0=_np(e0), pos0=np.array(pos0),
                u=_np(u), c1=_np(st1["c"]), s1=_np(st1["s"]), e1=_np(st1["e"]),
                dU=_np(dU), dc1=_np(dc), ds1=_np(ds), de1=_np(de),
                d_z=_np(z.grad), d_h=_np(h.grad), d_c0=_np(c0.grad), d_s0=_np(s0.grad), d_e0=_np(e0.grad),
                z2=_np(z2), h2=_np(h2), u2=_np(u2), c2=_np(st2["c"]), s2=_np(st2["s"]), e2=_np(st2["e"]),
                zs=_np(zs), hs=_np(hs), us=_np(torch.stack(us, 1)),
                cs=_np(st["c"]), ss=_np(st["s"]), es=_np(st["e"]), pos_end=np.array(int(st["pos"])),
                meta=np.array([B, T, d, L, dv, T2, steps]),
                **{"sd_" + k: v for k, v in sd.items()}, **grads)


def _tree_np(prefix, x, out):
    if isinstance(x, dict):
        for k, v in x.items():
            _tree_np(f"{prefix}.{k}", v, out)
    elif isinstance(x, (list, tuple)):
        for i, v in enumerate(x):
            _tree_np(f"{prefix}.{i}", v, out)
    elif torch.is_tensor(x):
        out[prefix] = _np(x)
    elif isinstance(x, (int, float)) and not isinstance(x, bool):
        out[prefix] = np.array(x)
    return out


def layer_fixture(gen, kind, B=2, T=45, steps=3):
    """A reference layer with random weights: prefill from its initial state, the output,
    the new state, every parameter and input gradient of sum(y * dY), then `steps` decode
    steps continuing from the prefill's state.  kind: "sca2" (SCA2Layer: CHeadRef + DHeadRef,
    sca2/ref.py:333-390), "gated" (GatedLayer: CHeadGated 2 heads with decay + DHeadSepQPolar
    + causal conv, sca2/arch_gatedc.py:199-256), "lapa" (LaplaceAttention, lapa/layer.py:551-600)."""
    torch.manual_seed(int(torch.randint(0, 2**31 - 1, (1,), generator=gen)))
    if kind == "lapa":
        import lapa.layer as LL
        layer = LL.LaplaceAttention(LL.LaplaceConfig(d=32, M=12, dv=8, L=8, ff=48, chunk=16,
                                                     theta_scale=0.3)).double()
        d = 32
    else:
        from sca2.ref import LayerCfg, SCA2Layer
        from sca2.arch_gatedc import GatedLayer
        if kind == "sca2":
            cfg = LayerCfg(d=32, Mc=16, Md=4, G=4, ff=48, freq="rope", theta_scale=0.3, max_len=64, dv=32)
            layer = SCA2Layer(cfg).double()
        else:
            # the reference's SCA2Layer passes rope_base / slow_frac, which its CHeadGated does not
            # take: build through a shim that drops them (the GatedLayer itself is unchanged)
            import sca2.arch_gatedc as AG
            orig = AG.CHeadGated
            AG.CHeadGated = lambda *a, rope_base=None, slow_frac=None, **kw: orig(*a, **kw)
            try:
                cfg = LayerCfg(d=32, Mc=16, Md=4, G=4, ff=48, freq="rope", theta_scale=0.3, max_len=64, dv=32,
                               c_heads=2, c_decay=True, conv=3)
                layer = GatedLayer(cfg).double()
            finally:
                AG.CHeadGated = orig
        d = cfg.d
    with torch.no_grad():  # move the read weights off their identity init
        for n, p in layer.named_parameters():
            if n.endswith("wr") or n.endswith("wi"):
                p.add_(0.3 * torch.randn(p.shape, generator=gen, dtype=torch.float64))
    x = torch.randn(B, T, d, generator=gen, dtype=torch.float64).requires_grad_(True)
    y, st = layer.prefill(x)
    dY = torch.randn(y.shape, generator=gen, dtype=torch.float64)
    (y * dY).sum().backward()
    out = dict(x=_np(x), y=_np(y), dY=_np(dY), d_x=_np(x.grad), meta=np.array([B, T, d, steps]))
    out.update({"sd_" + k: _np(v) for k, v in layer.state_dict().items()})
    out.update({"g_" + n: _np(p.grad) for n, p in layer.named_parameters() if p.grad is not None})
    _tree_np("st", st, out)
    xs = torch.randn(B, steps, d, generator=gen, dtype=torch.float64)
    st = {k: (v.detach() if torch.is_tensor(v) else v) for k, v in st.items()}
    st = _detach(st)
    ys = []
    with torch.no_grad():
        for t in range(steps):
            yt, st = layer.step(xs[:, t], st)
            ys.append(yt)
    out.update(xs=_np(xs), ys=_np(torch.stack(ys, 1)))
    _tree_np("sts", st, out)
    return out


def config1_fixture():
    """The first benchmark configuration at its own shape (tests/golden/config1.py): the
    reference GatedLayer (CHeadGated with 4 heads and decay, DHeadSepQPolar, chunk CTX = 64),
    built through the shim that drops rope_base / slow_frac, state dict from torch seed 0 with
    every 2-D weight re-drawn N(0, 0.02^2) and x ~ N(0, 1) by config1.draw, run in float64.
    Stored: the output y, the final state of both heads and z_prev, the gradient of
    sum(y * dY) for x and for every C-head parameter, and the state-dict entries that draw()
    does not regenerate."""
    sys.path.insert(0, os.path.dirname(os.path.abspath(__file__)))
    import config1 as C1
    import sca2.arch_gatedc as AG
    from sca2.ref import LayerCfg
    orig, ctx = AG.CHeadGated, AG.CHeadGated.CTX
    AG.CHeadGated.CTX = C1.CHUNK
    AG.CHeadGated = lambda *a, rope_base=None, slow_frac=None, **kw: orig(*a, **kw)
    try:
        torch.manual_seed(C1.SEED)
        layer = AG.GatedLayer(LayerCfg(**C1.LAYER))
        sd = layer.state_dict()
        w, x, dY = C1.draw(sd)
        sd.update(w)
        layer.load_state_dict(sd, strict=True)
        layer = layer.double()
        xd = x.double().requires_grad_(True)
        y, st = layer.prefill(xd)
        (y * dY.double()).sum().backward()
    finally:
        AG.CHeadGated = orig
        orig.CTX = ctx
    keep = set(C1.redrawn(sd))
    out = dict(y=_np(y).astype(np.float32), d_x=_np(xd.grad).astype(np.float32),
               meta=np.array([C1.B, C1.T, C1.LAYER["d"], C1.LAYER["c_heads"], C1.CHUNK]))
    out.update({"sd_" + k: _np(v) for k, v in layer.state_dict().items() if k not in keep})
    out.update({"g_" + n: _np(p.grad).astype(np.float32) for n, p in layer.named_parameters()
                if n.startswith("c.") and p.grad is not None})
    _tree_np("st", _detach(st), out)
    return out


def _detach(x):
    if isinstance(x, dict):
        return {k: _detach(v) for k, v in x.items()}
    if isinstance(x, (list, tuple)):
        return type(x)(_detach(v) for v in x)
    return x.detach() if torch.is_tensor(x) else x


def lm_fixture(gen, B=2, T=30, vocab=40, n_new=6):
    """lapa.model.LaplaceLM (2 LaplaceAttention layers, lapa/model.py): logits of a token
    batch, the gradients of the next-token cross entropy for every parameter, and a greedy
    continuation of a prompt (prefill + steps)."""
    import lapa.model as LM
    torch.manual_seed(int(torch.randint(0, 2**31 - 1, (1,), generator=gen)))
    lm = LM.LaplaceLM(vocab, d=32, n_layers=2, M=12, dv=8, L=8, ff=48, chunk=16, theta_scale=0.3).double()
    tok = torch.randint(0, vocab, (B, T + 1), generator=gen)
    logits = lm(tok[:, :-1])
    loss = torch.nn.functional.cross_entropy(logits.reshape(-1, vocab), tok[:, 1:].reshape(-1))
    loss.backward()
    prompt = torch.randint(0, vocab, (B, 9), generator=gen)
    with torch.no_grad():
        gen_ids = lm.generate(prompt, n_new, greedy=True)
    out = dict(tok=tok.numpy(), logits=_np(logits), loss=_np(loss), prompt=prompt.numpy(), gen=gen_ids.numpy(),
               meta=np.array([B, T, vocab, 32, 2, n_new]))
    out.update({"sd_" + k: _np(v) for k, v in lm.state_dict().items()})
    out.update({"g_" + n: _np(p.grad) for n, p in lm.named_parameters() if p.grad is not None})
    return out


def main(ref_root):
    sys.path.insert(0, ref_root)
    import sca2.arch_short  # noqa: F401  registers cdelta/damp/short (see registry import order)
    import sca2.arch_gatedc  # noqa: F401
    torch.set_default_dtype(torch.float32)
    gen = torch.Generator().manual_seed(20241201)
    _save("scan_longhead.npz", **longhead_scan(gen))
    _save("scan_longhead_chunkpath.npz", **longhead_scan(gen, T=37, path="chunk"))
    _save("step_longhead.npz", **longhead_step(gen))
    _save("scan_gated.npz", **gated_scan(gen))
    _save("scan_cdelta.npz", **cdelta_scan(gen))
    _save("scan_cdelta_damp.npz", **cdelta_scan(gen, damp=True))
    _save("gdn_fla.npz", **gdn_fla(gen))
    _save("head_longhead.npz", **head_longhead(gen))
    _save("head_gated.npz", **head_gated(gen))
    _save("head_dref.npz", **head_d(gen, "ref", M=4, G=4, dv=32))
    _save("head_dsepq.npz", **head_d(gen, "sepq", M=8, G=4, dv=16))
    _save("head_dpolar.npz", **head_d(gen, "polar", M=16, G=4, dv=16))
    _save("head_short_lapa.npz", **head_short(gen, "lapa", L=8, dv=6))
    _save("head_short_sca2.npz", **head_short(gen, "sca2", L=16, dv=8, T=37, T2=5, pos0=13))
    _save("layer_sca2.npz", **layer_fixture(gen, "sca2"))
    _save("layer_gated.npz", **layer_fixture(gen, "gated"))
    _save("layer_lapa.npz", **layer_fixture(gen, "lapa"))
    _save("lm_lapa.npz", **lm_fixture(gen))
    _save("layer_gated_config1.npz", **config1_fixture())


if __name__ == "__main__":
    ref = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("SCA2_REFERENCE")
    if not ref:
        sys.exit("usage: make_golden.py /path/to/reference   (or set SCA2_REFERENCE)")
    main(ref)
