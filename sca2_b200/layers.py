"""Layers around the heads, with the reference's layer protocol

    prefill(x, state=None) -> (y, state)     x (B,T,d)
    step(x_t, state)       -> (y_t, state)   one token (B,d)
    init_state(B, device[, dtype]);  forward(x) = prefill(x)[0]

and the reference's parameter names, so a reference layer's state_dict loads with
strict=True.  The heads are this package's (scan on the sm_100a kernels); norms, the
mix projection and the FFN are ordinary torch modules (cuBLAS GEMMs under autocast).

  LayerCfg          sca2/ref.py:281-331        (field for field)
  SCA2Layer         sca2/ref.py:333-390        norm -> (C head || D head) -> mix -> FFN
  GatedLayer        sca2/arch_gatedc.py:199-256  multi-head gated C head, causal conv on z
  ShortLayer*       sca2/arch_short.py:161-214   long C head + short DFT head in the D slot
  LaplaceAttention  lapa/layer.py:551-600      LapA: long head || short head
"""
from __future__ import annotations

import math
from dataclasses import dataclass
from typing import Optional

import torch
import torch.nn as nn
import torch.nn.functional as F

from . import heads
from .heads import LaplaceConfig


@dataclass
class LayerCfg:
    """Field for field the reference's LayerCfg (sca2/ref.py:281-331)."""
    d: int = 128
    Mc: int = 64
    Md: int = 16
    G: int = 8
    ff: int = 256
    freq: str = "dft"
    theta_scale: float = 0.0
    max_len: int = 128
    delta_rule: bool = False
    gated_read: bool = False
    dv: int = None
    c_heads: int = 1
    c_decay: bool = False
    c_decay_init: str = "gdn"
    c_sepq: bool = False
    conv: int = 0
    Ls: int = 16
    rope_base: float = 10000.0
    slow_frac: float = 0.0
    damp_mem: tuple = None
    lam_max: float = None
    gdn_heads: int = 3
    gdn_head_k: int = 60
    gdn_expand_v: float = 1.0


def _shift(z, z_prev):
    """h_t = z_{t-1}, with the state's last z before the first token."""
    return torch.cat([z_prev.to(z.dtype)[:, None], z[:, :-1]], 1)


class SCA2Layer(nn.Module):
    """sca2/ref.py:333-390: norm -> (C head || D head) -> mix -> residual -> FFN -> residual."""

    def __init__(self, cfg: LayerCfg, c_cls=None, d_cls=None):
        super().__init__()
        c_cls = c_cls or heads.CHeadRef
        d_cls = d_cls or heads.DHeadRef
        self.cfg = cfg
        d = cfg.d
        dv = cfg.dv if cfg.dv is not None else d // 2
        self.n = nn.LayerNorm(d)
        self.c = c_cls(d, cfg.Mc, freq=cfg.freq, theta_scale=cfg.theta_scale, max_len=cfg.max_len, dv=dv,
                       gated_read=cfg.gated_read, rope_base=cfg.rope_base, slow_frac=cfg.slow_frac)
        self.dh = d_cls(d, cfg.Md, cfg.G, dv=dv, max_len=cfg.max_len, delta_rule=cfg.delta_rule,
                        gated_read=cfg.gated_read)
        self.mix = nn.Linear(4 * dv, d)
        self.fn = nn.LayerNorm(d)
        self.ff = nn.Sequential(nn.Linear(d, cfg.ff), nn.GELU(), nn.Linear(cfg.ff, d))

    def init_state(self, B, device, dtype=torch.float32):
        return {"c": self.c.init_state(B, device, dtype), "d": self.dh.init_state(B, device, dtype),
                "z_prev": torch.zeros(B, self.cfg.d, device=device, dtype=dtype)}

    def forward(self, x):
        return self.prefill(x)[0]

    def _mixer(self, z, h, state):
        uc, cs = self.c.prefill(z, h, state["c"])
        ud, ds = self.dh.prefill(z, h, state["d"])
        return torch.cat([uc, ud], -1), {"c": cs, "d": ds}

    def prefill(self, x, state=None):
        B = x.size(0)
        st = state if state is not None else self.init_state(B, x.device, x.dtype)
        z = self.n(x)
        u, new = self._mixer(z, _shift(z, st["z_prev"]), st)
        x = x + self.mix(u)
        x = x + self.ff(self.fn(x))
        new["z_prev"] = z[:, -1]
        return x, new

    def step(self, x_t, state):
        z = self.n(x_t)
        h = state["z_prev"].to(z.dtype)
        uc, cs = self.c.step(z, h, state["c"])
        ud, ds = self.dh.step(z, h, state["d"])
        y = x_t + self.mix(torch.cat([uc, ud], -1))
        y = y + self.ff(self.fn(y))
        return y, {"c": cs, "d": ds, "z_prev": z}


class GatedLayer(SCA2Layer):
    """sca2/arch_gatedc.py:199-256: CHeadGated (cfg.c_heads heads, optional scalar decay and
    separate read key) in the C slot, DHeadSepQPolar by default in the D slot, and an
    optional causal depthwise conv of width cfg.conv on z before the heads."""

    def __init__(self, cfg: LayerCfg, c_cls=None, d_cls=None):
        d_cls = d_cls or heads.DHeadSepQPolar

        def c_make(d, M, **kw):
            return heads.CHeadGated(d, M, heads=cfg.c_heads, decay=cfg.c_decay, sepq=cfg.c_sepq,
                                    decay_init=cfg.c_decay_init, **kw)
        super().__init__(cfg, c_make, d_cls)
        self.k = cfg.conv
        if self.k:
            w = torch.zeros(cfg.d, 1, self.k)
            w[:, 0, -1] = 1.0
            self.cw = nn.Parameter(w)

    def init_state(self, B, device, dtype=torch.float32):
        st = super().init_state(B, device, dtype)
        if self.k:
            st["cbuf"] = torch.zeros(B, self.k - 1, self.cfg.d, device=device, dtype=dtype)
        return st

    def prefill(self, x, state=None):
        B = x.size(0)
        st = state if state is not None else self.init_state(B, x.device, x.dtype)
        z = self.n(x)
        cbuf = None
        if self.k:
            zz = torch.cat([st["cbuf"].to(z.dtype), z], 1)
            z = F.conv1d(zz.transpose(1, 2), self.cw.to(z.dtype), groups=self.cfg.d).transpose(1, 2)
            cbuf = zz[:, -(self.k - 1):]
        u, new = self._mixer(z, _shift(z, st["z_prev"]), st)
        x = x + self.mix(u)
        x = x + self.ff(self.fn(x))
        new["z_prev"] = z[:, -1]
        if self.k:
            new["cbuf"] = cbuf
        return x, new

    def step(self, x_t, state):
        z = self.n(x_t)
        new = {}
        if self.k:
            win = torch.cat([state["cbuf"].to(z.dtype), z[:, None]], 1)
            z = (win * self.cw[:, 0, :].t().to(z.dtype)[None]).sum(1)
            new["cbuf"] = win[:, 1:]
        h = state["z_prev"].to(z.dtype)
        uc, cs = self.c.step(z, h, state["c"])
        ud, ds = self.dh.step(z, h, state["d"])
        y = x_t + self.mix(torch.cat([uc, ud], -1))
        y = y + self.ff(self.fn(y))
        new.update({"c": cs, "d": ds, "z_prev": z})
        return y, new


class ShortLayer(SCA2Layer):
    """sca2/arch_short.py:161-177: a long C head (C_CLS) and the short DFT head CHeadShort in
    the D slot (window cfg.Ls); the damped long heads start just beyond the window and never
    forget faster than it (lam_max = 1 / Ls, memories in (Ls, 32 Ls))."""
    C_CLS = heads.CHeadDelta

    def __init__(self, cfg: LayerCfg, c_cls=None, d_cls=None):
        super().__init__(cfg, self.C_CLS, heads.DHeadSepQPolar)
        dv = cfg.dv if cfg.dv is not None else cfg.d // 2
        self.dh = heads.CHeadShort(cfg.d, cfg.Ls, dv, theta_scale=cfg.theta_scale or 0.02)
        if hasattr(self.c, "lam_raw"):
            lam_max = cfg.lam_max if cfg.lam_max is not None else 1.0 / cfg.Ls
            lo, hi = cfg.damp_mem if cfg.damp_mem is not None else (float(cfg.Ls), 32.0 * cfg.Ls)
            self.c.LAM_MAX = lam_max
            with torch.no_grad():
                mem = torch.exp(torch.empty(self.c.M).uniform_(math.log(lo), math.log(hi)))
                self.c.lam_raw.copy_(torch.log(torch.expm1(1.0 / mem)))


class ShortLayerDampH(ShortLayer):
    """sca2/arch_short.py:199-201: the half-persistent damped long head (cshort_damph)."""
    C_CLS = heads.CHeadDeltaDampHalf


class LaplaceAttention(nn.Module):
    """lapa/layer.py:551-600: norm -> (long head || short head) -> mix -> residual -> norm ->
    FFN -> residual."""

    def __init__(self, cfg: LaplaceConfig = LaplaceConfig()):
        super().__init__()
        self.cfg = cfg
        d, dv = cfg.d, cfg.dv
        self.n = nn.LayerNorm(d)
        self.long = heads.LongHead(cfg)
        self.short = heads.ShortHead(cfg)
        self.mix = nn.Linear(4 * dv, d)
        self.fn = nn.LayerNorm(d)
        self.ff = nn.Sequential(nn.Linear(d, cfg.ff), nn.GELU(), nn.Linear(cfg.ff, d))

    def init_state(self, B: int, device):
        return {"long": self.long.init_state(B, device), "short": self.short.init_state(B, device),
                "z_prev": torch.zeros(B, self.cfg.d, device=device, dtype=self.n.weight.dtype)}

    def forward(self, x):
        return self.prefill(x)[0]

    def prefill(self, x, state: Optional[dict] = None):
        B = x.size(0)
        st = state if state is not None else self.init_state(B, x.device)
        z = self.n(x)
        h = _shift(z, st["z_prev"])
        ul, sl = self.long.prefill(z, h, st["long"])
        us, ss = self.short.prefill(z, h, st["short"])
        x = x + self.mix(torch.cat([ul, us], -1))
        x = x + self.ff(self.fn(x))
        return x, {"long": sl, "short": ss, "z_prev": z[:, -1]}

    def step(self, x_t, state):
        z = self.n(x_t)
        h = state["z_prev"].to(z.dtype)
        ul, sl = self.long.step(z, h, state["long"])
        us, ss = self.short.step(z, h, state["short"])
        y = x_t + self.mix(torch.cat([ul, us], -1))
        y = y + self.ff(self.fn(y))
        return y, {"long": sl, "short": ss, "z_prev": z}

    def state_floats(self) -> int:
        cfg = self.cfg
        return 2 * cfg.M * cfg.dv + (cfg.L - 1) * (2 * cfg.L + cfg.dv) + cfg.d
