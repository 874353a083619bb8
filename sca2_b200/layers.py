"""Residual mixer layers around this package's heads, on the reference's layer protocol

    prefill(x, state=None) -> (y, state)     x (B,T,d)
    step(x_t, state)       -> (y_t, state)   one token (B,d)
    init_state(B, device[, dtype]);  forward(x) = prefill(x)[0]

Every layer family of the reference is one pre-norm residual block with a different set of
parallel sequence mixers ("head slots"), so this module has ONE block, `MixerLayer`, driven
by a slot table:

    z  = LN(x)  [-> causal depthwise conv of width k, with a (k-1)-token buffer in the state]
    h  = z shifted one token later (the state's z_prev before the first token)
    u_s, state_s = slot_s.prefill(z, h, state[s])          for every slot s, in table order
    y  = x + mix(concat_s u_s);   y = y + FFN(LN(y))

A slot is (module attribute, state key).  The families differ only in their table and head
constructors:

    family            slots (attribute:state key)   reference layer it loads weights of
    SCA2Layer         c:c, dh:d                     sca2/ref.py:333-390
    GatedLayer        c:c, dh:d  (+ conv)           sca2/arch_gatedc.py:199-256
    ShortLayer(DampH) c:c, dh:d  (dh = short head)  sca2/arch_short.py:161-214
    LaplaceAttention  long:long, short:short        lapa/layer.py:551-600

Parameter and state names follow those layers (n, <slots>, mix, fn, ff.0, ff.2, cw), so a
reference layer's state_dict loads with strict=True and decode states are interchangeable;
LayerCfg is the reference's configuration record field for field.  The heads run on the
sm_100a kernels; norms, the mix projection and the FFN are torch modules (cuBLAS under
autocast).
"""
from __future__ import annotations

import math
from dataclasses import dataclass
from typing import Dict, Optional, Sequence, Tuple

import torch
import torch.nn as nn
import torch.nn.functional as F

from . import heads, ops
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


class LayerNorm(nn.LayerNorm):
    """nn.LayerNorm (same parameters and state-dict names) whose CUDA fp32 forward and backward
    run on this package's row kernels (ops.layer_norm) for the widths they cover; autocast keeps
    LayerNorm in fp32, as torch does."""

    def forward(self, x):
        d = self.normalized_shape[-1]
        if (x.is_cuda and (x.dtype == torch.float32 or torch.is_autocast_enabled()) and self.elementwise_affine
                and self.bias is not None and len(self.normalized_shape) == 1 and ops.layer_norm_supported(d)):
            return ops.layer_norm(x, self.weight, self.bias, self.eps)
        return super().forward(x)


Slot = Tuple[str, str]  # (module attribute, state key)


class MixerLayer(nn.Module):
    """One pre-norm residual block over a table of parallel head slots (module docstring)."""

    def __init__(self, d: int, slots: Sequence[Tuple[str, str, nn.Module]], mix_in: int, ff: int, conv: int = 0):
        super().__init__()
        self.d = d
        self.n = LayerNorm(d)
        self.slots: Tuple[Slot, ...] = tuple((attr, key) for attr, key, _ in slots)
        for attr, _, module in slots:
            self.add_module(attr, module)
        self.mix = nn.Linear(mix_in, d)
        self.fn = LayerNorm(d)
        self.ff = nn.Sequential(nn.Linear(d, ff), nn.GELU(), nn.Linear(ff, d))
        self.k = conv
        if conv:
            w = torch.zeros(d, 1, conv)
            w[:, 0, -1] = 1.0  # identity tap at init: the conv starts as a no-op
            self.cw = nn.Parameter(w)

    # ---- state ------------------------------------------------------------------------
    def _head_state(self, head, B, device, dtype):
        return head.init_state(B, device, dtype)

    def init_state(self, B: int, device, dtype=torch.float32) -> Dict:
        st = {key: self._head_state(getattr(self, attr), B, device, dtype) for attr, key in self.slots}
        st["z_prev"] = torch.zeros(B, self.d, device=device, dtype=dtype)
        if self.k:
            st["cbuf"] = torch.zeros(B, self.k - 1, self.d, device=device, dtype=dtype)
        return st

    # ---- the residual tail shared by prefill and step ---------------------------------
    def _tail(self, x: torch.Tensor, us) -> torch.Tensor:
        if torch.is_autocast_enabled() and x.is_cuda:
            # the mix product reads its input in the autocast dtype: cast each slot's read-out
            # before joining them (the same elementwise rounding as casting the joined fp32
            # tensor, without materialising it; the gradients come back per slot, contiguous)
            dt = torch.get_autocast_dtype("cuda")
            us = [u.to(dt) for u in us]
        y = x + self.mix(torch.cat(us, -1))
        return y + self.ff(self.fn(y))

    def forward(self, x):
        return self.prefill(x)[0]

    def prefill(self, x: torch.Tensor, state: Optional[Dict] = None):
        st = state if state is not None else self.init_state(x.size(0), x.device, x.dtype)
        z = self.n(x)
        new = {}
        if self.k:  # causal depthwise conv over [buffer ; z], the last k-1 inputs kept
            zz = torch.cat([st["cbuf"].to(z.dtype), z], 1)
            new["cbuf"] = zz[:, zz.size(1) - (self.k - 1):]
            z = F.conv1d(zz.transpose(1, 2), self.cw.to(z.dtype), groups=self.d).transpose(1, 2)
        h = torch.cat([st["z_prev"].to(z.dtype).unsqueeze(1), z[:, :-1]], 1)
        us = []
        for attr, key in self.slots:
            u, new[key] = getattr(self, attr).prefill(z, h, st[key])
            us.append(u)
        new["z_prev"] = z[:, -1]
        return self._tail(x, us), new

    def step(self, x_t: torch.Tensor, state: Dict):
        z = self.n(x_t)
        new = {}
        if self.k:  # the conv's window is [buffer ; z_t]
            win = torch.cat([state["cbuf"].to(z.dtype), z.unsqueeze(1)], 1)
            new["cbuf"] = win[:, 1:]
            z = torch.einsum("bkd,dk->bd", win, self.cw[:, 0, :].to(z.dtype))
        h = state["z_prev"].to(z.dtype)
        us = []
        for attr, key in self.slots:
            u, new[key] = getattr(self, attr).step(z, h, state[key])
            us.append(u)
        new["z_prev"] = z
        return self._tail(x_t, us), new


# ---- the reference's layer families as slot tables --------------------------------------
def _dv(cfg: LayerCfg) -> int:
    return cfg.dv if cfg.dv is not None else cfg.d // 2


def _c_head(cfg: LayerCfg, c_cls, d: int, dv: int):
    return c_cls(d, cfg.Mc, freq=cfg.freq, theta_scale=cfg.theta_scale, max_len=cfg.max_len, dv=dv,
                 gated_read=cfg.gated_read, rope_base=cfg.rope_base, slow_frac=cfg.slow_frac)


def _d_head(cfg: LayerCfg, d_cls, d: int, dv: int):
    return d_cls(d, cfg.Md, cfg.G, dv=dv, max_len=cfg.max_len, delta_rule=cfg.delta_rule,
                 gated_read=cfg.gated_read)


class SCA2Layer(MixerLayer):
    """C head || D head (sca2/ref.py:333-390); c_cls / d_cls default to CHeadRef / DHeadRef."""

    def __init__(self, cfg: LayerCfg, c_cls=None, d_cls=None, conv: int = 0):
        dv = _dv(cfg)
        c = _c_head(cfg, c_cls or heads.CHeadRef, cfg.d, dv)
        dh = _d_head(cfg, d_cls or heads.DHeadRef, cfg.d, dv)
        super().__init__(cfg.d, [("c", "c", c), ("dh", "d", dh)], 4 * dv, cfg.ff, conv)
        self.cfg = cfg


class GatedLayer(SCA2Layer):
    """Multi-head gated C head (cfg.c_heads heads, optional scalar decay and separate read key)
    || DHeadSepQPolar by default, with a causal depthwise conv of width cfg.conv on z
    (sca2/arch_gatedc.py:199-256).  As in the reference, the C slot is always the gated head:
    c_cls is accepted for the layer-constructor protocol and not used."""

    def __init__(self, cfg: LayerCfg, c_cls=None, d_cls=None):
        def c_make(d, M, **kw):  # the C slot's constructor, given the cfg's gated knobs
            return heads.CHeadGated(d, M, heads=cfg.c_heads, decay=cfg.c_decay, sepq=cfg.c_sepq,
                                    decay_init=cfg.c_decay_init, **kw)
        super().__init__(cfg, c_make, d_cls or heads.DHeadSepQPolar, conv=cfg.conv)


class ShortLayer(MixerLayer):
    """A long C head (C_CLS) with the short DFT head in the D slot (window cfg.Ls,
    sca2/arch_short.py:161-177).  A damped long head starts just beyond the window and never
    forgets faster than it: lam <= lam_max (default 1 / Ls), memories drawn log-uniform in
    damp_mem (default (Ls, 32 Ls))."""
    C_CLS = heads.CHeadDelta

    def __init__(self, cfg: LayerCfg, c_cls=None, d_cls=None):
        dv = _dv(cfg)
        c = _c_head(cfg, self.C_CLS, cfg.d, dv)
        dh = heads.CHeadShort(cfg.d, cfg.Ls, dv, theta_scale=cfg.theta_scale or 0.02)
        super().__init__(cfg.d, [("c", "c", c), ("dh", "d", dh)], 4 * dv, cfg.ff)
        self.cfg = cfg
        if hasattr(c, "lam_raw"):
            c.LAM_MAX = cfg.lam_max if cfg.lam_max is not None else 1.0 / cfg.Ls
            lo, hi = cfg.damp_mem if cfg.damp_mem is not None else (float(cfg.Ls), 32.0 * cfg.Ls)
            with torch.no_grad():
                mem = torch.exp(torch.empty(c.M).uniform_(math.log(lo), math.log(hi)))
                c.lam_raw.copy_(torch.log(torch.expm1(1.0 / mem)))


class ShortLayerDampH(ShortLayer):
    """The half-persistent damped long head with the short head (sca2/arch_short.py:199-201)."""
    C_CLS = heads.CHeadDeltaDampHalf


class LaplaceAttention(MixerLayer):
    """Long head || short head (lapa/layer.py:551-600), configured by a LaplaceConfig."""

    def __init__(self, cfg: LaplaceConfig = LaplaceConfig()):
        super().__init__(cfg.d, [("long", "long", heads.LongHead(cfg)), ("short", "short", heads.ShortHead(cfg))],
                         4 * cfg.dv, cfg.ff)
        self.cfg = cfg

    def _head_state(self, head, B, device, dtype):
        return head.init_state(B, device)  # the LapA heads keep their own state dtype

    def init_state(self, B: int, device, dtype=None) -> Dict:
        return super().init_state(B, device, self.n.weight.dtype if dtype is None else dtype)

    def state_floats(self) -> int:
        """Decode-state floats per sequence: long head 2 M dv, short ring buffer, z_prev."""
        c = self.cfg
        return 2 * c.M * c.dv + (c.L - 1) * (2 * c.L + c.dv) + c.d
