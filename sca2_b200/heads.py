"""Drop-in heads whose scan runs on the sm_100a kernels of libsca2b200.so.

Each class keeps the reference head's parameter names, shapes and buffers, so a
reference state_dict loads with strict=True, and its protocol:

    prefill(z, h, state=None) -> (u, state)     z, h (B,T,d); u (B,T,2dv)
    step(z_t, h_t, state)     -> (u_t, state)   one token
    init_state(B, device[, dtype])
    forward(z, h) = prefill(z, h)[0]

The projections (K, V, bproj, a, rgate) stay ordinary cuBLAS GEMMs; the scan (phase codes,
decays, delta-rule solve, intra-chunk read, state carry) and the RMS read-out are the
hand-written kernels.  State dicts are the reference's: {"sr", "si"} fp32 plus a 0-dim
"pos" tensor (graph-capturable, sca2/decode.py:36-52).

  LongHead          lapa/layer.py:170-412            (per-mode decay, delta write)
  CHeadRef          sca2/ref.py:164-206              (additive write)
  CHeadDelta        sca2/arch_cdelta.py:92-206       (delta write)
  CHeadDeltaDamp*   sca2/arch_damp.py:43-259         (per-mode decay, delta write)
  CHeadGated        sca2/arch_gatedc.py:58-193       (H heads, scalar decay, additive)
  DHeadRef          sca2/ref.py:209-275              (D head: complex diagonal scan)
  DHeadSepQ(Polar)  sca2/arch_sepq.py:46-290         (D head, separable query; polar gate)
  ShortHead         lapa/layer.py:418-545            (exact L-tap window over a ring buffer)
  CHeadShort        sca2/arch_short.py:45-158        (the same read in the SCA2 D slot)
"""
from __future__ import annotations

import math
import os
from dataclasses import dataclass
from typing import Dict, Optional, Tuple

import torch
import torch.nn as nn
import torch.nn.functional as F

from . import ops

State = Dict[str, torch.Tensor]


# ----------------------------------------------------------------------------------------
#  configuration and frequency grids (same values as the reference's)
# ----------------------------------------------------------------------------------------
@dataclass
class LaplaceConfig:
    """Field-for-field the reference's LaplaceConfig (lapa/layer.py:82-114)."""
    d: int = 128
    M: int = 190
    dv: int = 56
    L: int = 16
    ff: int = 448
    theta_scale: float = 0.02
    persist: float = 0.5
    learn_persist: bool = False
    mem_range: Optional[Tuple[float, float]] = None
    lam_max: Optional[float] = None
    chunk: int = 128
    rope_base: float = 10000.0
    slow_frac: float = 0.0
    max_len: int = 1024
    long_path: str = "batched"
    gemm_dtype: Optional[torch.dtype] = None
    beta_init: float = -2.0


def rope_grid(M: int, base: float, slow_frac: float = 0.0, max_len: int = 1024) -> torch.Tensor:
    """omega_m = pi * base^(-m/(M-1)), optionally with a slow slice of periods
    [2 max_len, 20 max_len] (lapa/layer.py:126-139, sca2/ref.py:113-123)."""
    n_slow = int(round(slow_frac * M))
    n_fast = M - n_slow
    k = torch.arange(n_fast, dtype=torch.float32)
    fast = math.pi * base ** (-k / max(n_fast - 1, 1))
    if n_slow == 0:
        return fast
    per = torch.logspace(math.log10(2 * max_len), math.log10(20 * max_len), n_slow)
    return torch.cat([fast, 2 * math.pi / per])


def freq_grid(name: str, M: int, max_len: int = 128, base: float = 10000.0,
              slow_frac: float = 0.0) -> torch.Tensor:
    """The reference's C-head grids: dft 2 pi k/M, len 2 pi k/max_len, rope (sca2/ref.py:56-124)."""
    k = torch.arange(M, dtype=torch.float32)
    if name == "dft":
        return 2 * math.pi * k / M
    if name == "len":
        return 2 * math.pi * k / max_len
    if name == "rope":
        return rope_grid(M, base, slow_frac, max_len)
    raise ValueError(f"unknown freq grid {name!r}")


def _wd(p: torch.Tensor) -> torch.dtype:
    return torch.float64 if p.dtype == torch.float64 else torch.float32


def _rms(u: torch.Tensor, eps: float = 1e-6) -> torch.Tensor:
    """RMS read-out on the GPU kernel (sca2/ref.py:29-30)."""
    if u.dtype == torch.float64:
        raise TypeError("the sm_100a scan runs in float32 / bfloat16; float64 modules are a "
                        "reference-only configuration")
    return ops.rms(u, eps)


def _gated_out(head, u, z):
    """RMS read-out, or the raw read times rscale, optionally gated (sca2/ref.py:33-50)."""
    u = _rms(u) if getattr(head, "rms_read", True) else u * head.rscale
    return u * F.silu(head.rgate(z)) if getattr(head, "gated_read", False) else u


def _read_heads(head, o, z):
    """Read-out of a scan read o (..., H, 2, dvh) as u (..., 2 H dvh) = [re of every head | im
    of every head] through _gated_out (sca2/arch_gatedc.py:155-156, 168).  With the RMS read
    the head gathering and the RMS are one row kernel (ops.rms_heads), fp32 out."""
    if getattr(head, "rms_read", True) and o.shape[-1] % 4 == 0:
        u = ops.rms_heads(o)
        return u * F.silu(head.rgate(z)) if getattr(head, "gated_read", False) else u
    lead = o.shape[:-3]
    u = torch.cat([o[..., 0, :].reshape(*lead, -1), o[..., 1, :].reshape(*lead, -1)], -1)
    return _gated_out(head, u.float(), z)


def _value_dtype(z: torch.Tensor) -> torch.dtype:
    """Dtype handed to the kernel for v / o: the autocast dtype on CUDA (the reference's
    gemm_dtype policy, lapa/layer.py:225-230), else float32."""
    if torch.is_autocast_enabled() and z.is_cuda:
        dt = torch.get_autocast_dtype("cuda")
        return dt if dt in (torch.bfloat16, torch.float32) else torch.float32
    return torch.bfloat16 if z.dtype == torch.bfloat16 else torch.float32


def _gate_proj(lins, x: torch.Tensor):
    """[lin(x) for lin in lins] as one product with fp32 outputs whatever the autocast state.
    The decay and gate projections feed exponentials whose products run over the whole
    sequence, so a bf16 rounding of their outputs would compound along it.  Under autocast on
    CUDA the product is ops.linear16 (bf16 hi + lo operands, fp32 accumulation and output:
    about 16 significant bits, 2^7 finer than a bf16 output); otherwise one fp32 product."""
    w = torch.cat([lin.weight for lin in lins], 0) if len(lins) > 1 else lins[0].weight
    sizes = [lin.out_features for lin in lins]
    if torch.is_autocast_enabled() and x.is_cuda:
        outs = ops.linear16(x, w, sizes)
        outs = [o.view(*x.shape[:-1], o.shape[-1]) for o in outs]
    else:
        with torch.autocast(device_type=x.device.type, enabled=False):
            outs = F.linear(x.float(), w.float()).split(sizes, -1)
    return [o if lin.bias is None else o + lin.bias.float() for o, lin in zip(outs, lins)]


def _positions(T: int, pos: torch.Tensor, device) -> torch.Tensor:
    return (torch.arange(T, device=device, dtype=torch.float32) + pos.float())[:, None]


# ----------------------------------------------------------------------------------------
#  LapA long head
# ----------------------------------------------------------------------------------------
class LongHead(nn.Module):
    """lapa.layer.LongHead on the sm_100a scan: rope grid, damped accumulator with a
    learned per-mode decay, delta-rule write (lapa/layer.py:170-412)."""

    def __init__(self, cfg: LaplaceConfig):
        super().__init__()
        d, M, dv = cfg.d, cfg.M, cfg.dv
        self.d, self.M, self.dv, self.cfg = d, M, dv, cfg
        self.K = nn.Linear(d, M, False)
        self.V = nn.Linear(d, dv, False)
        self.theta = nn.Parameter(torch.zeros(M) if cfg.theta_scale == 0.0
                                  else cfg.theta_scale * torch.randn(M))
        self.wr = nn.Parameter(torch.ones(M))
        self.wi = nn.Parameter(torch.zeros(M))
        self.register_buffer("omega", rope_grid(M, cfg.rope_base, cfg.slow_frac, cfg.max_len))
        self.bproj = nn.Linear(d, 1, True)
        nn.init.zeros_(self.bproj.weight)
        nn.init.constant_(self.bproj.bias, cfg.beta_init)
        self.lam_max = cfg.lam_max if cfg.lam_max is not None else 1.0 / cfg.L
        lo, hi = cfg.mem_range if cfg.mem_range is not None else (float(cfg.L), 32.0 * cfg.L)
        mem = torch.exp(torch.empty(M).uniform_(math.log(lo), math.log(hi)))
        n_pin = int(round(cfg.persist * M))
        low = self.omega.abs().argsort()[:n_pin]
        if cfg.learn_persist:
            a = torch.logit((1.0 / mem / self.lam_max).clamp(1e-4, 1 - 1e-4))
            a[low] = -8.0
            self.lam_raw = nn.Parameter(a)
            self.register_buffer("lam_mask", torch.ones(M))
        else:
            self.lam_raw = nn.Parameter(torch.log(torch.expm1(1.0 / mem)))
            mask = torch.ones(M)
            if n_pin:
                mask[low] = 0.0
            self.register_buffer("lam_mask", mask)

    @property
    def wd(self) -> torch.dtype:
        return _wd(self.wr)

    def lam(self) -> torch.Tensor:
        if self.cfg.learn_persist:
            return self.lam_max * torch.sigmoid(self.lam_raw.float())
        return F.softplus(self.lam_raw.float()).clamp(max=self.lam_max) * self.lam_mask.float()

    def _phase(self, x: torch.Tensor, p: torch.Tensor) -> torch.Tensor:
        return self.K(x).float() * self.theta.float() + p * self.omega.float()

    def init_state(self, B: int, device) -> State:
        z = lambda: torch.zeros(B, self.M, self.dv, device=device, dtype=torch.float32)
        return {"sr": z(), "si": z(), "pos": torch.zeros((), device=device, dtype=torch.float32)}

    def forward(self, z, h):
        return self.prefill(z, h)[0]

    def prefill(self, z, h, state: Optional[State] = None):
        B, T, _ = z.shape
        st = state if state is not None else self.init_state(B, z.device)
        v = self.V(z).to(_value_dtype(z))[:, :, None]
        beta = torch.sigmoid(self.bproj(z).float())
        S0 = torch.cat([st["sr"], st["si"]], 1)[:, None].float()
        # phases K(x) theta + p omega formed inside the scan kernels where they cover the call
        o, S = ops.phase_scan_proj(self.K(h)[:, :, None], self.K(z)[:, :, None], self.theta[None], self.omega[None],
                                   st["pos"], v, beta, None, self.lam()[None], self.wr.float()[None],
                                   self.wi.float()[None], S0)
        u = (ops.rms_heads(o) if self.dv % 4 == 0 else _rms(o.reshape(B, T, 2 * self.dv))).view(B, T, -1)
        M = self.M
        return u.to(z.dtype), {"sr": S[:, 0, :M], "si": S[:, 0, M:], "pos": st["pos"] + T}

    def step(self, z_t, h_t, state: State):
        M = self.M
        p = state["pos"].float()
        phw = self._phase(h_t, p)[:, None]
        phq = self._phase(z_t, p)[:, None]
        v = self.V(z_t).float()[:, None]
        beta = torch.sigmoid(self.bproj(z_t).float())
        S = torch.cat([state["sr"], state["si"]], 1)[:, None].float().contiguous()
        o, S = ops.phase_step(phw, phq, v, beta, None, self.lam()[None], self.wr.float()[None],
                              self.wi.float()[None], S, S_out=S)
        u = _rms(o.reshape(-1, 2 * self.dv)).to(z_t.dtype)
        return u, {"sr": S[:, 0, :M], "si": S[:, 0, M:], "pos": state["pos"] + 1}


# ----------------------------------------------------------------------------------------
#  sca2 C heads
# ----------------------------------------------------------------------------------------
class CHeadBase(nn.Module):
    """Parameter container of the reference's C heads (sca2/ref.py:130-163)."""

    def __init__(self, d, M, freq="dft", theta_scale=0.0, max_len=128, dv=None,
                 gated_read=False, rope_base=10000.0, slow_frac=0.0):
        super().__init__()
        self.d, self.M, self.dv = d, M, (d // 2 if dv is None else dv)
        self.freq, self.theta_scale, self.max_len = freq, theta_scale, max_len
        self.K = nn.Linear(d, M, False)
        self.V = nn.Linear(d, self.dv, False)
        self.theta = nn.Parameter(torch.zeros(M) if theta_scale == 0.0 else theta_scale * torch.randn(M))
        self.register_buffer("omega", freq_grid(freq, M, max_len, rope_base, slow_frac))
        self.wr = nn.Parameter(torch.ones(M))
        self.wi = nn.Parameter(torch.zeros(M))
        self.gated_read = gated_read
        if gated_read:
            self.rgate = nn.Linear(d, 2 * self.dv, bias=False)

    def init_state(self, B, device, dtype=torch.float32):
        z = torch.zeros(B, self.M, self.dv, device=device, dtype=torch.float32)
        return {"sr": z, "si": z.clone(), "pos": torch.zeros((), device=device, dtype=torch.float32),
                "empty": True}

    def forward(self, z, h):
        return self.prefill(z, h)[0]


class _PhaseHead(CHeadBase):
    """Single-head phase-coded C head on ops.phase_scan / ops.phase_step; subclasses choose
    the write gate (_beta), the decay (_lam), the value (_value) and the read-out (_out)."""

    def _beta(self, z):
        return None

    def _pw(self, h, p):
        return self.K(h).float() * self.theta.float() + p * self.omega.float()

    def _pq(self, z, p):
        return self.K(z).float() * self.theta.float() + p * self.omega.float()

    def _value(self, z, h):
        return self.V(z)

    def _out(self, u, z):
        return _gated_out(self, u, z)

    def _lam(self):
        return None

    def prefill(self, z, h, state=None):
        B, T, _ = z.shape
        st = state if state is not None else self.init_state(B, z.device)
        lam = self._lam()
        S0 = None if st.get("empty", False) else torch.cat([st["sr"], st["si"]], 1)[:, None].float()
        v = self._value(z, h).to(_value_dtype(z))[:, :, None]
        if type(self)._pw is _PhaseHead._pw and type(self)._pq is _PhaseHead._pq:
            # phases K(x) theta + p omega formed inside the scan kernels where they cover the call
            o, S = ops.phase_scan_proj(self.K(h)[:, :, None], self.K(z)[:, :, None], self.theta[None],
                                       self.omega[None], st["pos"], v, self._beta(z), None,
                                       None if lam is None else lam[None], self.wr.float()[None],
                                       self.wi.float()[None], S0)
        else:
            p = _positions(T, st["pos"], z.device)
            o, S = ops.phase_scan(self._pw(h, p)[:, :, None], self._pq(z, p)[:, :, None], v, self._beta(z), None,
                                  None if lam is None else lam[None], self.wr.float()[None],
                                  self.wi.float()[None], S0)
        M = self.M
        u = self._out(o.reshape(B, T, 2 * self.dv).float(), z).to(z.dtype)
        return u, {"sr": S[:, 0, :M], "si": S[:, 0, M:], "pos": st["pos"] + T, "empty": False}

    def step(self, z_t, h_t, state):
        M = self.M
        p = state["pos"].float()
        lam = self._lam()
        S = torch.cat([state["sr"], state["si"]], 1)[:, None].float().contiguous()
        o, S = ops.phase_step(self._pw(h_t, p)[:, None], self._pq(z_t, p)[:, None],
                              self._value(z_t, h_t).float()[:, None], self._beta(z_t),
                              None, None if lam is None else lam[None], self.wr.float()[None],
                              self.wi.float()[None], S, S_out=S)
        u = self._out(o.reshape(-1, 2 * self.dv), z_t).to(z_t.dtype)
        return u, {"sr": S[:, 0, :M], "si": S[:, 0, M:], "pos": state["pos"] + 1, "empty": False}


class CHeadRef(_PhaseHead):
    """Additive complex write read with wr + i wi, sca2/ref.py:164-206 (the default C head
    of SCA2Layer): the scan with no erase gate and no decay; u = rms(o)."""

    def _out(self, u, z):
        return _rms(u)


class CHeadDelta(_PhaseHead):
    """Error-correcting (delta) complex write, sca2/arch_cdelta.py:92-206."""
    CTX = int(os.environ.get("SCA2_CTX_CHUNK", 256))

    def __init__(self, *a, cdelta_init=-2.0, **kw):
        super().__init__(*a, **kw)
        self.bproj = nn.Linear(self.d, 1, True)
        nn.init.zeros_(self.bproj.weight)
        nn.init.constant_(self.bproj.bias, cdelta_init)

    def _beta(self, z):
        return torch.sigmoid(self.bproj(z).float())


class CHeadDeltaDamp(CHeadDelta):
    """cdelta with a learned per-mode decay on the accumulator, sca2/arch_damp.py:43-69."""
    LAM_MAX = 0.125
    PERSIST = 0.0

    def __init__(self, *a, mem_range=(64.0, 4096.0), **kw):
        super().__init__(*a, **kw)
        lo, hi = mem_range
        mem = torch.exp(torch.empty(self.M).uniform_(math.log(lo), math.log(hi)))
        self.lam_raw = nn.Parameter(torch.log(torch.expm1(1.0 / mem)))
        n_pin = int(round(self.PERSIST * self.M))
        mask = torch.ones(self.M)
        if n_pin:
            mask[self.omega.abs().argsort()[:n_pin]] = 0.0
        self.register_buffer("lam_mask", mask)

    def lam(self):
        return F.softplus(self.lam_raw.float()).clamp(max=self.LAM_MAX) * self.lam_mask.float()

    def _lam(self):
        return self.lam()


class CHeadDeltaDampHalf(CHeadDeltaDamp):
    PERSIST = 0.5


class CHeadDeltaDampHalfFast(CHeadDeltaDampHalf):
    LAM_MAX = min(2.0, 60.0 / CHeadDelta.CTX)


class CHeadGated(CHeadBase):
    """Multi-head C head with a data-dependent scalar decay per head, optional separate
    read key (sepq) and gated read-out (sca2/arch_gatedc.py:58-193)."""
    CTX = int(os.environ.get("SCA2_CTX_CHUNK", 256))

    def __init__(self, d, M, freq="dft", theta_scale=0.0, max_len=128, dv=None,
                 gated_read=False, heads=1, decay=False, sepq=False, decay_init="gdn",
                 rope_base=10000.0, slow_frac=0.0):
        super().__init__(d, M, freq, theta_scale, max_len, dv, gated_read, rope_base, slow_frac)
        assert M % heads == 0 and self.dv % heads == 0
        self.H, self.Mh, self.dvh = heads, M // heads, self.dv // heads
        self.decay, self.sepq = decay, sepq
        if sepq:
            self.Kq = nn.Linear(d, M, False)
            with torch.no_grad():
                self.Kq.weight.copy_(self.K.weight)
        if decay:
            self.a = nn.Linear(d, heads, False)
            if decay_init == "soft":
                A = torch.ones(heads)
                dt = torch.full((heads,), 0.01)
            else:
                A = torch.empty(heads).uniform_(1, 16)
                dt = torch.exp(torch.rand(heads) * (math.log(0.1) - math.log(0.001))
                               + math.log(0.001)).clamp(min=1e-4)
            self.A_log = nn.Parameter(torch.log(A))
            self.dt_bias = nn.Parameter(dt + torch.log(-torch.expm1(-dt)))

    def init_state(self, B, device, dtype=torch.float32):
        z = torch.zeros(B, self.H, self.Mh, self.dvh, device=device, dtype=torch.float32)
        return {"sr": z, "si": z.clone(), "pos": torch.zeros((), device=device, dtype=torch.float32),
                "empty": True}

    def _phases(self, z, h, p):
        kq = self.Kq(z) if self.sepq else self.K(z)
        th, om = self.theta.float(), self.omega.float()
        return self.K(h).float() * th + p * om, kq.float() * th + p * om

    def _logdecay(self, z):
        return -torch.exp(self.A_log.float()) * F.softplus(_gate_proj((self.a,), z)[0] + self.dt_bias.float())

    def prefill(self, z, h, state=None):
        B, T, _ = z.shape
        H, Mh, dvh = self.H, self.Mh, self.dvh
        st = state if state is not None else self.init_state(B, z.device)
        g = self._logdecay(z) if self.decay else None
        S0 = None if st.get("empty", False) else torch.cat([st["sr"], st["si"]], 2).float()
        kq = self.Kq(z) if self.sepq else self.K(z)
        # phases K(x) theta + p omega formed inside the scan kernels where they cover the call
        o, S = ops.phase_scan_proj(self.K(h).view(B, T, H, Mh), kq.view(B, T, H, Mh), self.theta.view(H, Mh),
                                   self.omega.view(H, Mh), st["pos"],
                                   self.V(z).to(_value_dtype(z)).view(B, T, H, dvh), None, g, None,
                                   self.wr.float().view(H, Mh), self.wi.float().view(H, Mh), S0)
        u = _read_heads(self, o, z).to(z.dtype)
        return u, {"sr": S[:, :, :Mh], "si": S[:, :, Mh:], "pos": st["pos"] + T, "empty": False}

    def step(self, z_t, h_t, state):
        B = z_t.size(0)
        H, Mh, dvh = self.H, self.Mh, self.dvh
        p = state["pos"].float()
        pw, pq = self._phases(z_t, h_t, p)
        g = self._logdecay(z_t) if self.decay else None
        S = torch.cat([state["sr"], state["si"]], 2).float().contiguous()
        o, S = ops.phase_step(pw.view(B, H, Mh), pq.view(B, H, Mh), self.V(z_t).float().view(B, H, dvh),
                              None, g, None, self.wr.float().view(H, Mh), self.wi.float().view(H, Mh),
                              S, S_out=S)
        u = _read_heads(self, o, z_t).to(z_t.dtype)
        return u, {"sr": S[:, :, :Mh], "si": S[:, :, Mh:], "pos": state["pos"] + 1, "empty": False}


# ----------------------------------------------------------------------------------------
#  D heads: complex diagonal scan with a read contracted over M rows (ops.dscan)
# ----------------------------------------------------------------------------------------
class DHeadRef(nn.Module):
    """sca2/ref.py:209-275: s_t = a_t s_{t-1} + v_t per (m, j) with the cartesian gate
    a = tanh(gr(h)) / sqrt 2 + i tanh(gi(h)) / sqrt 2 shared by groups of dv / G channels,
    read with the normalised query q(z) and contracted over m; u = rms([A | Bv])."""

    def __init__(self, d, M=16, G=8, dv=None, max_len=None, delta_rule=False, gated_read=False):
        super().__init__()
        self.d, self.M, self.G, self.dv = d, M, G, (d // 2 if dv is None else dv)
        self.gated_read = gated_read
        if gated_read:
            self.rgate = nn.Linear(d, 2 * self.dv, bias=False)
        self.max_len = max_len
        self.delta_rule = delta_rule
        assert self.dv % G == 0
        self.gs = self.dv // G
        self.V = nn.Linear(d, self.dv, False)
        self.gr = nn.Linear(d, M * G)
        self.gi = nn.Linear(d, M * G)
        self.qr = nn.Linear(d, M * self.dv, False)
        self.qi = nn.Linear(d, M * self.dv, False)

    def init_state(self, B, device, dtype=torch.float32):
        return {"sr": torch.zeros(B, self.M, self.dv, device=device, dtype=torch.float32),
                "si": torch.zeros(B, self.M, self.dv, device=device, dtype=torch.float32)}

    def _gate(self, h, B, T):
        s2 = 1.0 / math.sqrt(2.0)
        sr, si = _gate_proj((self.gr, self.gi), h)
        return (torch.tanh(sr).view(B, T, self.M, self.G) * s2, torch.tanh(si).view(B, T, self.M, self.G) * s2)

    def _scan(self, z, h, state):
        B, T, _ = z.shape
        st = state if state is not None else self.init_state(B, z.device)
        a_re, a_im = self._gate(h, B, T)
        qr = self.qr(z).view(B, T, self.M, self.dv)
        qi = self.qi(z).view(B, T, self.M, self.dv)
        qn = torch.sqrt(qr.square() + qi.square() + 1e-6)
        ab, (sr, si) = ops.dscan(a_re, a_im, self.V(z), qr / qn, qi / qn, (st["sr"], st["si"]))
        return ab.reshape(B, T, 2 * self.dv), {"sr": sr, "si": si}

    def prefill(self, z, h, state=None):
        u, st = self._scan(z, h, state)
        return _rms(u).to(z.dtype), st

    def forward(self, z, h):
        return self.prefill(z, h)[0]

    def step(self, z_t, h_t, state):
        u, st = self.prefill(z_t[:, None], h_t[:, None], state)
        return u[:, 0], st


class DHeadSepQ(nn.Module):
    """sca2/arch_sepq.py:46-178 (plain write): the same diagonal scan with a separable
    query, alpha (B,T,M) contracted over m inside the scan and beta (B,T,dv) applied to
    [A | Bv] afterwards, then the (optionally gated) RMS read-out."""

    def __init__(self, d, M=16, G=8, dv=None, max_len=None, delta_rule=False, gated_read=False):
        super().__init__()
        self.d, self.M, self.G, self.dv = d, M, G, (d // 2 if dv is None else dv)
        self.max_len = max_len
        self.gated_read = gated_read
        if gated_read:
            self.rgate = nn.Linear(d, 2 * self.dv, bias=False)
        self.delta_rule = "exact" if delta_rule is True else delta_rule
        if self.delta_rule:
            raise NotImplementedError("the delta-rule D head is not on the B200 scan path")
        assert self.dv % G == 0
        self.gs = self.dv // G
        self.V = nn.Linear(d, self.dv, False)
        self.gr = nn.Linear(d, M * G)
        self.gi = nn.Linear(d, M * G)
        self.qa_r = nn.Linear(d, M, False)
        self.qa_i = nn.Linear(d, M, False)
        self.qb_r = nn.Linear(d, self.dv, False)
        self.qb_i = nn.Linear(d, self.dv, False)

    init_state = DHeadRef.init_state

    def _gate(self, h, B, T):
        s2 = 1.0 / math.sqrt(2.0)
        sr, si = _gate_proj((self.gr, self.gi), h)
        return (torch.tanh(sr).view(B, T, self.M, self.G) * s2, torch.tanh(si).view(B, T, self.M, self.G) * s2)

    def _queries(self, z):
        """The four query projections [qa_r | qa_i] (B,T,2M) and [qb_r | qb_i] (B,T,2dv) as
        one product.  The separable query is normalised per (token, mode) and per (token,
        channel), and the gradient of q / |q| scales with 1 / |q|: under autocast the product
        keeps about 16 bits (ops.linear16: bf16 hi + lo operands, fp32 output), so a small q
        keeps its relative precision; otherwise it is one fp32 product."""
        B, T, _ = z.shape
        w = torch.cat([self.qa_r.weight, self.qa_i.weight, self.qb_r.weight, self.qb_i.weight], 0)
        if torch.is_autocast_enabled() and z.is_cuda:
            qa, qb = ops.linear16(z, w, (2 * self.M, 2 * self.dv))
            return qa.view(B, T, 2 * self.M), qb.view(B, T, 2 * self.dv)
        with torch.autocast(device_type=z.device.type, enabled=False):
            y = F.linear(z.float(), w.float())
        return y[..., :2 * self.M], y[..., 2 * self.M:]

    def prefill(self, z, h, state=None):
        B, T, _ = z.shape
        M = self.M
        st = state if state is not None else self.init_state(B, z.device)
        a_re, a_im = self._gate(h, B, T)
        qa, qb = self._queries(z)
        ar, ai = qa[..., :M], qa[..., M:]
        an = torch.rsqrt(ar.square() + ai.square() + 1e-6)
        ab, (sr, si) = ops.dscan(a_re, a_im, self.V(z), ar * an, ai * an, (st["sr"], st["si"]), sep=True)
        if getattr(self, "rms_read", True):  # channel-query normalisation, combine and RMS fused
            u = ops.sepq_read(ab, qb)
            if self.gated_read:
                u = u * F.silu(self.rgate(z))
        else:
            br, bi = qb[..., :self.dv], qb[..., self.dv:]
            bn = torch.rsqrt(br.square() + bi.square() + 1e-6)
            A, Bv = ab[:, :, 0], ab[:, :, 1]
            br, bi = br * bn, bi * bn
            u = _gated_out(self, torch.cat([br * A + bi * Bv, br * Bv - bi * A], -1), z)
        return u.to(z.dtype), {"sr": sr, "si": si}

    def forward(self, z, h):
        return self.prefill(z, h)[0]

    def step(self, z_t, h_t, state):
        u, st = self.prefill(z_t[:, None], h_t[:, None], state)
        return u[:, 0], st


class DHeadSepQPolar(DHeadSepQ):
    """sca2/arch_sepq.py:181-290: the gate emitted in log-polar form,
    a = exp(-softplus(gr(h))) e^{i gi(h)}."""

    def _gate(self, h, B, T):
        sr, si = _gate_proj((self.gr, self.gi), h)
        mag = torch.exp(-F.softplus(sr)).view(B, T, self.M, self.G)
        ph = si.view(B, T, self.M, self.G)
        return mag * torch.cos(ph), mag * torch.sin(ph)


# ----------------------------------------------------------------------------------------
#  short heads: exact L-tap window read over a ring buffer (ops.short_read)
# ----------------------------------------------------------------------------------------
class ShortHead(nn.Module):
    """lapa/layer.py:418-545: the DFT-grid short head.  Phases phi = K(h) theta + (p mod L)
    omega (write) and psi = K(z) theta + (p mod L) omega (read); the read is the exact window
    sum over the last L writes, the state the ring buffer of the L-1 previous writes.  Runs in
    float32 with autocast off (lapa/layer.py:55-56: the Dirichlet comb cancels only in fp32)."""

    def __init__(self, cfg: LaplaceConfig):
        super().__init__()
        d, L, dv = cfg.d, cfg.L, cfg.dv
        self.d, self.L, self.dv = d, L, dv
        self.K = nn.Linear(d, L, False)
        self.V = nn.Linear(d, dv, False)
        self.theta = nn.Parameter((cfg.theta_scale or 0.02) * torch.randn(L))
        self.wr = nn.Parameter(torch.ones(L))
        self.wi = nn.Parameter(torch.zeros(L))
        self.register_buffer("omega", (torch.arange(L, dtype=torch.float64) * (2 * math.pi / L)).float())

    def init_state(self, B: int, device, dtype=torch.float32) -> State:
        n, L = self.L - 1, self.L
        return {"c": torch.ones(B, n, L, device=device, dtype=torch.float32),
                "s": torch.zeros(B, n, L, device=device, dtype=torch.float32),
                "e": torch.zeros(B, n, self.dv, device=device, dtype=torch.float32),
                "pos": torch.zeros((), device=device, dtype=torch.long)}

    def _read(self, z, h, state):
        B, T, _ = z.shape
        st = state if state is not None else self.init_state(B, z.device)
        with torch.autocast(device_type="cuda", enabled=False):
            zf, hf = z.float(), h.float()
            o, (c, s, e) = ops.short_read(self.K(hf), self.K(zf), self.V(zf), self.theta, self.omega, self.wr,
                                          self.wi, (st["c"], st["s"], st["e"]), st["pos"])
        return o, {"c": c, "s": s, "e": e, "pos": st["pos"] + T}

    def prefill(self, z, h, state: Optional[State] = None):
        o, st = self._read(z, h, state)
        return _rms(o).to(z.dtype), st

    def forward(self, z, h):
        return self.prefill(z, h)[0]

    def step(self, z_t, h_t, state: State):
        u, st = self.prefill(z_t[:, None], h_t[:, None], state)
        return u[:, 0], st


class CHeadShort(ShortHead):
    """sca2/arch_short.py:45-158: the same window read in the SCA2 D slot, read out through
    _gated_out (RMS, or raw x rscale, optionally gated; sca2/ref.py:33-50)."""

    def __init__(self, d, L, dv, theta_scale=0.02):
        nn.Module.__init__(self)
        self.d, self.L, self.dv = d, L, dv
        self.K = nn.Linear(d, L, False)
        self.V = nn.Linear(d, dv, False)
        self.theta = nn.Parameter(theta_scale * torch.randn(L))
        self.wr = nn.Parameter(torch.ones(L))
        self.wi = nn.Parameter(torch.zeros(L))
        self.register_buffer("omega", (torch.arange(L, dtype=torch.float64) * (2 * math.pi / L))
                             .to(torch.get_default_dtype()))

    def prefill(self, z, h, state: Optional[State] = None):
        o, st = self._read(z, h, state)
        return _gated_out(self, o, z).to(z.dtype), st
