"""Differentiable scan ops over the C ABI (torch tensors in, torch tensors out).

    phase_scan(phw, phq, v, beta, g, lam, wr, wi, S0)     -> o (B,T,H,2,V), S (B,H,2Mh,V)
    key_scan(q, k, v, g, beta, scale, S0, v_times_beta)   -> o (B,T,H,V),   S (B,H,K,V)
    phase_step(...) / key_step(...)                       one decode token, state in place
    dscan(a_re, a_im, v, c_re, c_im, S0, sep)             D-head diagonal scan
    short_read(kh, kz, v, theta, omega, wr, wi, state)    short-head window read
    rms(x, eps)                                           per-row RMS read-out
    sepq_read(ab, q)                                      separable D-head read-out + RMS
    rms_heads(o)                                          multi-head read gathered + RMS
    layer_norm(x, w, b, eps)                              the layers' LayerNorm (fwd + bwd kernels)
    linear16(x, w, sizes)                                 x w^T to 16 bits on bf16 tensor cores

Every op runs the CUDA kernels of libsca2b200.so on the current stream.  There is no
CPU path: a CPU tensor or a missing library raises.  Device memory (outputs, saved
chunk states, gradients) comes from the PyTorch caching allocator; the library itself
allocates nothing.
"""
from __future__ import annotations

from typing import Optional, Tuple

import torch

from . import _lib
from ._lib import Out, ScanArgs, ScanGrads, Tok

_DT = {torch.float32: _lib.SCA2_F32, torch.bfloat16: _lib.SCA2_BF16}


def _stream():
    return torch.cuda.current_stream().cuda_stream


def _ptr(t: Optional[torch.Tensor]):
    return None if t is None else t.data_ptr()


def _need_cuda(*ts):
    dev = None
    for t in ts:
        if t is None:
            continue
        if not t.is_cuda:
            raise _lib.Sca2Error("sca2_b200 ops run on CUDA tensors only (no CPU path)")
        if dev is None:
            dev = t.device
        elif t.device != dev:
            raise _lib.Sca2Error("all tensors must be on the same CUDA device")
    return dev


def _inner(t: torch.Tensor) -> torch.Tensor:
    """Make the innermost dimension contiguous (strides of the others are passed through)."""
    return t if t.stride(-1) == 1 or t.size(-1) == 1 else t.contiguous()


def _tok(t: Optional[torch.Tensor], step: bool = False) -> Tok:
    """(B,T,H,C) or (B,T,H) tensor -> Tok; for a step, (B,H,C) or (B,H) (T stride 0)."""
    if t is None:
        return Tok(None, 0, 0, 0)
    if step:
        return Tok(t.data_ptr(), t.stride(0), 0, t.stride(1))
    return Tok(t.data_ptr(), t.stride(0), t.stride(1), t.stride(2))


def _out(t: torch.Tensor) -> Out:
    """(B,T,H,R,V) -> Out."""
    return Out(t.data_ptr(), t.stride(0), t.stride(1), t.stride(2), t.stride(3))


def _f32(t):
    return None if t is None else t.float()


# ======================================================================================
#  phase-coded scan
# ======================================================================================
def _phase_args(phw, phq, v, beta, g, lam, wr, wi, S0):
    B, T, H, Mh = phw.shape
    a = ScanArgs()
    a.flavor = _lib.FLAVOR_PHASE
    a.B, a.T, a.H, a.K, a.V = B, T, H, 2 * Mh, v.shape[-1]
    a.io_dtype = _DT[v.dtype]
    a.v_times_beta = 0
    a.q_scale = 1.0
    a.phw, a.phq, a.v = _tok(phw), _tok(phq), _tok(v)
    a.beta, a.g = _tok(beta), _tok(g)
    a.lam, a.wr, a.wi, a.S0 = _ptr(lam), _ptr(wr), _ptr(wi), _ptr(S0)
    return a


def _check_phase(phw, phq, v, beta, g, lam, wr, wi, S0):
    if phw.dim() != 4 or phq.shape != phw.shape:
        raise _lib.Sca2Error(f"phases must be (B,T,H,Mh) and equal-shaped, got {tuple(phw.shape)}"
                             f" and {tuple(phq.shape)}")
    B, T, H, Mh = phw.shape
    if v.dim() != 4 or tuple(v.shape[:3]) != (B, T, H):
        raise _lib.Sca2Error(f"v must be (B,T,H,V) with (B,T,H)={B, T, H}, got {tuple(v.shape)}")
    if v.dtype not in _DT:
        raise _lib.Sca2Error(f"v dtype {v.dtype} unsupported (float32 or bfloat16)")
    for n, t in (("beta", beta), ("g", g)):
        if t is not None and tuple(t.shape) != (B, T, H):
            raise _lib.Sca2Error(f"{n} must be (B,T,H), got {tuple(t.shape)}")
    for n, t in (("lam", lam), ("wr", wr), ("wi", wi)):
        if t is not None and tuple(t.shape) != (H, Mh):
            raise _lib.Sca2Error(f"{n} must be (H,Mh)={(H, Mh)}, got {tuple(t.shape)}")
    if S0 is not None and tuple(S0.shape) != (B, H, 2 * Mh, v.shape[-1]):
        raise _lib.Sca2Error(f"S0 must be (B,H,2Mh,V), got {tuple(S0.shape)}")


def _slots(T: int) -> int:
    """Saved-state slots of the chunk-state buffer (the library's sca2_num_chunks)."""
    return 4 * ((T + 63) // 64) if T > 0 else 0


def _fwd_infer(a, pp, o: Out, S: torch.Tensor, dev: torch.device, what: str):
    """Forward without saved chunk states (sca2_scan_fwd_work): where the tensor-core path covers
    the call, every chunk's delta-rule inverse is formed chunk-parallel into a work buffer first
    and the chunk walk reads it instead of inverting inside its sequential loop."""
    lib = _lib.load()
    n = int(lib.sca2_scan_fwd_work_bytes(C_ref(a)))
    work = torch.empty(n, device=dev, dtype=torch.uint8) if n > 0 else None
    _lib.check(lib.sca2_scan_fwd_work(C_ref(a), None if pp is None else C_ref(pp), o, _ptr(S), _ptr(work), n,
                                      _stream()), what)


@torch.library.custom_op("sca2b200::phase_scan_fwd", mutates_args=())
def _phase_scan_fwd(phw: torch.Tensor, phq: torch.Tensor, v: torch.Tensor, beta: Optional[torch.Tensor],
                    g: Optional[torch.Tensor], lam: Optional[torch.Tensor], wr: torch.Tensor, wi: torch.Tensor,
                    S0: Optional[torch.Tensor], save: bool) -> Tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """sca2_scan_fwd: o (B,T,H,2,V), S (B,H,2Mh,V) and, with save, the chunk-state buffer
    for the backward (else an empty tensor)."""
    _need_cuda(phw, phq, v, beta, g, lam, wr, wi, S0)
    phw, phq = _inner(phw.float()), _inner(phq.float())
    v = _inner(v)
    beta, g = _f32(beta), _f32(g)
    lam = None if lam is None else lam.float().contiguous()
    wr, wi = wr.float().contiguous(), wi.float().contiguous()
    S0 = None if S0 is None else S0.float().contiguous()
    a = _phase_args(phw, phq, v, beta, g, lam, wr, wi, S0)
    B, T, H, Mh = phw.shape
    V = v.shape[-1]
    o = torch.empty(B, T, H, 2, V, device=v.device, dtype=v.dtype)
    S = torch.empty(B, H, 2 * Mh, V, device=v.device, dtype=torch.float32)
    cs = (torch.empty(B, H, _slots(T), 2 * Mh, V, device=v.device, dtype=torch.float32) if save
          else torch.empty(0, device=v.device, dtype=torch.float32))
    if save:
        _lib.check(_lib.load().sca2_scan_fwd(C_ref(a), _out(o), _ptr(S), _ptr(cs), _stream()), "scan_fwd")
    else:
        _fwd_infer(a, None, _out(o), S, v.device, "scan_fwd")
    return o, S, cs


@_phase_scan_fwd.register_fake
def _(phw, phq, v, beta, g, lam, wr, wi, S0, save):
    B, T, H, Mh = phw.shape
    V = v.shape[-1]
    return (v.new_empty(B, T, H, 2, V), v.new_empty(B, H, 2 * Mh, V, dtype=torch.float32),
            v.new_empty((B, H, _slots(T), 2 * Mh, V) if save else (0,), dtype=torch.float32))


@torch.library.custom_op("sca2b200::phase_scan_bwd", mutates_args=())
def _phase_scan_bwd(phw: torch.Tensor, phq: torch.Tensor, v: torch.Tensor, beta: Optional[torch.Tensor],
                    g: Optional[torch.Tensor], lam: Optional[torch.Tensor], wr: torch.Tensor, wi: torch.Tensor,
                    S0: Optional[torch.Tensor], cs: torch.Tensor, do: torch.Tensor, dS: Optional[torch.Tensor]
                    ) -> Tuple[torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor,
                               torch.Tensor, torch.Tensor, torch.Tensor]:
    """sca2_scan_bwd: gradients of (phw, phq, v, beta, g, lam, wr, wi, S0); an input given
    as None gets an empty gradient."""
    phw, phq = _inner(phw.float()), _inner(phq.float())
    v = _inner(v)
    beta, g = _f32(beta), _f32(g)
    lam = None if lam is None else lam.float().contiguous()
    wr, wi = wr.float().contiguous(), wi.float().contiguous()
    S0 = None if S0 is None else S0.float().contiguous()
    B, T, H, Mh = phw.shape
    V = v.shape[-1]
    dev = v.device
    do = do.to(v.dtype)
    if do.stride(-1) != 1:
        do = do.contiguous()
    dS = None if dS is None else dS.float().contiguous()
    a = _phase_args(phw, phq, v, beta, g, lam, wr, wi, S0)
    z = lambda *sh: torch.empty(*sh, device=dev, dtype=torch.float32)  # written (overwrite mode)
    E = lambda: torch.empty(0, device=dev, dtype=torch.float32)  # the gradient of an absent input
    dphw, dphq = z(B, T, H, Mh), z(B, T, H, Mh)
    dv = torch.empty(B, T, H, V, device=dev, dtype=v.dtype)
    dbeta = z(B, T, H) if beta is not None else None
    dg = z(B, T, H) if g is not None else None
    dlam = z(H, Mh) if lam is not None else None
    dwr, dwi = z(H, Mh), z(H, Mh)
    dS0 = torch.empty(B, H, 2 * Mh, V, device=dev, dtype=torch.float32)
    gr = ScanGrads()
    gr.dphw, gr.dphq, gr.dv = _tok(dphw), _tok(dphq), _tok(dv)
    gr.dbeta, gr.dg = _tok(dbeta), _tok(dg)
    gr.dlam, gr.dwr, gr.dwi, gr.dS0 = _ptr(dlam), _ptr(dwr), _ptr(dwi), _ptr(dS0)
    gr.overwrite = 1
    _lib.check(_lib.load().sca2_scan_bwd(C_ref(a), _out(do), _ptr(dS), _ptr(cs), C_ref(gr), _stream()),
               "scan_bwd")
    return (dphw, dphq, dv, E() if dbeta is None else dbeta, E() if dg is None else dg,
            E() if dlam is None else dlam, dwr, dwi, dS0 if S0 is not None else E())


@_phase_scan_bwd.register_fake
def _(phw, phq, v, beta, g, lam, wr, wi, S0, cs, do, dS):
    B, T, H, Mh = phw.shape
    V = v.shape[-1]
    f = lambda *sh: v.new_empty(*sh, dtype=torch.float32)
    return (f(B, T, H, Mh), f(B, T, H, Mh), v.new_empty(B, T, H, V), f(B, T, H) if beta is not None else f(0),
            f(B, T, H) if g is not None else f(0), f(H, Mh) if lam is not None else f(0), f(H, Mh), f(H, Mh),
            f(B, H, 2 * Mh, V) if S0 is not None else f(0))


def _phase_setup(ctx, inputs, output):
    phw, phq, v, beta, g, lam, wr, wi, S0, save = inputs
    ctx.save_for_backward(phw, phq, v, beta, g, lam, wr, wi, S0, output[2])


def _phase_backward(ctx, do, dS, dcs):
    phw, phq, v, beta, g, lam, wr, wi, S0, cs = ctx.saved_tensors
    if do is None:
        do = torch.zeros(*phw.shape[:3], 2, v.shape[-1], device=v.device, dtype=v.dtype)
    grads = torch.ops.sca2b200.phase_scan_bwd(phw, phq, v, beta, g, lam, wr, wi, S0, cs, do, dS)
    ni = ctx.needs_input_grad
    ins = (phw, phq, v, beta, g, lam, wr, wi, S0)
    return tuple(gd if (ni[k] and ins[k] is not None) else None for k, gd in enumerate(grads)) + (None,)


_phase_scan_fwd.register_autograd(_phase_backward, setup_context=_phase_setup)


def _wants_grad(*ts):
    return torch.is_grad_enabled() and any(t is not None and t.requires_grad for t in ts)


def C_ref(x):
    import ctypes
    return ctypes.byref(x)


def phase_scan(phw, phq, v, beta=None, g=None, lam=None, wr=None, wi=None, S0=None
               ) -> Tuple[torch.Tensor, torch.Tensor]:
    """Phase-coded decayed-state scan (the C head / long head of the reference).

    phw, phq (B,T,H,Mh) write / read phases (fp32); v (B,T,H,V) fp32 or bf16;
    beta, g (B,T,H) erase gate and scalar log-decay (None: additive / no decay);
    lam (H,Mh) per-mode decay; wr, wi (H,Mh) spectral read weights; S0 (B,H,2Mh,V)
    incoming state [sr ; si].  Returns the raw read o (B,T,H,2,V) in v's dtype
    ([re, im] along dim 3) and the final fp32 state.  Differentiable in every input.
    """
    _check_phase(phw, phq, v, beta, g, lam, wr, wi, S0)
    if wr is None or wi is None:
        raise _lib.Sca2Error("wr and wi are required")
    _need_cuda(phw, phq, v, beta, g, lam, wr, wi, S0)
    save = _wants_grad(phw, phq, v, beta, g, lam, wr, wi, S0)
    o, S, _ = torch.ops.sca2b200.phase_scan_fwd(phw, phq, v, beta, g, lam, wr, wi, S0, save)
    return o, S


# ======================================================================================
#  phase-coded scan with the phases formed in the kernels from the projections
# ======================================================================================
def _pp(kh, theta, omega, pos):
    pp = _lib.PhaseProj()
    pp.dtype = _DT[kh.dtype]
    pp.theta, pp.omega, pp.pos = theta.data_ptr(), omega.data_ptr(), _ptr(pos)
    return pp


@torch.library.custom_op("sca2b200::phase_scan_proj_fwd", mutates_args=())
def _phase_scan_proj_fwd(kh: torch.Tensor, kz: torch.Tensor, v: torch.Tensor, beta: Optional[torch.Tensor],
                         g: Optional[torch.Tensor], lam: Optional[torch.Tensor], wr: torch.Tensor, wi: torch.Tensor,
                         S0: Optional[torch.Tensor], theta: torch.Tensor, omega: torch.Tensor,
                         pos: Optional[torch.Tensor], save: bool) -> Tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """sca2_scan_fwd_proj: as phase_scan_fwd with phi = kh theta + (pos + t) omega and psi
    = kz theta + (pos + t) omega formed inside the kernels."""
    a = _phase_args(kh, kz, v, beta, g, lam, wr, wi, S0)
    B, T, H, Mh = kh.shape
    V = v.shape[-1]
    o = torch.empty(B, T, H, 2, V, device=v.device, dtype=v.dtype)
    S = torch.empty(B, H, 2 * Mh, V, device=v.device, dtype=torch.float32)
    cs = (torch.empty(B, H, _slots(T), 2 * Mh, V, device=v.device, dtype=torch.float32) if save
          else torch.empty(0, device=v.device, dtype=torch.float32))
    pp = _pp(kh, theta, omega, pos)
    if save:
        _lib.check(_lib.load().sca2_scan_fwd_proj(C_ref(a), C_ref(pp), _out(o), _ptr(S), _ptr(cs), _stream()),
                   "scan_fwd_proj")
    else:
        _fwd_infer(a, pp, _out(o), S, v.device, "scan_fwd_proj")
    return o, S, cs


@_phase_scan_proj_fwd.register_fake
def _(kh, kz, v, beta, g, lam, wr, wi, S0, theta, omega, pos, save):
    B, T, H, Mh = kh.shape
    V = v.shape[-1]
    return (v.new_empty(B, T, H, 2, V), v.new_empty(B, H, 2 * Mh, V, dtype=torch.float32),
            v.new_empty((B, H, _slots(T), 2 * Mh, V) if save else (0,), dtype=torch.float32))


@torch.library.custom_op("sca2b200::phase_scan_proj_bwd", mutates_args=())
def _phase_scan_proj_bwd(kh: torch.Tensor, kz: torch.Tensor, v: torch.Tensor, beta: Optional[torch.Tensor],
                         g: Optional[torch.Tensor], lam: Optional[torch.Tensor], wr: torch.Tensor, wi: torch.Tensor,
                         S0: Optional[torch.Tensor], theta: torch.Tensor, omega: torch.Tensor,
                         pos: Optional[torch.Tensor], cs: torch.Tensor, do: torch.Tensor, dS: Optional[torch.Tensor]
                         ) -> Tuple[torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor,
                                    torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor]:
    """sca2_scan_bwd_proj: gradients of (kh, kz, v, beta, g, lam, wr, wi, S0, theta)."""
    B, T, H, Mh = kh.shape
    V = v.shape[-1]
    dev = v.device
    do = do.to(v.dtype)
    if do.stride(-1) != 1:
        do = do.contiguous()
    dS = None if dS is None else dS.float().contiguous()
    a = _phase_args(kh, kz, v, beta, g, lam, wr, wi, S0)
    z = lambda *sh: torch.empty(*sh, device=dev, dtype=torch.float32)  # written (overwrite mode)
    E = lambda: torch.empty(0, device=dev, dtype=torch.float32)
    dkh, dkz = torch.empty_like(kh), torch.empty_like(kz)
    dv = torch.empty(B, T, H, V, device=dev, dtype=v.dtype)
    dbeta = z(B, T, H) if beta is not None else None
    dg = z(B, T, H) if g is not None else None
    dlam = z(H, Mh) if lam is not None else None
    dwr, dwi = z(H, Mh), z(H, Mh)
    dS0 = torch.empty(B, H, 2 * Mh, V, device=dev, dtype=torch.float32)
    dth = torch.empty(H, Mh, device=dev, dtype=torch.float32)
    gr = ScanGrads()
    gr.dphw, gr.dphq, gr.dv = _tok(dkh), _tok(dkz), _tok(dv)
    gr.dbeta, gr.dg = _tok(dbeta), _tok(dg)
    gr.dlam, gr.dwr, gr.dwi, gr.dS0 = _ptr(dlam), _ptr(dwr), _ptr(dwi), _ptr(dS0)
    gr.overwrite = 1
    lib = _lib.load()
    wk = torch.empty((lib.sca2_scan_proj_work_bytes(B, T, H, Mh) + 3) // 4, device=dev, dtype=torch.float32)
    _lib.check(lib.sca2_scan_bwd_proj(C_ref(a), C_ref(_pp(kh, theta, omega, pos)), _out(do), _ptr(dS), _ptr(cs),
                                      C_ref(gr), dth.data_ptr(), wk.data_ptr(), _stream()), "scan_bwd_proj")
    return (dkh, dkz, dv, E() if dbeta is None else dbeta, E() if dg is None else dg,
            E() if dlam is None else dlam, dwr, dwi, dS0 if S0 is not None else E(), dth)


@_phase_scan_proj_bwd.register_fake
def _(kh, kz, v, beta, g, lam, wr, wi, S0, theta, omega, pos, cs, do, dS):
    B, T, H, Mh = kh.shape
    V = v.shape[-1]
    f = lambda *sh: v.new_empty(*sh, dtype=torch.float32)
    return (torch.empty_like(kh), torch.empty_like(kz), v.new_empty(B, T, H, V),
            f(B, T, H) if beta is not None else f(0), f(B, T, H) if g is not None else f(0),
            f(H, Mh) if lam is not None else f(0), f(H, Mh), f(H, Mh), f(B, H, 2 * Mh, V) if S0 is not None else f(0),
            f(H, Mh))


def _proj_setup(ctx, inputs, output):
    ctx.save_for_backward(*inputs[:12], output[2])


def _proj_backward(ctx, do, dS, dcs):
    kh, kz, v, beta, g, lam, wr, wi, S0, theta, omega, pos, cs = ctx.saved_tensors
    if do is None:
        do = torch.zeros(*kh.shape[:3], 2, v.shape[-1], device=v.device, dtype=v.dtype)
    gr = torch.ops.sca2b200.phase_scan_proj_bwd(kh, kz, v, beta, g, lam, wr, wi, S0, theta, omega, pos, cs, do, dS)
    ni = ctx.needs_input_grad
    ins = (kh, kz, v, beta, g, lam, wr, wi, S0)
    out = [gd if (ni[j] and ins[j] is not None) else None for j, gd in enumerate(gr[:9])]
    return tuple(out) + (gr[9] if ni[9] else None, None, None, None)


_phase_scan_proj_fwd.register_autograd(_proj_backward, setup_context=_proj_setup)


def _proj_ok(kh, v) -> bool:
    """Whether the projected-phase kernels cover this call (the rule of
    sca2_scan_proj_supported): tensor-core path (bf16 values, K = 2 Mh = 64, V a multiple
    of 64) and 16-byte aligned projection rows."""
    if kh.dim() != 4 or kh.shape[-1] != 32 or v.dtype != torch.bfloat16 or v.shape[-1] % 64 or kh.shape[1] == 0:
        return False
    if kh.dtype not in _DT or kh.stride(-1) != 1:
        return False
    q = 8 if kh.dtype == torch.bfloat16 else 4
    return kh.data_ptr() % 16 == 0 and all(s % q == 0 for s in kh.stride()[:3])


def phase_scan_proj(kh, kz, theta, omega, pos, v, beta=None, g=None, lam=None, wr=None, wi=None, S0=None):
    """The phase scan fed by the head's projections: kh, kz (B,T,H,Mh) = K(h), K(z) (fp32 or
    bf16), theta, omega (H,Mh), pos a 0-dim fp32 tensor (position of token 0) or None; the
    phases phi = kh theta + (pos + t) omega, psi = kz theta + (pos + t) omega are formed inside
    the kernels when the tensor-core path covers the call, and in torch otherwise (same
    expression, then ops.phase_scan).  Returns (o, S) as phase_scan; differentiable in kh, kz,
    theta and the scan's inputs."""
    if wr is None or wi is None:
        raise _lib.Sca2Error("wr and wi are required")
    _need_cuda(kh, kz, theta, omega, pos, v, beta, g, lam, wr, wi, S0)
    if _proj_ok(kh, v) and _proj_ok(kz, v) and kh.dtype == kz.dtype and kh.shape == kz.shape:
        th, om = theta.float().contiguous(), omega.float().contiguous()
        ps = None if pos is None else pos.float().reshape(())
        lam_ = None if lam is None else lam.float().contiguous()
        w1, w2 = wr.float().contiguous(), wi.float().contiguous()
        S0_ = None if S0 is None else S0.float().contiguous()
        b_, g_ = _f32(beta), _f32(g)
        _check_phase(kh, kz, v, b_, g_, lam_, w1, w2, S0_)
        save = _wants_grad(kh, kz, v, b_, g_, lam_, w1, w2, S0_, th)
        o, S, _ = torch.ops.sca2b200.phase_scan_proj_fwd(kh, kz, v, b_, g_, lam_, w1, w2, S0_, th, om, ps, save)
        return o, S
    T = kh.shape[1]
    p = torch.arange(T, device=kh.device, dtype=torch.float32)[:, None, None]
    if pos is not None:
        p = p + pos.float()
    th, om = theta.float(), omega.float()
    return phase_scan(kh.float() * th + p * om, kz.float() * th + p * om, v, beta, g, lam, wr, wi, S0)


# ======================================================================================
#  explicit-key (GDN) scan
# ======================================================================================
def _key_args(q, k, v, g, beta, lam, S0, scale, v_times_beta):
    B, T, H, K = k.shape
    a = ScanArgs()
    a.flavor = _lib.FLAVOR_KEY
    a.B, a.T, a.H, a.K, a.V = B, T, H, K, v.shape[-1]
    a.io_dtype = _DT[v.dtype]
    a.v_times_beta = 1 if v_times_beta else 0
    a.q_scale = float(scale)
    a.phw, a.phq, a.v = _tok(k), _tok(q), _tok(v)
    a.beta, a.g = _tok(beta), _tok(g)
    a.lam, a.wr, a.wi, a.S0 = _ptr(lam), None, None, _ptr(S0)
    return a


@torch.library.custom_op("sca2b200::key_scan_fwd", mutates_args=())
def _key_scan_fwd(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, g: Optional[torch.Tensor],
                  beta: Optional[torch.Tensor], lam: Optional[torch.Tensor], S0: Optional[torch.Tensor], scale: float,
                  v_times_beta: bool, save: bool) -> Tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """sca2_scan_fwd, key flavour: o (B,T,H,V), S (B,H,K,V), chunk states (or empty)."""
    _need_cuda(q, k, v, g, beta, lam, S0)
    dt = v.dtype
    q, k, v = _inner(q.to(dt)), _inner(k.to(dt)), _inner(v)
    g, beta = _f32(g), _f32(beta)
    lam = None if lam is None else lam.float().contiguous()
    S0 = None if S0 is None else S0.float().contiguous()
    a = _key_args(q, k, v, g, beta, lam, S0, scale, v_times_beta)
    B, T, H, K = k.shape
    V = v.shape[-1]
    o = torch.empty(B, T, H, V, device=v.device, dtype=dt)
    S = torch.empty(B, H, K, V, device=v.device, dtype=torch.float32)
    cs = (torch.empty(B, H, _slots(T), K, V, device=v.device, dtype=torch.float32) if save
          else torch.empty(0, device=v.device, dtype=torch.float32))
    if save:
        _lib.check(_lib.load().sca2_scan_fwd(C_ref(a), _out(o.unsqueeze(3)), _ptr(S), _ptr(cs), _stream()),
                   "scan_fwd")
    else:
        _fwd_infer(a, None, _out(o.unsqueeze(3)), S, v.device, "scan_fwd")
    return o, S, cs


@_key_scan_fwd.register_fake
def _(q, k, v, g, beta, lam, S0, scale, v_times_beta, save):
    B, T, H, K = k.shape
    V = v.shape[-1]
    return (v.new_empty(B, T, H, V), v.new_empty(B, H, K, V, dtype=torch.float32),
            v.new_empty((B, H, _slots(T), K, V) if save else (0,), dtype=torch.float32))


def _key_grads_io(v, K, lam):
    """Whether the key-flavour backward returns dq, dk in the io dtype: bf16 at K = V = 128
    without lam (the chunk-parallel path writes them so); otherwise fp32."""
    return v.dtype == torch.bfloat16 and K == 128 and v.shape[-1] == 128 and lam is None


def _rows16(x):
    """16-byte aligned rows of a (B,T,H,C) tensor with a contiguous channel axis."""
    return x.data_ptr() % 16 == 0 and all(s % 8 == 0 for s in x.stride()[:3])


@torch.library.custom_op("sca2b200::key_scan_bwd", mutates_args=("cs",))
def _key_scan_bwd(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, g: Optional[torch.Tensor],
                  beta: Optional[torch.Tensor], lam: Optional[torch.Tensor], S0: Optional[torch.Tensor], scale: float,
                  v_times_beta: bool, cs: torch.Tensor, do: torch.Tensor, dS: Optional[torch.Tensor]
                  ) -> Tuple[torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor,
                             torch.Tensor]:
    """sca2_scan_bwd, key flavour: gradients of (q, k, v, g, beta, lam, S0).

    cs is declared mutated: on the chunk-parallel path (bf16, K = V = 128, no lam) the backward
    uses the slots of the chunk-state buffer that the forward leaves free as its workspace.
    What the forward saved there is left intact, so the backward may run again on the same
    buffer (retain_graph)."""
    dt = v.dtype
    q, k, v = _inner(q.to(dt)), _inner(k.to(dt)), _inner(v)
    g, beta = _f32(g), _f32(beta)
    lam = None if lam is None else lam.float().contiguous()
    S0 = None if S0 is None else S0.float().contiguous()
    B, T, H, K = k.shape
    V = v.shape[-1]
    dev = v.device
    do = do.to(dt)
    if do.stride(-1) != 1:
        do = do.contiguous()
    do5 = do.unsqueeze(3)
    dS = None if dS is None else dS.float().contiguous()
    a = _key_args(q, k, v, g, beta, lam, S0, scale, v_times_beta)
    z = lambda *sh: torch.empty(*sh, device=dev, dtype=torch.float32)  # written (overwrite mode)
    E = lambda: torch.empty(0, device=dev, dtype=torch.float32)
    # dq, dk come back in the io dtype where the kernels write it (bf16, K = V = 128, no lam)
    gio = _key_grads_io(v, K, lam)
    direct = gio and all(_rows16(x) for x in (q, k, v))
    dk, dq = (torch.empty(B, T, H, K, device=dev, dtype=dt) for _ in range(2)) if direct else (z(B, T, H, K), z(B, T, H, K))
    dv = torch.empty(B, T, H, V, device=dev, dtype=dt)
    dbeta = z(B, T, H) if beta is not None else None
    dg = z(B, T, H) if g is not None else None
    dlam = z(H, K) if lam is not None else None
    dS0 = torch.empty(B, H, K, V, device=dev, dtype=torch.float32)
    gr = ScanGrads()
    gr.dphw, gr.dphq, gr.dv = _tok(dk), _tok(dq), _tok(dv)
    gr.dbeta, gr.dg = _tok(dbeta), _tok(dg)
    gr.dlam, gr.dwr, gr.dwi, gr.dS0 = _ptr(dlam), None, None, _ptr(dS0)
    gr.overwrite = 1
    gr.grad_io_dtype = 1 if direct else 0
    _lib.check(_lib.load().sca2_scan_bwd(C_ref(a), _out(do5), _ptr(dS), _ptr(cs), C_ref(gr), _stream()),
               "scan_bwd")
    if gio and not direct:
        dq, dk = dq.to(dt), dk.to(dt)
    return (dq, dk, dv, E() if dg is None else dg, E() if dbeta is None else dbeta, E() if dlam is None else dlam,
            dS0 if S0 is not None else E())


@_key_scan_bwd.register_fake
def _(q, k, v, g, beta, lam, S0, scale, v_times_beta, cs, do, dS):
    B, T, H, K = k.shape
    V = v.shape[-1]
    f = lambda *sh: v.new_empty(*sh, dtype=torch.float32)
    if _key_grads_io(v, K, lam):
        return (v.new_empty(B, T, H, K), v.new_empty(B, T, H, K), v.new_empty(B, T, H, V),
                f(B, T, H) if g is not None else f(0), f(B, T, H) if beta is not None else f(0), f(0),
                f(B, H, K, V) if S0 is not None else f(0))
    return (f(B, T, H, K), f(B, T, H, K), v.new_empty(B, T, H, V), f(B, T, H) if g is not None else f(0),
            f(B, T, H) if beta is not None else f(0), f(H, K) if lam is not None else f(0),
            f(B, H, K, V) if S0 is not None else f(0))


def _key_setup(ctx, inputs, output):
    q, k, v, g, beta, lam, S0, scale, vtb, save = inputs
    ctx.save_for_backward(q, k, v, g, beta, lam, S0)
    # the chunk-state buffer is kept outside save_for_backward: key_scan_bwd declares it mutated
    # (its free slots are the backward's workspace), which would otherwise make autograd refuse
    # a second backward over a retained graph although the saved slots are untouched
    ctx.cs = output[2].detach()
    ctx.scale, ctx.vtb = scale, vtb


def _key_backward(ctx, do, dS, dcs):
    q, k, v, g, beta, lam, S0 = ctx.saved_tensors
    cs = ctx.cs
    if do is None:
        do = torch.zeros(*k.shape[:3], v.shape[-1], device=v.device, dtype=v.dtype)
    grads = torch.ops.sca2b200.key_scan_bwd(q, k, v, g, beta, lam, S0, ctx.scale, ctx.vtb, cs, do, dS)
    ni = ctx.needs_input_grad
    ins = (q, k, v, g, beta, lam, S0)
    return tuple(gd if (ni[j] and ins[j] is not None) else None for j, gd in enumerate(grads)) + (None, None, None)


_key_scan_fwd.register_autograd(_key_backward, setup_context=_key_setup)


def key_scan(q, k, v, g=None, beta=None, scale=None, S0=None, lam=None, v_times_beta=True):
    """Explicit-key delta scan in fla's gated-delta-rule convention:
    S~ = exp(g) S;  e = beta (v - k^T S~)  (v_times_beta) or v - beta k^T S~;  S = S~ + k e^T;
    o = scale q^T S.  q, k (B,T,H,K), v (B,T,H,V) same dtype (fp32/bf16); g, beta (B,T,H);
    S0 (B,H,K,V).  scale defaults to K^-1/2.  Returns o (B,T,H,V), S (B,H,K,V) fp32."""
    if k.dim() != 4 or q.shape != k.shape or tuple(v.shape[:3]) != tuple(k.shape[:3]):
        raise _lib.Sca2Error("q, k must be (B,T,H,K) and v (B,T,H,V)")
    if v.dtype not in _DT:
        raise _lib.Sca2Error(f"v dtype {v.dtype} unsupported (float32 or bfloat16)")
    if v_times_beta and beta is None:
        raise _lib.Sca2Error("v_times_beta needs beta")
    K = k.shape[-1]
    scale = K ** -0.5 if scale is None else float(scale)
    _need_cuda(q, k, v, g, beta, lam, S0)
    save = _wants_grad(q, k, v, g, beta, lam, S0)
    o, S, _ = torch.ops.sca2b200.key_scan_fwd(q, k, v, g, beta, lam, S0, scale, bool(v_times_beta), save)
    return o, S


def chunk_gated_delta_rule(q, k, v, g, beta, chunk_size: int = 64, scale=None,
                           initial_state=None, output_final_state: bool = False):
    """Drop-in for fla's (naive_)chunk_gated_delta_rule as called by the reference's GDN
    baseline (lapa/benchmarks/baselines.py:111-120): same argument order and returns.
    chunk_size is accepted for signature compatibility; the kernel picks its own chunk
    (the closed form is chunk-size invariant)."""
    o, S = key_scan(q, k, v, g, beta, scale, initial_state)
    return o, (S if output_final_state else None)


# ======================================================================================
#  decode step
# ======================================================================================
def _phase_step_args(phw, phq, v, beta, g, lam, wr, wi):
    B, H, Mh = phw.shape
    a = ScanArgs()
    a.flavor = _lib.FLAVOR_PHASE
    a.B, a.T, a.H, a.K, a.V = B, 1, H, 2 * Mh, v.shape[-1]
    a.io_dtype = _DT[v.dtype]
    a.q_scale = 1.0
    a.phw, a.phq, a.v = _tok(phw, True), _tok(phq, True), _tok(v, True)
    a.beta, a.g = _tok(beta, True), _tok(g, True)
    a.lam, a.wr, a.wi, a.S0 = _ptr(lam), _ptr(wr), _ptr(wi), None
    return a


def _phase_step_run(phw, phq, v, beta, g, lam, wr, wi, S, S_out):
    B, H, Mh = phw.shape
    V = v.shape[-1]
    phw, phq, v = _inner(phw.float()), _inner(phq.float()), _inner(v)
    beta, g = _f32(beta), _f32(g)
    lam = None if lam is None else lam.float().contiguous()
    wr, wi = wr.float().contiguous(), wi.float().contiguous()
    a = _phase_step_args(phw, phq, v, beta, g, lam, wr, wi)
    o = torch.empty(B, H, 2, V, device=v.device, dtype=v.dtype)
    _lib.check(_lib.load().sca2_scan_step(C_ref(a), S.data_ptr(), S_out.data_ptr(), _out(o.unsqueeze(1)),
                                          _stream()), "scan_step")
    return o


@torch.library.custom_op("sca2b200::phase_step", mutates_args=("S_out",))
def _phase_step_out(phw: torch.Tensor, phq: torch.Tensor, v: torch.Tensor, beta: Optional[torch.Tensor],
                    g: Optional[torch.Tensor], lam: Optional[torch.Tensor], wr: torch.Tensor, wi: torch.Tensor,
                    S: torch.Tensor, S_out: torch.Tensor) -> torch.Tensor:
    """sca2_scan_step, phase flavour: reads S, writes the new state into S_out, returns o."""
    return _phase_step_run(phw, phq, v, beta, g, lam, wr, wi, S, S_out)


@torch.library.custom_op("sca2b200::phase_step_", mutates_args=("S",))
def _phase_step_inplace(phw: torch.Tensor, phq: torch.Tensor, v: torch.Tensor, beta: Optional[torch.Tensor],
                        g: Optional[torch.Tensor], lam: Optional[torch.Tensor], wr: torch.Tensor, wi: torch.Tensor,
                        S: torch.Tensor) -> torch.Tensor:
    """sca2_scan_step with the state updated in place."""
    return _phase_step_run(phw, phq, v, beta, g, lam, wr, wi, S, S)


def _phase_step_fake(phw, phq, v, beta, g, lam, wr, wi, S, S_out=None):
    B, H, Mh = phw.shape
    return v.new_empty(B, H, 2, v.shape[-1])


_phase_step_out.register_fake(_phase_step_fake)
_phase_step_inplace.register_fake(_phase_step_fake)


def phase_step(phw, phq, v, beta, g, lam, wr, wi, S, S_out=None):
    """One token for every (b, h): phw, phq (B,H,Mh) fp32, v (B,H,V), beta/g (B,H) or None,
    lam/wr/wi (H,Mh), S (B,H,2Mh,V) fp32.  Returns o (B,H,2,V) in v's dtype and the new
    state (written into S_out, default a new tensor; pass S_out=S to update in place)."""
    _need_cuda(phw, phq, v, beta, g, lam, wr, wi, S)
    B, H, Mh = phw.shape
    V = v.shape[-1]
    if S.dtype != torch.float32 or not S.is_contiguous() or tuple(S.shape) != (B, H, 2 * Mh, V):
        raise _lib.Sca2Error("state must be a contiguous fp32 (B,H,2Mh,V) tensor")
    if S_out is S:
        return torch.ops.sca2b200.phase_step_(phw, phq, v, beta, g, lam, wr, wi, S), S
    S_out = torch.empty_like(S) if S_out is None else S_out
    return torch.ops.sca2b200.phase_step(phw, phq, v, beta, g, lam, wr, wi, S, S_out), S_out


def _key_step_run(q, k, v, g, beta, S, S_out, scale, v_times_beta):
    B, H, K = k.shape
    V = v.shape[-1]
    dt = v.dtype
    q, k, v = _inner(q.to(dt)), _inner(k.to(dt)), _inner(v)
    g, beta = _f32(g), _f32(beta)
    a = ScanArgs()
    a.flavor = _lib.FLAVOR_KEY
    a.B, a.T, a.H, a.K, a.V = B, 1, H, K, V
    a.io_dtype = _DT[dt]
    a.v_times_beta = 1 if v_times_beta else 0
    a.q_scale = float(scale)
    a.phw, a.phq, a.v = _tok(k, True), _tok(q, True), _tok(v, True)
    a.beta, a.g = _tok(beta, True), _tok(g, True)
    a.lam = a.wr = a.wi = a.S0 = None
    o = torch.empty(B, H, V, device=v.device, dtype=dt)
    _lib.check(_lib.load().sca2_scan_step(C_ref(a), S.data_ptr(), S_out.data_ptr(), _out(o[:, None, :, None]),
                                          _stream()), "scan_step")
    return o


@torch.library.custom_op("sca2b200::key_step", mutates_args=("S_out",))
def _key_step_out(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, g: Optional[torch.Tensor],
                  beta: Optional[torch.Tensor], S: torch.Tensor, S_out: torch.Tensor, scale: float,
                  v_times_beta: bool) -> torch.Tensor:
    """sca2_scan_step, key flavour: reads S, writes the new state into S_out, returns o."""
    return _key_step_run(q, k, v, g, beta, S, S_out, scale, v_times_beta)


@torch.library.custom_op("sca2b200::key_step_", mutates_args=("S",))
def _key_step_inplace(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, g: Optional[torch.Tensor],
                      beta: Optional[torch.Tensor], S: torch.Tensor, scale: float, v_times_beta: bool) -> torch.Tensor:
    """sca2_scan_step, key flavour, state updated in place."""
    return _key_step_run(q, k, v, g, beta, S, S, scale, v_times_beta)


@_key_step_out.register_fake
def _(q, k, v, g, beta, S, S_out, scale, v_times_beta):
    return v.new_empty(*k.shape[:2], v.shape[-1])


@_key_step_inplace.register_fake
def _(q, k, v, g, beta, S, scale, v_times_beta):
    return v.new_empty(*k.shape[:2], v.shape[-1])


def key_step(q, k, v, g, beta, S, scale=None, S_out=None, v_times_beta=True):
    """One GDN token (fla naive_recurrent_gated_delta_rule with T = 1): q, k (B,H,K),
    v (B,H,V), g, beta (B,H), S (B,H,K,V) fp32 -> o (B,H,V), new state."""
    _need_cuda(q, k, v, g, beta, S)
    B, H, K = k.shape
    V = v.shape[-1]
    if S.dtype != torch.float32 or not S.is_contiguous() or tuple(S.shape) != (B, H, K, V):
        raise _lib.Sca2Error("state must be a contiguous fp32 (B,H,K,V) tensor")
    scale = K ** -0.5 if scale is None else float(scale)
    if S_out is S:
        return torch.ops.sca2b200.key_step_(q, k, v, g, beta, S, scale, bool(v_times_beta)), S
    S_out = torch.empty_like(S) if S_out is None else S_out
    return torch.ops.sca2b200.key_step(q, k, v, g, beta, S, S_out, scale, bool(v_times_beta)), S_out


# ======================================================================================
#  D-head diagonal scan
# ======================================================================================
def _dscan_args(a_re, a_im, v, c_re, c_im, S0, sep):
    B, T, M, G = a_re.shape
    a = _lib.DScanArgs()
    a.B, a.T, a.M, a.G, a.V, a.sep = B, T, M, G, v.shape[-1], 1 if sep else 0
    a.a_re, a.a_im, a.v, a.c_re, a.c_im = (x.data_ptr() for x in (a_re, a_im, v, c_re, c_im))
    a.S0_re = S0[0].data_ptr() if S0 is not None else None
    a.S0_im = S0[1].data_ptr() if S0 is not None else None
    return a


def _dscan_work(lib, B, T, M, G, V, device, blocks):
    if not blocks:
        return None
    n = lib.sca2_dscan_work_bytes(B, T, M, G, V)
    return torch.empty((n + 3) // 4, device=device, dtype=torch.float32) if n > 0 else None


@torch.library.custom_op("sca2b200::dscan_fwd", mutates_args=())
def _dscan_fwd(a_re: torch.Tensor, a_im: torch.Tensor, v: torch.Tensor, c_re: torch.Tensor, c_im: torch.Tensor,
               S0_re: Optional[torch.Tensor], S0_im: Optional[torch.Tensor], sep: bool, blocks: bool, save: bool
               ) -> Tuple[torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor]:
    """sca2_dscan_fwd: ab (B,T,2,V), S_re, S_im (B,M,V), checkpoints (or empty)."""
    B, T, M, G = a_re.shape
    V = v.shape[-1]
    S0 = (S0_re, S0_im) if S0_re is not None else None
    a = _dscan_args(a_re, a_im, v, c_re, c_im, S0, sep)
    ab = torch.empty(B, T, 2, V, device=v.device, dtype=torch.float32)
    S_re = torch.empty(B, M, V, device=v.device, dtype=torch.float32)
    S_im = torch.empty_like(S_re)
    lib = _lib.load()
    ck = (torch.empty(B, lib.sca2_dscan_num_ckpt(T), 2, M, V, device=v.device) if save
          else torch.empty(0, device=v.device))
    wk = _dscan_work(lib, B, T, M, G, V, v.device, blocks)
    _lib.check(lib.sca2_dscan_fwd(C_ref(a), ab.data_ptr(), S_re.data_ptr(), S_im.data_ptr(),
                                  ck.data_ptr() if save else None, _ptr(wk), _stream()), "dscan_fwd")
    return ab, S_re, S_im, ck


@_dscan_fwd.register_fake
def _(a_re, a_im, v, c_re, c_im, S0_re, S0_im, sep, blocks, save):
    B, T, M, G = a_re.shape
    V = v.shape[-1]
    f = lambda *sh: v.new_empty(*sh, dtype=torch.float32)
    return f(B, T, 2, V), f(B, M, V), f(B, M, V), (f(B, (T + 15) // 16, 2, M, V) if save else f(0))


@torch.library.custom_op("sca2b200::dscan_bwd", mutates_args=())
def _dscan_bwd(a_re: torch.Tensor, a_im: torch.Tensor, v: torch.Tensor, c_re: torch.Tensor, c_im: torch.Tensor,
               S0_re: Optional[torch.Tensor], S0_im: Optional[torch.Tensor], sep: bool, blocks: bool,
               ck: torch.Tensor, dab: torch.Tensor, dS_re: Optional[torch.Tensor], dS_im: Optional[torch.Tensor]
               ) -> Tuple[torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor,
                          torch.Tensor]:
    """sca2_dscan_bwd: gradients of (a_re, a_im, v, c_re, c_im, S0_re, S0_im)."""
    S0 = (S0_re, S0_im) if S0_re is not None else None
    a = _dscan_args(a_re, a_im, v, c_re, c_im, S0, sep)
    da_re, da_im = torch.zeros_like(a_re), torch.zeros_like(a_im)
    dv = torch.empty_like(v)
    dc_re = torch.zeros_like(c_re) if sep else torch.empty_like(c_re)
    dc_im = torch.zeros_like(c_im) if sep else torch.empty_like(c_im)
    dS0_re = torch.empty_like(S0_re) if S0 is not None else None
    dS0_im = torch.empty_like(S0_im) if S0 is not None else None
    g = _lib.DScanGrads()
    g.da_re, g.da_im, g.dv, g.dc_re, g.dc_im = (x.data_ptr() for x in (da_re, da_im, dv, dc_re, dc_im))
    g.dS0_re, g.dS0_im = _ptr(dS0_re), _ptr(dS0_im)
    dab = dab.contiguous()
    dS_re = dS_re.contiguous() if dS_re is not None else None
    dS_im = dS_im.contiguous() if dS_im is not None else None
    lib = _lib.load()
    B, T, M, G = a_re.shape
    wk = _dscan_work(lib, B, T, M, G, v.shape[-1], v.device, blocks)
    _lib.check(lib.sca2_dscan_bwd(C_ref(a), dab.data_ptr(), _ptr(dS_re), _ptr(dS_im), ck.data_ptr(),
                                  C_ref(g), _ptr(wk), _stream()), "dscan_bwd")
    E = lambda: torch.empty(0, device=v.device)
    return (da_re, da_im, dv, dc_re, dc_im, dS0_re if dS0_re is not None else E(),
            dS0_im if dS0_im is not None else E())


@_dscan_bwd.register_fake
def _(a_re, a_im, v, c_re, c_im, S0_re, S0_im, sep, blocks, ck, dab, dS_re, dS_im):
    e = lambda t: torch.empty_like(t) if t is not None else v.new_empty(0)
    return (torch.empty_like(a_re), torch.empty_like(a_im), torch.empty_like(v), torch.empty_like(c_re),
            torch.empty_like(c_im), e(S0_re), e(S0_im))


def _dscan_setup(ctx, inputs, output):
    a_re, a_im, v, c_re, c_im, S0_re, S0_im, sep, blocks, save = inputs
    ctx.save_for_backward(a_re, a_im, v, c_re, c_im, S0_re, S0_im, output[3])
    ctx.sep, ctx.blocks = sep, blocks


def _dscan_backward(ctx, dab, dS_re, dS_im, dck):
    a_re, a_im, v, c_re, c_im, S0_re, S0_im, ck = ctx.saved_tensors
    if dab is None:
        dab = torch.zeros(*a_re.shape[:2], 2, v.shape[-1], device=v.device)
    g = torch.ops.sca2b200.dscan_bwd(a_re, a_im, v, c_re, c_im, S0_re, S0_im, ctx.sep, ctx.blocks, ck, dab,
                                     dS_re, dS_im)
    ni = ctx.needs_input_grad
    ins = (a_re, a_im, v, c_re, c_im, S0_re, S0_im)
    return tuple(x if (ni[j] and ins[j] is not None) else None for j, x in enumerate(g)) + (None, None, None)


_dscan_fwd.register_autograd(_dscan_backward, setup_context=_dscan_setup)


def dscan(a_re, a_im, v, c_re, c_im, S0: Optional[Tuple[torch.Tensor, torch.Tensor]] = None, sep: bool = False,
          blocks: bool = True):
    """D-head diagonal scan (sca2/ref.py:239-275, sca2/arch_sepq.py:110-178): complex gate
    a (B,T,M,G), values v (B,T,V), read coefficients c (B,T,M,V), or (B,T,M) with sep,
    initial state (sr, si) each (B,M,V) -> ab (B,T,2,V) = [A | Bv] and the final (sr, si).
    fp32; differentiable in every input.  blocks=True runs long sequences as 16-token blocks
    in parallel (a small workspace); False keeps one sequential pass per (b, m, j)."""
    _need_cuda(a_re, a_im, v, c_re, c_im, *(S0 or ()))
    f = lambda x: x.to(torch.float32).contiguous()
    a_re, a_im, v, c_re, c_im = f(a_re), f(a_im), f(v), f(c_re), f(c_im)
    S0_re, S0_im = (f(S0[0]), f(S0[1])) if S0 is not None else (None, None)
    save = _wants_grad(a_re, a_im, v, c_re, c_im, S0_re, S0_im)
    ab, S_re, S_im, _ = torch.ops.sca2b200.dscan_fwd(a_re, a_im, v, c_re, c_im, S0_re, S0_im, bool(sep),
                                                      bool(blocks), save)
    return ab, (S_re, S_im)


# ======================================================================================
#  short head: exact L-tap window read
# ======================================================================================
def _short_args(kh, kz, v, theta, omega, wr, wi, c0, s0, e0, pos):
    B, T, L = kh.shape
    a = _lib.ShortArgs()
    a.B, a.T, a.L, a.dv = B, T, L, v.shape[-1]
    a.pos = _ptr(pos)
    a.kh, a.kz, a.v = kh.data_ptr(), kz.data_ptr(), v.data_ptr()
    a.theta, a.omega, a.wr, a.wi = theta.data_ptr(), omega.data_ptr(), wr.data_ptr(), wi.data_ptr()
    a.c0, a.s0, a.e0 = _ptr(c0), _ptr(s0), _ptr(e0)
    return a


@torch.library.custom_op("sca2b200::short_fwd", mutates_args=())
def _short_fwd(kh: torch.Tensor, kz: torch.Tensor, v: torch.Tensor, theta: torch.Tensor, omega: torch.Tensor,
               wr: torch.Tensor, wi: torch.Tensor, c0: Optional[torch.Tensor], s0: Optional[torch.Tensor],
               e0: Optional[torch.Tensor], pos: Optional[torch.Tensor]
               ) -> Tuple[torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor]:
    """sca2_short_fwd: o (B,T,2dv) and the new ring buffer (c, s, e)."""
    B, T, L = kh.shape
    dv = v.shape[-1]
    n = L - 1
    a = _short_args(kh, kz, v, theta, omega, wr, wi, c0, s0, e0, pos)
    o = torch.empty(B, T, 2 * dv, device=v.device, dtype=torch.float32)
    c1 = torch.empty(B, n, L, device=v.device, dtype=torch.float32)
    s1, e1 = torch.empty_like(c1), torch.empty(B, n, dv, device=v.device, dtype=torch.float32)
    _lib.check(_lib.load().sca2_short_fwd(C_ref(a), o.data_ptr() if T else None, _ptr(c1) if n else None,
                                          _ptr(s1) if n else None, _ptr(e1) if n else None, _stream()), "short_fwd")
    return o, c1, s1, e1


@_short_fwd.register_fake
def _(kh, kz, v, theta, omega, wr, wi, c0, s0, e0, pos):
    B, T, L = kh.shape
    dv = v.shape[-1]
    f = lambda *sh: v.new_empty(*sh, dtype=torch.float32)
    return f(B, T, 2 * dv), f(B, L - 1, L), f(B, L - 1, L), f(B, L - 1, dv)


@torch.library.custom_op("sca2b200::short_bwd", mutates_args=())
def _short_bwd(kh: torch.Tensor, kz: torch.Tensor, v: torch.Tensor, theta: torch.Tensor, omega: torch.Tensor,
               wr: torch.Tensor, wi: torch.Tensor, c0: Optional[torch.Tensor], s0: Optional[torch.Tensor],
               e0: Optional[torch.Tensor], pos: Optional[torch.Tensor], dO: torch.Tensor,
               dc1: Optional[torch.Tensor], ds1: Optional[torch.Tensor], de1: Optional[torch.Tensor]
               ) -> Tuple[torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor,
                          torch.Tensor, torch.Tensor, torch.Tensor]:
    """sca2_short_bwd: gradients of (kh, kz, v, theta, wr, wi, c0, s0, e0)."""
    B, T, L = kh.shape
    dv = v.shape[-1]
    a = _short_args(kh, kz, v, theta, omega, wr, wi, c0, s0, e0, pos)
    lib = _lib.load()
    g = _lib.ShortGrads()
    dkh, dkz, dvv = torch.empty_like(kh), torch.empty_like(kz), torch.empty_like(v)
    dth, dwr, dwi = torch.empty_like(theta), torch.empty_like(wr), torch.empty_like(wi)
    E = lambda: torch.empty(0, device=v.device)
    dc0 = torch.empty_like(c0) if c0 is not None else E()
    ds0 = torch.empty_like(s0) if s0 is not None else E()
    de0 = torch.empty_like(e0) if e0 is not None else E()
    g.dkh, g.dkz, g.dv = dkh.data_ptr(), dkz.data_ptr(), dvv.data_ptr()
    g.dtheta, g.dwr, g.dwi = dth.data_ptr(), dwr.data_ptr(), dwi.data_ptr()
    g.dc0 = dc0.data_ptr() if c0 is not None and dc0.numel() else None
    g.ds0 = ds0.data_ptr() if s0 is not None and ds0.numel() else None
    g.de0 = de0.data_ptr() if e0 is not None and de0.numel() else None
    c = lambda x: x.contiguous() if x is not None and x.numel() else None
    dO, dc1, ds1, de1 = dO.contiguous(), c(dc1), c(ds1), c(de1)
    nw = lib.sca2_short_work_bytes(B, T, L, dv)
    wk = torch.empty((nw + 3) // 4, device=v.device, dtype=torch.float32) if nw > 0 else None
    _lib.check(lib.sca2_short_bwd(C_ref(a), dO.data_ptr() if T else None, _ptr(dc1), _ptr(ds1), _ptr(de1),
                                  C_ref(g), _ptr(wk), _stream()), "short_bwd")
    return dkh, dkz, dvv, dth, dwr, dwi, dc0, ds0, de0


@_short_bwd.register_fake
def _(kh, kz, v, theta, omega, wr, wi, c0, s0, e0, pos, dO, dc1, ds1, de1):
    e = lambda t: torch.empty_like(t) if t is not None else v.new_empty(0)
    return (torch.empty_like(kh), torch.empty_like(kz), torch.empty_like(v), torch.empty_like(theta),
            torch.empty_like(wr), torch.empty_like(wi), e(c0), e(s0), e(e0))


def _short_setup(ctx, inputs, output):
    ctx.save_for_backward(*inputs)


def _short_backward(ctx, dO, dc1, ds1, de1):
    kh, kz, v, theta, omega, wr, wi, c0, s0, e0, pos = ctx.saved_tensors
    if dO is None:
        dO = torch.zeros(*kh.shape[:2], 2 * v.shape[-1], device=v.device)
    g = torch.ops.sca2b200.short_bwd(kh, kz, v, theta, omega, wr, wi, c0, s0, e0, pos, dO, dc1, ds1, de1)
    dkh, dkz, dvv, dth, dwr, dwi, dc0, ds0, de0 = g
    ni = ctx.needs_input_grad
    out = [dkh, dkz, dvv, dth, None, dwr, dwi, dc0 if c0 is not None else None, ds0 if s0 is not None else None,
           de0 if e0 is not None else None, None]
    return tuple(x if ni[j] else None for j, x in enumerate(out))


_short_fwd.register_autograd(_short_backward, setup_context=_short_setup)


def short_read(kh, kz, v, theta, omega, wr, wi, state=None, pos=None):
    """Short-head window read (lapa/layer.py:418-545, sca2/arch_short.py:45-158):
    kh, kz (B,T,L) = K(h), K(z); v (B,T,dv) = V(z); theta, omega, wr, wi (L); state =
    (c, s, e) ring buffer of the L-1 previous writes or None (init_state); pos a 0-dim
    integer tensor (position of token 0) or None.  Returns o (B,T,2dv) = [Re | Im] and the
    new buffer (c, s, e).  fp32; differentiable in kh, kz, v, theta, wr, wi and the state."""
    _need_cuda(kh, kz, v, theta, omega, wr, wi, *(state or ()))
    f = lambda x: x.to(torch.float32).contiguous() if x is not None else None
    kh, kz, v, theta, omega, wr, wi = (f(x) for x in (kh, kz, v, theta, omega, wr, wi))
    c0, s0, e0 = (f(x) for x in state) if state is not None else (None, None, None)
    if pos is not None:
        pos = pos.to(device=v.device, dtype=torch.int64).reshape(())
    o, c1, s1, e1 = torch.ops.sca2b200.short_fwd(kh, kz, v, theta, omega, wr, wi, c0, s0, e0, pos)
    return o, (c1, s1, e1)


# ======================================================================================
#  RMS read-out
# ======================================================================================
@torch.library.custom_op("sca2b200::rms_fwd", mutates_args=())
def _rms_fwd(x: torch.Tensor, eps: float) -> torch.Tensor:
    """sca2_rms_fwd on a contiguous fp32 / bf16 tensor, rows over the last dimension."""
    D = x.shape[-1]
    u = torch.empty_like(x)
    _lib.check(_lib.load().sca2_rms_fwd(x.data_ptr(), u.data_ptr(), x.numel() // D, D, float(eps), _DT[x.dtype],
                                        _stream()), "rms_fwd")
    return u


@_rms_fwd.register_fake
def _(x, eps):
    return torch.empty_like(x)


@torch.library.custom_op("sca2b200::rms_bwd", mutates_args=())
def _rms_bwd(x: torch.Tensor, du: torch.Tensor, eps: float) -> torch.Tensor:
    """sca2_rms_bwd: dx from x and du (same shape and dtype)."""
    D = x.shape[-1]
    du = du.to(x.dtype).contiguous()
    dx = torch.empty_like(x)
    _lib.check(_lib.load().sca2_rms_bwd(x.data_ptr(), du.data_ptr(), dx.data_ptr(), x.numel() // D, D, float(eps),
                                        _DT[x.dtype], _stream()), "rms_bwd")
    return dx


@_rms_bwd.register_fake
def _(x, du, eps):
    return torch.empty_like(x)


def _rms_setup(ctx, inputs, output):
    ctx.save_for_backward(inputs[0])
    ctx.eps = inputs[1]


def _rms_backward(ctx, du):
    (x,) = ctx.saved_tensors
    return torch.ops.sca2b200.rms_bwd(x, du, ctx.eps), None


_rms_fwd.register_autograd(_rms_backward, setup_context=_rms_setup)


def rms(x: torch.Tensor, eps: float = 1e-6) -> torch.Tensor:
    """u = x * rsqrt(mean(x^2, -1) + eps) (sca2/ref.py:29-30), on the GPU kernel."""
    _need_cuda(x)
    if x.dtype not in _DT:
        x = x.float()
    return torch.ops.sca2b200.rms_fwd(x.contiguous(), float(eps))


# ======================================================================================
#  separable D-head read-out (RMS fused) and the 16-bit projections
# ======================================================================================
def _rows(x: torch.Tensor, width: int) -> torch.Tensor:
    """x as a (rows, width) matrix with unit column stride (a view where the strides allow)."""
    if x.stride(-1) != 1:
        x = x.contiguous()
    try:
        return x.view(-1, width)
    except RuntimeError:
        return x.contiguous().view(-1, width)


@torch.library.custom_op("sca2b200::sepq_read_fwd", mutates_args=())
def _sepq_read_fwd(ab: torch.Tensor, q: torch.Tensor, eps_q: float, eps: float) -> torch.Tensor:
    """sca2_sepq_read_fwd: ab (..., 2, dv) and q (..., 2 dv) = [br | bi] -> (..., 2 dv) fp32."""
    dv = ab.shape[-1]
    q2 = _rows(q, 2 * dv)
    rows = q2.shape[0]
    out = torch.empty(*ab.shape[:-2], 2 * dv, device=ab.device, dtype=torch.float32)
    _lib.check(_lib.load().sca2_sepq_read_fwd(ab.data_ptr(), q2.data_ptr(), q2.data_ptr() + 4 * dv, q2.stride(0),
                                              out.data_ptr(), rows, dv, float(eps_q), float(eps), _stream()),
               "sepq_read_fwd")
    return out


@_sepq_read_fwd.register_fake
def _(ab, q, eps_q, eps):
    return ab.new_empty(*ab.shape[:-2], 2 * ab.shape[-1], dtype=torch.float32)


@torch.library.custom_op("sca2b200::sepq_read_bwd", mutates_args=())
def _sepq_read_bwd(ab: torch.Tensor, q: torch.Tensor, dout: torch.Tensor, eps_q: float,
                   eps: float) -> Tuple[torch.Tensor, torch.Tensor]:
    """sca2_sepq_read_bwd: gradients of ab (..., 2, dv) and of q (..., 2 dv)."""
    dv = ab.shape[-1]
    q2 = _rows(q, 2 * dv)
    rows = q2.shape[0]
    dout = dout.float().contiguous()
    dab = torch.empty(ab.shape, device=ab.device, dtype=torch.float32)
    dq = torch.empty(rows, 2 * dv, device=ab.device, dtype=torch.float32)
    _lib.check(_lib.load().sca2_sepq_read_bwd(ab.data_ptr(), q2.data_ptr(), q2.data_ptr() + 4 * dv, q2.stride(0),
                                              dout.data_ptr(), dab.data_ptr(), dq.data_ptr(),
                                              dq.data_ptr() + 4 * dv, 2 * dv, rows, dv, float(eps_q), float(eps),
                                              _stream()), "sepq_read_bwd")
    return dab, dq.view(q.shape)


@_sepq_read_bwd.register_fake
def _(ab, q, dout, eps_q, eps):
    return ab.new_empty(ab.shape, dtype=torch.float32), q.new_empty(q.shape, dtype=torch.float32)


def _sepq_setup(ctx, inputs, output):
    ab, q, ctx.eps_q, ctx.eps = inputs
    ctx.save_for_backward(ab, q)


def _sepq_backward(ctx, dout):
    ab, q = ctx.saved_tensors
    dab, dq = torch.ops.sca2b200.sepq_read_bwd(ab, q, dout, ctx.eps_q, ctx.eps)
    return dab, dq, None, None


_sepq_read_fwd.register_autograd(_sepq_backward, setup_context=_sepq_setup)


def sepq_read(ab: torch.Tensor, q: torch.Tensor, eps_q: float = 1e-6, eps: float = 1e-6) -> torch.Tensor:
    """Separable D-head read-out with the RMS fused (sca2/arch_sepq.py:93-104, sca2/ref.py:29-30):
    ab (..., 2, dv) = [A | Bv] from dscan(sep=True), q (..., 2 dv) = [br | bi] the raw channel
    query (unit last stride; any single row stride) ->
    rms([n (br A + bi Bv) | n (br Bv - bi A)]), n = rsqrt(br^2 + bi^2 + eps_q).  fp32."""
    _need_cuda(ab, q)
    if ab.dtype != torch.float32 or q.dtype != torch.float32:
        raise TypeError("sepq_read takes fp32 ab and q")
    return torch.ops.sca2b200.sepq_read_fwd(ab.contiguous(), q, float(eps_q), float(eps))


@torch.library.custom_op("sca2b200::layer_norm_fwd", mutates_args=())
def _layer_norm_fwd(x: torch.Tensor, w: torch.Tensor, b: torch.Tensor,
                    eps: float) -> Tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """sca2_layer_norm_fwd: x (..., d) fp32 contiguous -> y, and the rows' mean and rstd."""
    d = x.shape[-1]
    rows = x.numel() // d
    y = torch.empty_like(x)
    mean = torch.empty(rows, device=x.device, dtype=torch.float32)
    rstd = torch.empty(rows, device=x.device, dtype=torch.float32)
    _lib.check(_lib.load().sca2_layer_norm_fwd(x.data_ptr(), w.data_ptr(), b.data_ptr(), y.data_ptr(), mean.data_ptr(),
                                               rstd.data_ptr(), rows, d, float(eps), _stream()), "layer_norm_fwd")
    return y, mean, rstd


@_layer_norm_fwd.register_fake
def _(x, w, b, eps):
    rows = x.numel() // x.shape[-1]
    return torch.empty_like(x), x.new_empty(rows), x.new_empty(rows)


@torch.library.custom_op("sca2b200::layer_norm_bwd", mutates_args=())
def _layer_norm_bwd(x: torch.Tensor, w: torch.Tensor, mean: torch.Tensor, rstd: torch.Tensor,
                    dy: torch.Tensor) -> Tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """sca2_layer_norm_bwd: dx, dw, db."""
    d = x.shape[-1]
    rows = x.numel() // d
    lib = _lib.load()
    dy = dy.float().contiguous()
    dx = torch.empty_like(x)
    dw = torch.empty(d, device=x.device, dtype=torch.float32)
    db = torch.empty(d, device=x.device, dtype=torch.float32)
    work = torch.empty(max(1, lib.sca2_layer_norm_work_floats(rows, d)), device=x.device, dtype=torch.float32)
    _lib.check(lib.sca2_layer_norm_bwd(x.data_ptr(), w.data_ptr(), mean.data_ptr(), rstd.data_ptr(), dy.data_ptr(),
                                       dx.data_ptr(), dw.data_ptr(), db.data_ptr(), work.data_ptr(), rows, d,
                                       _stream()), "layer_norm_bwd")
    return dx, dw, db


@_layer_norm_bwd.register_fake
def _(x, w, mean, rstd, dy):
    return torch.empty_like(x), w.new_empty(w.shape), w.new_empty(w.shape)


def _ln_setup(ctx, inputs, output):
    x, w, _, _ = inputs
    _, mean, rstd = output
    ctx.save_for_backward(x, w, mean, rstd)


def _ln_backward(ctx, dy, _dmean, _drstd):
    x, w, mean, rstd = ctx.saved_tensors
    dx, dw, db = torch.ops.sca2b200.layer_norm_bwd(x, w, mean, rstd, dy)
    return dx, dw, db, None


_layer_norm_fwd.register_autograd(_ln_backward, setup_context=_ln_setup)


def layer_norm_supported(d: int) -> bool:
    return bool(_lib.load().sca2_layer_norm_supported(int(d)))


def layer_norm(x: torch.Tensor, w: torch.Tensor, b: torch.Tensor, eps: float = 1e-5) -> torch.Tensor:
    """torch.nn.functional.layer_norm over the last dimension on the fused row kernels (fp32;
    d = 128 ... 1024 in steps of 128, layer_norm_supported)."""
    _need_cuda(x, w, b)
    y, _, _ = torch.ops.sca2b200.layer_norm_fwd(x.float().contiguous(), w.float().contiguous(),
                                                b.float().contiguous(), float(eps))
    return y


@torch.library.custom_op("sca2b200::rms_heads_fwd", mutates_args=())
def _rms_heads_fwd(o: torch.Tensor, eps: float) -> torch.Tensor:
    """sca2_rms_heads_fwd: o (..., H, 2, dvh) contiguous fp32 / bf16 -> (..., 2 H dvh) fp32."""
    H, dvh = o.shape[-3], o.shape[-1]
    D = 2 * H * dvh
    u = torch.empty(*o.shape[:-3], D, device=o.device, dtype=torch.float32)
    _lib.check(_lib.load().sca2_rms_heads_fwd(o.data_ptr(), _DT[o.dtype], u.data_ptr(), o.numel() // D, H, dvh,
                                              float(eps), _stream()), "rms_heads_fwd")
    return u


@_rms_heads_fwd.register_fake
def _(o, eps):
    return o.new_empty(*o.shape[:-3], 2 * o.shape[-3] * o.shape[-1], dtype=torch.float32)


@torch.library.custom_op("sca2b200::rms_heads_bwd", mutates_args=())
def _rms_heads_bwd(o: torch.Tensor, du: torch.Tensor, eps: float) -> torch.Tensor:
    """sca2_rms_heads_bwd: the gradient of o (its shape and dtype) from du (..., 2 H dvh)."""
    H, dvh = o.shape[-3], o.shape[-1]
    D = 2 * H * dvh
    du = du.float().contiguous()
    do = torch.empty_like(o)
    _lib.check(_lib.load().sca2_rms_heads_bwd(o.data_ptr(), _DT[o.dtype], du.data_ptr(), do.data_ptr(), o.numel() // D,
                                              H, dvh, float(eps), _stream()), "rms_heads_bwd")
    return do


@_rms_heads_bwd.register_fake
def _(o, du, eps):
    return torch.empty_like(o)


def _rms_heads_setup(ctx, inputs, output):
    o, ctx.eps = inputs
    ctx.save_for_backward(o)


def _rms_heads_backward(ctx, du):
    (o,) = ctx.saved_tensors
    return torch.ops.sca2b200.rms_heads_bwd(o, du, ctx.eps), None


_rms_heads_fwd.register_autograd(_rms_heads_backward, setup_context=_rms_heads_setup)


def rms_heads(o: torch.Tensor, eps: float = 1e-6) -> torch.Tensor:
    """RMS read-out of a multi-head read (sca2/arch_gatedc.py:155-156 with _gated_out's RMS):
    o (..., H, 2, dvh) -> rms([re of every head | im of every head]) (..., 2 H dvh) fp32, the
    gathering fused into the row kernel.  dvh % 4 == 0."""
    _need_cuda(o)
    if o.dtype not in _DT:
        o = o.float()
    if o.shape[-2] != 2 or o.shape[-1] % 4:
        raise ValueError("rms_heads takes (..., H, 2, dvh) reads with dvh % 4 == 0")
    return torch.ops.sca2b200.rms_heads_fwd(o.contiguous(), float(eps))


def split_bf16(x: torch.Tensor, lo_blocks: Tuple[bool, ...]) -> torch.Tensor:
    """sca2_split_bf16: x (rows, cols) fp32 -> (rows, len(lo_blocks) * cols) bf16 whose column
    block b is bf16(x) (False) or bf16(x - bf16(x)) (True)."""
    _need_cuda(x)
    x2 = _rows(x.float(), x.shape[-1])
    rows, cols = x2.shape
    nb = len(lo_blocks)
    out = torch.empty(rows, nb * cols, device=x.device, dtype=torch.bfloat16)
    mask = sum(1 << b for b, lo in enumerate(lo_blocks) if lo)
    _lib.check(_lib.load().sca2_split_bf16(x2.data_ptr(), rows, cols, x2.stride(0), out.data_ptr(), nb * cols, nb, mask,
                                           _stream()), "split_bf16")
    return out


def _mm32(a: torch.Tensor, b: torch.Tensor) -> torch.Tensor:
    """a @ b for bf16 operands with fp32 output (cuBLAS, fp32 accumulation, no output rounding)."""
    return torch.mm(a, b, out_dtype=torch.float32)


class _Linear16(torch.autograd.Function):
    """y = x w^T with x and w each split into bf16 hi + lo: ONE bf16 GEMM over the stacked
    contraction [xh | xh | xl] . [wh | wl | wh]^T = xh wh + xh wl + xl wh, fp32 output.  The
    backward splits dy the same way: dx = [dyh | dyh | dyl] . [wh ; wl ; wh] (one GEMM) and
    dw = dyh^T (xh + xl) + dyl^T xh (two GEMMs), all with fp32 outputs."""

    @staticmethod
    def forward(ctx, x2, w, sizes):
        with torch.autocast(device_type="cuda", enabled=False):
            X3 = split_bf16(x2, (False, False, True))
            W3 = split_bf16(w, (False, True, False))
            y = _mm32(X3, W3.t())
        ctx.save_for_backward(X3, W3)
        ctx.sizes = sizes
        return tuple(y.split(list(sizes), 1))

    @staticmethod
    def backward(ctx, *dys):
        X3, W3 = ctx.saved_tensors
        R, d, N = X3.shape[0], X3.shape[1] // 3, W3.shape[0]
        parts = [g.float() if g is not None else torch.zeros(R, n, device=X3.device) for g, n in zip(dys, ctx.sizes)]
        with torch.autocast(device_type="cuda", enabled=False):
            Y3 = split_bf16(torch.cat(parts, 1) if len(parts) > 1 else parts[0], (False, False, True))
            dx = dw = None
            if ctx.needs_input_grad[0]:
                dx = _mm32(Y3, torch.cat([W3[:, :d], W3[:, d:2 * d], W3[:, :d]], 0))
            if ctx.needs_input_grad[1]:
                a = _mm32(Y3[:, :N].t(), X3[:, d:])
                dw = a[:, :d] + a[:, d:] + _mm32(Y3[:, 2 * N:].t(), X3[:, :d])
        return dx, dw, None


def linear16(x: torch.Tensor, w: torch.Tensor, sizes: Tuple[int, ...]) -> Tuple[torch.Tensor, ...]:
    """x (..., d) fp32 times w (N, d)^T to about 16 significant bits on bf16 tensor cores (see
    _Linear16), returned as the column groups `sizes` (summing to N), each (rows, size) fp32
    with rows = x.numel() / d.  Differentiable in x and w."""
    _need_cuda(x, w)
    if sum(sizes) != w.shape[0]:
        raise ValueError("linear16: the column groups must cover the rows of w")
    return _Linear16.apply(_rows(x.float(), x.shape[-1]), w.float(), tuple(sizes))


# ======================================================================================
#  preallocated plans (benchmarks, CUDA-graph capture)
# ======================================================================================
class PhaseScanPlan:
    """A phase-flavour scan with every output / saved / gradient buffer allocated once, so
    fwd() and bwd() are exactly one library call each and can be timed or captured in a CUDA
    graph.  overwrite=True: the gradients are written (the library initialises them); False:
    they accumulate and bwd() zero-fills them first."""

    def __init__(self, phw, phq, v, beta=None, g=None, lam=None, wr=None, wi=None, S0=None,
                 need_grad=True, overwrite=True):
        _check_phase(phw, phq, v, beta, g, lam, wr, wi, S0)
        _need_cuda(phw, phq, v, beta, g, lam, wr, wi, S0)
        self.inp = dict(phw=_inner(phw.float()), phq=_inner(phq.float()), v=_inner(v),
                        beta=_f32(beta), g=_f32(g), lam=None if lam is None else lam.float().contiguous(),
                        wr=wr.float().contiguous(), wi=wi.float().contiguous(),
                        S0=None if S0 is None else S0.float().contiguous())
        i = self.inp
        B, T, H, Mh = i["phw"].shape
        V = i["v"].shape[-1]
        dev, dt = i["v"].device, i["v"].dtype
        self.shape = (B, T, H, Mh, V)
        self.args = _phase_args(i["phw"], i["phq"], i["v"], i["beta"], i["g"], i["lam"], i["wr"], i["wi"], i["S0"])
        self.o = torch.empty(B, T, H, 2, V, device=dev, dtype=dt)
        self.S = torch.empty(B, H, 2 * Mh, V, device=dev, dtype=torch.float32)
        self.lib = _lib.load()
        self.cs = None
        if need_grad:
            NC = self.lib.sca2_num_chunks(T)
            self.cs = torch.empty(B, H, NC, 2 * Mh, V, device=dev, dtype=torch.float32)
            z = lambda *s: torch.zeros(*s, device=dev, dtype=torch.float32)
            self.grads = dict(phw=z(B, T, H, Mh), phq=z(B, T, H, Mh),
                              v=torch.empty(B, T, H, V, device=dev, dtype=dt),
                              beta=z(B, T, H) if beta is not None else None,
                              g=z(B, T, H) if g is not None else None,
                              lam=z(H, Mh) if lam is not None else None, wr=z(H, Mh), wi=z(H, Mh),
                              S0=torch.empty(B, H, 2 * Mh, V, device=dev, dtype=torch.float32))
            gr = ScanGrads()
            G = self.grads
            gr.dphw, gr.dphq, gr.dv = _tok(G["phw"]), _tok(G["phq"]), _tok(G["v"])
            gr.dbeta, gr.dg = _tok(G["beta"]), _tok(G["g"])
            gr.dlam, gr.dwr, gr.dwi, gr.dS0 = _ptr(G["lam"]), _ptr(G["wr"]), _ptr(G["wi"]), _ptr(G["S0"])
            gr.overwrite = 1 if overwrite else 0
            self.gr = gr
            # overwrite: the library initialises every gradient itself; else they accumulate
            self._acc = [] if overwrite else [t for k, t in G.items() if t is not None and k not in ("v", "S0")]

    def fwd(self):
        _lib.check(self.lib.sca2_scan_fwd(C_ref(self.args), _out(self.o), _ptr(self.S), _ptr(self.cs),
                                          _stream()), "scan_fwd")
        return self.o, self.S

    def zero_grads(self):
        for t in self._acc:
            t.zero_()

    def bwd(self, dO, dS=None, zero=True):
        if zero:
            self.zero_grads()
        _lib.check(self.lib.sca2_scan_bwd(C_ref(self.args), _out(dO), _ptr(dS), _ptr(self.cs), C_ref(self.gr),
                                          _stream()), "scan_bwd")
        return self.grads


class PhaseStepPlan:
    """Decode step with fixed buffers: step(t) advances the state in place using the inputs
    of token t from preloaded (B,T,H,...) tensors; capturable in a CUDA graph."""

    def __init__(self, phw, phq, v, beta, g, lam, wr, wi, S):
        _need_cuda(phw, phq, v, beta, g, lam, wr, wi, S)
        B, T, H, Mh = phw.shape
        V = v.shape[-1]
        if S.dtype != torch.float32 or not S.is_contiguous() or tuple(S.shape) != (B, H, 2 * Mh, V):
            raise _lib.Sca2Error("state must be a contiguous fp32 (B,H,2Mh,V) tensor")
        self.inp = dict(phw=_inner(phw.float()), phq=_inner(phq.float()), v=_inner(v),
                        beta=_f32(beta), g=_f32(g), lam=None if lam is None else lam.float().contiguous(),
                        wr=wr.float().contiguous(), wi=wi.float().contiguous())
        self.S = S
        self.o = torch.empty(B, 1, H, 2, V, device=v.device, dtype=v.dtype)
        self.lib = _lib.load()
        self.args = []
        i = self.inp
        for t in range(T):
            a = ScanArgs()
            a.flavor = _lib.FLAVOR_PHASE
            a.B, a.T, a.H, a.K, a.V = B, 1, H, 2 * Mh, V
            a.io_dtype = _DT[v.dtype]
            a.q_scale = 1.0
            sl = lambda x: None if x is None else x[:, t]
            a.phw, a.phq, a.v = _tok(sl(i["phw"]), True), _tok(sl(i["phq"]), True), _tok(sl(i["v"]), True)
            a.beta, a.g = _tok(sl(i["beta"]), True), _tok(sl(i["g"]), True)
            a.lam, a.wr, a.wi, a.S0 = _ptr(i["lam"]), _ptr(i["wr"]), _ptr(i["wi"]), None
            self.args.append(a)

    def step(self, t):
        p = self.S.data_ptr()
        _lib.check(self.lib.sca2_scan_step(C_ref(self.args[t]), p, p, _out(self.o), _stream()), "scan_step")
        return self.o


def phase_scan_fwd_bwd_noalloc(phw, phq, v, beta, g, lam, wr, wi, dO, S0=None, dS=None):
    """Forward and backward of the phase scan in ONE library call that allocates nothing on
    the device and takes no workspace (sca2_scan_fwd_bwd_noalloc): for callers that cannot
    allocate device memory.  The saved chunk data live in the library's static 16 MiB device
    array: sca2_num_chunks(T) = 4*ceil(T/64) slots of 2Mh*V fp32 per (b, h), so
    B*H*4*ceil(T/64)*2Mh*V*4 bytes must fit; calls that overlap on the GPU race on that array.  This wrapper allocates the outputs with torch only for convenience; a caller
    without an allocator passes its own buffers through the C ABI.  Returns
    (o, S, grads dict) with the same meaning as phase_scan + autograd."""
    _check_phase(phw, phq, v, beta, g, lam, wr, wi, S0)
    _need_cuda(phw, phq, v, beta, g, lam, wr, wi, S0, dO, dS)
    phw, phq, v = _inner(phw.float()), _inner(phq.float()), _inner(v)
    beta, g = _f32(beta), _f32(g)
    lam = None if lam is None else lam.float().contiguous()
    wr, wi = wr.float().contiguous(), wi.float().contiguous()
    S0 = None if S0 is None else S0.float().contiguous()
    dO = dO.to(v.dtype)
    if dO.stride(-1) != 1:
        dO = dO.contiguous()
    dS = None if dS is None else dS.float().contiguous()
    B, T, H, Mh = phw.shape
    V = v.shape[-1]
    dev = v.device
    a = _phase_args(phw, phq, v, beta, g, lam, wr, wi, S0)
    o = torch.empty(B, T, H, 2, V, device=dev, dtype=v.dtype)
    S = torch.empty(B, H, 2 * Mh, V, device=dev, dtype=torch.float32)
    z = lambda *s: torch.zeros(*s, device=dev, dtype=torch.float32)
    G = dict(phw=z(B, T, H, Mh), phq=z(B, T, H, Mh), v=torch.empty(B, T, H, V, device=dev, dtype=v.dtype),
             beta=z(B, T, H) if beta is not None else None, g=z(B, T, H) if g is not None else None,
             lam=z(H, Mh) if lam is not None else None, wr=z(H, Mh), wi=z(H, Mh),
             S0=torch.empty(B, H, 2 * Mh, V, device=dev, dtype=torch.float32))
    gr = ScanGrads()
    gr.dphw, gr.dphq, gr.dv = _tok(G["phw"]), _tok(G["phq"]), _tok(G["v"])
    gr.dbeta, gr.dg = _tok(G["beta"]), _tok(G["g"])
    gr.dlam, gr.dwr, gr.dwi, gr.dS0 = _ptr(G["lam"]), _ptr(G["wr"]), _ptr(G["wi"]), _ptr(G["S0"])
    _lib.check(_lib.load().sca2_scan_fwd_bwd_noalloc(C_ref(a), _out(o), _ptr(S), _out(dO), _ptr(dS), C_ref(gr),
                                                     _stream()), "scan_fwd_bwd_noalloc")
    return o, S, G
