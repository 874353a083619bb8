"""Shared helpers for the parity tests."""
from __future__ import annotations

import numpy as np
import torch


def relerr(a, b) -> float:
    """Max abs deviation over max |reference| (the reference's metric, sca2/iso.py:27-36)."""
    a = np.asarray(a.detach().double().cpu() if torch.is_tensor(a) else a, np.float64)
    b = np.asarray(b.detach().double().cpu() if torch.is_tensor(b) else b, np.float64)
    return float(np.abs(a - b).max() / max(np.abs(b).max(), 1e-30))


def cosine(a, b) -> float:
    a = np.asarray(a.detach().double().cpu() if torch.is_tensor(a) else a, np.float64).ravel()
    b = np.asarray(b.detach().double().cpu() if torch.is_tensor(b) else b, np.float64).ravel()
    return float(a @ b / max(np.linalg.norm(a) * np.linalg.norm(b), 1e-300))


def rms_np(o, axis=-1, eps=1e-6):
    return o / np.sqrt((o * o).mean(axis, keepdims=True) + eps)


# Parity bars (north star): fp32 <= 1e-4 relative; bf16 inputs with fp32 state:
# max-abs <= 2e-2 on unit-RMS outputs (relative to max |ref| for gradients) and cosine >= 0.9999.
TOL_F32 = 1e-4
TOL_BF16_ABS = 2e-2
TOL_BF16_COS = 0.9999


def cuda(x, dtype=torch.float32, grad=False):
    if x is None:
        return None
    t = torch.as_tensor(np.ascontiguousarray(x)).to("cuda", dtype)
    return t.requires_grad_(grad) if grad else t


def seeded_phase_inputs(B, T, H, Mh, V, seed=0, beta=True, g=False, lam=True, S0=True,
                        pos_scale=1.0, lam_max=1.0 / 16):
    """Seeded kernel-level inputs of the phase flavour, with the shapes and value
    distributions of the benchmark workload: phi, psi = p * omega_rope + theta * N(0,1),
    beta = sigmoid(N(0,1)), lam = min(softplus(N(0,1)), lam_max), g = -softplus(N(0,1))."""
    rng = np.random.default_rng(seed)
    p = np.arange(T, dtype=np.float64)[:, None] * pos_scale
    om = np.pi * 1e4 ** (-np.arange(Mh) / max(Mh - 1, 1))
    phw = (p * om)[None, :, None, :] + rng.standard_normal((B, T, H, Mh))
    phq = (p * om)[None, :, None, :] + rng.standard_normal((B, T, H, Mh))
    v = rng.standard_normal((B, T, H, V))
    sp = lambda x: np.log1p(np.exp(x))
    out = dict(phw=phw.astype(np.float32), phq=phq.astype(np.float32), v=v,
               beta=(1 / (1 + np.exp(-rng.standard_normal((B, T, H))))) if beta else None,
               g=(-sp(rng.standard_normal((B, T, H)))) if g else None,
               lam=np.minimum(sp(rng.standard_normal((H, Mh))), lam_max) if lam else None,
               wr=1.0 + 0.3 * rng.standard_normal((H, Mh)), wi=0.3 * rng.standard_normal((H, Mh)),
               S0=0.3 * rng.standard_normal((B, H, 2 * Mh, V)) if S0 else None)
    out["dO"] = rng.standard_normal((B, T, H, 2, V))
    out["dS"] = rng.standard_normal((B, H, 2 * Mh, V)) if S0 else None
    return out
