"""Sequence-parallel prefill of one long sequence (phase-coded heads).

The scan is linear in its state: for a slab of tokens, the state leaving the slab is
S_out = P S_in + S_r, where S_r is the state reached from S_in = 0 and P (K x K per (b, h))
carries an incoming state through the slab's decays and erases.  Because every value column
evolves independently under the same keys and gates, one scan gives both: the values are
extended with K zero columns and the initial state with the identity, so the state leaving
the slab is [S_r | P].

Two levels use this:
  * within a GPU, a slab is split into `split` consecutive sub-slabs that run as extra batch
    rows (a view, no copy), so a single sequence fills the SMs instead of one CTA per head;
  * across ranks (torch.distributed, NCCL), every rank holds one slab of the sequence;
    the ranks' slab maps are all-gathered (K x (V + K) fp32 per (b, h)) and each rank
    composes the maps of the ranks before it into its incoming state.
Maps are composed on the device as an inclusive prefix of affine maps in log2(n) rounds of
batched products.  Then every sub-slab is scanned once more from its true incoming state,
which gives the outputs.  (The reads are affine in the incoming state as well, and the map
scan's outputs for the identity columns are their linear part, but those outputs are rounded
to the values' bf16: a correction built from them missed the bf16 bar, so the outputs come
from the second scan.)  This is the long-sequence path of lapa/layer.py:298-366 (the same
chunk scan over a 131072-token sequence), spread over the GPUs of one box.
"""
from __future__ import annotations

from typing import Callable, Optional

import torch

from . import ops


def _slab_map(scan, phw, phq, v, beta, g, lam, wr, wi, sdt):
    """[S_r | P] of every batch row: state leaving the rows from S0 = 0, and the K x K
    transfer of an incoming state."""
    B, T, H, Mh = phw.shape
    V, K = v.shape[-1], 2 * Mh
    v_ext = torch.cat([v, v.new_zeros(B, T, H, K)], -1)
    S0 = torch.zeros(B, H, K, V + K, device=v.device, dtype=sdt)
    S0[..., V:] = torch.eye(K, device=v.device, dtype=sdt)
    _, S = scan(phw, phq, v_ext, beta, g, lam, wr, wi, S0)
    return S[..., :V], S[..., V:]


def _compose_prefix(P, S):
    """Inclusive prefix of affine maps x -> P_s x + S_s over the leading axis (segments in
    sequence order): (P~_s, S~_s) maps the state entering segment 0 to the state leaving
    segment s.  log2(n) rounds of batched products (Hillis-Steele), all on the device, no
    per-segment host loop.  P (n, ..., K, K), S (n, ..., K, V)."""
    n, o = P.shape[0], 1
    while o < n:
        P, S = (torch.cat([P[:o], torch.matmul(P[o:], P[:-o])], 0),
                torch.cat([S[:o], torch.matmul(P[o:], S[:-o]) + S[o:]], 0))
        o *= 2
    return P, S


def _entering(Pp, Sp, S_in):
    """States entering each segment, given the inclusive prefix (Pp, Sp) of the segments' maps
    and the state entering the first: S_in, then Pp[s - 1] S_in + Sp[s - 1]."""
    later = torch.matmul(Pp[:-1], S_in.unsqueeze(0)) + Sp[:-1]
    return torch.cat([S_in.unsqueeze(0), later], 0)


def _as_rows(x, split):
    """(B, T, ...) -> (B * split, T / split, ...) (a view for contiguous inputs)."""
    if x is None:
        return None
    B, T = x.shape[:2]
    return x.reshape(B * split, T // split, *x.shape[2:])


def sp_phase_prefill(phw, phq, v, beta=None, g=None, lam=None, wr=None, wi=None, S0=None,
                     split: Optional[int] = None, group=None,
                     scan: Callable = None, state_dtype=torch.float32):
    """Prefill of a sequence whose tokens are distributed over the ranks of `group` (this
    rank holds tokens [rank * T, (rank + 1) * T) of every batch row; T a multiple of
    64 * split).  Returns this rank's outputs o (B, T, H, 2, V) and the state leaving the
    whole sequence (B, H, 2Mh, V) fp32 on every rank.  group=None and no initialised
    process group: one rank.  `scan` defaults to the CUDA scan (ops.phase_scan), whose
    states are fp32 (state_dtype)."""
    import torch.distributed as dist

    scan = scan or ops.phase_scan
    distributed = dist.is_available() and dist.is_initialized()
    world = dist.get_world_size(group) if distributed else 1
    rank = dist.get_rank(group) if distributed else 0
    B, T, H, Mh = phw.shape
    V, K = v.shape[-1], 2 * Mh
    if split is None:  # enough rows to fill the GPU: B * H * split >= 128
        split = 1
        while B * H * split < 128 and T % (64 * split * 2) == 0:
            split *= 2
    if T % split:
        raise ValueError(f"slab length {T} is not a multiple of split={split}")
    rows = lambda x: _as_rows(x, split)
    with torch.no_grad():
        # 1. map of every sub-slab, then of this rank's slab (the prefix over its sub-slabs)
        sdt = state_dtype
        Sr, P = _slab_map(scan, rows(phw), rows(phq), rows(v), rows(beta), rows(g), lam, wr, wi, sdt)
        Sr = Sr.reshape(B, split, H, K, V).transpose(0, 1)   # (split, B, H, K, V)
        P = P.reshape(B, split, H, K, K).transpose(0, 1)     # (split, B, H, K, K)
        Pp, Sp = _compose_prefix(P, Sr)
        # 2. exchange the slab maps
        mine = torch.cat([Sp[-1], Pp[-1]], -1).contiguous()  # (B, H, K, V + K)
        if world > 1:
            every = [torch.empty_like(mine) for _ in range(world)]
            dist.all_gather(every, mine, group=group)
            every = torch.stack(every, 0)
        else:
            every = mine[None]
        # 3. incoming state of this rank, then of each sub-slab
        S_first = torch.zeros(B, H, K, V, device=v.device, dtype=sdt) if S0 is None else S0.to(sdt)
        Rp, Rs = _compose_prefix(every[..., V:], every[..., :V])
        S_end = torch.matmul(Rp[-1], S_first) + Rs[-1]
        S_rank = _entering(Rp, Rs, S_first)[rank]
        S_in_subs = _entering(Pp, Sp, S_rank)                # (split, B, H, K, V)
        S_in_rows = S_in_subs.transpose(0, 1).reshape(B * split, H, K, V).contiguous()
        # 4. outputs: every sub-slab scanned again from its true incoming state
        o, _ = scan(rows(phw), rows(phq), rows(v), rows(beta), rows(g), lam, wr, wi, S_in_rows)
    return o.reshape(B, T, *o.shape[2:]), S_end
