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
    folds the maps of the ranks before it into its incoming state.
Then every sub-slab is scanned once more from its true incoming state, which gives the
outputs.  This is the long-sequence path of lapa/layer.py:298-366 (the same chunk scan
over a 131072-token sequence), spread over the GPUs of one box.
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


def _fold(P, S, S_in):
    """Incoming states of consecutive segments: S_in(0) = S_in, S_in(s+1) = P_s S_in(s) + S_s.
    P (n, ..., K, K), S (n, ..., K, V); returns (n, ..., K, V) and the state leaving the last."""
    out = []
    cur = S_in
    for s in range(P.shape[0]):
        out.append(cur)
        cur = torch.matmul(P[s], cur) + S[s]
    return torch.stack(out, 0), cur


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
        # 1. map of every sub-slab, then of this rank's slab
        sdt = state_dtype
        Sr, P = _slab_map(scan, rows(phw), rows(phq), rows(v), rows(beta), rows(g), lam, wr, wi, sdt)
        Sr = Sr.reshape(B, split, H, K, V).transpose(0, 1)   # (split, B, H, K, V)
        P = P.reshape(B, split, H, K, K).transpose(0, 1)     # (split, B, H, K, K)
        zeros = torch.zeros(B, H, K, V, device=v.device, dtype=sdt)
        _, slab_S = _fold(P, Sr, zeros)                      # S_r of the slab
        slab_P = torch.eye(K, device=v.device, dtype=sdt).expand(B, H, K, K)
        for s in range(split):
            slab_P = torch.matmul(P[s], slab_P)
        # 2. exchange the slab maps
        mine = torch.cat([slab_S, slab_P], -1).contiguous()  # (B, H, K, V + K)
        if world > 1:
            every = [torch.empty_like(mine) for _ in range(world)]
            dist.all_gather(every, mine, group=group)
            every = torch.stack(every, 0)
        else:
            every = mine[None]
        # 3. incoming state of this rank, then of each sub-slab
        S_first = zeros if S0 is None else S0.to(sdt)
        S_in_ranks, S_end = _fold(every[..., V:], every[..., :V], S_first)
        S_in_subs, _ = _fold(P, Sr, S_in_ranks[rank])        # (split, B, H, K, V)
        S_in_rows = S_in_subs.transpose(0, 1).reshape(B * split, H, K, V).contiguous()
        # 4. outputs from the true incoming states
        o, _ = scan(rows(phw), rows(phq), rows(v), rows(beta), rows(g), lam, wr, wi, S_in_rows)
    return o.reshape(B, T, *o.shape[2:]), S_end
