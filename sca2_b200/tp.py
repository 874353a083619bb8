"""Head-sharded (tensor-parallel) multi-head C head, for layers whose batch is smaller than
the number of GPUs.

When B < N, sharding a layer over the batch leaves GPUs idle.  The scan of a multi-head gated
C head (sca2/arch_gatedc.py:58-193) is independent per head, so here each rank of a
torch.distributed group owns H / N of the heads: it projects z and h onto its heads' rows of
K (Kq), V and the decay logit only, runs the phase scan of those heads, and the ranks'
raw reads are all-gathered along the head axis (one collective in the forward).  Everything
after that -- the read-out (RMS over all heads), the D head, mix, FFN -- runs replicated on
every rank, on identical inputs, so:

  * the backward of the gather needs no communication: every rank holds the full gradient of
    the gathered read and takes its own heads' slice;
  * z and h feed only this rank's heads through the sharded part, so the gradient they receive
    from it is the rank's share: one all-reduce (sum) of that share in the backward;
  * the sharded parameters (K, Kq, V, a, A_log, dt_bias, theta, wr, wi) receive gradients only
    in their owner's rows: `reduce_sharded_grads` sums them over the group after the backward,
    which gives every rank the full gradient; replicated parameters already agree.

Parameters are kept whole on every rank (the state dict is the reference's, unchanged); the
decode state of the C head is this rank's heads only.  Layer-level: `shard_layer(layer,
group)` switches the C slot of a GatedLayer (or any MixerLayer whose C slot is a CHeadGated).
"""
from __future__ import annotations

from typing import Optional

import torch
import torch.distributed as dist
import torch.nn.functional as F

from . import heads, ops


class _GatherHeads(torch.autograd.Function):
    """All-gather of the ranks' head slices along dim 2 (heads); backward: own slice."""

    @staticmethod
    def forward(ctx, x, group, world: int, rank: int):
        parts = [torch.empty_like(x) for _ in range(world)]
        dist.all_gather(parts, x.contiguous(), group=group)
        ctx.sl = (rank * x.shape[2], (rank + 1) * x.shape[2])
        return torch.cat(parts, 2)

    @staticmethod
    def backward(ctx, g):
        a, b = ctx.sl
        return g[:, :, a:b].contiguous(), None, None, None


class _ShareGrad(torch.autograd.Function):
    """Identity; backward: sum of the ranks' gradient shares."""

    @staticmethod
    def forward(ctx, x, group):
        ctx.group = group
        return x.view_as(x)

    @staticmethod
    def backward(ctx, g):
        g = g.contiguous().clone()
        dist.all_reduce(g, group=ctx.group)
        return g, None


SHARDED = ("K", "Kq", "V", "a", "A_log", "dt_bias", "theta", "wr", "wi")


class ShardedCHeadGated(heads.CHeadGated):
    """A CHeadGated whose scan runs on this rank's heads only (module docstring).  Made from a
    built head by `shard_head`, so its parameters and their names are the original's."""

    def _tp_setup(self, group):
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        if self.H % self.world:
            raise ValueError(f"{self.H} heads do not split over {self.world} ranks")
        self.Hr = self.H // self.world
        self.h0 = self.rank * self.Hr

    def init_state(self, B, device, dtype=torch.float32):
        z = torch.zeros(B, self.Hr, self.Mh, self.dvh, device=device, dtype=torch.float32)
        return {"sr": z, "si": z.clone(), "pos": torch.zeros((), device=device, dtype=torch.float32),
                "empty": True}

    def _local(self, z, h):
        """This rank's projections: K(h), K(z) or Kq(z), V(z) and the log-decay of its heads."""
        Mh, dvh, a0, a1 = self.Mh, self.dvh, self.h0, self.h0 + self.Hr
        kz_w = (self.Kq if self.sepq else self.K).weight[a0 * Mh:a1 * Mh]
        kh = F.linear(h, self.K.weight[a0 * Mh:a1 * Mh])
        kz = F.linear(z, kz_w)
        v = F.linear(z, self.V.weight[a0 * dvh:a1 * dvh])
        g = None
        if self.decay:
            with torch.autocast(device_type=z.device.type, enabled=False):
                logit = F.linear(z.float(), self.a.weight[a0:a1].float())
            g = -torch.exp(self.A_log[a0:a1].float()) * F.softplus(logit + self.dt_bias[a0:a1].float())
        return kh, kz, v, g

    def _params(self):
        a0, a1 = self.h0, self.h0 + self.Hr
        H, Mh = self.H, self.Mh
        return (self.theta.view(H, Mh)[a0:a1], self.omega.view(H, Mh)[a0:a1],
                self.wr.float().view(H, Mh)[a0:a1], self.wi.float().view(H, Mh)[a0:a1])

    def _read_out(self, o, z):
        """o (B,T,H,2,dvh) of every head -> the head's read-out u (B,T,2dv), replicated."""
        return heads._read_heads(self, o, z).to(z.dtype)

    def prefill(self, z, h, state=None):
        B, T, _ = z.shape
        st = state if state is not None else self.init_state(B, z.device)
        zs, hs = _ShareGrad.apply(z, self.group), _ShareGrad.apply(h, self.group)
        kh, kz, v, g = self._local(zs, hs)
        th, om, wr, wi = self._params()
        S0 = None if st.get("empty", False) else torch.cat([st["sr"], st["si"]], 2).float()
        o, S = ops.phase_scan_proj(kh.view(B, T, self.Hr, self.Mh), kz.view(B, T, self.Hr, self.Mh), th, om,
                                   st["pos"], v.to(heads._value_dtype(z)).view(B, T, self.Hr, self.dvh), None, g,
                                   None, wr, wi, S0)
        u = self._read_out(_GatherHeads.apply(o, self.group, self.world, self.rank), z)
        Mh = self.Mh
        return u, {"sr": S[:, :, :Mh], "si": S[:, :, Mh:], "pos": st["pos"] + T, "empty": False}

    def step(self, z_t, h_t, state):
        B = z_t.size(0)
        p = state["pos"].float()
        kh, kz, v, g = self._local(z_t, h_t)
        th, om, wr, wi = self._params()
        pw = kh.float().view(B, self.Hr, self.Mh) * th.float() + p * om.float()
        pq = kz.float().view(B, self.Hr, self.Mh) * th.float() + p * om.float()
        S = torch.cat([state["sr"], state["si"]], 2).float().contiguous()
        o, S = ops.phase_step(pw, pq, v.float().view(B, self.Hr, self.dvh), None, g, None, wr, wi, S, S_out=S)
        parts = [torch.empty_like(o) for _ in range(self.world)]
        dist.all_gather(parts, o.contiguous(), group=self.group)
        u = self._read_out(torch.cat(parts, 1), z_t)
        Mh = self.Mh
        return u, {"sr": S[:, :, :Mh], "si": S[:, :, Mh:], "pos": state["pos"] + 1, "empty": False}


def shard_head(head: heads.CHeadGated, group=None) -> ShardedCHeadGated:
    """Turn a built CHeadGated into its head-sharded form in place (same parameters)."""
    if not isinstance(head, heads.CHeadGated):
        raise TypeError("head sharding covers the multi-head gated C head (CHeadGated)")
    head.__class__ = ShardedCHeadGated
    head._tp_setup(group)
    return head


def shard_layer(layer, group=None):
    """Shard the C slot of a layer (GatedLayer or another MixerLayer with a CHeadGated in
    slot "c") over the ranks of `group`; returns the layer."""
    shard_head(layer.c, group)
    return layer


def reduce_sharded_grads(module, group=None):
    """After the backward: sum the gradients of every sharded head's parameters over the group
    (each rank filled only its own heads' rows)."""
    for m in module.modules():
        if isinstance(m, ShardedCHeadGated):
            for name in SHARDED:
                sub = getattr(m, name, None)
                ps = [sub] if isinstance(sub, torch.nn.Parameter) else list(sub.parameters()) if sub is not None else []
                for prm in ps:
                    if prm.grad is not None:
                        dist.all_reduce(prm.grad, group=group)
