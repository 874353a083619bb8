"""Layer-level parity case of the first benchmark configuration (SCA2 layer forward, fp32).

One GatedLayer (multi-head gated C head, sca2/arch_gatedc.py:58-256) at the configuration's
shape: B = 2, T = 512, d_model = 256, four C heads of d_head 64 (Mc = 128, dv = 256, so
Mh = 32 complex modes and 64 value columns per head), per-head scalar decay, rope grid with
theta_scale = 0.02, chunk 64, the layer's default D head (DHeadSepQPolar) with Md = 4, G = 8,
ff = 256.  Seed 0: every 2-D weight matrix (the projections) is re-drawn N(0, 0.02^2) after
construction and the input is x ~ N(0, 1).

The weights and inputs are not stored in the fixture: `draw` regenerates them from one CPU
torch.Generator stream, in a fixed order (the 2-D ".weight" entries of the state dict sorted by
name, then x, then the upstream gradient dY), so make_golden.py and the GPU test see the same
values.  Everything else of the state dict (norms, biases, theta, read weights, decay
parameters, the D head's vectors, buffers) is stored.
"""
from __future__ import annotations

import torch

B, T = 2, 512
LAYER = dict(d=256, Mc=128, Md=4, G=8, ff=256, freq="rope", theta_scale=0.02, max_len=512, dv=256,
             c_heads=4, c_decay=True)
CHUNK = 64
SEED = 0
STD = 0.02


def redrawn(state_dict) -> list:
    """Names of the entries that `draw` replaces: the 2-D weight matrices, sorted."""
    return sorted(k for k, v in state_dict.items() if k.endswith(".weight") and v.dim() == 2)


def draw(state_dict):
    """(weights, x, dY): the re-drawn 2-D weights {name: fp32 tensor}, the input x (B, T, d) and
    the upstream gradient dY (B, T, d), all fp32 on the CPU, from one generator seeded SEED."""
    g = torch.Generator().manual_seed(SEED)
    w = {k: STD * torch.randn(tuple(state_dict[k].shape), generator=g, dtype=torch.float32)
         for k in redrawn(state_dict)}
    d = LAYER["d"]
    x = torch.randn((B, T, d), generator=g, dtype=torch.float32)
    dY = torch.randn((B, T, d), generator=g, dtype=torch.float32)
    return w, x, dY
