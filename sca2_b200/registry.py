"""Plugin registry with the reference's interface (sca2/registry.py:9-32).

    register(name, c_cls=None, d_cls=None, note="", wrap=None, layer_cls=None, arch=False)
    build(name, cfg=None, seed=0, device="cpu", dtype=torch.float32)
    VARIANTS  name -> {"c", "d", "note", "wrap", "layer", "arch"}

This package rebuilds the scan of the C heads, not the layer around it nor the D head, so
a variant here names this package's C-head class and takes the layer and D-head classes
from the caller (the reference's SCA2Layer / GatedLayer and its D heads).  `install`
registers every C head of this package into the reference's own registry, which is how
a reference user switches to the B200 scan:

    import sca2.registry, sca2_b200.registry
    sca2_b200.registry.install(sca2.registry)      # adds "b200_delta", "b200_gated", ...
    layer = sca2.registry.build("b200_gated", cfg, device="cuda")
"""
from __future__ import annotations

import torch

from . import heads

VARIANTS = {}

# C heads of this package and the reference heads they replace (same constructor
# arguments, parameters and state dicts)
C_HEADS = {
    "b200_delta": (heads.CHeadDelta, "CHeadDelta (sca2/arch_cdelta.py:92-206), scan on sm_100a"),
    "b200_damp": (heads.CHeadDeltaDamp, "CHeadDeltaDamp (sca2/arch_damp.py:43-259), scan on sm_100a"),
    "b200_damp_half": (heads.CHeadDeltaDampHalf, "CHeadDeltaDampHalf (sca2/arch_damp.py), scan on sm_100a"),
    "b200_gated": (heads.CHeadGated, "CHeadGated (sca2/arch_gatedc.py:58-193), scan on sm_100a"),
}


def register(name, c_cls=None, d_cls=None, note="", wrap=None, layer_cls=None, arch=False):
    """Register a (C head, D head[, layer]) triple under `name`; returns the name.  As in the
    reference, `wrap` is an optional post-build callable that must keep the prefill / step
    contract and `arch=True` marks a different function rather than a faster schedule."""
    VARIANTS[name] = {"c": c_cls, "d": d_cls, "note": note, "wrap": wrap, "layer": layer_cls, "arch": arch}
    return name


def build(name, cfg=None, seed=0, device="cpu", dtype=torch.float32):
    """Instantiate variant `name`: layer_cls(cfg, c_cls, d_cls) seeded with `seed`, moved to
    device / dtype, wrapped if the variant has a wrap.  cfg and the layer class come from the
    caller's layer family (the reference's LayerCfg / SCA2Layer when the variant was
    registered without one, which requires the reference package)."""
    v = VARIANTS[name]
    layer = v["layer"]
    if layer is None or cfg is None:
        from sca2.ref import LayerCfg, SCA2Layer  # the reference's layer family
        layer = layer or SCA2Layer
        cfg = cfg or LayerCfg()
    torch.manual_seed(seed)
    m = layer(cfg, v["c"], v["d"]) if v["d"] is not None else layer(cfg, v["c"])
    m = m.to(device=device, dtype=dtype)
    return v["wrap"](m) if v["wrap"] else m


# short-window layers of the reference (sca2/arch_short.py:161-214): a long C head with the
# short DFT head CHeadShort in the D slot.  The layer class fixes its C head (C_CLS), so the
# B200 variant subclasses it with this package's C head and swaps the D slot after building.
SHORT_LAYERS = {
    "b200_cshort": ("ShortLayer", heads.CHeadDelta, "cshort (sca2/arch_short.py:161-177) on sm_100a"),
    "b200_cshort_damph": ("ShortLayerDampH", heads.CHeadDeltaDampHalf,
                          "cshort_damph (sca2/arch_short.py:199-201) on sm_100a"),
}


def use_b200_short(layer):
    """wrap= hook: replace the reference CHeadShort in a built layer's D slot (`dh`) by
    heads.CHeadShort with the same weights and read-out attributes."""
    old = layer.dh
    new = heads.CHeadShort(old.d, old.L, old.dv)
    for a in ("rms_read", "gated_read", "rscale", "rgate"):
        if hasattr(old, a):
            setattr(new, a, getattr(old, a))
    new.load_state_dict(old.state_dict(), strict=True)
    p = next(old.parameters())
    layer.dh = new.to(device=p.device, dtype=p.dtype)
    return layer


def install(target=None, d_cls=None, layer_cls=None):
    """Register this package's C heads into `target` (a registry module with the reference's
    register(), e.g. sca2.registry), or into this module when target is None.  With the
    reference registry as target, the short-window layers are registered too (B200 C head
    and B200 short head)."""
    reg = target.register if target is not None else register
    names = []
    for name, (cls, note) in C_HEADS.items():
        names.append(reg(name, c_cls=cls, d_cls=d_cls, note=note, layer_cls=layer_cls))
    if target is not None:
        import importlib
        try:
            ash = importlib.import_module(target.__name__.rsplit(".", 1)[0] + ".arch_short")
        except ImportError:
            ash = None
        for name, (base, c_cls, note) in SHORT_LAYERS.items() if ash is not None else ():
            lcls = type(name + "_layer", (getattr(ash, base),), {"C_CLS": c_cls})
            names.append(reg(name, c_cls=c_cls, d_cls=None, note=note, wrap=use_b200_short,
                             layer_cls=lcls, arch=True))
    return names
