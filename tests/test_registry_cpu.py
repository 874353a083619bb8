"""The plugin registry mirror: same interface as the reference's sca2/registry.py, and a
reference layer built with this package's C head through the reference's own registry
loads the reference layer's weights unchanged (CPU, construction only)."""
import inspect
import os
import sys

import pytest
import torch

from sca2_b200 import heads, registry

# the reference checkout: SCA2_REFERENCE, else a folder named "reference" beside this
# repository; the tests skip when neither exists (e.g. on a machine without the sources)
REF = os.environ.get("SCA2_REFERENCE") or os.path.join(
    os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__)))), "reference")


def _ref_registry():
    if not os.path.isdir(REF):
        pytest.skip("reference sources not present")
    sys.dont_write_bytecode = True  # never write caches next to the reference sources
    if REF not in sys.path:
        sys.path.insert(0, REF)
    try:
        import sca2.registry as r
    except Exception as e:  # pragma: no cover - reference import problems
        pytest.skip(f"reference registry not importable: {e}")
    return r


def test_interface_matches_reference():
    ref = _ref_registry()
    for fn in ("register", "build"):
        a, b = inspect.signature(getattr(registry, fn)), inspect.signature(getattr(ref, fn))
        assert list(a.parameters) == list(b.parameters), fn
        for n in a.parameters:
            assert a.parameters[n].default == b.parameters[n].default, (fn, n)


def test_install_and_build_with_reference_layer():
    ref = _ref_registry()
    from sca2.arch_cdelta import CHeadDelta as RefCHeadDelta
    from sca2.ref import LayerCfg
    names = registry.install(ref)
    assert "b200_delta" in names and "b200_delta" in ref.VARIANTS
    cfg = LayerCfg(d=64, Mc=32, Md=4, G=4, dv=32)
    mine = ref.build("b200_delta", cfg, seed=0)
    assert isinstance(mine.c, heads.CHeadDelta)
    name = ref.register("ref_delta_check", c_cls=RefCHeadDelta)
    theirs = ref.build(name, cfg, seed=0)
    mine.load_state_dict(theirs.state_dict(), strict=True)
    for k, v in theirs.state_dict().items():
        assert torch.equal(mine.state_dict()[k], v), k


def test_local_registry_build():
    class Layer(torch.nn.Module):
        def __init__(self, cfg, c_cls, d_cls=None):
            super().__init__()
            self.c = c_cls(cfg["d"], cfg["M"], dv=cfg["dv"])

    registry.install(layer_cls=Layer)
    m = registry.build("b200_delta", {"d": 32, "M": 16, "dv": 16}, seed=1)
    assert isinstance(m.c, heads.CHeadDelta)


def test_install_short_layers_into_reference():
    """The short-window layers build through the reference registry with this package's C
    head and short head, and load the reference layer's weights unchanged."""
    ref = _ref_registry()
    from sca2.ref import LayerCfg
    registry.install(ref)
    cfg = LayerCfg(d=64, Mc=32, Md=4, G=4, dv=32)
    for name, ref_name in (("b200_cshort", "cshort"), ("b200_cshort_damph", "cshort_damph")):
        mine = ref.build(name, cfg, seed=0)
        assert isinstance(mine.dh, heads.CHeadShort)
        assert isinstance(mine.c, registry.SHORT_LAYERS[name][1])
        theirs = ref.build(ref_name, cfg, seed=0)
        mine.load_state_dict(theirs.state_dict(), strict=True)
        for k, v in theirs.state_dict().items():
            assert torch.equal(mine.state_dict()[k], v), k
