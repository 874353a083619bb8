"""The first benchmark configuration at its own shape against the reference: one GatedLayer
(B = 2, T = 512, d_model = 256, four C heads of d_head 64 with scalar decay, chunk 64, seed 0,
projections N(0, 0.02^2); tests/golden/config1.py) -- the output y, the final state of both
heads and z_prev, and the gradients of x and of every C-head parameter, from the reference's
own GatedLayer run in float64 (tests/golden/layer_gated_config1.npz).

fp32: 1e-4 relative.  bf16 autocast (the layer and LM benchmarks' precision): the output, the
layer's increment y - x and the input gradient at max-abs <= 2e-2 relative to max |ref| and
cosine >= 0.9999; the same bar for LaplaceAttention against its float64 fixture."""
import numpy as np
import pytest
import torch

from tests._util import TOL_BF16_ABS, TOL_BF16_COS, TOL_F32, cosine, cuda, relerr
from tests.golden import config1 as C1
from tests.golden import fixtures as fx


def _layer(device):
    from sca2_b200 import layers
    return layers.GatedLayer(layers.LayerCfg(**C1.LAYER)).to(device)


def _loaded(device):
    """Our GatedLayer with the fixture's state dict (stored entries + the re-drawn weights),
    strict loading; plus x and dY."""
    f = fx.load("layer_gated_config1.npz")
    layer = _layer("cpu")
    sd = {k[3:]: torch.tensor(f[k]).float() for k in f if k.startswith("sd_")}
    w, x, dY = C1.draw(layer.state_dict())
    sd.update(w)
    layer.load_state_dict(sd, strict=True)
    return f, layer.to(device), x.to(device), dY.to(device)


def test_config1_state_dict_matches_reference_layout():
    """CPU: our GatedLayer at the configuration has exactly the reference's state-dict entries
    (the stored ones plus the re-drawn weight matrices), so the fixture loads strictly."""
    f, layer, x, dY = _loaded("cpu")
    stored = {k[3:] for k in f if k.startswith("sd_")}
    assert stored | set(C1.redrawn(layer.state_dict())) == set(layer.state_dict())
    assert tuple(f["meta"]) == (C1.B, C1.T, C1.LAYER["d"], C1.LAYER["c_heads"], C1.CHUNK)


def _state_checks(f, st):
    for key, ours in (("st.c.sr", st["c"]["sr"]), ("st.c.si", st["c"]["si"]), ("st.d.sr", st["d"]["sr"]),
                      ("st.d.si", st["d"]["si"]), ("st.z_prev", st["z_prev"])):
        ref = f[key]
        got = ours.detach().float().reshape(ref.shape)
        yield key, relerr(got, ref), cosine(got, ref)
    assert float(st["c"]["pos"]) == float(f["st.c.pos"])


@pytest.mark.gpu
def test_config1_fp32_vs_reference():
    f, layer, x, dY = _loaded("cuda")
    x.requires_grad_(True)
    y, st = layer.prefill(x)
    (y * dY).sum().backward()
    assert relerr(y, f["y"]) < TOL_F32
    for key, err, _ in _state_checks(f, st):
        assert err < TOL_F32, key
    assert relerr(x.grad, f["d_x"]) < TOL_F32
    for n, p in layer.named_parameters():
        if "g_" + n in f:
            assert relerr(p.grad, f["g_" + n]) < TOL_F32, n


def _bf16_bar(got, ref, what, abs_bar=TOL_BF16_ABS):
    e, c = relerr(got, ref), cosine(got, ref)
    assert e < abs_bar and c > TOL_BF16_COS, (what, e, c)



@pytest.mark.gpu
def test_config1_bf16_autocast_vs_reference():
    f, layer, x, dY = _loaded("cuda")
    x.requires_grad_(True)
    with torch.autocast("cuda", dtype=torch.bfloat16):
        y, st = layer.prefill(x)
    (y.float() * dY).sum().backward()
    xr = x.detach().cpu().double().numpy()
    _bf16_bar(y, f["y"], "y")
    _bf16_bar(y.detach().float().cpu().double().numpy() - xr, f["y"] - xr, "y - x")
    _bf16_bar(x.grad, f["d_x"], "d_x")
    for key, err, cos in _state_checks(f, st):
        assert err < TOL_BF16_ABS and cos > TOL_BF16_COS, (key, err, cos)


@pytest.mark.gpu
def test_laplace_attention_bf16_autocast_vs_reference():
    """LaplaceAttention (long head + short head, lapa/layer.py:551-600) under bf16 autocast
    against the reference's float64 layer fixture."""
    from sca2_b200 import layers
    from sca2_b200.heads import LaplaceConfig
    f = fx.load("layer_lapa.npz")
    layer = layers.LaplaceAttention(LaplaceConfig(d=32, M=12, dv=8, L=8, ff=48, chunk=16, theta_scale=0.3)).cuda()
    layer.load_state_dict({k[3:]: torch.tensor(f[k]).float() for k in f if k.startswith("sd_")}, strict=True)
    x = cuda(f["x"], torch.float32, True)
    with torch.autocast("cuda", dtype=torch.bfloat16):
        y, _ = layer.prefill(x)
    (y.float() * cuda(f["dY"])).sum().backward()
    xr = np.asarray(f["x"], np.float64)
    _bf16_bar(y, f["y"], "y")
    _bf16_bar(y.detach().float().cpu().double().numpy() - xr, f["y"] - xr, "y - x")
    _bf16_bar(x.grad, f["d_x"], "d_x")
