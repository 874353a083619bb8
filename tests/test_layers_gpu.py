"""Whole layers and the LM on the GPU against the reference (fixtures made by the reference's
SCA2Layer, GatedLayer, LaplaceAttention and LaplaceLM in float64): outputs, new states,
every parameter / input gradient, decode steps, greedy generation, and the CUDA-graph
decoder against eager decoding.  fp32 bar: 1e-4 relative."""
import numpy as np
import pytest
import torch

from tests._util import TOL_F32, cuda, relerr
from tests.golden import fixtures as fx

pytestmark = pytest.mark.gpu


def _build(kind):
    from sca2_b200 import layers
    if kind == "sca2":
        return layers.SCA2Layer(layers.LayerCfg(d=32, Mc=16, Md=4, G=4, ff=48, freq="rope", theta_scale=0.3,
                                                max_len=64, dv=32))
    if kind == "gated":
        return layers.GatedLayer(layers.LayerCfg(d=32, Mc=16, Md=4, G=4, ff=48, freq="rope", theta_scale=0.3,
                                                 max_len=64, dv=32, c_heads=2, c_decay=True, conv=3))
    from sca2_b200.heads import LaplaceConfig
    return layers.LaplaceAttention(LaplaceConfig(d=32, M=12, dv=8, L=8, ff=48, chunk=16, theta_scale=0.3))


def _get(tree, path):
    for k in path:
        tree = tree[int(k)] if isinstance(tree, (list, tuple)) else tree[k]
    return tree


def _check_state(f, prefix, st):
    n = 0
    for key in f:
        if key.startswith(prefix + "."):
            ours = _get(st, key.split(".")[1:])
            ref = f[key]
            if torch.is_tensor(ours):
                ours = ours.detach().float().reshape(ref.shape)
                assert relerr(ours, ref) < TOL_F32, key
            else:
                assert float(ours) == float(ref), key
            n += 1
    assert n > 0


@pytest.mark.parametrize("kind", ["sca2", "gated", "lapa"])
def test_layer_vs_reference(kind):
    f = fx.load(f"layer_{kind}.npz")
    layer = _build(kind).cuda()
    layer.load_state_dict({k[3:]: torch.tensor(f[k]).float() for k in f if k.startswith("sd_")}, strict=True)
    x = cuda(f["x"], torch.float32, True)
    y, st = layer.prefill(x)
    (y * cuda(f["dY"])).sum().backward()
    assert relerr(y, f["y"]) < TOL_F32
    assert relerr(x.grad, f["d_x"]) < TOL_F32
    for n, p in layer.named_parameters():
        if "g_" + n in f:
            assert relerr(p.grad, f["g_" + n]) < TOL_F32, n
    _check_state(f, "st", st)
    with torch.no_grad():
        for t in range(f["xs"].shape[1]):
            yt, st = layer.step(cuda(f["xs"][:, t]), st)
            assert relerr(yt, f["ys"][:, t]) < TOL_F32, t
    _check_state(f, "sts", st)


def test_lm_vs_reference_and_graph_decode():
    from sca2_b200 import lm as L
    f = fx.load("lm_lapa.npz")
    B, T, vocab, d, n_layers, n_new = (int(x) for x in f["meta"])
    model = L.LaplaceLM(vocab, d=d, n_layers=n_layers, M=12, dv=8, L=8, ff=48, chunk=16, theta_scale=0.3).cuda()
    model.load_state_dict({k[3:]: torch.tensor(f[k]).float() for k in f if k.startswith("sd_")}, strict=True)
    tok = torch.tensor(f["tok"], device="cuda")
    logits = model(tok[:, :-1])
    loss = torch.nn.functional.cross_entropy(logits.reshape(-1, vocab), tok[:, 1:].reshape(-1))
    loss.backward()
    assert relerr(logits, f["logits"]) < TOL_F32
    for n, p in model.named_parameters():
        assert relerr(p.grad, f["g_" + n]) < TOL_F32, n
    prompt = torch.tensor(f["prompt"], device="cuda")
    ids = model.generate(prompt, n_new, greedy=True)
    assert torch.equal(ids.cpu(), torch.tensor(f["gen"]))
    # the whole decode step as one CUDA graph gives the same tokens
    with torch.no_grad():
        logits, st = model.prefill(prompt)
        dec = L.GraphDecoder(model, st)
        first = logits[:, -1].argmax(-1)
        gen = dec.generate(first, n_new - 1)
    assert torch.equal(torch.cat([prompt, first[:, None], gen], 1).cpu(), torch.tensor(f["gen"]))


def test_gated_lm_train_step_decreases_loss():
    """A small GatedLM trains (bf16 autocast, AdamW) on a fixed Zipf batch: the loss falls."""
    from sca2_b200 import lm as L
    from sca2_b200.layers import LayerCfg
    torch.manual_seed(0)
    cfg = LayerCfg(d=64, Mc=32, Md=4, G=8, ff=128, freq="rope", theta_scale=0.02, max_len=256, dv=64,
                   c_heads=2, c_decay=True)
    model = L.GatedLM(128, cfg, n_layers=2).cuda()
    L.init_weights(model)
    opt = torch.optim.AdamW(model.parameters(), lr=3e-3)
    tok = L.zipf_tokens(4, 129, 128, seed=1, device="cuda")
    losses = [float(L.train_step(model, opt, tok)) for _ in range(20)]
    assert np.isfinite(losses).all() and losses[-1] < 0.8 * losses[0]
