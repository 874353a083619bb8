"""Layer and LM classes on the CPU (construction only: the heads' kernels need a GPU): the
reference layers' and LM's state_dicts load with strict=True, and the Zipf corpus of the
LM benchmark is seeded and Zipf-shaped."""
import numpy as np
import torch

from tests.golden import fixtures as fx
from tests.test_layers_gpu import _build


def test_layer_state_dicts_load():
    for kind in ("sca2", "gated", "lapa"):
        f = fx.load(f"layer_{kind}.npz")
        _build(kind).load_state_dict({k[3:]: torch.tensor(f[k]).float() for k in f if k.startswith("sd_")},
                                     strict=True)


def test_lm_state_dict_loads():
    from sca2_b200 import lm as L
    f = fx.load("lm_lapa.npz")
    B, T, vocab, d, n_layers, n_new = (int(x) for x in f["meta"])
    model = L.LaplaceLM(vocab, d=d, n_layers=n_layers, M=12, dv=8, L=8, ff=48, chunk=16, theta_scale=0.3)
    model.load_state_dict({k[3:]: torch.tensor(f[k]).float() for k in f if k.startswith("sd_")}, strict=True)


def test_zipf_tokens():
    from sca2_b200.lm import zipf_tokens
    a, b = zipf_tokens(8, 2048, 16384, seed=3), zipf_tokens(8, 2048, 16384, seed=3)
    assert torch.equal(a, b) and a.shape == (8, 2048) and int(a.min()) >= 0 and int(a.max()) < 16384
    counts = np.sort(np.bincount(a.flatten().numpy(), minlength=16384))[::-1]
    r = np.arange(1, 51)
    slope = np.polyfit(np.log(r), np.log(counts[:50] + 1e-9), 1)[0]
    assert -1.4 < slope < -0.8
