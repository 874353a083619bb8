"""GPU parity of the tensor-core (tcgen05) scan kernels: bf16 inputs, fp32 state.

Bars (north star): max-abs <= 2e-2 on unit-RMS outputs, relative max error <= 2e-2 on
states and gradients, cosine >= 0.9999, all against the oracle on the same bf16-rounded
inputs.  Every test also checks that no tensor-core wait timed out (device fault word).
"""
import numpy as np
import pytest
import torch

from oracle import scan as ora
from tests._util import TOL_BF16_ABS, TOL_BF16_COS, cosine, cuda, relerr, rms_np, seeded_phase_inputs

pytestmark = pytest.mark.gpu


def _bf16r(x):
    return torch.tensor(x).bfloat16().double().numpy()


def _kernel_names(fn):
    from torch.profiler import ProfilerActivity, profile
    with profile(activities=[ProfilerActivity.CUDA]) as prof:
        fn()
        torch.cuda.synchronize()
    return [e.name for e in prof.events() if e.device_type.name == "CUDA"]


def _no_faults():
    from sca2_b200 import _lib
    assert _lib.device_faults() == 0


TC_PHASE = [
    # B, T, H, Mh, V, beta, g, lam, S0
    (2, 200, 3, 32, 64, True, True, True, True),
    (1, 64, 2, 32, 64, True, False, True, False),
    (2, 130, 2, 64, 64, True, True, True, True),     # K = 128, R = 2 (fp32 path: shared memory)
    (1, 257, 1, 32, 32, False, False, False, True),  # additive, V = 32
    (3, 1, 2, 32, 64, True, True, True, True),
    (1, 100, 2, 32, 96, True, False, True, True),    # V = 96: not a multiple of 64 (fp32 path)
    (2, 150, 2, 32, 128, True, True, True, True),    # value block 128
]


@pytest.mark.parametrize("case", TC_PHASE)
def test_tc_phase_forward(case):
    from sca2_b200 import ops
    B, T, H, Mh, V, be, g, lam, s0 = case
    d = seeded_phase_inputs(B, T, H, Mh, V, seed=B * T + V, beta=be, g=g, lam=lam, S0=s0)
    d["v"] = _bf16r(d["v"])
    t = {k: cuda(d[k]) for k in ("phw", "phq", "beta", "g", "lam", "wr", "wi", "S0")}
    with torch.no_grad():
        o, S = ops.phase_scan(t["phw"], t["phq"], cuda(d["v"], torch.bfloat16), t["beta"], t["g"], t["lam"],
                              t["wr"], t["wi"], t["S0"])
    torch.cuda.synchronize()
    _no_faults()
    ro, rS = ora.phase_forward(d["phw"].astype(np.float64), d["phq"].astype(np.float64), d["v"], d["beta"],
                               d["g"], d["lam"], d["wr"], d["wi"], d["S0"], chunked=True, C=64)
    u = rms_np(o.double().cpu().numpy().reshape(B, T, H, -1))
    ru = rms_np(ro.reshape(B, T, H, -1))
    assert np.abs(u - ru).max() < TOL_BF16_ABS and cosine(u, ru) > TOL_BF16_COS
    assert relerr(S, rS) < TOL_BF16_ABS and cosine(S, rS) > TOL_BF16_COS


@pytest.mark.parametrize("shape", [(2, 150, 2, 64, 64), (1, 300, 2, 128, 128)])
def test_tc_key_forward(shape):
    from sca2_b200 import ops
    B, T, H, K, V = shape
    rng = np.random.default_rng(K + T)
    nrm = lambda x: x / np.linalg.norm(x, axis=-1, keepdims=True)
    q, k = _bf16r(nrm(rng.standard_normal((B, T, H, K)))), _bf16r(nrm(rng.standard_normal((B, T, H, K))))
    v = _bf16r(rng.standard_normal((B, T, H, V)))
    g = -np.log1p(np.exp(rng.standard_normal((B, T, H))))
    beta = 1 / (1 + np.exp(-rng.standard_normal((B, T, H))))
    S0 = 0.3 * rng.standard_normal((B, H, K, V))
    with torch.no_grad():
        o, S = ops.key_scan(cuda(q, torch.bfloat16), cuda(k, torch.bfloat16), cuda(v, torch.bfloat16),
                            cuda(g), cuda(beta), S0=cuda(S0))
    torch.cuda.synchronize()
    _no_faults()
    ro, rS = ora.gdn_forward(q, k, v, g, beta, S0=S0, chunked=True, C=64)
    assert relerr(o, ro) < TOL_BF16_ABS and cosine(o, ro) > TOL_BF16_COS
    assert relerr(S, rS) < TOL_BF16_ABS and cosine(S, rS) > TOL_BF16_COS


def test_tc_kernel_is_what_runs():
    """bf16 inference dispatches to the tcgen05 kernel (checked by kernel name)."""
    from sca2_b200 import ops
    d = seeded_phase_inputs(1, 128, 2, 32, 64, seed=3)
    t = {k: cuda(d[k]) for k in ("phw", "phq", "beta", "lam", "wr", "wi")}
    v = cuda(d["v"], torch.bfloat16)

    def run():
        with torch.no_grad():
            ops.phase_scan(t["phw"], t["phq"], v, t["beta"], None, t["lam"], t["wr"], t["wi"])
    names = _kernel_names(run)
    assert any("scan_fwd_tc" in n for n in names), names


def test_tc_full_size_slices():
    """Benchmark shape (B=8, T=4096, H=16, Mh=32, V=64), bf16 inference: four sequences vs the oracle."""
    from sca2_b200 import ops
    B, T, H, Mh, V = 8, 4096, 16, 32, 64
    d = seeded_phase_inputs(B, T, H, Mh, V, seed=77, S0=False)
    d["v"] = _bf16r(d["v"])
    t = {k: cuda(d[k]) for k in ("phw", "phq", "beta", "lam", "wr", "wi")}
    with torch.no_grad():
        o, S = ops.phase_scan(t["phw"], t["phq"], cuda(d["v"], torch.bfloat16), t["beta"], None, t["lam"],
                              t["wr"], t["wi"])
    torch.cuda.synchronize()
    _no_faults()
    for b, h in ((0, 0), (7, 15), (2, 9), (5, 4)):
        sl = lambda x: None if x is None else x[b:b + 1, :, h:h + 1]
        ro, rS = ora.phase_forward(sl(d["phw"]).astype(np.float64), sl(d["phq"]).astype(np.float64), sl(d["v"]),
                                   sl(d["beta"]), None, d["lam"][h:h + 1], d["wr"][h:h + 1], d["wi"][h:h + 1],
                                   None, chunked=True, C=64)
        u = rms_np(o[b:b + 1, :, h:h + 1].double().cpu().numpy().reshape(1, T, 1, -1))
        ru = rms_np(ro.reshape(1, T, 1, -1))
        assert np.abs(u - ru).max() < TOL_BF16_ABS and cosine(u, ru) > TOL_BF16_COS
        assert relerr(S[b:b + 1, h:h + 1], rS) < TOL_BF16_ABS
