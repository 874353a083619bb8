"""GPU parity of the inference forward with a work buffer (sca2_scan_fwd_work).

Without saved chunk states, the tensor-core forward at K = 64 first forms the delta-rule
inverse of every 64-token chunk chunk-parallel into a caller work buffer, and the chunk walk
reads it instead of inverting inside its sequential loop.  The ops layer takes this path for
every forward that keeps no autograd graph.  Checked here, through the C ABI:
  * against the numpy oracle (pinned to the reference's fixtures) at the bf16 bar;
  * against sca2_scan_fwd with no chunk states (the walk that inverts in its loop);
  * ragged lengths, T = 1, two value blocks per sequence (V = 128), scalar decay, the additive
    write, the explicit-key flavour and the projected-phase form;
  * the work-size query and the refusal of a short work buffer.
"""
import numpy as np
import pytest
import torch

from oracle import scan as ora
from tests._util import TOL_BF16_ABS, TOL_BF16_COS, cosine, cuda, relerr, rms_np, seeded_phase_inputs

pytestmark = pytest.mark.gpu


def _ops():
    from sca2_b200 import ops
    return ops


def _phase_tensors(d):
    t = {k: cuda(d[k], torch.float32) for k in ("phw", "phq", "beta", "g", "lam", "wr", "wi", "S0")}
    t["v"] = cuda(d["v"], torch.bfloat16)
    return t


def _no_work_forward(t):
    """sca2_scan_fwd without chunk states: the walk inverts each chunk inside its loop."""
    ops = _ops()
    from sca2_b200 import _lib
    a = ops._phase_args(t["phw"], t["phq"], t["v"], t["beta"], t["g"], t["lam"], t["wr"], t["wi"], t["S0"])
    B, T, H, Mh = t["phw"].shape
    V = t["v"].shape[-1]
    o = torch.empty(B, T, H, 2, V, device="cuda", dtype=torch.bfloat16)
    S = torch.empty(B, H, 2 * Mh, V, device="cuda", dtype=torch.float32)
    _lib.check(_lib.load().sca2_scan_fwd(ops.C_ref(a), ops._out(o), ops._ptr(S), None, ops._stream()), "scan_fwd")
    return o, S


CASES = [  # B, T, H, Mh, V, beta, g, lam, S0
    (2, 200, 2, 32, 64, True, True, True, True),
    (1, 256, 3, 32, 128, True, False, True, True),
    (2, 64, 1, 32, 64, False, True, False, False),
    (1, 1, 2, 32, 64, True, False, True, True),
    (3, 129, 2, 32, 64, True, False, True, False),
]


@pytest.mark.parametrize("case", CASES)
def test_phase_inference_work(case):
    B, T, H, Mh, V, be, g, lam, s0 = case
    ops = _ops()
    from sca2_b200 import _lib
    d = seeded_phase_inputs(B, T, H, Mh, V, seed=11 * T + V, beta=be, g=g, lam=lam, S0=s0)
    d["v"] = torch.tensor(d["v"]).bfloat16().double().numpy()
    t = _phase_tensors(d)
    a = ops._phase_args(t["phw"], t["phq"], t["v"], t["beta"], t["g"], t["lam"], t["wr"], t["wi"], t["S0"])
    nc = (T + 63) // 64
    assert _lib.load().sca2_scan_fwd_work_bytes(ops.C_ref(a)) == B * H * nc * 64 * 64 * 2
    with torch.no_grad():
        o, S = ops.phase_scan(t["phw"], t["phq"], t["v"], t["beta"], t["g"], t["lam"], t["wr"], t["wi"], t["S0"])
    torch.cuda.synchronize()
    ro, rS = ora.phase_forward(d["phw"].astype(np.float64), d["phq"].astype(np.float64), d["v"], d["beta"], d["g"],
                               d["lam"], d["wr"], d["wi"], d["S0"], chunked=True, C=32)
    u, ru = rms_np(o.double().cpu().numpy().reshape(B, T, H, -1)), rms_np(ro.reshape(B, T, H, -1))
    assert np.abs(u - ru).max() < TOL_BF16_ABS and cosine(u, ru) > TOL_BF16_COS
    assert relerr(S, rS) < TOL_BF16_ABS and cosine(S, rS) > TOL_BF16_COS
    o2, S2 = _no_work_forward(t)
    torch.cuda.synchronize()
    u2 = rms_np(o2.double().cpu().numpy().reshape(B, T, H, -1))
    assert np.abs(u - u2).max() < TOL_BF16_ABS and cosine(u, u2) > TOL_BF16_COS
    assert relerr(S, S2) < TOL_BF16_ABS and cosine(S, S2) > TOL_BF16_COS
    assert _lib.device_faults() == 0


def test_key_inference_work():
    ops = _ops()
    from sca2_b200 import _lib
    B, T, H, K, V = 2, 130, 2, 64, 64
    rng = np.random.default_rng(5)
    nrm = lambda x: x / np.linalg.norm(x, axis=-1, keepdims=True)
    bf = lambda x: torch.tensor(x).bfloat16().double().numpy()
    q, k, v = bf(nrm(rng.standard_normal((B, T, H, K)))), bf(nrm(rng.standard_normal((B, T, H, K)))), \
        bf(rng.standard_normal((B, T, H, V)))
    g = -np.log1p(np.exp(rng.standard_normal((B, T, H))))
    beta = 1 / (1 + np.exp(-rng.standard_normal((B, T, H))))
    S0 = 0.3 * rng.standard_normal((B, H, K, V))
    tq, tk, tv = (cuda(x, torch.bfloat16) for x in (q, k, v))
    tg, tb, tS = cuda(g), cuda(beta), cuda(S0)
    a = ops._key_args(tq, tk, tv, tg, tb, None, tS, 1.0, False)
    assert _lib.load().sca2_scan_fwd_work_bytes(ops.C_ref(a)) == B * H * 3 * 64 * 64 * 2
    with torch.no_grad():
        o, S = ops.key_scan(tq, tk, tv, tg, tb, S0=tS)
    ro, rS = ora.gdn_forward(q, k, v, g, beta, S0=S0, chunked=True, C=32)
    assert relerr(o, ro) < TOL_BF16_ABS and cosine(o, ro) > TOL_BF16_COS
    assert relerr(S, rS) < TOL_BF16_ABS and cosine(S, rS) > TOL_BF16_COS


def test_proj_inference_work():
    """Projected phases without a graph: the work path with the phases formed in the kernels,
    against the same call with the phases formed in torch (fp32 phase path, bf16 values)."""
    ops = _ops()
    B, T, H, Mh, V = 2, 100, 2, 32, 64
    gen = torch.Generator(device="cuda").manual_seed(3)
    rn = lambda *s: torch.randn(*s, device="cuda", generator=gen)
    kh, kz = rn(B, T, H, Mh).bfloat16(), rn(B, T, H, Mh).bfloat16()
    theta = 0.5 + rn(H, Mh).abs()
    omega = torch.pi * 1e4 ** (-torch.arange(Mh, device="cuda") / (Mh - 1))
    omega = omega.expand(H, Mh).contiguous()
    pos = torch.tensor(17.0, device="cuda")
    v = rn(B, T, H, V).bfloat16()
    beta = torch.sigmoid(rn(B, T, H))
    lam = torch.nn.functional.softplus(rn(H, Mh)).clamp(max=1 / 16)
    wr, wi = 1 + 0.3 * rn(H, Mh), 0.3 * rn(H, Mh)
    with torch.no_grad():
        o, S = ops.phase_scan_proj(kh, kz, theta, omega, pos, v, beta, None, lam, wr, wi)
        p = torch.arange(T, device="cuda", dtype=torch.float32)[:, None, None] + pos
        phw = kh.float() * theta + p * omega
        phq = kz.float() * theta + p * omega
        o2, S2 = ops.phase_scan(phw, phq, v, beta, None, lam, wr, wi)
    u = rms_np(o.double().cpu().numpy().reshape(B, T, H, -1))
    u2 = rms_np(o2.double().cpu().numpy().reshape(B, T, H, -1))
    assert np.abs(u - u2).max() < TOL_BF16_ABS and cosine(u, u2) > TOL_BF16_COS
    assert relerr(S, S2) < TOL_BF16_ABS and cosine(S, S2) > TOL_BF16_COS


def test_work_query_and_refusal():
    ops = _ops()
    from sca2_b200 import _lib
    lib = _lib.load()
    d = seeded_phase_inputs(1, 70, 1, 32, 64, seed=1)
    t = _phase_tensors(d)
    a = ops._phase_args(t["phw"], t["phq"], t["v"], t["beta"], t["g"], t["lam"], t["wr"], t["wi"], t["S0"])
    need = lib.sca2_scan_fwd_work_bytes(ops.C_ref(a))
    assert need == 2 * 64 * 64 * 2
    o = torch.empty(1, 70, 1, 2, 64, device="cuda", dtype=torch.bfloat16)
    S = torch.empty(1, 1, 64, 64, device="cuda")
    short = torch.empty(need // 2, device="cuda", dtype=torch.uint8)
    rc = lib.sca2_scan_fwd_work(ops.C_ref(a), None, ops._out(o), ops._ptr(S), short.data_ptr(), need // 2,
                                ops._stream())
    assert rc == _lib.SCA2_ERR_ARG
    # fp32 values: no tensor-core path, no work buffer, the call runs the fp32 kernels
    t32 = dict(t, v=t["v"].float())
    a32 = ops._phase_args(t32["phw"], t32["phq"], t32["v"], t32["beta"], t32["g"], t32["lam"], t32["wr"], t32["wi"],
                          t32["S0"])
    assert lib.sca2_scan_fwd_work_bytes(ops.C_ref(a32)) == 0
