"""GPU parity of the CUDA scan (forward, backward, decode step) through the C ABI.

Checks, in order of strength:
  1. golden fixtures produced by the reference's own heads (fp64 autograd): fp32 <= 1e-4;
  2. the numpy oracle (pinned to those fixtures) on seeded inputs of several shapes,
     gate combinations and ragged lengths, fp32 and bf16;
  3. full-size benchmark shapes: chosen (batch, head) sequences against the oracle, plus
     size-independent properties (split prefill == one prefill, decode == prefill).
"""
import numpy as np
import pytest
import torch

from oracle import scan as ora
from tests._util import (TOL_BF16_ABS, TOL_BF16_COS, TOL_F32, cosine, cuda, relerr, rms_np,
                         seeded_phase_inputs)
from tests.golden import fixtures as fx

pytestmark = pytest.mark.gpu


def _ops():
    from sca2_b200 import ops
    return ops


def _run_phase(inp, dO=None, dS=None, dtype=torch.float32, grad=True):
    ops = _ops()
    t = {k: cuda(inp[k], torch.float32, grad) for k in ("phw", "phq", "beta", "g", "lam", "wr", "wi", "S0")}
    t["v"] = cuda(inp["v"], dtype, grad)
    o, S = ops.phase_scan(t["phw"], t["phq"], t["v"], t["beta"], t["g"], t["lam"], t["wr"], t["wi"], t["S0"])
    grads = None
    if grad and dO is not None:
        loss = (o.float() * cuda(dO)).sum()
        if dS is not None:
            loss = loss + (S * cuda(dS)).sum()
        loss.backward()
        grads = {k: (None if t[k] is None else t[k].grad) for k in t}
    return o, S, grads


# ------------------------------------------------------------------------------------------
#  1. golden fixtures (reference autograd, fp64) -> fp32 kernels
# ------------------------------------------------------------------------------------------
@pytest.mark.parametrize("name", ["scan_longhead.npz", "scan_longhead_chunkpath.npz"])
def test_golden_longhead(name):
    inp, out = fx.longhead(name)
    o, S, gr = _run_phase(inp, out["dO"], out["dS"])
    assert relerr(o, out["o"]) < TOL_F32
    assert relerr(S, out["S"]) < TOL_F32
    ref = out["grads"]
    for n in ("phw", "phq", "v", "wr", "wi", "S0"):
        assert relerr(gr[n], ref[n]) < TOL_F32, n
    b = inp["beta"]
    assert relerr(gr["beta"].double().cpu().numpy() * b * (1 - b), ref["blogit"]) < TOL_F32
    dlr = gr["lam"].double().cpu().numpy() * out["lam_raw_sig"] * out["lam_mask"]
    assert relerr(dlr, ref["lam_raw"]) < TOL_F32


@pytest.mark.parametrize("damp", [False, True])
def test_golden_cdelta(damp):
    inp, out = fx.cdelta(damp)
    o, S, gr = _run_phase(inp, out["dO"], out["dS"])
    assert relerr(o, out["o"]) < TOL_F32 and relerr(S, out["S"]) < TOL_F32
    for n in ("phw", "phq", "v", "wr", "wi", "S0"):
        assert relerr(gr[n], out["grads"][n]) < TOL_F32, n
    b = inp["beta"]
    assert relerr(gr["beta"].double().cpu().numpy() * b * (1 - b), out["grads"]["blogit"]) < TOL_F32
    if damp:
        assert relerr(gr["lam"].double().cpu().numpy() * out["lam_raw_sig"], out["grads"]["lam_raw"]) < TOL_F32


def test_golden_gated():
    inp, out = fx.gated()
    o, S, gr = _run_phase(inp, out["dO"], out["dS"])
    assert relerr(o, out["o"]) < TOL_F32 and relerr(S, out["S"]) < TOL_F32
    for n in ("phw", "phq", "v", "wr", "wi", "S0"):
        assert relerr(gr[n], out["grads"][n]) < TOL_F32, n
    dxg = gr["g"].double().cpu().numpy() * -(1.0 / (1.0 + np.exp(-out["xg"])))
    assert relerr(dxg, out["grads"]["xg"]) < TOL_F32


def test_golden_longhead_step():
    ops = _ops()
    inp, out = fx.longhead_step()
    T = inp["phw"].shape[1]
    S = cuda(inp["S0"]).contiguous()
    outs = []
    for t in range(T):
        o, S = ops.phase_step(cuda(inp["phw"][:, t]), cuda(inp["phq"][:, t]), cuda(inp["v"][:, t]),
                              cuda(inp["beta"][:, t]), None, cuda(inp["lam"]), cuda(inp["wr"]),
                              cuda(inp["wi"]), S)
        outs.append(o)
    assert relerr(torch.stack(outs, 1), out["o"]) < TOL_F32
    assert relerr(S, out["S"]) < TOL_F32


def test_golden_gdn_fla():
    ops = _ops()
    f = fx.gdn()
    t = {k: cuda(f[k], torch.float32, True) for k in ("q", "k", "v", "g", "beta", "S0")}
    o, S = ops.chunk_gated_delta_rule(t["q"], t["k"], t["v"], t["g"], t["beta"], initial_state=t["S0"],
                                      output_final_state=True)
    tol = 2e-5 + TOL_F32  # the fixture itself is fp32 (fla casts to float32)
    assert relerr(o, f["o"]) < tol and relerr(S, f["S"]) < tol
    ((o * cuda(f["dO"])).sum() + (S * cuda(f["dS"])).sum()).backward()
    for n in ("q", "k", "v", "g", "beta", "S0"):
        assert relerr(t[n].grad, f["d_" + n]) < tol, n
    # decode step == fla's recurrent form
    S1 = cuda(f["S0"]).contiguous()
    outs = []
    for i in range(f["q"].shape[1]):
        o1, S1 = ops.key_step(cuda(f["q"][:, i]), cuda(f["k"][:, i]), cuda(f["v"][:, i]),
                              cuda(f["g"][:, i]), cuda(f["beta"][:, i]), S1)
        outs.append(o1)
    assert relerr(torch.stack(outs, 1), f["o_rec"]) < tol and relerr(S1, f["S_rec"]) < tol


# ------------------------------------------------------------------------------------------
#  2. seeded inputs vs the oracle
# ------------------------------------------------------------------------------------------
CASES = [
    # B, T, H, Mh, V, beta, g, lam
    (2, 100, 3, 16, 40, True, True, True),
    (1, 65, 2, 32, 64, True, False, True),
    (2, 33, 1, 8, 5, False, True, False),
    (1, 1, 2, 4, 3, True, True, True),
    (3, 31, 2, 64, 32, True, True, True),
    (1, 257, 1, 32, 96, False, False, False),
]


def _oracle_phase(d, with_grad=True):
    o, S = ora.phase_forward(d["phw"].astype(np.float64), d["phq"].astype(np.float64), d["v"],
                             d["beta"], d["g"], d["lam"], d["wr"], d["wi"], d["S0"], chunked=True, C=32)
    gr = None
    if with_grad:
        gr = ora.phase_backward(d["phw"].astype(np.float64), d["phq"].astype(np.float64), d["v"],
                                d["beta"], d["g"], d["lam"], d["wr"], d["wi"], d["S0"], d["dO"], d["dS"],
                                chunked=True, C=32)
    return o, S, gr


@pytest.mark.parametrize("case", CASES)
def test_phase_vs_oracle_fp32(case):
    B, T, H, Mh, V, be, g, lam = case
    d = seeded_phase_inputs(B, T, H, Mh, V, seed=T + V, beta=be, g=g, lam=lam)
    o, S, gr = _run_phase(d, d["dO"], d["dS"])
    ro, rS, rg = _oracle_phase(d)
    assert relerr(o, ro) < TOL_F32 and relerr(S, rS) < TOL_F32
    for n in ("phw", "phq", "v", "beta", "g", "lam", "wr", "wi", "S0"):
        if rg[n] is not None:
            assert relerr(gr[n], rg[n]) < TOL_F32, n


@pytest.mark.parametrize("case", CASES[:3])
def test_phase_vs_oracle_bf16(case):
    B, T, H, Mh, V, be, g, lam = case
    d = seeded_phase_inputs(B, T, H, Mh, V, seed=7 * T + V, beta=be, g=g, lam=lam)
    d["v"] = torch.tensor(d["v"]).bfloat16().double().numpy()      # same bf16-rounded inputs
    d["dO"] = torch.tensor(d["dO"]).bfloat16().double().numpy()
    o, S, gr = _run_phase(d, d["dO"], d["dS"], dtype=torch.bfloat16)
    ro, rS, rg = _oracle_phase(d)
    u, ru = rms_np(o.detach().double().cpu().numpy().reshape(B, T, H, -1)), rms_np(ro.reshape(B, T, H, -1))
    assert np.abs(u - ru).max() < TOL_BF16_ABS and cosine(u, ru) > TOL_BF16_COS
    assert relerr(S, rS) < TOL_BF16_ABS and cosine(S, rS) > TOL_BF16_COS
    for n in ("phw", "phq", "v", "beta", "g", "lam", "wr", "wi", "S0"):
        if rg[n] is not None:
            assert relerr(gr[n], rg[n]) < TOL_BF16_ABS and cosine(gr[n], rg[n]) > TOL_BF16_COS, n


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("shape", [(2, 70, 2, 8, 6), (1, 129, 3, 32, 48)])
def test_key_vs_oracle(shape, dtype):
    ops = _ops()
    B, T, H, K, V = shape
    rng = np.random.default_rng(K * T)
    nrm = lambda x: x / np.linalg.norm(x, axis=-1, keepdims=True)
    q, k = nrm(rng.standard_normal((B, T, H, K))), nrm(rng.standard_normal((B, T, H, K)))
    v = rng.standard_normal((B, T, H, V))
    if dtype == torch.bfloat16:
        q, k, v = (torch.tensor(x).bfloat16().double().numpy() for x in (q, k, v))
    g = -np.log1p(np.exp(rng.standard_normal((B, T, H))))
    beta = 1 / (1 + np.exp(-rng.standard_normal((B, T, H))))
    S0 = 0.3 * rng.standard_normal((B, H, K, V))
    dO = rng.standard_normal((B, T, H, V))
    if dtype == torch.bfloat16:
        dO = torch.tensor(dO).bfloat16().double().numpy()
    t = dict(q=cuda(q, dtype, True), k=cuda(k, dtype, True), v=cuda(v, dtype, True),
             g=cuda(g, torch.float32, True), beta=cuda(beta, torch.float32, True),
             S0=cuda(S0, torch.float32, True))
    o, S = ops.key_scan(t["q"], t["k"], t["v"], t["g"], t["beta"], S0=t["S0"])
    (o.float() * cuda(dO)).sum().backward()
    ro, rS = ora.gdn_forward(q, k, v, g, beta, S0=S0, chunked=True, C=32)
    rg = ora.gdn_backward(q, k, v, g, beta, dO, S0=S0, chunked=True, C=32)
    if dtype == torch.float32:
        assert relerr(o, ro) < TOL_F32 and relerr(S, rS) < TOL_F32
        for n in rg:
            assert relerr(t[n].grad, rg[n]) < TOL_F32, n
    else:
        assert relerr(o, ro) < TOL_BF16_ABS and cosine(o, ro) > TOL_BF16_COS
        for n in rg:
            assert relerr(t[n].grad, rg[n]) < TOL_BF16_ABS and cosine(t[n].grad, rg[n]) > TOL_BF16_COS, n


@pytest.mark.parametrize("case", [(3, 5, 2, 16, 24, True, True, True), (2, 4, 4, 64, 128, True, False, True),
                                  (1, 3, 1, 6, 5, False, True, False),
                                  # persistent kernel, more (b, h) items than SMs (K = V = 128 and 64)
                                  (20, 3, 16, 64, 128, True, True, True), (10, 3, 16, 32, 64, True, False, True)])
def test_phase_step_vs_oracle(case):
    ops = _ops()
    B, T, H, Mh, V, be, g, lam = case
    d = seeded_phase_inputs(B, T, H, Mh, V, seed=3, beta=be, g=g, lam=lam)
    ro, rS = ora.phase_forward(d["phw"].astype(np.float64), d["phq"].astype(np.float64), d["v"], d["beta"],
                               d["g"], d["lam"], d["wr"], d["wi"], d["S0"])
    S = cuda(d["S0"]).contiguous()
    outs = []
    for t in range(T):
        sl = lambda x: None if x is None else cuda(x[:, t])
        o, S = ops.phase_step(sl(d["phw"]), sl(d["phq"]), sl(d["v"]), sl(d["beta"]), sl(d["g"]),
                              cuda(d["lam"]), cuda(d["wr"]), cuda(d["wi"]), S, S_out=S)
        outs.append(o)
    assert relerr(torch.stack(outs, 1), ro) < TOL_F32 and relerr(S, rS) < TOL_F32


def test_empty_sequence():
    ops = _ops()
    d = seeded_phase_inputs(2, 0, 2, 8, 8)
    o, S, _ = _run_phase(d, grad=False)
    assert o.shape[1] == 0 and relerr(S, d["S0"].astype(np.float32)) == 0.0


def test_strided_inputs():
    """Phases as views of a (B,T,H*Mh) projection and v as a slice of a wider tensor."""
    ops = _ops()
    B, T, H, Mh, V = 2, 50, 3, 8, 16
    d = seeded_phase_inputs(B, T, H, Mh, V, seed=11)
    big = torch.randn(B, T, H * Mh + 5, device="cuda")
    big[..., :H * Mh] = cuda(d["phw"]).reshape(B, T, H * Mh)
    phw = big[..., :H * Mh].unflatten(-1, (H, Mh))
    vv = torch.randn(B, T, H, V + 4, device="cuda")
    vv[..., :V] = cuda(d["v"])
    o, S = ops.phase_scan(phw, cuda(d["phq"]), vv[..., :V], cuda(d["beta"]), None, cuda(d["lam"]),
                          cuda(d["wr"]), cuda(d["wi"]), cuda(d["S0"]))
    ro, rS, _ = _oracle_phase(d, with_grad=False)
    assert relerr(o, ro) < TOL_F32 and relerr(S, rS) < TOL_F32


def test_errors_are_raised():
    ops = _ops()
    from sca2_b200._lib import Sca2Error
    d = seeded_phase_inputs(1, 8, 1, 4, 4)
    with pytest.raises(Sca2Error):
        ops.phase_scan(cuda(d["phw"]), cuda(d["phq"])[:, :4], cuda(d["v"]), wr=cuda(d["wr"]), wi=cuda(d["wi"]))
    with pytest.raises(Sca2Error):  # CPU tensors: no CPU path
        ops.phase_scan(torch.tensor(d["phw"]), torch.tensor(d["phq"]), torch.tensor(d["v"]).float(),
                       wr=torch.tensor(d["wr"]).float(), wi=torch.tensor(d["wi"]).float())
    with pytest.raises(Sca2Error):  # K > 128 is unsupported
        dd = seeded_phase_inputs(1, 4, 1, 80, 4)
        ops.phase_scan(cuda(dd["phw"]), cuda(dd["phq"]), cuda(dd["v"]), wr=cuda(dd["wr"]), wi=cuda(dd["wi"]))


# ------------------------------------------------------------------------------------------
#  3. full-size shapes
# ------------------------------------------------------------------------------------------
def test_full_size_phase_slices_bf16():
    """Benchmark workload (B=8, T=4096, H=16, d_head=64 -> Mh=32, V=64, bf16 v / dO, per-mode lam,
    delta beta): the whole batch runs on the GPU, four (b, h) sequences are checked against the
    oracle, fwd and bwd."""
    B, T, H, Mh, V = 8, 4096, 16, 32, 64
    d = seeded_phase_inputs(B, T, H, Mh, V, seed=2024, S0=False)
    d["v"] = torch.tensor(d["v"]).bfloat16().double().numpy()
    d["dO"] = torch.tensor(d["dO"]).bfloat16().double().numpy()
    o, S, gr = _run_phase(d, d["dO"], None, dtype=torch.bfloat16)
    for b, h in ((0, 0), (3, 7), (7, 15), (5, 2)):
        sl = {k: (None if d[k] is None else d[k][b:b + 1, :, h:h + 1])
              for k in ("phw", "phq", "v", "beta", "g", "dO")}
        sl.update(lam=d["lam"][h:h + 1], wr=d["wr"][h:h + 1], wi=d["wi"][h:h + 1], S0=None, dS=None)
        ro, rS, rg = _oracle_phase(sl)
        oo = o[b:b + 1, :, h:h + 1].detach().double().cpu().numpy()
        u, ru = rms_np(oo.reshape(1, T, 1, -1)), rms_np(ro.reshape(1, T, 1, -1))
        assert np.abs(u - ru).max() < TOL_BF16_ABS and cosine(u, ru) > TOL_BF16_COS
        assert relerr(S[b:b + 1, h:h + 1], rS) < TOL_BF16_ABS
        for n in ("phw", "phq", "v", "beta"):
            gg = gr[n][b:b + 1, :, h:h + 1]
            assert relerr(gg, rg[n]) < TOL_BF16_ABS and cosine(gg, rg[n]) > TOL_BF16_COS, n


def test_full_size_properties_fp32():
    """Size-independent properties at the benchmark shape in fp32: a prefill split at an
    arbitrary token equals one prefill; decode steps continuing a prefill equal the prefill."""
    ops = _ops()
    B, T, H, Mh, V = 8, 4096, 16, 32, 64
    d = seeded_phase_inputs(B, T, H, Mh, V, seed=99, g=True)
    t = {k: cuda(d[k]) for k in ("phw", "phq", "v", "beta", "g", "lam", "wr", "wi", "S0")}
    args = lambda a, b: [None if t[k] is None else t[k][:, a:b] for k in ("phw", "phq", "v", "beta", "g")]
    o, S = ops.phase_scan(*args(0, T), t["lam"], t["wr"], t["wi"], t["S0"])
    cut = 1500
    o1, S1 = ops.phase_scan(*args(0, cut), t["lam"], t["wr"], t["wi"], t["S0"])
    o2, S2 = ops.phase_scan(*args(cut, T), t["lam"], t["wr"], t["wi"], S1)
    assert relerr(torch.cat([o1, o2], 1), o) < TOL_F32 and relerr(S2, S) < TOL_F32
    Sd = S1.clone()
    for i in range(cut, cut + 8):
        od, Sd = ops.phase_step(t["phw"][:, i], t["phq"][:, i], t["v"][:, i], t["beta"][:, i], t["g"][:, i],
                                t["lam"], t["wr"], t["wi"], Sd, S_out=Sd)
        assert relerr(od, o[:, i]) < TOL_F32
    assert torch.isfinite(o).all() and torch.isfinite(S).all()


def test_full_size_key_slices():
    """Delta-rule workload (B=4, T=8192, H=8, K=V=128, bf16): two sequences vs the oracle."""
    ops = _ops()
    B, T, H, K, V = 4, 8192, 8, 128, 128
    gen = torch.Generator(device="cuda").manual_seed(5)
    rn = lambda *s: torch.randn(*s, device="cuda", generator=gen)
    q = torch.nn.functional.normalize(rn(B, T, H, K), dim=-1).bfloat16()
    k = torch.nn.functional.normalize(rn(B, T, H, K), dim=-1).bfloat16()
    v = rn(B, T, H, V).bfloat16()
    g = -torch.nn.functional.softplus(rn(B, T, H))
    beta = torch.sigmoid(rn(B, T, H))
    o, S = ops.key_scan(q, k, v, g, beta)
    for b, h in ((0, 0), (3, 6)):
        np_ = lambda x: x[b:b + 1, :, h:h + 1].double().cpu().numpy()
        ro, rS = ora.gdn_forward(np_(q), np_(k), np_(v), np_(g), np_(beta), chunked=True, C=64)
        oo = o[b:b + 1, :, h:h + 1]
        assert relerr(oo, ro) < TOL_BF16_ABS and cosine(oo, ro) > TOL_BF16_COS
        assert relerr(S[b:b + 1, h:h + 1], rS) < TOL_BF16_ABS


@pytest.mark.parametrize("shape", [(12, 3, 16, 64, 64), (3, 4, 2, 128, 128)])
def test_key_step_vs_oracle(shape):
    """GDN decode steps (persistent kernel for K = V = 64 / 128) against the oracle's scan."""
    ops = _ops()
    B, T, H, K, V = shape
    rng = np.random.default_rng(B * K + T)
    nrm = lambda x: x / np.linalg.norm(x, axis=-1, keepdims=True)
    q, k = nrm(rng.standard_normal((B, T, H, K))), nrm(rng.standard_normal((B, T, H, K)))
    v = rng.standard_normal((B, T, H, V))
    g = -np.log1p(np.exp(rng.standard_normal((B, T, H))))
    beta = 1 / (1 + np.exp(-rng.standard_normal((B, T, H))))
    S0 = 0.3 * rng.standard_normal((B, H, K, V))
    ro, rS = ora.gdn_forward(q, k, v, g, beta, S0=S0)
    S = cuda(S0).contiguous()
    outs = []
    for t in range(T):
        o, S = ops.key_step(cuda(q[:, t]), cuda(k[:, t]), cuda(v[:, t]), cuda(g[:, t]), cuda(beta[:, t]), S, S_out=S)
        outs.append(o)
    assert relerr(torch.stack(outs, 1), ro) < TOL_F32 and relerr(S, rS) < TOL_F32
