"""Chunk-parallel training path of the explicit-key delta rule (K = V = 128, bf16 inputs, fp32
state): forward with saved chunk data + backward, against the numpy oracle.

Cases follow the gated-delta-rule workload (q, k L2-normalised, beta = sigmoid, g = -softplus):
ragged T (a partial last chunk), T = 1, no decay, the additive write (no beta), the erase form
without the value pre-scaled by beta, incoming state and state gradient; plus two (b, h)
sequences of the full B=4, T=8192, H=8 workload.  bf16 bar: max-abs / max-ref <= 2e-2 and
cosine >= 0.9999 on the outputs, the final state and every gradient.
"""
import numpy as np
import pytest
import torch

from oracle import scan as ora
from tests._util import TOL_BF16_ABS, TOL_BF16_COS, cosine, cuda, relerr

pytestmark = pytest.mark.gpu

K = V = 128


def _bf16r(x):
    return torch.tensor(np.asarray(x, np.float32)).bfloat16().double().numpy()


def _inputs(B, T, H, seed, g=True, beta=True, S0=True, dS=True):
    rng = np.random.default_rng(seed)
    nrm = lambda x: x / np.linalg.norm(x, axis=-1, keepdims=True)
    d = dict(q=_bf16r(nrm(rng.standard_normal((B, T, H, K)))), k=_bf16r(nrm(rng.standard_normal((B, T, H, K)))),
             v=_bf16r(rng.standard_normal((B, T, H, V))), dO=_bf16r(rng.standard_normal((B, T, H, V))))
    d["g"] = -np.log1p(np.exp(rng.standard_normal((B, T, H)))) if g else None
    d["beta"] = 1 / (1 + np.exp(-rng.standard_normal((B, T, H)))) if beta else None
    d["S0"] = 0.3 * rng.standard_normal((B, H, K, V)) if S0 else None
    d["dS"] = 0.3 * rng.standard_normal((B, H, K, V)) if dS else None
    return d


def _oracle(d, vtb):
    """Outputs, final state and gradients in float64 (oracle.scan's chunk closed form)."""
    scale = K ** -0.5
    if vtb:
        o, S = ora.gdn_forward(d["q"], d["k"], d["v"], d["g"], d["beta"], S0=d["S0"], chunked=True)
        g = ora.gdn_backward(d["q"], d["k"], d["v"], d["g"], d["beta"], d["dO"], S0=d["S0"], dS_final=d["dS"],
                             chunked=True)
        return o, S, g
    Q = (scale * d["q"])[..., None]
    o, S = ora.forward_chunked(d["k"], Q, d["v"], d["beta"], d["g"], None, 1.0, d["S0"])
    g = ora.backward_chunked(d["k"], Q, d["v"], d["beta"], d["g"], None, 1.0, d["S0"], d["dO"][:, :, :, None],
                             d["dS"])
    g["q"] = scale * g.pop("Q")[..., 0]
    return o[:, :, :, 0], S, g


def _run(d, vtb):
    from sca2_b200 import ops
    t = {n: (None if d[n] is None else cuda(d[n], torch.bfloat16 if n in "qkv" else torch.float32, True))
         for n in ("q", "k", "v", "g", "beta", "S0")}
    o, S = ops.key_scan(t["q"], t["k"], t["v"], t["g"], t["beta"], S0=t["S0"], v_times_beta=vtb)
    loss = (o.float() * cuda(d["dO"])).sum()
    if d["dS"] is not None:
        loss = loss + (S * cuda(d["dS"])).sum()
    loss.backward()
    torch.cuda.synchronize()
    return o, S, {n: (None if x is None else x.grad) for n, x in t.items()}


def _check(name, a, r):
    e, c = relerr(a, r), cosine(a, r)
    assert e < TOL_BF16_ABS and c > TOL_BF16_COS, (name, e, c)


CASES = [
    # B, T, H, g, beta, v_times_beta, S0, dS
    (2, 200, 2, True, True, True, True, True),
    (1, 64, 3, False, True, True, False, False),
    (2, 130, 1, True, False, False, True, True),
    (1, 129, 2, True, True, False, False, True),
    (3, 1, 2, True, True, True, True, False),
]


def test_cp_path_is_what_runs():
    """Training forward dispatches to the chunk-parallel kernels: its saved data has their
    layout (slot 4c+1 of chunk 0 holds T = (I + L)^{-1} in fp32 at float offset 64 V, after E in bf16:
    ones on the diagonal, zeros above it), not the fp32 path's per-32-token states."""
    from sca2_b200 import _lib, ops
    d = _inputs(1, 130, 2, seed=1)
    t = {n: cuda(d[n], torch.bfloat16 if n in "qkv" else torch.float32) for n in ("q", "k", "v", "g", "beta")}
    o, S, cs = torch.ops.sca2b200.key_scan_fwd(t["q"], t["k"], t["v"], t["g"], t["beta"], None, None, K ** -0.5,
                                               True, True)
    torch.cuda.synchronize()
    assert _lib.device_faults() == 0
    assert cs.shape == (1, 2, ops._slots(130), K, V)
    Tm = cs[0, 1, 1].reshape(-1)[64 * V:64 * V + 64 * 64].reshape(64, 64).double().cpu()
    assert torch.equal(torch.diagonal(Tm), torch.ones(64, dtype=torch.float64))
    assert torch.equal(torch.triu(Tm, 1), torch.zeros(64, 64, dtype=torch.float64))
    assert torch.tril(Tm, -1).abs().sum() > 0


@pytest.mark.parametrize("case", CASES)
def test_cp_train_vs_oracle(case):
    from sca2_b200 import _lib
    B, T, H, g, be, vtb, s0, ds = case
    d = _inputs(B, T, H, seed=B * T + H, g=g, beta=be, S0=s0, dS=ds)
    o, S, gr = _run(d, vtb)
    assert _lib.device_faults() == 0
    ro, rS, rg = _oracle(d, vtb)
    _check("o", o, ro)
    _check("S", S, rS)
    for n in ("q", "k", "v", "g", "beta", "S0"):
        if rg.get(n) is not None and gr.get(n) is not None:
            _check(n, gr[n], rg[n])


def test_cp_full_size_slices():
    """B=4, T=8192, H=8, K=V=128 training step; two (b, h) sequences against the oracle."""
    from sca2_b200 import _lib, ops
    B, T, H = 4, 8192, 8
    gen = torch.Generator(device="cuda").manual_seed(9)
    rn = lambda *s: torch.randn(*s, device="cuda", generator=gen)
    q = torch.nn.functional.normalize(rn(B, T, H, K), dim=-1).bfloat16().requires_grad_(True)
    k = torch.nn.functional.normalize(rn(B, T, H, K), dim=-1).bfloat16().requires_grad_(True)
    v = rn(B, T, H, V).bfloat16().requires_grad_(True)
    g = (-torch.nn.functional.softplus(rn(B, T, H))).requires_grad_(True)
    beta = torch.sigmoid(rn(B, T, H)).requires_grad_(True)
    dO = rn(B, T, H, V).bfloat16()
    o, S = ops.key_scan(q, k, v, g, beta)
    torch.autograd.backward(o, dO)
    torch.cuda.synchronize()
    assert _lib.device_faults() == 0
    for b, h in ((0, 0), (3, 6)):
        sl = lambda x: x[b:b + 1, :, h:h + 1].detach().double().cpu().numpy()
        d = dict(q=sl(q), k=sl(k), v=sl(v), g=sl(g), beta=sl(beta), dO=sl(dO), S0=None, dS=None)
        ro, rS, rg = _oracle(d, True)
        _check("o", o[b:b + 1, :, h:h + 1], ro)
        _check("S", S[b:b + 1, h:h + 1], rS)
        for n, x in (("q", q), ("k", k), ("v", v), ("g", g), ("beta", beta)):
            _check(n, x.grad[b:b + 1, :, h:h + 1], rg[n])


def test_cp_grad_dtypes_agree():
    """dq / dk written in bf16 (grad_io_dtype = 1, what the torch op uses) equal the fp32 ones of the
    same backward (grad_io_dtype = 0) up to bf16 rounding; grad_io_dtype = 1 is refused where the
    chunk-parallel path does not run."""
    from sca2_b200 import _lib, ops
    d = _inputs(2, 150, 2, seed=4)
    t = {n: cuda(d[n], torch.bfloat16 if n in "qkv" else torch.float32) for n in ("q", "k", "v", "g", "beta")}
    dO = cuda(d["dO"], torch.bfloat16)
    sc = K ** -0.5
    o, S, cs = torch.ops.sca2b200.key_scan_fwd(t["q"], t["k"], t["v"], t["g"], t["beta"], None, None, sc, True, True)
    dq16, dk16 = torch.ops.sca2b200.key_scan_bwd(t["q"], t["k"], t["v"], t["g"], t["beta"], None, None, sc, True, cs,
                                                 dO, None)[:2]
    assert dq16.dtype == torch.bfloat16 and dk16.dtype == torch.bfloat16

    def bwd(gio, k_width=K, cs_=cs, tt=t):
        B, T, H = 2, 150, 2
        a = ops._key_args(tt["q"], tt["k"], tt["v"], tt["g"], tt["beta"], None, None, sc, True)
        f = lambda *sh, dt=torch.float32: torch.empty(*sh, device="cuda", dtype=dt)
        gdt = torch.bfloat16 if gio else torch.float32
        dk, dq, dv = f(B, T, H, k_width, dt=gdt), f(B, T, H, k_width, dt=gdt), f(B, T, H, V, dt=torch.bfloat16)
        db, dg = f(B, T, H), f(B, T, H)
        gr = _lib.ScanGrads()
        gr.dphw, gr.dphq, gr.dv = ops._tok(dk), ops._tok(dq), ops._tok(dv)
        gr.dbeta, gr.dg = ops._tok(db), ops._tok(dg)
        gr.overwrite, gr.grad_io_dtype = 1, gio
        rc = _lib.load().sca2_scan_bwd(ops.C_ref(a), ops._out(dO.unsqueeze(3)), None, ops._ptr(cs_), ops.C_ref(gr),
                                       ops._stream())
        return rc, dq, dk
    rc, dq32, dk32 = bwd(0)
    assert rc == 0
    torch.cuda.synchronize()
    for a16, a32 in ((dq16, dq32), (dk16, dk32)):  # one bf16 rounding apart
        assert (a16.float() - a32).abs().max() <= 2 ** -8 * a32.abs().max()
    # K = 64: the tensor-core walk runs instead, which writes fp32 only
    d64 = {n: x[..., :64].contiguous() if n in "qk" else x for n, x in t.items()}
    o2, S2, cs2 = torch.ops.sca2b200.key_scan_fwd(d64["q"], d64["k"], d64["v"], d64["g"], d64["beta"], None, None,
                                                  sc, True, True)
    rc, _, _ = bwd(1, 64, cs2, d64)
    assert rc == _lib.SCA2_ERR_UNSUPPORTED
