"""The custom ops under torch's own checks and torch.compile: torch.library.opcheck (schema,
fake implementation, autograd registration, AOT dispatch) for each op, and whole heads traced
with fullgraph=True (no graph break: every kernel call is a registered op) giving the eager
outputs and gradients."""
import pytest
import torch

from tests._util import relerr

pytestmark = pytest.mark.gpu


def _phase_inputs(B=2, T=100, H=2, Mh=32, V=64, grad=True):
    g = torch.Generator(device="cuda").manual_seed(0)
    rn = lambda *s: torch.randn(*s, device="cuda", generator=g)
    t = dict(phw=rn(B, T, H, Mh), phq=rn(B, T, H, Mh), v=rn(B, T, H, V).bfloat16(),
             beta=torch.sigmoid(rn(B, T, H)), lam=0.05 * torch.rand(H, Mh, device="cuda", generator=g),
             wr=1 + 0.3 * rn(H, Mh), wi=0.3 * rn(H, Mh))
    if grad:
        for k in ("phw", "phq", "v", "beta"):
            t[k].requires_grad_(True)
    return t


def test_opcheck_phase_scan():
    from sca2_b200 import ops  # noqa: F401
    t = _phase_inputs()
    args = (t["phw"], t["phq"], t["v"], t["beta"], None, t["lam"], t["wr"], t["wi"], None, True)
    torch.library.opcheck(torch.ops.sca2b200.phase_scan_fwd, args,
                          test_utils=("test_schema", "test_autograd_registration", "test_faketensor"))


def test_opcheck_key_scan_bwd_chunk_parallel():
    """The explicit-key backward at bf16, K = V = 128 writes its workspace into the chunk-state
    buffer: opcheck's schema test checks that the op declares that mutation."""
    from sca2_b200 import ops
    g = torch.Generator(device="cuda").manual_seed(2)
    rn = lambda *s: torch.randn(*s, device="cuda", generator=g)
    B, T, H, K = 1, 130, 2, 128
    q = torch.nn.functional.normalize(rn(B, T, H, K), dim=-1).bfloat16()
    k = torch.nn.functional.normalize(rn(B, T, H, K), dim=-1).bfloat16()
    v = rn(B, T, H, K).bfloat16()
    gg = -torch.nn.functional.softplus(rn(B, T, H))
    beta = torch.sigmoid(rn(B, T, H))
    o, S, cs = torch.ops.sca2b200.key_scan_fwd(q, k, v, gg, beta, None, None, K ** -0.5, True, True)
    do = rn(B, T, H, K).bfloat16()
    args = (q, k, v, gg, beta, None, None, K ** -0.5, True, cs, do, None)
    torch.library.opcheck(torch.ops.sca2b200.key_scan_bwd, args, test_utils=("test_schema", "test_faketensor"))
    # a second backward over the retained graph reads the forward's saved slots, which the
    # first backward left intact: it gives the same gradients again
    vv = v.clone().requires_grad_(True)
    o2, _ = ops.key_scan(q, k, vv, gg, beta)
    o2.backward(do, retain_graph=True)
    g1 = vv.grad.clone()
    o2.backward(do)
    assert relerr(vv.grad, 2 * g1) < 1e-2


@pytest.mark.parametrize("op", ["rms", "dscan", "short"])
def test_opcheck_small_ops(op):
    from sca2_b200 import ops  # noqa: F401
    g = torch.Generator(device="cuda").manual_seed(1)
    rn = lambda *s: torch.randn(*s, device="cuda", generator=g, requires_grad=True)
    if op == "rms":
        torch.library.opcheck(torch.ops.sca2b200.rms_fwd, (rn(4, 10, 64), 1e-6))
    elif op == "dscan":
        args = (0.5 * rn(2, 70, 4, 8), 0.5 * rn(2, 70, 4, 8), rn(2, 70, 64), rn(2, 70, 4), rn(2, 70, 4), None, None,
                True, True, True)
        torch.library.opcheck(torch.ops.sca2b200.dscan_fwd, args,
                              test_utils=("test_schema", "test_autograd_registration", "test_faketensor"))
    else:
        L, dv = 8, 16
        om = torch.arange(L, device="cuda", dtype=torch.float32) * (6.283185307179586 / L)
        args = (rn(2, 50, L), rn(2, 50, L), rn(2, 50, dv), rn(L), om, rn(L), rn(L), None, None, None, None)
        torch.library.opcheck(torch.ops.sca2b200.short_fwd, args,
                              test_utils=("test_schema", "test_autograd_registration", "test_faketensor"))


def test_long_head_compiles_fullgraph():
    """A LapA long head's prefill + backward traced by torch.compile without graph breaks."""
    from sca2_b200 import heads
    torch.manual_seed(0)
    head = heads.LongHead(heads.LaplaceConfig(d=64, M=32, dv=64, chunk=64, theta_scale=0.3)).cuda()
    z = torch.randn(2, 130, 64, device="cuda", requires_grad=True)
    h = torch.randn(2, 130, 64, device="cuda", requires_grad=True)

    def run(fn):
        z.grad = h.grad = None
        for p in head.parameters():
            p.grad = None
        u, st = fn(z, h)
        (u.square().sum() + st["sr"].sum()).backward()
        return [u.detach(), st["sr"].detach(), z.grad.clone(), h.grad.clone()] + [p.grad.clone() for p in head.parameters()]

    eager = run(lambda a, b: head.prefill(a, b))
    comp = run(torch.compile(lambda a, b: head.prefill(a, b), fullgraph=True))
    # outputs and input gradients at the fp32 bar; the per-mode parameter gradients are sums
    # over tokens with cancellation, and inductor's fused elementwise code rounds the phases
    # (positions x omega up to ~400 rad) differently from eager, so they get 1e-2
    for k, (x, y) in enumerate(zip(comp, eager)):
        assert relerr(x, y) < (1e-4 if k < 4 else 1e-2), k


def test_short_head_step_compiles_fullgraph():
    from sca2_b200 import heads
    torch.manual_seed(0)
    head = heads.ShortHead(heads.LaplaceConfig(d=32, L=8, dv=16)).cuda()
    st = head.init_state(3, "cuda")
    z, h = torch.randn(3, 32, device="cuda"), torch.randn(3, 32, device="cuda")
    with torch.no_grad():
        u0, s0 = head.step(z, h, st)
        u1, s1 = torch.compile(head.step, fullgraph=True)(z, h, st)
    assert relerr(u1, u0) < 1e-5 and relerr(s1["e"], s0["e"]) < 1e-6
