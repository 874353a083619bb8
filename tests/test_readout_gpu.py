"""Separable D-head read-out (RMS fused) and the 16-bit projection ops against float64 torch
references of the reference's expressions (sca2/arch_sepq.py:93-104, sca2/ref.py:29-30):
forward and every gradient, vector and scalar kernel paths, strided query rows, empty input;
the bf16 hi / lo split bit for bit."""
import pytest
import torch

from tests._util import TOL_F32, relerr

pytestmark = pytest.mark.gpu


def _read_ref(ab, q, eps_q=1e-6, eps=1e-6):
    dv = ab.shape[-1]
    A, Bv = ab[..., 0, :], ab[..., 1, :]
    br, bi = q[..., :dv], q[..., dv:]
    n = torch.rsqrt(br.square() + bi.square() + eps_q)
    br, bi = br * n, bi * n
    u = torch.cat([br * A + bi * Bv, br * Bv - bi * A], -1)
    return u * torch.rsqrt(u.square().mean(-1, keepdim=True) + eps)


@pytest.mark.parametrize("shape,dv,strided", [((2, 37), 64, False), ((3, 5), 37, False), ((4, 96), 1024, True),
                                              ((1, 7), 6, True), ((2, 3), 128, False)])
def test_sepq_read_vs_torch(shape, dv, strided):
    from sca2_b200 import ops
    g = torch.Generator(device="cuda").manual_seed(dv)
    ab = torch.randn(*shape, 2, dv, device="cuda", generator=g)
    base = torch.randn(*shape, 2 * dv + (24 if strided else 0), device="cuda", generator=g)
    q = base[..., 8:8 + 2 * dv] if strided else base  # a column slice: row stride 2 dv + 24
    q = q.detach().requires_grad_(True)
    ab = ab.requires_grad_(True)
    dout = torch.randn(*shape, 2 * dv, device="cuda", generator=g)
    out = ops.sepq_read(ab, q)
    out.backward(dout)
    a64, q64 = ab.detach().double().requires_grad_(True), q.detach().double().requires_grad_(True)
    ref = _read_ref(a64, q64)
    ref.backward(dout.double())
    assert relerr(out, ref) < TOL_F32
    assert relerr(ab.grad, a64.grad) < TOL_F32 and relerr(q.grad, q64.grad) < TOL_F32


def test_sepq_read_empty():
    from sca2_b200 import ops
    ab = torch.zeros(2, 0, 2, 16, device="cuda")
    q = torch.zeros(2, 0, 32, device="cuda")
    assert ops.sepq_read(ab, q).shape == (2, 0, 32)


@pytest.mark.parametrize("rows,cols,lo", [(33, 64, (False, False, True)), (5, 37, (False, True)), (7, 8, (True,))])
def test_split_bf16_exact(rows, cols, lo):
    from sca2_b200 import ops
    x = torch.randn(rows, cols, device="cuda") * torch.logspace(-3, 3, cols, device="cuda")
    out = ops.split_bf16(x, lo)
    hi = x.to(torch.bfloat16)
    lo_v = (x - hi.float()).to(torch.bfloat16)
    for b, is_lo in enumerate(lo):
        blk = out[:, b * cols:(b + 1) * cols]
        assert torch.equal(blk, lo_v if is_lo else hi)


def test_linear16_16_bits():
    """Output and both gradients to about 16 significant bits (bar 2e-4 relative to the largest
    value), an order of magnitude inside bf16 and far inside the bf16 parity bar."""
    from sca2_b200 import ops
    g = torch.Generator(device="cuda").manual_seed(3)
    x = torch.randn(3, 50, 96, device="cuda", generator=g).requires_grad_(True)
    w = (0.05 * torch.randn(40, 96, device="cuda", generator=g)).requires_grad_(True)
    ya, yb = ops.linear16(x, w, (8, 32))
    da, db = torch.randn(150, 8, device="cuda", generator=g), torch.randn(150, 32, device="cuda", generator=g)
    ((ya * da).sum() + (yb * db).sum()).backward()
    x64, w64 = x.detach().double().requires_grad_(True), w.detach().double().requires_grad_(True)
    y64 = x64.reshape(150, 96) @ w64.t()
    (y64 * torch.cat([da, db], 1).double()).sum().backward()
    assert relerr(torch.cat([ya, yb], 1), y64) < 2e-4
    assert relerr(x.grad, x64.grad) < 2e-4 and relerr(w.grad, w64.grad) < 2e-4


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("lead,H,dvh", [((2, 33), 4, 64), ((5,), 1, 12), ((1, 3), 16, 8)])
def test_rms_heads_vs_torch(dtype, lead, H, dvh):
    """Gathered multi-head RMS read-out (sca2/arch_gatedc.py:155-156 + sca2/ref.py:29-30):
    fp32 output and the input gradient in the input's dtype (fp32 bar; bf16 inputs: the
    gradient's own bf16 rounding, 1e-2 relative)."""
    from sca2_b200 import ops
    g = torch.Generator(device="cuda").manual_seed(H * dvh)
    o = torch.randn(*lead, H, 2, dvh, device="cuda", generator=g).to(dtype).requires_grad_(True)
    du = torch.randn(*lead, 2 * H * dvh, device="cuda", generator=g)
    u = ops.rms_heads(o)
    u.backward(du)
    o64 = o.detach().double().requires_grad_(True)
    cat = torch.cat([o64[..., 0, :].reshape(*lead, -1), o64[..., 1, :].reshape(*lead, -1)], -1)
    ref = cat * torch.rsqrt(cat.square().mean(-1, keepdim=True) + 1e-6)
    ref.backward(du.double())
    assert u.dtype == torch.float32 and o.grad.dtype == dtype
    assert relerr(u, ref) < TOL_F32
    assert relerr(o.grad, o64.grad) < (TOL_F32 if dtype == torch.float32 else 1e-2)


@pytest.mark.parametrize("d,rows", [(1024, 300), (768, 33), (128, 5000), (384, 1)])
def test_layer_norm_vs_torch(d, rows):
    """The layers' LayerNorm kernels against torch.nn.functional.layer_norm in float64: output,
    input, weight and bias gradients (fp32 bar), many rows per CTA in the backward's sums."""
    from sca2_b200 import ops
    g = torch.Generator(device="cuda").manual_seed(d + rows)
    x = (3 * torch.randn(rows, d, device="cuda", generator=g) + 1).requires_grad_(True)
    w = torch.randn(d, device="cuda", generator=g).requires_grad_(True)
    b = torch.randn(d, device="cuda", generator=g).requires_grad_(True)
    dy = torch.randn(rows, d, device="cuda", generator=g)
    assert ops.layer_norm_supported(d)
    y = ops.layer_norm(x, w, b, 1e-5)
    y.backward(dy)
    x64, w64, b64 = (t.detach().double().requires_grad_(True) for t in (x, w, b))
    ref = torch.nn.functional.layer_norm(x64, (d,), w64, b64, 1e-5)
    ref.backward(dy.double())
    assert relerr(y, ref) < TOL_F32
    for t, r in ((x, x64), (w, w64), (b, b64)):
        assert relerr(t.grad, r.grad) < TOL_F32
