"""The allocation-free entry point sca2_scan_fwd_bwd_noalloc, for callers that cannot
allocate device memory (a plugin inside a runtime that owns the device memory pool, or a
path where cudaMalloc must not be called): its chunk states live in the library's static
16 MiB device array instead of a caller workspace.

Checked through the C ABI against the two-call path (sca2_scan_fwd + sca2_scan_bwd with a
caller-provided chunk-state buffer), on two calls in a row, so that the second call reuses
the shared array the first one left behind.  Kept in its own file, collected last.
"""
import ctypes

import numpy as np
import pytest
import torch

from tests._util import (TOL_BF16_ABS, TOL_BF16_COS, TOL_F32, cosine, cuda, relerr,
                         seeded_phase_inputs)

pytestmark = pytest.mark.gpu

NAMES = ("phw", "phq", "v", "beta", "g", "lam", "wr", "wi", "S0")


def _two_call(d, dtype):
    from sca2_b200 import ops
    t = {k: cuda(d[k]) for k in NAMES}
    t["v"] = cuda(d["v"], dtype)
    plan = ops.PhaseScanPlan(t["phw"], t["phq"], t["v"], t["beta"], t["g"], t["lam"], t["wr"], t["wi"], t["S0"])
    o, S = plan.fwd()
    grads = plan.bwd(cuda(d["dO"], dtype), cuda(d["dS"]))
    return o.clone(), S.clone(), {k: (None if x is None else x.clone()) for k, x in grads.items()}, t


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_noalloc_matches_two_call_path(dtype):
    from sca2_b200 import ops
    d = seeded_phase_inputs(2, 100, 3, 16, 40, seed=31, beta=True, g=True, lam=True)
    ro, rS, rg, t = _two_call(d, dtype)
    for call in range(2):  # the second call reuses what the first left in the shared array
        o, S, G = ops.phase_scan_fwd_bwd_noalloc(t["phw"], t["phq"], t["v"], t["beta"], t["g"], t["lam"],
                                                 t["wr"], t["wi"], cuda(d["dO"], dtype), t["S0"],
                                                 cuda(d["dS"]))
        torch.cuda.synchronize()
        if dtype == torch.float32:
            assert relerr(o, ro) < TOL_F32 and relerr(S, rS) < TOL_F32, call
            for k in rg:
                if rg[k] is not None:
                    assert relerr(G[k], rg[k]) < TOL_F32, (call, k)
        else:
            assert relerr(o, ro) < TOL_BF16_ABS and cosine(o, ro) > TOL_BF16_COS, call
            for k in rg:
                if rg[k] is not None:
                    assert relerr(G[k], rg[k]) < TOL_BF16_ABS and cosine(G[k], rg[k]) > TOL_BF16_COS, (call, k)


def test_noalloc_phase_tensor_core_shape():
    """bf16, K = 2 Mh = 64, V = 64: the tensor-core path (chunk-parallel inversion, saved T, E
    and P in the shared array)."""
    from sca2_b200 import ops
    d = seeded_phase_inputs(1, 200, 2, 32, 64, seed=32, beta=True, g=False, lam=True)
    ro, rS, rg, t = _two_call(d, torch.bfloat16)
    for call in range(2):
        o, S, G = ops.phase_scan_fwd_bwd_noalloc(t["phw"], t["phq"], t["v"], t["beta"], t["g"], t["lam"],
                                                 t["wr"], t["wi"], cuda(d["dO"], torch.bfloat16), t["S0"],
                                                 cuda(d["dS"]))
        torch.cuda.synchronize()
        assert relerr(o, ro) < TOL_BF16_ABS and cosine(o, ro) > TOL_BF16_COS, call
        assert relerr(S, rS) < TOL_BF16_ABS and cosine(S, rS) > TOL_BF16_COS, call
        for k in rg:
            if rg[k] is not None:
                assert relerr(G[k], rg[k]) < TOL_BF16_ABS and cosine(G[k], rg[k]) > TOL_BF16_COS, (call, k)


def _key_call(lib, a, o, S, cs, do, grads, noalloc):
    """One forward + backward of the explicit-key scan through the C ABI: the two-call path
    with a caller chunk-state buffer, or the allocation-free entry point."""
    from sca2_b200 import _lib, ops
    st = torch.cuda.current_stream().cuda_stream
    gr = _lib.ScanGrads()
    gr.dphw, gr.dphq, gr.dv = ops._tok(grads["k"]), ops._tok(grads["q"]), ops._tok(grads["v"])
    gr.dbeta, gr.dg = ops._tok(grads["beta"]), ops._tok(grads["g"])
    gr.dS0 = grads["S0"].data_ptr()
    gr.overwrite = 1
    oo, dd = ops._out(o.unsqueeze(3)), ops._out(do.unsqueeze(3))
    if noalloc:
        rc = lib.sca2_scan_fwd_bwd_noalloc(ctypes.byref(a), oo, S.data_ptr(), dd, None, ctypes.byref(gr), st)
        assert rc == 0, lib.sca2_last_error().decode()
        return
    assert lib.sca2_scan_fwd(ctypes.byref(a), oo, S.data_ptr(), cs.data_ptr(), st) == 0, lib.sca2_last_error()
    assert lib.sca2_scan_bwd(ctypes.byref(a), dd, None, cs.data_ptr(), ctypes.byref(gr), st) == 0, \
        lib.sca2_last_error()


def test_noalloc_key_chunk_parallel_shape():
    """bf16 explicit keys at K = V = 128 (B = 1, H = 2, T = 256: 2 MiB of the array): the
    chunk-parallel path, whose backward also uses the shared array as its workspace."""
    from sca2_b200 import _lib, ops
    lib = _lib.load()
    g = torch.Generator(device="cuda").manual_seed(33)
    rn = lambda *s: torch.randn(*s, device="cuda", generator=g)
    B, T, H, K = 1, 256, 2, 128
    q = torch.nn.functional.normalize(rn(B, T, H, K), dim=-1).bfloat16()
    k = torch.nn.functional.normalize(rn(B, T, H, K), dim=-1).bfloat16()
    v = rn(B, T, H, K).bfloat16()
    gg = -torch.nn.functional.softplus(rn(B, T, H))
    beta = torch.sigmoid(rn(B, T, H))
    S0 = 0.3 * rn(B, H, K, K)
    do = rn(B, T, H, K).bfloat16()
    a = ops._key_args(q, k, v, gg, beta, None, S0, K ** -0.5, True)
    need = B * H * lib.sca2_num_chunks(T) * K * K * 4
    assert need <= _lib.SCA2_NOALLOC_SCRATCH_BYTES

    def buffers():
        f = lambda *s: torch.empty(*s, device="cuda", dtype=torch.float32)
        return (torch.empty(B, T, H, K, device="cuda", dtype=torch.bfloat16), f(B, H, K, K),
                dict(k=f(B, T, H, K), q=f(B, T, H, K), v=torch.empty(B, T, H, K, device="cuda", dtype=torch.bfloat16),
                     beta=f(B, T, H), g=f(B, T, H), S0=f(B, H, K, K)))

    ro, rS, rg = buffers()
    cs = torch.empty(B, H, lib.sca2_num_chunks(T), K, K, device="cuda", dtype=torch.float32)
    _key_call(lib, a, ro, rS, cs, do, rg, noalloc=False)
    for call in range(2):
        o, S, G = buffers()
        _key_call(lib, a, o, S, None, do, G, noalloc=True)
        torch.cuda.synchronize()
        assert relerr(o, ro) < TOL_BF16_ABS and cosine(o, ro) > TOL_BF16_COS, call
        assert relerr(S, rS) < TOL_BF16_ABS and cosine(S, rS) > TOL_BF16_COS, call
        for name in rg:
            assert relerr(G[name], rg[name]) < TOL_BF16_ABS and cosine(G[name], rg[name]) > TOL_BF16_COS, \
                (call, name)


def test_noalloc_rejects_oversized_problems():
    """A problem whose chunk states exceed the static array is refused before any launch."""
    from sca2_b200 import _lib, ops
    d = seeded_phase_inputs(1, 8, 1, 4, 4, seed=1)
    t = {k: cuda(d[k]) for k in NAMES}
    a = ops._phase_args(t["phw"], t["phq"], t["v"], t["beta"], t["g"], t["lam"], t["wr"], t["wi"], t["S0"])
    a.B, a.T, a.H, a.K, a.V = 64, 4096, 16, 64, 64   # 2 GiB of chunk states
    gr = _lib.ScanGrads()
    rc = _lib.load().sca2_scan_fwd_bwd_noalloc(ctypes.byref(a), _lib.Out(), None, _lib.Out(), None,
                                               ctypes.byref(gr), torch.cuda.current_stream().cuda_stream)
    assert rc == _lib.SCA2_ERR_ARG
    msg = _lib.load().sca2_last_error().decode()
    assert "scratch" in msg and str(_lib.SCA2_NOALLOC_SCRATCH_BYTES) in msg
