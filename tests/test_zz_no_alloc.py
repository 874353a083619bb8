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
