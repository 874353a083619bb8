"""The torch custom ops (torch.ops.sca2b200.*) without a GPU: every op is registered, and
its fake (meta) implementation gives the shapes and dtypes the CUDA implementation returns,
so torch.compile can trace the heads through them.  The chunk-state slot count of the fake
forward equals the library's sca2_num_chunks."""
import torch
from torch._subclasses.fake_tensor import FakeTensorMode

from sca2_b200 import _lib, ops  # noqa: F401  (registers the ops)

OPS = ["phase_scan_fwd", "phase_scan_bwd", "key_scan_fwd", "key_scan_bwd", "phase_step", "phase_step_",
       "key_step", "key_step_", "dscan_fwd", "dscan_bwd", "short_fwd", "short_bwd", "rms_fwd", "rms_bwd"]


def test_ops_registered():
    for n in OPS:
        assert hasattr(torch.ops.sca2b200, n), n


def test_slot_count_matches_library():
    lib = _lib.load()
    for T in (1, 63, 64, 65, 4096, 4097):
        assert ops._slots(T) == lib.sca2_num_chunks(T)


def test_fake_shapes():
    with FakeTensorMode():
        d = "cuda"
        B, T, H, Mh, V = 2, 100, 2, 32, 64
        phw = torch.empty(B, T, H, Mh, device=d)
        v = torch.empty(B, T, H, V, device=d, dtype=torch.bfloat16)
        beta = torch.empty(B, T, H, device=d)
        w = torch.empty(H, Mh, device=d)
        o, S, cs = torch.ops.sca2b200.phase_scan_fwd(phw, phw, v, beta, None, w, w, w, None, True)
        assert o.shape == (B, T, H, 2, V) and o.dtype == torch.bfloat16
        assert S.shape == (B, H, 2 * Mh, V) and cs.shape == (B, H, ops._slots(T), 2 * Mh, V)
        g = torch.ops.sca2b200.phase_scan_bwd(phw, phw, v, beta, None, w, w, w, None, cs, o, None)
        assert [tuple(x.shape) for x in g] == [(B, T, H, Mh), (B, T, H, Mh), (B, T, H, V), (B, T, H), (0,),
                                               (H, Mh), (H, Mh), (H, Mh), (0,)]
        q = torch.empty(B, T, H, 128, device=d, dtype=torch.bfloat16)
        vk = torch.empty(B, T, H, 128, device=d, dtype=torch.bfloat16)
        o, S, cs = torch.ops.sca2b200.key_scan_fwd(q, q, vk, beta, beta, None, None, 0.1, True, False)
        assert o.shape == (B, T, H, 128) and S.shape == (B, H, 128, 128) and cs.numel() == 0
        St = torch.empty(B, H, 2 * Mh, V, device=d)
        ph = torch.empty(B, H, Mh, device=d)
        ot = torch.ops.sca2b200.phase_step_(ph, ph, torch.empty(B, H, V, device=d), None, None, None, w, w, St)
        assert ot.shape == (B, H, 2, V)
        a = torch.empty(B, T, 4, 8, device=d)
        ab, sr, si, ck = torch.ops.sca2b200.dscan_fwd(a, a, torch.empty(B, T, 64, device=d),
                                                      torch.empty(B, T, 4, device=d), torch.empty(B, T, 4, device=d),
                                                      None, None, True, True, True)
        assert ab.shape == (B, T, 2, 64) and sr.shape == (B, 4, 64) and ck.shape == (B, (T + 15) // 16, 2, 4, 64)
        L, dv = 16, 32
        kh = torch.empty(B, T, L, device=d)
        th = torch.empty(L, device=d)
        o, c1, s1, e1 = torch.ops.sca2b200.short_fwd(kh, kh, torch.empty(B, T, dv, device=d), th, th, th, th,
                                                     None, None, None, None)
        assert o.shape == (B, T, 2 * dv) and c1.shape == (B, L - 1, L) and e1.shape == (B, L - 1, dv)
        x = torch.empty(B, T, 128, device=d)
        assert torch.ops.sca2b200.rms_fwd(x, 1e-6).shape == x.shape
