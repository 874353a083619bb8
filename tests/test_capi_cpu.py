"""C ABI checks that need no GPU: the library loads, exports every function the header
declares, and the ctypes mirror of each struct has the C layout (compiled with gcc)."""
import ctypes
import os
import re
import shutil
import subprocess
import tempfile

import pytest

from sca2_b200 import _lib

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "sca2b200.h")


def _declared():
    src = open(HEADER).read()
    return sorted(set(re.findall(r"SCA2_API\s+[\w\s\*]*?\b(sca2_\w+)\s*\(", src)))


def test_library_exports_every_declared_symbol():
    lib = _lib.load()
    names = _declared()
    assert names, "no SCA2_API declarations found"
    for n in names:
        assert hasattr(lib, n), n
    assert sorted(n for n, _, _ in _lib.SIGNATURES) == names
    assert b"sm_100a" in lib.sca2_version()
    # four saved-state slots per 64-token chunk
    assert lib.sca2_num_chunks(4096) == 256 and lib.sca2_num_chunks(1) == 4 and lib.sca2_num_chunks(65) == 8
    assert lib.sca2_num_chunks(0) == 0


@pytest.mark.skipif(shutil.which("gcc") is None, reason="gcc not available")
def test_struct_layout_matches_header():
    probe = r"""
#include <stddef.h>
#include <stdio.h>
#include "sca2b200.h"
#define F(T, f) printf(#T "." #f " %zu\n", offsetof(T, f));
int main(void) {
  printf("sca2_tok %zu\nsca2_out %zu\nsca2_scan_args %zu\nsca2_scan_grads %zu\n",
         sizeof(sca2_tok), sizeof(sca2_out), sizeof(sca2_scan_args), sizeof(sca2_scan_grads));
  F(sca2_scan_args, q_scale) F(sca2_scan_args, phw) F(sca2_scan_args, g) F(sca2_scan_args, lam)
  F(sca2_scan_args, S0) F(sca2_scan_grads, dg) F(sca2_scan_grads, dlam) F(sca2_scan_grads, dS0)
  F(sca2_scan_grads, overwrite) F(sca2_scan_grads, grad_io_dtype)
  printf("sca2_dscan_args %zu\nsca2_dscan_grads %zu\n", sizeof(sca2_dscan_args), sizeof(sca2_dscan_grads));
  F(sca2_dscan_args, sep) F(sca2_dscan_args, a_re) F(sca2_dscan_args, S0_im)
  F(sca2_dscan_grads, dv) F(sca2_dscan_grads, dS0_im)
  printf("sca2_short_args %zu\nsca2_short_grads %zu\n", sizeof(sca2_short_args), sizeof(sca2_short_grads));
  F(sca2_short_args, pos) F(sca2_short_args, kh) F(sca2_short_args, omega) F(sca2_short_args, e0)
  F(sca2_short_grads, dv) F(sca2_short_grads, dtheta) F(sca2_short_grads, de0)
  printf("sca2_phase_proj %zu\n", sizeof(sca2_phase_proj));
  F(sca2_phase_proj, theta) F(sca2_phase_proj, pos)
  return 0;
}
"""
    with tempfile.TemporaryDirectory() as d:
        c = os.path.join(d, "probe.c")
        open(c, "w").write(probe)
        exe = os.path.join(d, "probe")
        subprocess.run(["gcc", "-I", os.path.dirname(HEADER), c, "-o", exe], check=True)
        out = dict(line.split() for line in subprocess.run([exe], capture_output=True, text=True,
                                                           check=True).stdout.splitlines())
    assert int(out["sca2_tok"]) == ctypes.sizeof(_lib.Tok)
    assert int(out["sca2_out"]) == ctypes.sizeof(_lib.Out)
    assert int(out["sca2_scan_args"]) == ctypes.sizeof(_lib.ScanArgs)
    assert int(out["sca2_scan_grads"]) == ctypes.sizeof(_lib.ScanGrads)
    assert int(out["sca2_dscan_args"]) == ctypes.sizeof(_lib.DScanArgs)
    assert int(out["sca2_dscan_grads"]) == ctypes.sizeof(_lib.DScanGrads)
    assert int(out["sca2_short_args"]) == ctypes.sizeof(_lib.ShortArgs)
    assert int(out["sca2_short_grads"]) == ctypes.sizeof(_lib.ShortGrads)
    assert int(out["sca2_phase_proj"]) == ctypes.sizeof(_lib.PhaseProj)
    for key, val in out.items():
        if "." in key:
            st, field = key.split(".")
            cls = {"sca2_scan_args": _lib.ScanArgs, "sca2_scan_grads": _lib.ScanGrads,
                   "sca2_dscan_args": _lib.DScanArgs, "sca2_dscan_grads": _lib.DScanGrads,
                   "sca2_short_args": _lib.ShortArgs, "sca2_short_grads": _lib.ShortGrads,
                   "sca2_phase_proj": _lib.PhaseProj}[st]
            assert getattr(cls, field).offset == int(val), key


def test_ops_refuse_cpu_tensors():
    """No CPU fallback: the product path raises on CPU tensors instead of computing."""
    import torch
    from sca2_b200 import ops
    x = torch.zeros(1, 4, 1, 2)
    with pytest.raises(_lib.Sca2Error):
        ops.phase_scan(x, x, torch.zeros(1, 4, 1, 3), wr=torch.ones(1, 2), wi=torch.zeros(1, 2))


def test_row_ops_refuse_cpu_tensors():
    """The read-out, split, 16-bit projection and LayerNorm ops have no CPU path either."""
    import torch
    from sca2_b200 import ops
    with pytest.raises(_lib.Sca2Error):
        ops.sepq_read(torch.zeros(2, 3, 2, 8), torch.zeros(2, 3, 16))
    with pytest.raises(_lib.Sca2Error):
        ops.rms_heads(torch.zeros(2, 3, 4, 2, 8))
    with pytest.raises(_lib.Sca2Error):
        ops.split_bf16(torch.zeros(4, 8), (False, True))
    with pytest.raises(_lib.Sca2Error):
        ops.linear16(torch.zeros(4, 8), torch.zeros(6, 8), (6,))
    with pytest.raises(_lib.Sca2Error):
        ops.layer_norm(torch.zeros(4, 128), torch.ones(128), torch.zeros(128))


def test_row_ops_entry_points_refuse_bad_sizes():
    """Argument checks of the new entry points run on the host before any launch (no device
    pointer is dereferenced), so they can be exercised without a GPU."""
    lib = _lib.load()
    assert lib.sca2_sepq_read_fwd(None, None, None, 4, None, 3, 8, 1e-6, 1e-6, None) != 0  # ld_q < dv
    assert lib.sca2_split_bf16(None, 2, 8, 8, None, 16, 9, 0, None) != 0                  # nblk > 8
    assert lib.sca2_rms_heads_fwd(None, 0, None, 2, 2, 6, 1e-6, None) != 0                # dvh % 4
    assert lib.sca2_layer_norm_supported(1024) == 1 and lib.sca2_layer_norm_supported(1000) == 0
    assert lib.sca2_layer_norm_fwd(None, None, None, None, None, None, 2, 1000, 1e-5, None) != 0
    assert lib.sca2_layer_norm_work_floats(0, 1024) == 0 and lib.sca2_layer_norm_work_floats(64, 1024) > 0


def test_inference_work_entry_refuses_bad_arguments():
    """The inference forward with a work buffer checks its arguments on the host before any
    launch: no argument struct is an error, and its work-size query answers 0 for it."""
    lib = _lib.load()
    assert lib.sca2_scan_fwd_work_bytes(None) == 0
    assert lib.sca2_scan_fwd_work(None, None, _lib.Out(None, 0, 0, 0, 0), None, None, 0, None) == _lib.SCA2_ERR_ARG
