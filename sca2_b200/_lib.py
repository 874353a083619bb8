"""ctypes binding of libsca2b200.so (include/sca2b200.h).

The library is loaded from this package folder; there is no fallback: if it is missing
or fails to load, every op raises.  Structures mirror the C declarations field by field.
"""
from __future__ import annotations

import ctypes as C
import os
import threading

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libsca2b200.so")

SCA2_OK, SCA2_ERR_ARG, SCA2_ERR_UNSUPPORTED, SCA2_ERR_CUDA = 0, 1, 2, 3
SCA2_F32, SCA2_BF16 = 0, 1
SCA2_NOALLOC_SCRATCH_BYTES = 16 << 20  # include/sca2b200.h
FLAVOR_PHASE, FLAVOR_KEY = 0, 1


class Tok(C.Structure):
    _fields_ = [("ptr", C.c_void_p), ("sb", C.c_int64), ("st", C.c_int64), ("sh", C.c_int64)]


class Out(C.Structure):
    _fields_ = [("ptr", C.c_void_p), ("sb", C.c_int64), ("st", C.c_int64), ("sh", C.c_int64),
                ("sr", C.c_int64)]


class ScanArgs(C.Structure):
    _fields_ = [
        ("flavor", C.c_int32), ("B", C.c_int32), ("T", C.c_int32), ("H", C.c_int32),
        ("K", C.c_int32), ("V", C.c_int32), ("io_dtype", C.c_int32), ("v_times_beta", C.c_int32),
        ("q_scale", C.c_float),
        ("phw", Tok), ("phq", Tok), ("v", Tok), ("beta", Tok), ("g", Tok),
        ("lam", C.c_void_p), ("wr", C.c_void_p), ("wi", C.c_void_p), ("S0", C.c_void_p),
    ]


class ScanGrads(C.Structure):
    _fields_ = [
        ("dphw", Tok), ("dphq", Tok), ("dv", Tok), ("dbeta", Tok), ("dg", Tok),
        ("dlam", C.c_void_p), ("dwr", C.c_void_p), ("dwi", C.c_void_p), ("dS0", C.c_void_p),
        ("overwrite", C.c_int32), ("grad_io_dtype", C.c_int32),
    ]


class DScanArgs(C.Structure):
    _fields_ = [
        ("B", C.c_int32), ("T", C.c_int32), ("M", C.c_int32), ("G", C.c_int32), ("V", C.c_int32),
        ("sep", C.c_int32),
        ("a_re", C.c_void_p), ("a_im", C.c_void_p), ("v", C.c_void_p), ("c_re", C.c_void_p),
        ("c_im", C.c_void_p), ("S0_re", C.c_void_p), ("S0_im", C.c_void_p),
    ]


class PhaseProj(C.Structure):
    _fields_ = [("dtype", C.c_int32), ("theta", C.c_void_p), ("omega", C.c_void_p), ("pos", C.c_void_p)]


class ShortArgs(C.Structure):
    _fields_ = [
        ("B", C.c_int32), ("T", C.c_int32), ("L", C.c_int32), ("dv", C.c_int32),
        ("pos", C.c_void_p), ("kh", C.c_void_p), ("kz", C.c_void_p), ("v", C.c_void_p),
        ("theta", C.c_void_p), ("omega", C.c_void_p), ("wr", C.c_void_p), ("wi", C.c_void_p),
        ("c0", C.c_void_p), ("s0", C.c_void_p), ("e0", C.c_void_p),
    ]


class ShortGrads(C.Structure):
    _fields_ = [
        ("dkh", C.c_void_p), ("dkz", C.c_void_p), ("dv", C.c_void_p), ("dtheta", C.c_void_p),
        ("dwr", C.c_void_p), ("dwi", C.c_void_p), ("dc0", C.c_void_p), ("ds0", C.c_void_p),
        ("de0", C.c_void_p),
    ]


class DScanGrads(C.Structure):
    _fields_ = [
        ("da_re", C.c_void_p), ("da_im", C.c_void_p), ("dv", C.c_void_p), ("dc_re", C.c_void_p),
        ("dc_im", C.c_void_p), ("dS0_re", C.c_void_p), ("dS0_im", C.c_void_p),
    ]


# (name, restype, argtypes) of every exported symbol, in header order
SIGNATURES = [
    ("sca2_scan_fwd", C.c_int, [C.POINTER(ScanArgs), Out, C.c_void_p, C.c_void_p, C.c_void_p]),
    ("sca2_scan_value_tma", C.c_int, [C.POINTER(ScanArgs)]),
    ("sca2_num_chunks", C.c_int32, [C.c_int32]),
    ("sca2_scan_bwd", C.c_int, [C.POINTER(ScanArgs), Out, C.c_void_p, C.c_void_p,
                                C.POINTER(ScanGrads), C.c_void_p]),
    ("sca2_scan_step", C.c_int, [C.POINTER(ScanArgs), C.c_void_p, C.c_void_p, Out, C.c_void_p]),
    ("sca2_sepq_read_fwd", C.c_int, [C.c_void_p, C.c_void_p, C.c_void_p, C.c_int64, C.c_void_p, C.c_int64,
                                     C.c_int32, C.c_float, C.c_float, C.c_void_p]),
    ("sca2_sepq_read_bwd", C.c_int, [C.c_void_p, C.c_void_p, C.c_void_p, C.c_int64, C.c_void_p, C.c_void_p,
                                     C.c_void_p, C.c_void_p, C.c_int64, C.c_int64, C.c_int32, C.c_float, C.c_float,
                                     C.c_void_p]),
    ("sca2_layer_norm_supported", C.c_int, [C.c_int32]),
    ("sca2_layer_norm_fwd", C.c_int, [C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p,
                                      C.c_int64, C.c_int32, C.c_float, C.c_void_p]),
    ("sca2_layer_norm_work_floats", C.c_size_t, [C.c_int64, C.c_int32]),
    ("sca2_layer_norm_bwd", C.c_int, [C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p,
                                      C.c_void_p, C.c_void_p, C.c_void_p, C.c_int64, C.c_int32, C.c_void_p]),
    ("sca2_rms_heads_fwd", C.c_int, [C.c_void_p, C.c_int32, C.c_void_p, C.c_int64, C.c_int32, C.c_int32, C.c_float,
                                     C.c_void_p]),
    ("sca2_rms_heads_bwd", C.c_int, [C.c_void_p, C.c_int32, C.c_void_p, C.c_void_p, C.c_int64, C.c_int32, C.c_int32,
                                     C.c_float, C.c_void_p]),
    ("sca2_split_bf16", C.c_int, [C.c_void_p, C.c_int64, C.c_int32, C.c_int64, C.c_void_p, C.c_int64, C.c_int32,
                                  C.c_uint32, C.c_void_p]),
    ("sca2_rms_fwd", C.c_int, [C.c_void_p, C.c_void_p, C.c_int64, C.c_int32, C.c_float,
                               C.c_int32, C.c_void_p]),
    ("sca2_rms_bwd", C.c_int, [C.c_void_p, C.c_void_p, C.c_void_p, C.c_int64, C.c_int32,
                               C.c_float, C.c_int32, C.c_void_p]),
    ("sca2_dscan_num_ckpt", C.c_int32, [C.c_int32]),
    ("sca2_dscan_work_bytes", C.c_int64, [C.c_int32, C.c_int32, C.c_int32, C.c_int32, C.c_int32]),
    ("sca2_dscan_fwd", C.c_int, [C.POINTER(DScanArgs), C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p,
                                 C.c_void_p, C.c_void_p]),
    ("sca2_dscan_bwd", C.c_int, [C.POINTER(DScanArgs), C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p,
                                 C.POINTER(DScanGrads), C.c_void_p, C.c_void_p]),
    ("sca2_scan_proj_supported", C.c_int, [C.POINTER(ScanArgs), C.POINTER(PhaseProj), C.c_int32]),
    ("sca2_scan_fwd_proj", C.c_int, [C.POINTER(ScanArgs), C.POINTER(PhaseProj), Out, C.c_void_p, C.c_void_p,
                                     C.c_void_p]),
    ("sca2_scan_proj_work_bytes", C.c_int64, [C.c_int32, C.c_int32, C.c_int32, C.c_int32]),
    ("sca2_scan_fwd_work_bytes", C.c_int64, [C.POINTER(ScanArgs)]),
    ("sca2_scan_fwd_work", C.c_int, [C.POINTER(ScanArgs), C.POINTER(PhaseProj), Out, C.c_void_p, C.c_void_p,
                                     C.c_int64, C.c_void_p]),
    ("sca2_scan_bwd_proj", C.c_int, [C.POINTER(ScanArgs), C.POINTER(PhaseProj), Out, C.c_void_p, C.c_void_p,
                                     C.POINTER(ScanGrads), C.c_void_p, C.c_void_p, C.c_void_p]),
    ("sca2_short_fwd", C.c_int, [C.POINTER(ShortArgs), C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p,
                                 C.c_void_p]),
    ("sca2_short_work_bytes", C.c_int64, [C.c_int32, C.c_int32, C.c_int32, C.c_int32]),
    ("sca2_short_bwd", C.c_int, [C.POINTER(ShortArgs), C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p,
                                 C.POINTER(ShortGrads), C.c_void_p, C.c_void_p]),
    ("sca2_scan_fwd_bwd_noalloc", C.c_int, [C.POINTER(ScanArgs), Out, C.c_void_p, Out, C.c_void_p,
                                            C.POINTER(ScanGrads), C.c_void_p]),
    ("sca2_fault_status", C.c_int, [C.POINTER(C.c_uint32)]),
    ("sca2_last_error", C.c_char_p, []),
    ("sca2_version", C.c_char_p, []),
]

_lib = None
_lock = threading.Lock()


class Sca2Error(RuntimeError):
    pass


def load(path: str = LIB_PATH):
    """Load (once) and return the library handle with typed symbols."""
    global _lib
    with _lock:
        if _lib is not None:
            return _lib
        if not os.path.exists(path):
            raise Sca2Error(
                f"{path} is missing: build it with `python -m sca2_b200.build` "
                "(there is no CPU or PyTorch fallback for the scan)")
        lib = C.CDLL(path)
        for name, res, args in SIGNATURES:
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        _lib = lib
        return lib


def device_faults() -> int:
    """Read and clear the device fault word (bit 0: a tensor-core wait timed out)."""
    f = C.c_uint32(0)
    check(load().sca2_fault_status(C.byref(f)), "fault_status")
    return int(f.value)


def check(rc: int, what: str):
    if rc != SCA2_OK:
        msg = load().sca2_last_error().decode(errors="replace")
        kind = {SCA2_ERR_ARG: "invalid argument", SCA2_ERR_UNSUPPORTED: "unsupported",
                SCA2_ERR_CUDA: "CUDA error"}.get(rc, f"error {rc}")
        raise Sca2Error(f"{what}: {kind}: {msg}")
