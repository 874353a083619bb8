"""sincos_big (Cody-Waite reduction + SFU sine/cosine, used to build the phase codes of the
tensor-core kernels and of the short head) against float64 and against CUDA's sincosf over
the phase range of the benchmark workload (|phi| up to pi * 4096 plus noise)."""
import ctypes
import os
import subprocess

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu
HERE = os.path.dirname(os.path.abspath(__file__))


@pytest.fixture(scope="module")
def harness(tmp_path_factory):
    so = str(tmp_path_factory.mktemp("sincos") / "libsincos.so")
    subprocess.run(["nvcc", "-gencode", "arch=compute_100a,code=sm_100a", "-O3", "-std=c++17", "-Xcompiler",
                    "-fPIC", "-shared", "-o", so, os.path.join(HERE, "cuda", "sincos_check.cu")], check=True)
    lib = ctypes.CDLL(so)
    lib.sincos_check.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int]
    return lib


def test_sincos_big_error(harness):
    rng = np.random.default_rng(0)
    x = np.concatenate([rng.uniform(-np.pi, np.pi, 1 << 16), rng.uniform(-2e4, 2e4, 1 << 18),
                        np.arange(4096)[:, None].repeat(8, 1).ravel() * np.pi * 1e4 ** -np.linspace(0, 1, 8).repeat(4096)[: 4096 * 8]
                        ]).astype(np.float32)
    xt = torch.tensor(x, device="cuda")
    out = torch.empty(len(x), 4, device="cuda")
    assert harness.sincos_check(xt.data_ptr(), out.data_ptr(), len(x)) == 0
    o = out.double().cpu().numpy()
    xd = x.astype(np.float64)
    err_big = max(np.abs(o[:, 0] - np.sin(xd)).max(), np.abs(o[:, 1] - np.cos(xd)).max())
    err_lib = max(np.abs(o[:, 2] - np.sin(xd)).max(), np.abs(o[:, 3] - np.cos(xd)).max())
    assert err_big < 4e-6, (err_big, err_lib)
