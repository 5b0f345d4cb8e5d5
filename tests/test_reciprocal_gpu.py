"""The Sinkhorn-Knopp kernels' reciprocal (rcp_rn in sinkhorn_n4.cuh: the
hardware approximation plus one Newton step on a fused multiply-add) is the
correctly rounded reciprocal: equal to CUDA's __frcp_rn on every one of the
2^32 float inputs, bit for bit, with the kernels' flush-to-zero; and the
kernels' factor sk_inv(s, 1e-8) equals (s > 1e-8 ? __frcp_rn(s) : 0) on all of
them.  The check is a small CUDA program built here against the shipped
header."""
import os
import shutil
import subprocess

import pytest

from conftest import ROOT

pytestmark = pytest.mark.gpu

CSRC = os.path.join(ROOT, "mhc-proj_b200", "csrc")
NVCC = os.path.join(os.environ.get("CUDA_HOME", "/usr/local/cuda"), "bin", "nvcc")


def test_rcp_rn_equals_frcp_rn_on_all_inputs(tmp_path):
    if not os.path.exists(NVCC) and shutil.which("nvcc") is None:
        pytest.skip("nvcc is not available")
    exe = str(tmp_path / "rcp_exhaustive")
    src = os.path.join(ROOT, "tests", "rcp_exhaustive.cu")
    subprocess.run([NVCC if os.path.exists(NVCC) else "nvcc", "-O3", "-std=c++17",
                    "-gencode", "arch=compute_100a,code=sm_100a", "-ftz=true", "-prec-div=true",
                    "-prec-sqrt=true", "-fmad=true", "-I", CSRC, "-o", exe, src], check=True)
    out = subprocess.run([exe], check=True, capture_output=True, text=True, timeout=300).stdout
    assert "status=no error" in out, out
    assert "mismatches=0" in out.splitlines()[0], out
