"""The forward after the caller resets the device.

The persistent forward needs a per-function attribute (100 KB of dynamic
shared memory per block) that belongs to the CUDA context.  A process that
calls cudaDeviceReset and projects again gets a new context without it; the
launcher must set it again rather than fail.  Run in a fresh process that
uses the CUDA runtime directly (no PyTorch state to invalidate); a regression
shows as a non-zero status, not a fault."""
import os
import subprocess
import sys

import pytest

pytestmark = pytest.mark.gpu

SCRIPT = r"""
import ctypes, sys
import numpy as np
sys.path.insert(0, sys.argv[1])
from mhc_proj import capi
L = capi.lib()
rt = ctypes.CDLL("libcudart.so.12")
rt.cudaMalloc.argtypes = [ctypes.POINTER(ctypes.c_void_p), ctypes.c_size_t]
rt.cudaMemcpy.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_size_t, ctypes.c_int]
rt.cudaFree.argtypes = [ctypes.c_void_p]
n = 1 << 16  # above the small-batch threshold: the persistent kernel
R = np.random.default_rng(0).standard_normal((n, 4, 4), dtype=np.float32)

def project():
    dR, dT = ctypes.c_void_p(), ctypes.c_void_p()
    assert rt.cudaMalloc(ctypes.byref(dR), R.nbytes) == 0 and rt.cudaMalloc(ctypes.byref(dT), R.nbytes) == 0
    assert rt.cudaMemcpy(dR, R.ctypes.data, R.nbytes, 1) == 0
    status = L.mhc_birkhoff_proj_n4(dR, dT, ctypes.c_float(1e-6), n, None)
    T = np.empty_like(R)
    assert rt.cudaMemcpy(T.ctypes.data, dT, R.nbytes, 2) == 0
    rt.cudaFree(dR); rt.cudaFree(dT)
    return status, T

s1, T1 = project()
assert rt.cudaDeviceReset() == 0
s2, T2 = project()
print(s1, s2, int(np.array_equal(T1.view(np.int32), T2.view(np.int32))))
"""


def test_forward_after_device_reset():
    pkg = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "mhc-proj_b200")
    out = subprocess.run([sys.executable, "-c", SCRIPT, pkg], capture_output=True, text=True, timeout=300)
    assert out.returncode == 0, out.stderr
    assert out.stdout.split()[-3:] == ["0", "0", "1"], out.stdout
