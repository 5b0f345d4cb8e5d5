"""The no-allocation form of the fused H_res backward
(mhc_birkhoff_proj_n4_hres_backward_noalloc), for callers that cannot
allocate device memory -- a framework or serving engine that owns the
device's memory pool, or a loop that cannot afford cudaMalloc/cudaFree
synchronising the device.  It keeps its partial sums in a fixed array inside
the library instead of a caller workspace.

Collected last on purpose (the file name), so that a run that stops at the
first failure has run every other test before it; it also passes on its own
in a fresh process.  Two calls in a row, on different batches and sizes, each
give the bits of the workspace entry point on the same inputs (the tests'
tolerance for this backward is bitwise) -- the fixed array needs no reset
between calls."""
import os
import subprocess
import sys

import pytest
import torch

from mhc_proj import capi

pytestmark = pytest.mark.gpu


def inputs(n, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    H = torch.randn(n, 24, device="cuda", generator=g)
    rms = torch.rand(n, device="cuda", generator=g) * 1.5 + 0.5
    a = torch.tensor([0.9], device="cuda")
    b = torch.randn(16, device="cuda", generator=g) + 2.0 * torch.eye(4, device="cuda").reshape(16)
    G = torch.randn(n, 4, 4, device="cuda", generator=g)
    h = H[:, 8:24]
    T = capi.birkhoff_proj_n4_hres_tensor(h, rms, a, b)
    return G, T, h, rms, a


def outputs(n):
    return (torch.empty(n, 16, device="cuda"), torch.empty(n, device="cuda"), torch.empty((), device="cuda"),
            torch.empty(4, 4, device="cuda"))


def with_workspace(G, T, h, rms, a):
    n = h.shape[0]
    dh, drms, dalpha, db = outputs(n)
    nbytes = capi.birkhoff_proj_n4_hres_backward_workspace(n)
    ws = torch.empty(nbytes // 4, device="cuda")
    capi.birkhoff_proj_n4_hres_backward(G.data_ptr(), T.data_ptr(), h.data_ptr(), h.stride(0), rms.data_ptr(),
                                        a.data_ptr(), dh.data_ptr(), 16, drms.data_ptr(), dalpha.data_ptr(),
                                        db.data_ptr(), n, ws.data_ptr(), nbytes,
                                        torch.cuda.current_stream().cuda_stream)
    return dh, drms, dalpha, db


def without_allocation(G, T, h, rms, a):
    n = h.shape[0]
    dh, drms, dalpha, db = outputs(n)
    capi.birkhoff_proj_n4_hres_backward_noalloc(G.data_ptr(), T.data_ptr(), h.data_ptr(), h.stride(0),
                                                rms.data_ptr(), a.data_ptr(), dh.data_ptr(), 16, drms.data_ptr(),
                                                dalpha.data_ptr(), db.data_ptr(), n,
                                                torch.cuda.current_stream().cuda_stream)
    return dh, drms, dalpha, db


def same_bits(x, y):
    return torch.equal(x.contiguous().view(torch.int32), y.contiguous().view(torch.int32))


# The fixed array holds 1024 rows of partial sums.  The workspace form gives
# the same bits when it also uses at most 1024 blocks (one resident wave on
# this GPU); on a GPU with a larger wave its batch sums are added in another
# order and only agree to rounding.
NOALLOC_ROWS = 1024


def wave_fits(n):
    return capi.birkhoff_proj_n4_hres_backward_workspace(n) // (17 * 4) <= NOALLOC_ROWS


def agree(x, y, bitwise):
    if bitwise:
        return same_bits(x, y)
    return torch.allclose(x, y, rtol=1e-5, atol=1e-6)


def test_two_calls_in_a_row_match_the_workspace_entry_point():
    first = inputs(1 << 20, 1)
    second = inputs(77777, 2)
    got1 = without_allocation(*first)
    got2 = without_allocation(*second)  # reuses the same scratch right after the first call
    want1 = with_workspace(*first)
    want2 = with_workspace(*second)
    torch.cuda.synchronize()
    for g, w in zip(got1, want1):
        assert agree(g, w, wave_fits(1 << 20))
    for g, w in zip(got2, want2):
        assert agree(g, w, wave_fits(77777))


def test_empty_batch_writes_zero_sums():
    G, T, h, rms, a = inputs(0, 3)
    dh, drms, dalpha, db = outputs(0)
    dalpha.fill_(5.0)
    db.fill_(5.0)
    capi.birkhoff_proj_n4_hres_backward_noalloc(0, 0, 0, 24, 0, a.data_ptr(), 0, 16, 0, dalpha.data_ptr(),
                                                db.data_ptr(), 0, torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    assert float(dalpha) == 0.0 and bool((db == 0).all())


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_each_device_uses_its_own_array():
    """The array is looked up on the first call on each device: a call on the
    second GPU, right after one on the first, still matches the workspace
    form there, and the first GPU's results stay right afterwards."""
    first = inputs(50001, 3)
    got0 = without_allocation(*first)
    with torch.cuda.device(1):
        second = inputs(60007, 4)
        got1 = without_allocation(*second)
        want1 = with_workspace(*second)
        torch.cuda.synchronize()
        for g, w in zip(got1, want1):
            assert agree(g, w, wave_fits(60007))
    want0 = with_workspace(*first)
    again0 = without_allocation(*first)
    torch.cuda.synchronize()
    for g, a, w in zip(got0, again0, want0):
        assert agree(g, w, wave_fits(50001)) and same_bits(a, g)


FIRST_CALL_IN_CAPTURE = r"""
import sys
sys.path.insert(0, sys.argv[1])
import torch
from mhc_proj import capi
n = 4096
G = torch.randn(n, 4, 4, device="cuda"); T = torch.rand(n, 4, 4, device="cuda")
h = torch.randn(n, 16, device="cuda"); rms = torch.ones(n, device="cuda"); a = torch.ones(1, device="cuda")
dh = torch.empty(n, 16, device="cuda"); drms = torch.empty(n, device="cuda")
dalpha = torch.empty((), device="cuda"); db = torch.empty(4, 4, device="cuda")
args = (G.data_ptr(), T.data_ptr(), h.data_ptr(), 16, rms.data_ptr(), a.data_ptr(), dh.data_ptr(), 16,
        drms.data_ptr(), dalpha.data_ptr(), db.data_ptr(), n)
L = capi.lib()
s = torch.cuda.Stream()
torch.cuda.synchronize()
g = torch.cuda.CUDAGraph()
with torch.cuda.graph(g, stream=s):
    status = L.mhc_birkhoff_proj_n4_hres_backward_noalloc(*args, s.cuda_stream)
del g
print(status)
"""


def test_first_call_during_capture_is_refused():
    """In a fresh process the first call must look the array's address up;
    made inside a stream capture it launches nothing and returns
    MHC_ERR_CAPTURE instead of running the lookup inside the capture."""
    pkg = os.path.dirname(os.path.dirname(capi.__file__))
    out = subprocess.run([sys.executable, "-c", FIRST_CALL_IN_CAPTURE, pkg], capture_output=True, text=True,
                         timeout=300)
    assert out.returncode == 0, out.stderr
    assert int(out.stdout.strip().splitlines()[-1]) == capi.MHC_ERR_CAPTURE
