"""Small batches take the two-lanes-per-matrix forward (batches up to 2^13
matrices; mhc_birkhoff_proj_n4 and mhc_birkhoff_proj_n4_ex dispatch by N).
It must give the reference kernel's bits and the persistent kernel's (the
stats entry point always runs the persistent kernel), on every distribution,
on both sides of the threshold, for the native storage types and strides."""
import pytest
import torch

import mhc_proj
import oracle
from mhc_proj import capi
from mhc_proj.workloads import make_logits

pytestmark = pytest.mark.gpu

PAIR_MAX_N = 1 << 13


def same_bits(a, b):
    return torch.equal(a.contiguous().view(torch.int16 if a.element_size() == 2 else torch.int32),
                       b.contiguous().view(torch.int16 if b.element_size() == 2 else torch.int32))


def persistent(R, tol):
    n = R.shape[0]
    T = torch.empty_like(R)
    it = torch.empty(n, dtype=torch.int32, device="cuda")
    gn = torch.empty(n, device="cuda")
    capi.birkhoff_proj_n4_stats(R.data_ptr(), T.data_ptr(), tol, n, it.data_ptr(), gn.data_ptr(),
                                torch.cuda.current_stream().cuda_stream)
    return T


@pytest.mark.parametrize("kind", ["normal", "sigma_mix", "mixture", "wide", "uniform"])
@pytest.mark.parametrize("n", [1, 2, 15, 16, 17, 1000, PAIR_MAX_N, PAIR_MAX_N + 1])
@pytest.mark.parametrize("tol", [1e-6, 0.0, float("inf")])
def test_small_batches_bitwise(kind, n, tol):
    R = make_logits(kind, n, seed=n + 3)
    T = capi.birkhoff_proj_n4_tensor(R, tol)
    assert same_bits(T, persistent(R, tol))
    if oracle.RefCuda.available():
        ref = oracle.RefCuda()
        Tr = torch.empty_like(R)
        ref.birkhoff_proj_n4(R.data_ptr(), Tr.data_ptr(), tol, n, torch.cuda.current_stream().cuda_stream)
        torch.cuda.synchronize()
        assert same_bits(T, Tr)


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16, torch.float16])
@pytest.mark.parametrize("stride,offset", [(16, 0), (24, 8), (20, 4), (16, 1)])
def test_small_native_types_and_strides(dtype, stride, offset):
    n = 3001
    full = make_logits("sigma_mix", n * stride // 16 + 2, seed=stride).reshape(-1)
    buf = torch.empty(n * stride + 16, device="cuda", dtype=dtype)
    buf.copy_(full[: buf.numel()].to(dtype))
    R = torch.as_strided(buf, (n, 4, 4), (stride, 4, 1), offset)
    T = mhc_proj.torch.birkhoff_proj_n4(R, 1e-6)["T"]
    expected = persistent(R.float().contiguous(), 1e-6).to(dtype)
    assert T.dtype == dtype and same_bits(T, expected)


def test_nonfinite_small_batch():
    R = make_logits("normal", 257, seed=9)
    R[3, 1, 2] = float("nan")
    R[7, 0, 0] = float("inf")
    R[9, 3, 3] = -float("inf")
    R[11] = 1e30
    R[12] = 0.0
    R[13, 2, 1] = -0.0
    T = capi.birkhoff_proj_n4_tensor(R)
    assert same_bits(T, persistent(R, 1e-6))


# --- the small-batch backward (two lanes per matrix up to the same threshold) --

def backward(G, T):
    D = torch.empty_like(G)
    capi.birkhoff_proj_n4_backward(G.data_ptr(), T.data_ptr(), D.data_ptr(), G.shape[0],
                                   torch.cuda.current_stream().cuda_stream)
    return D


@pytest.mark.parametrize("kind", ["normal", "sigma_mix", "wide"])
@pytest.mark.parametrize("n", [1, 2, 17, 1000, PAIR_MAX_N])
def test_small_backward_bitwise(kind, n):
    """Against the reference kernel, and against the one-thread-per-matrix
    kernel (the same matrices padded past the threshold)."""
    R = make_logits(kind, n, seed=n + 7)
    G = make_logits("normal", n, seed=n + 8)
    T = capi.birkhoff_proj_n4_tensor(R)
    D = backward(G, T)
    pad = PAIR_MAX_N + 1
    Gp = torch.cat([G, make_logits("normal", pad, seed=1)])
    Tp = torch.cat([T, capi.birkhoff_proj_n4_tensor(make_logits(kind, pad, seed=2))])
    assert same_bits(D, backward(Gp, Tp)[:n])
    if oracle.RefCuda.available():
        ref = oracle.RefCuda()
        Dr = torch.empty_like(G)
        ref.birkhoff_proj_n4_backward(G.data_ptr(), T.data_ptr(), Dr.data_ptr(), n,
                                      torch.cuda.current_stream().cuda_stream)
        torch.cuda.synchronize()
        assert same_bits(D, Dr)


@pytest.mark.parametrize("gdt", [torch.float32, torch.bfloat16, torch.float16])
@pytest.mark.parametrize("tdt", [torch.float32, torch.bfloat16])
def test_small_backward_native_types(gdt, tdt):
    n = 3001
    R = make_logits("sigma_mix", n, seed=5)
    T32 = capi.birkhoff_proj_n4_tensor(R)
    G32 = make_logits("normal", n, seed=6)
    Tb = torch.empty(n * 24 + 16, device="cuda", dtype=tdt)
    T = torch.as_strided(Tb, (n, 4, 4), (24, 4, 1), 8)
    T.copy_(T32.to(tdt))
    Gb = torch.empty(n * 20 + 16, device="cuda", dtype=gdt)
    G = torch.as_strided(Gb, (n, 4, 4), (20, 4, 1), 4)
    G.copy_(G32.to(gdt))
    D = mhc_proj.torch.birkhoff_proj_n4_backward(G, T)["D"]
    expected = backward(G.float().contiguous(), T.float().contiguous()).to(gdt)
    assert D.dtype == gdt and same_bits(D, expected)
