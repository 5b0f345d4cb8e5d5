"""The PyTorch-facing API on the GPU: the autograd modules and the low-level
functions behave like the reference package (mhc_proj/module.py,
src/solvers_torch.cpp) and give the C-ABI kernels' results."""
import json
import os

import numpy as np
import pytest
import torch

import mhc_proj
import oracle
from conftest import GOLDEN
from mhc_proj.workloads import make_logits
from mhc_proj import capi

pytestmark = pytest.mark.gpu


def test_module_forward_backward_equals_kernels():
    x = make_logits("sigma_mix", 10000, seed=1).requires_grad_(True)
    G = make_logits("normal", 10000, seed=2)
    T = mhc_proj.MHCProjectionN4(tol=1e-6)(x)
    (T * G).sum().backward()
    T2 = capi.birkhoff_proj_n4_tensor(x.detach())
    assert torch.equal(T.detach(), T2)
    assert torch.equal(x.grad, capi.birkhoff_proj_n4_backward_tensor(G, T2))


def test_low_level_functions_return_dicts():
    R = make_logits("normal", 1000, seed=3)
    out = mhc_proj.torch.birkhoff_proj_n4(R, 1e-6, unused_kwarg=True)
    assert set(out) == {"T"}
    D = mhc_proj.torch.birkhoff_proj_n4_backward(R, out["T"], another=1)
    assert set(D) == {"D"}
    assert set(mhc_proj.torch.sinkhorn_knopp_n4(R.exp())) == {"T"}
    assert set(mhc_proj.torch.sinkhorn_knopp_n4_backward(R, R.exp())) == {"D"}


def test_dtype_and_device_round_trip():
    R = make_logits("normal", 777, seed=4)
    T32 = mhc_proj.torch.birkhoff_proj_n4(R)["T"]
    T64 = mhc_proj.torch.birkhoff_proj_n4(R.double())["T"]
    assert T64.dtype == torch.float64 and T64.is_cuda
    assert torch.equal(T64.float(), T32)
    Tcpu = mhc_proj.torch.birkhoff_proj_n4(R.cpu())["T"]
    assert Tcpu.device.type == "cpu" and torch.equal(Tcpu, T32.cpu())
    Tbf = mhc_proj.torch.birkhoff_proj_n4(R.bfloat16())["T"]
    assert Tbf.dtype == torch.bfloat16
    # the backward follows G's dtype/device for both G and T
    D = mhc_proj.torch.birkhoff_proj_n4_backward(R.double().cpu(), T32)["D"]
    assert D.dtype == torch.float64 and D.device.type == "cpu"


def test_non_contiguous_and_batched_shapes():
    base = make_logits("normal", 2 * 3 * 5, seed=5).view(2, 3, 5, 4, 4)
    x = base.transpose(0, 1)  # non-contiguous 5-D input
    T = mhc_proj.MHCProjectionN4()(x)
    assert T.shape == x.shape
    ref = capi.birkhoff_proj_n4_tensor(x.reshape(-1, 4, 4).contiguous()).view(x.shape)
    assert torch.equal(T, ref)
    xt = make_logits("normal", 64, seed=6).transpose(1, 2)
    assert torch.equal(mhc_proj.torch.birkhoff_proj_n4(xt)["T"], capi.birkhoff_proj_n4_tensor(xt.contiguous()))


def test_empty_batch():
    R = torch.empty(0, 4, 4, device="cuda")
    assert mhc_proj.torch.birkhoff_proj_n4(R)["T"].shape == (0, 4, 4)
    assert mhc_proj.torch.birkhoff_proj_n4_backward(R, R)["D"].shape == (0, 4, 4)
    assert mhc_proj.MHCProjectionN4()(R).shape == (0, 4, 4)


def test_sinkhorn_iteration_limit_raises_value_error():
    M = make_logits("normal", 8, seed=7).exp()
    with pytest.raises(ValueError):
        mhc_proj.torch.sinkhorn_knopp_n4_backward(M, M, 21)
    mhc_proj.torch.sinkhorn_knopp_n4(M, 50)  # the forward has no limit


def test_sinkhorn_module_matches_vanilla():
    x = make_logits("normal", 20000, seed=8).requires_grad_(True)
    G = make_logits("normal", 20000, seed=9)
    T = mhc_proj.MHCSinkhornN4(max_iter=20)(x)
    (T * G).sum().backward()
    P, dR = oracle.vanilla_sinkhorn(x.detach(), G)
    assert (T.detach() - P).abs().max().item() < 1e-5
    assert (x.grad - dR).abs().max().item() < 1e-5


def test_runs_on_the_current_stream():
    R = make_logits("mixture", 1 << 18, seed=10)
    expected = capi.birkhoff_proj_n4_tensor(R)
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        T = mhc_proj.torch.birkhoff_proj_n4(R)["T"]
        D = mhc_proj.torch.birkhoff_proj_n4_backward(R, T)["D"]
    torch.cuda.current_stream().wait_stream(s)
    assert torch.equal(T, expected)
    assert torch.equal(D, capi.birkhoff_proj_n4_backward_tensor(R, expected))


def test_readme_example():
    """README.md:27-133 run as written: CUDA RNG with seed 123, N = 2."""
    vals = json.load(open(os.path.join(GOLDEN, "readme_values.json")))
    torch.manual_seed(123)
    x = torch.randn(2, 4, 4, device="cuda")
    x.requires_grad_(True)
    G = torch.randn(2, 4, 4, device="cuda")
    P2 = mhc_proj.MHCProjectionN4(tol=1e-6)(x)
    torch.sum(G * P2).backward()
    half = 0.5e-4 + 1e-7
    assert np.max(np.abs(P2.detach().cpu().numpy().ravel() - np.array(vals["P_module"]))) <= half
    assert np.max(np.abs(x.grad.cpu().numpy().ravel() - np.array(vals["dx_module"]))) <= half
    P3 = mhc_proj.torch.birkhoff_proj_n4(x.detach(), tol=1e-6)["T"]
    D3 = mhc_proj.torch.birkhoff_proj_n4_backward(G, P3)["D"]
    assert np.max(np.abs(P3.cpu().numpy().ravel() - np.array(vals["P_lowlevel"]))) <= half
    assert np.max(np.abs(D3.cpu().numpy().ravel() - np.array(vals["D_lowlevel"]))) <= half
    ex = np.load(os.path.join(GOLDEN, "readme_example.npz"))
    assert np.array_equal(P3.cpu().numpy().view(np.uint32), ex["T_ref"].view(np.uint32))


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_second_device_keeps_its_index():
    R = make_logits("normal", 1000, seed=12).to("cuda:1")
    T = mhc_proj.torch.birkhoff_proj_n4(R)["T"]
    assert T.device == R.device
    assert torch.equal(T.cpu(), capi.birkhoff_proj_n4_tensor(R.to("cuda:0")).cpu())


def test_sinkhorn_module_uses_fused_kernels_and_keeps_other_dtypes():
    x = make_logits("normal", 4096, seed=13)
    G = make_logits("normal", 4096, seed=14)
    # fp32 CUDA: fused kernels, same bits as the reference's composition
    xa = x.clone().requires_grad_(True)
    T = mhc_proj.MHCSinkhornN4()(xa)
    (T * G).sum().backward()
    M = torch.exp(x)
    assert torch.equal(T.detach(), mhc_proj.torch.sinkhorn_knopp_n4(M)["T"])
    assert torch.equal(xa.grad, mhc_proj.torch.sinkhorn_knopp_n4_backward(G, M)["D"] * M)
    # float64: the reference composition in the input dtype
    xd = x.double().requires_grad_(True)
    Td = mhc_proj.MHCSinkhornN4()(xd)
    assert Td.dtype == torch.float64
    (Td * G.double()).sum().backward()
    assert xd.grad.dtype == torch.float64
    assert (xd.grad.float() - xa.grad).abs().max().item() < 1e-5


def test_fused_logits_backward_iteration_limit():
    R = make_logits("normal", 8, seed=15)
    with pytest.raises(ValueError):
        mhc_proj.torch.sinkhorn_knopp_n4_logits_backward(R, R, 21)


@pytest.mark.parametrize("kind", ["normal", "wide"])
def test_convergence_stats(kind):
    """return_stats=True adds per-matrix Newton iteration counts and final
    gradient norms; T is unchanged.  A matrix reports gnorm >= tol exactly
    when it stopped at the 20-iteration cap."""
    R = make_logits(kind, 1 << 16, seed=21)
    out = mhc_proj.torch.birkhoff_proj_n4(R, 1e-6, return_stats=True)
    assert set(out) == {"T", "iters", "gnorm"}
    assert torch.equal(out["T"], mhc_proj.torch.birkhoff_proj_n4(R, 1e-6)["T"])
    it, gn = out["iters"], out["gnorm"]
    assert it.dtype == torch.int32 and int(it.min()) >= 0 and int(it.max()) <= 20
    capped = gn >= 1e-6
    assert bool((it[capped] == 20).all())
    # the reported norm is the l1 norm of the first three column sums minus one
    c = out["T"].double().sum(1)[:, :3]
    assert torch.allclose(gn.double(), (c - 1).abs().sum(1), atol=2e-6)
    if kind == "wide":
        assert int(capped.sum()) > 0


def test_cuda_graph_capture_and_replay():
    """Forward and backward captured in a CUDA graph replay to the same bits as
    eager calls (the launchers make no runtime calls that capture forbids
    once a device has been seen)."""
    R = make_logits("sigma_mix", 1 << 16, seed=31)
    G = make_logits("normal", 1 << 16, seed=32)
    T0 = mhc_proj.torch.birkhoff_proj_n4(R)["T"]
    D0 = mhc_proj.torch.birkhoff_proj_n4_backward(G, T0)["D"]
    Rs, Gs = R.clone(), G.clone()
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):  # warm-up on the capture stream
        mhc_proj.torch.birkhoff_proj_n4(Rs)
    torch.cuda.current_stream().wait_stream(s)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        T = mhc_proj.torch.birkhoff_proj_n4(Rs)["T"]
        D = mhc_proj.torch.birkhoff_proj_n4_backward(Gs, T)["D"]
    Rs.copy_(make_logits("normal", 1 << 16, seed=33))
    g.replay()
    torch.cuda.synchronize()
    assert torch.equal(T, mhc_proj.torch.birkhoff_proj_n4(Rs)["T"])
    Rs.copy_(R)
    g.replay()
    torch.cuda.synchronize()
    assert torch.equal(T, T0) and torch.equal(D, D0)


def test_cuda_graph_capture_sinkhorn():
    """The fused Sinkhorn pair also captures and replays to the eager bits."""
    R = make_logits("normal", 1 << 14, seed=41)
    G = make_logits("normal", 1 << 14, seed=42)
    T0 = mhc_proj.torch.sinkhorn_knopp_n4_logits(R)["T"]
    D0 = mhc_proj.torch.sinkhorn_knopp_n4_logits_backward(G, R)["D"]
    Rs, Gs = R.clone(), G.clone()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        T = mhc_proj.torch.sinkhorn_knopp_n4_logits(Rs)["T"]
        D = mhc_proj.torch.sinkhorn_knopp_n4_logits_backward(Gs, Rs)["D"]
    g.replay()
    torch.cuda.synchronize()
    assert torch.equal(T, T0) and torch.equal(D, D0)
