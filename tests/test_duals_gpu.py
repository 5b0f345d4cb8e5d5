"""Saving the duals instead of T: the forward also writes the final beta,
the backward rebuilds T from R and beta with the forward's arithmetic.  Both
must give the plain path's bits: T, and D for the same G."""
import pytest
import torch

import mhc_proj
from mhc_proj import capi
from mhc_proj.workloads import make_logits

pytestmark = pytest.mark.gpu


def same_bits(a, b):
    return torch.equal(a.contiguous().view(torch.int32), b.contiguous().view(torch.int32))


@pytest.mark.parametrize("kind", ["normal", "sigma_mix", "mixture", "wide", "uniform"])
def test_duals_rebuild_t_and_d_bitwise(kind):
    n = (1 << 20) + 7
    R = make_logits(kind, n, seed=61)
    G = make_logits("normal", n, seed=62)
    T = capi.birkhoff_proj_n4_tensor(R)
    Td, beta = capi.birkhoff_proj_n4_duals_tensor(R)
    D = capi.birkhoff_proj_n4_backward_tensor(G, T)
    Dd = capi.birkhoff_proj_n4_backward_duals_tensor(G, R, beta)
    torch.cuda.synchronize()
    assert same_bits(Td, T)
    assert same_bits(Dd, D)
    assert bool((beta[:, 3] == 0).all())  # beta_3 is pinned at zero (either sign)


def test_duals_edge_inputs():
    n = 4096
    R = make_logits("normal", n, seed=63)
    R[0] = 0.0                                  # uniform: converged at beta = 0 after the column pass
    ds = torch.full((4, 4), 0.1, device="cuda") + 0.6 * torch.eye(4, device="cuda")
    R[1] = ds.log()                             # exp(R) already doubly stochastic
    R[2, 1, 2] = float("nan")
    R[3, 0, 0] = float("inf")
    R[4] = 1e30
    R[5, 2] = -1e4
    G = make_logits("normal", n, seed=64)
    T = capi.birkhoff_proj_n4_tensor(R)
    Td, beta = capi.birkhoff_proj_n4_duals_tensor(R)
    D = capi.birkhoff_proj_n4_backward_tensor(G, T)
    Dd = capi.birkhoff_proj_n4_backward_duals_tensor(G, R, beta)
    torch.cuda.synchronize()
    assert same_bits(Td, T) and same_bits(Dd, D)
    assert bool((beta[0] == 0).all())


def test_duals_unaligned_and_ragged():
    for n in (1, 31, 33, 1000):
        R = make_logits("sigma_mix", n, seed=65 + n)
        G = make_logits("normal", n, seed=66 + n)
        T = capi.birkhoff_proj_n4_tensor(R)
        D = capi.birkhoff_proj_n4_backward_tensor(G, T)
        rb = torch.empty(n * 16 + 1, device="cuda")
        Rm = rb[1:].view(n, 4, 4)
        Rm.copy_(R)
        tb = torch.empty(n * 16 + 1, device="cuda")
        bb = torch.empty(n * 4 + 1, device="cuda")
        capi.birkhoff_proj_n4_duals(Rm.data_ptr(), tb[1:].data_ptr(), bb[1:].data_ptr(), 1e-6, n,
                                    torch.cuda.current_stream().cuda_stream)
        db = torch.empty(n * 16 + 1, device="cuda")
        gb = torch.empty(n * 16 + 1, device="cuda")
        gb[1:].copy_(G.reshape(-1))
        capi.birkhoff_proj_n4_backward_duals(gb[1:].data_ptr(), Rm.data_ptr(), bb[1:].data_ptr(), db[1:].data_ptr(),
                                             n, torch.cuda.current_stream().cuda_stream)
        torch.cuda.synchronize()
        assert same_bits(tb[1:].view(n, 4, 4), T) and same_bits(db[1:].view(n, 4, 4), D)


def test_module_save_duals_gives_the_same_gradients():
    n = 65536
    x = make_logits("sigma_mix", n, seed=67).view(256, 256, 4, 4)
    G = make_logits("normal", n, seed=68).view(256, 256, 4, 4)
    grads = []
    for save in (False, True):
        xi = x.clone().requires_grad_(True)
        T = mhc_proj.MHCProjectionN4(tol=1e-6, save_duals=save)(xi)
        (T * G).sum().backward()
        grads.append((T.detach(), xi.grad))
    assert same_bits(grads[0][0], grads[1][0]) and same_bits(grads[0][1], grads[1][1])


def test_binding_return_duals():
    R = make_logits("normal", 1000, seed=69)
    out = mhc_proj.torch.birkhoff_proj_n4(R, 1e-6, return_duals=True)
    assert set(out) == {"T", "beta"} and tuple(out["beta"].shape) == (1000, 4)
    assert same_bits(out["T"], mhc_proj.torch.birkhoff_proj_n4(R, 1e-6)["T"])
    G = make_logits("normal", 1000, seed=70)
    D = mhc_proj.torch.birkhoff_proj_n4_backward_duals(G, R, out["beta"])["D"]
    assert same_bits(D, mhc_proj.torch.birkhoff_proj_n4_backward(G, out["T"])["D"])
