"""Parity of the CUDA kernels, called through the C ABI, with the reference.

The reference's own CUDA kernels, compiled unmodified from its sources into
oracle/_ref/libmhcref.so, run on the same device buffers; the Newton forward
and the IFT backward must agree bit for bit.  The golden fixtures recorded
from the reference (tests/golden) are checked too, as are the vanilla
PyTorch Sinkhorn-Knopp (forward and autograd, within 1e-5) for the
Sinkhorn-Knopp pair, and the CPU oracle."""
import numpy as np
import pytest
import torch

import oracle
from conftest import golden_cases, load_golden
from mhc_proj.workloads import make_logits
from mhc_proj import capi

pytestmark = pytest.mark.gpu
TOL = 1e-5


@pytest.fixture(scope="module")
def ref():
    if not oracle.RefCuda.available():
        pytest.skip("oracle/_ref/libmhcref.so is not built (needs the reference sources)")
    return oracle.RefCuda()


def bitwise_equal(a, b):
    return torch.equal(a.contiguous().view(torch.int32), b.contiguous().view(torch.int32))


def stream():
    return torch.cuda.current_stream().cuda_stream


def ref_forward(ref, R, tol=1e-6):
    T = torch.empty_like(R)
    ref.birkhoff_proj_n4(R.data_ptr(), T.data_ptr(), tol, R.shape[0], stream())
    return T


def ref_backward(ref, G, T):
    D = torch.empty_like(G)
    ref.birkhoff_proj_n4_backward(G.data_ptr(), T.data_ptr(), D.data_ptr(), G.shape[0], stream())
    return D


CONFIGS = [
    ("normal", 1 << 20),        # Newton forward workload, N = 2^20, N(0,1)
    ("sigma_mix", 2097152),     # training-shaped: 32 layers x 16 seqs x 4096 tokens
    ("mixture", 1 << 22),       # mixture of the multi-GPU sweep
    ("wide", 1 << 20),
    ("uniform", 1 << 18),
]


@pytest.mark.parametrize("kind,n", CONFIGS)
def test_forward_and_backward_bitwise(ref, kind, n):
    R = make_logits(kind, n, seed=1000 + n)
    G = make_logits("normal", n, seed=7)
    T = capi.birkhoff_proj_n4_tensor(R)
    Tr = ref_forward(ref, R)
    assert bitwise_equal(T, Tr)
    D = capi.birkhoff_proj_n4_backward_tensor(G, T)
    Dr = ref_backward(ref, G, Tr)
    assert bitwise_equal(D, Dr)


@pytest.mark.parametrize("n", [1, 2, 31, 32, 33, 127, 4097, 100003])
def test_ragged_batch_sizes(ref, n):
    R = make_logits("sigma_mix", n, seed=n)
    G = make_logits("normal", n, seed=n + 1)
    T = capi.birkhoff_proj_n4_tensor(R)
    assert bitwise_equal(T, ref_forward(ref, R))
    assert bitwise_equal(capi.birkhoff_proj_n4_backward_tensor(G, T), ref_backward(ref, G, T))


@pytest.mark.parametrize("offset", [1, 2, 3, 5])
def test_unaligned_pointers(ref, offset):
    n = 3001
    R = make_logits("normal", n, seed=3)
    G = make_logits("normal", n, seed=4)
    bufs = [torch.empty(n * 16 + offset, device="cuda") for _ in range(4)]
    Ru, Gu, Tu, Du = (b[offset:].view(n, 4, 4) for b in bufs)
    Ru.copy_(R)
    Gu.copy_(G)
    capi.birkhoff_proj_n4(Ru.data_ptr(), Tu.data_ptr(), 1e-6, n, stream())
    capi.birkhoff_proj_n4_backward(Gu.data_ptr(), Tu.data_ptr(), Du.data_ptr(), n, stream())
    Tr = ref_forward(ref, R)
    assert bitwise_equal(Tu, Tr)
    assert bitwise_equal(Du, ref_backward(ref, G, Tr))


@pytest.mark.parametrize("tol", [1e-3, 1e-5, 1e-7, 0.0, float("inf")])
def test_tolerances(ref, tol):
    R = make_logits("mixture", 50000, seed=11)
    assert bitwise_equal(capi.birkhoff_proj_n4_tensor(R, tol=tol), ref_forward(ref, R, tol))


def test_nonfinite_inputs(ref):
    R = make_logits("normal", 4096, seed=5)
    flat = R.view(-1)
    flat[::97] = float("nan")
    flat[13::89] = float("inf")
    flat[29::83] = float("-inf")
    flat[41::79] = 1e30
    T = capi.birkhoff_proj_n4_tensor(R)
    assert bitwise_equal(T, ref_forward(ref, R))
    G = make_logits("normal", 4096, seed=6)
    Tr = ref_forward(ref, R)
    assert bitwise_equal(capi.birkhoff_proj_n4_backward_tensor(G, Tr), ref_backward(ref, G, Tr))


@pytest.mark.parametrize("case", golden_cases())
def test_golden_fixtures(case):
    g = load_golden(case)
    R = torch.from_numpy(g["R"]).cuda()
    T = capi.birkhoff_proj_n4_tensor(R)
    assert np.array_equal(T.cpu().numpy().view(np.uint32), g["T_ref"].view(np.uint32))
    D = capi.birkhoff_proj_n4_backward_tensor(torch.from_numpy(g["G"]).cuda(), torch.from_numpy(g["T_ref"]).cuda())
    assert np.array_equal(D.cpu().numpy().view(np.uint32), g["D_ref"].view(np.uint32))
    Tsk = capi.sinkhorn_knopp_n4_tensor(torch.from_numpy(g["M"]).cuda(), 20)
    assert np.array_equal(Tsk.cpu().numpy().view(np.uint32), g["T_sk_ref"].view(np.uint32))


def test_against_cpu_oracle():
    R = make_logits("normal", 1 << 14, seed=21)
    G = make_logits("normal", 1 << 14, seed=22)
    T = capi.birkhoff_proj_n4_tensor(R)
    To = oracle.birkhoff_proj_n4(R.cpu().numpy(), 1e-6)
    assert np.max(np.abs(T.cpu().numpy() - To)) < TOL
    D = capi.birkhoff_proj_n4_backward_tensor(G, T)
    Do = oracle.birkhoff_proj_n4_backward(G.cpu().numpy(), T.cpu().numpy())
    assert np.max(np.abs(D.cpu().numpy() - Do)) < TOL


def test_doubly_stochastic_at_workload_size(ref):
    """Rows sum to one (by construction, to rounding) and columns to within
    1e-5 wherever the reference's Newton converges.  A few matrices in a
    million stop at the 20-iteration cap with a column sum a little past
    1e-5; the reference returns the same bits for them."""
    R = make_logits("normal", 1 << 22, seed=0)
    T = capi.birkhoff_proj_n4_tensor(R)
    Tr = ref_forward(ref, R)
    assert bitwise_equal(T, Tr)
    T = T.double()
    assert (T.sum(2) - 1).abs().max().item() < 1e-6
    col = (T.sum(1) - 1).abs().amax(1)
    assert (col > TOL).float().mean().item() < 1e-5
    assert col.max().item() < 1e-4
    assert T.min().item() >= 0


# ---- Sinkhorn-Knopp pair -------------------------------------------------

@pytest.mark.parametrize("kind", ["normal", "sigma_mix", "wide"])
@pytest.mark.parametrize("iters", [0, 1, 7, 20, 35])
def test_sinkhorn_forward_bitwise(ref, kind, iters):
    M = torch.exp(make_logits(kind, 1 << 16, seed=iters))
    T = capi.sinkhorn_knopp_n4_tensor(M, iters)
    Tr = torch.empty_like(M)
    ref.sinkhorn_knopp_n4(M.data_ptr(), Tr.data_ptr(), M.shape[0], iters, stream())
    assert bitwise_equal(T, Tr)


def test_sinkhorn_pair_matches_vanilla_autograd():
    """The Sinkhorn-Knopp kernel configuration: N = 2^22, x ~ N(0,1), 20
    iterations; forward and dR within 1e-5 of the vanilla PyTorch SK20."""
    n = 1 << 22
    x = make_logits("normal", n, seed=123)
    G = make_logits("normal", n, seed=124)
    M = torch.exp(x)
    T = capi.sinkhorn_knopp_n4_tensor(M, 20)
    dR = capi.sinkhorn_knopp_n4_backward_tensor(G, M, 20) * M
    P, dRv = oracle.vanilla_sinkhorn(x, G)
    assert (T - P).abs().max().item() < TOL
    assert (dR - dRv).abs().max().item() < TOL


@pytest.mark.parametrize("iters", [1, 2, 3, 4, 5, 9, 16, 19, 20])
def test_sinkhorn_backward_every_iteration_count(iters):
    """The exact VJP for every iteration count: against the oracle's (the
    row/column form differentiated step by step, with correctly rounded
    reciprocals) within 2e-6, relative where |dM| > 1 -- the kernel forms the
    gradient from the forward's potentials with the hardware reciprocal (one
    ulp), and dM = dR / M grows where M is small -- and dR within 1e-5 of
    vanilla autograd."""
    n = 4096
    M = torch.exp(make_logits("normal", n, seed=iters))
    G = make_logits("normal", n, seed=iters + 50)
    D = capi.sinkhorn_knopp_n4_backward_tensor(G, M, iters)
    Do = oracle.sinkhorn_knopp_n4_backward(G.cpu().numpy(), M.cpu().numpy(), iters, 1e-8, exact=True)
    assert (np.abs(D.cpu().numpy() - Do) <= 2e-6 * np.maximum(1.0, np.abs(Do))).all()
    x = torch.log(M)
    _, dRv = oracle.vanilla_sinkhorn(x, G, iters=iters)
    assert (D * M - dRv).abs().max().item() < TOL


@pytest.mark.parametrize("iters", [1, 2, 5, 20])
def test_sinkhorn_backward_masked_rows_and_columns(iters):
    """Rows and columns whose sums fall to eps or below get a zero factor
    (sinkhorn_knopp.cuh:851-906).  The kernel takes its masks from the first
    iteration only (no later row or column can fall that low); the oracle
    tests every iteration.  Matrices with a row of logits -40 (row sum below
    eps), a column of -40 (its sum below eps after the row step), both, two
    such rows, and rows or columns just above the threshold: the same zero
    pattern, dR = dM * M within 2e-6, and dM within 2e-6 relative wherever
    M > 1e-6 (below that dM = dR / M carries both sides' rounding, amplified)."""
    n = 4096
    g = torch.Generator().manual_seed(70 + iters)
    R = torch.randn(n, 4, 4, generator=g)
    for m in range(n):
        i, j, c = m % 4, (m // 4) % 4, m % 8
        if c in (1, 3):
            R[m, i, :] = -40.0
        if c in (2, 3):
            R[m, :, j] = -40.0
        if c == 4:
            R[m, i, :] = -19.5  # row sum 1.3e-8: just above eps
        if c == 5:
            R[m, :, j] = -21.0
        if c == 6:
            R[m, i, :] = -40.0
            R[m, (i + 1) % 4, :] = -40.0
    G = torch.randn(n, 4, 4, generator=g)
    M = torch.exp(R)
    D = capi.sinkhorn_knopp_n4_backward_tensor(G.cuda(), M.cuda(), iters).cpu().numpy()
    Mn = M.numpy()
    Do = oracle.sinkhorn_knopp_n4_backward(G.numpy(), Mn, iters, 1e-8, exact=True)
    assert np.array_equal(D == 0, Do == 0)
    assert (np.abs(D * Mn - Do * Mn) <= 2e-6).all()
    big = Mn > 1e-6
    assert (np.abs(D - Do)[big] <= 2e-6 * np.maximum(1.0, np.abs(Do[big]))).all()


def test_sinkhorn_backward_zero_iterations_is_identity():
    M = torch.exp(make_logits("normal", 1000, seed=1))
    G = make_logits("normal", 1000, seed=2)
    assert torch.equal(capi.sinkhorn_knopp_n4_backward_tensor(G, M, 0), G)


# ---- fused exp + Sinkhorn-Knopp (logits input) -------------------------------

@pytest.mark.parametrize("kind", ["normal", "sigma_mix", "uniform"])
@pytest.mark.parametrize("iters", [0, 1, 5, 20])
def test_fused_logits_equals_exp_then_kernel(kind, iters):
    """sinkhorn_knopp_n4_logits(R) is bit for bit the kernel on torch.exp(R),
    and its backward is bit for bit the M-gradient times torch.exp(R) (the
    reference's MHCSinkhornN4 composition, module.py:50,70)."""
    n = 1 << 16
    R = make_logits(kind, n, seed=31 + iters)
    G = make_logits("normal", n, seed=32 + iters)
    M = torch.exp(R)
    assert bitwise_equal(capi.sinkhorn_knopp_n4_logits_tensor(R, iters), capi.sinkhorn_knopp_n4_tensor(M, iters))
    D_unfused = capi.sinkhorn_knopp_n4_backward_tensor(G, M, iters) * M
    assert bitwise_equal(capi.sinkhorn_knopp_n4_logits_backward_tensor(G, R, iters), D_unfused)


def test_fused_logits_wide_inputs_within_tolerance():
    """With N(0,100) logits exp(R) has subnormal entries, which the kernels
    flush like the reference; agreement is then to the last few ulps."""
    n = 1 << 16
    R = make_logits("wide", n, seed=40)
    G = make_logits("normal", n, seed=41)
    M = torch.exp(R)
    assert (capi.sinkhorn_knopp_n4_logits_tensor(R, 20) - capi.sinkhorn_knopp_n4_tensor(M, 20)).abs().max().item() < 1e-6
    D_unfused = capi.sinkhorn_knopp_n4_backward_tensor(G, M, 20) * M
    D = capi.sinkhorn_knopp_n4_logits_backward_tensor(G, R, 20)
    assert torch.allclose(D, D_unfused, rtol=1e-5, atol=1e-6)


def test_fused_logits_matches_vanilla_autograd():
    n = 1 << 20
    x = make_logits("normal", n, seed=123)
    G = make_logits("normal", n, seed=124)
    T = capi.sinkhorn_knopp_n4_logits_tensor(x, 20)
    dR = capi.sinkhorn_knopp_n4_logits_backward_tensor(G, x, 20)
    P, dRv = oracle.vanilla_sinkhorn(x, G)
    assert (T - P).abs().max().item() < TOL
    assert (dR - dRv).abs().max().item() < TOL


# ---- fuzzing: arbitrary inputs, bit for bit -----------------------------------

from hypothesis import HealthCheck, given, settings, strategies as st  # noqa: E402
from hypothesis.extra.numpy import arrays  # noqa: E402

_any32 = st.floats(width=32, allow_nan=True, allow_infinity=True, allow_subnormal=True)


@settings(max_examples=40, deadline=None, suppress_health_check=[HealthCheck.function_scoped_fixture])
@given(R=arrays(np.float32, (96, 4, 4), elements=_any32), G=arrays(np.float32, (96, 4, 4), elements=_any32),
       tol=st.sampled_from([1e-6, 1e-3, 0.0]))
def test_fuzz_against_reference(ref, R, G, tol):
    Rd = torch.from_numpy(R).cuda()
    Gd = torch.from_numpy(G).cuda()
    T = capi.birkhoff_proj_n4_tensor(Rd, tol=tol)
    Tr = ref_forward(ref, Rd, tol)
    assert bitwise_equal(T, Tr)
    assert bitwise_equal(capi.birkhoff_proj_n4_backward_tensor(Gd, Tr), ref_backward(ref, Gd, Tr))


@settings(max_examples=40, deadline=None)
@given(scale=st.floats(0.05, 12.0), shift=st.floats(-30.0, 5.0), iters=st.integers(1, 20),
       seed=st.integers(0, 2**31 - 1), masked=st.booleans())
def test_fuzz_sinkhorn_backward_against_oracle(scale, shift, iters, seed, masked):
    """The SK backward (from the forward's potentials, the first iteration's
    masks) against the oracle's step-by-step exact VJP on random scales of
    the logits (up to N(0, 144)), shifts that push whole matrices towards eps,
    random iteration counts and, optionally, rows and columns of -40 planted
    in.  dR = dM * M, what a caller uses, within 2e-6; rows whose sum is at
    most eps exactly zero on both sides; dM itself within 2e-6 relative where
    M > 1e-6 on well-conditioned draws (on ill-conditioned ones dM = dR / M
    carries each form's rounding, amplified, in both)."""
    n = 256
    g = torch.Generator().manual_seed(seed)
    R = torch.randn(n, 4, 4, generator=g) * scale + shift
    if masked:
        R[::5, 1, :] = -40.0
        R[2::7, :, 2] = -40.0
    G = torch.randn(n, 4, 4, generator=g)
    M = torch.exp(R)
    D = capi.sinkhorn_knopp_n4_backward_tensor(G.cuda(), M.cuda(), iters).cpu().numpy()
    Mn = M.numpy()
    Do = oracle.sinkhorn_knopp_n4_backward(G.numpy(), Mn, iters, 1e-8, exact=True)
    assert (np.abs(D * Mn - Do * Mn) <= 2e-6).all()
    rows = Mn.sum(2) <= 1e-8
    assert (D[rows] == 0).all() and (Do[rows] == 0).all()
    if scale <= 1.0 and shift >= -5.0:
        big = Mn > 1e-6
        assert (np.abs(D - Do)[big] <= 2e-6 * np.maximum(1.0, np.abs(Do[big]))).all()


def test_sinkhorn_batch_beyond_int32_element_indexing():
    """The fused Sinkhorn-Knopp pair on N = 2^27 + 5 matrices (2^31 + 80
    elements per tensor): slices at both ends and across the 2^31-element
    boundary equal separate launches on those slices, bit for bit."""
    n = (1 << 27) + 5
    free, _ = torch.cuda.mem_get_info()
    if free < 5 * n * 64:
        pytest.skip("needs ~45 GB of free device memory")
    R = torch.empty(n, 4, 4, device="cuda")
    for i in range(0, n, 1 << 24):
        m = min(1 << 24, n - i)
        R[i:i + m] = make_logits("normal", m, seed=91 + i // (1 << 24))
    G = torch.empty_like(R).normal_()
    T = capi.sinkhorn_knopp_n4_logits_tensor(R, 20)
    D = capi.sinkhorn_knopp_n4_logits_backward_tensor(G, R, 20)
    edge = (1 << 27) - 1000
    for a, b in [(0, 4096), (edge, edge + 2000), (n - 3000, n)]:
        assert bitwise_equal(T[a:b], capi.sinkhorn_knopp_n4_logits_tensor(R[a:b].contiguous(), 20))
        assert bitwise_equal(D[a:b], capi.sinkhorn_knopp_n4_logits_backward_tensor(G[a:b].contiguous(),
                                                                                   R[a:b].contiguous(), 20))
    del R, G, T, D
    torch.cuda.empty_cache()


def test_batch_beyond_int32_element_indexing():
    """N = 2^27 + 5 matrices (2^31 + 80 elements per tensor): past the point
    where the reference's 32-bit element index N*16 overflows
    (birkhoff_proj_n4.cu:510).  Slices at both ends and across the 2^31
    element boundary must equal separate launches on those slices."""
    n = (1 << 27) + 5
    free, _ = torch.cuda.mem_get_info()
    if free < 5 * n * 64:
        pytest.skip("needs ~45 GB of free device memory")
    R = torch.empty(n, 4, 4, device="cuda")
    for i in range(0, n, 1 << 24):  # fill in chunks to bound the generator's temporaries
        m = min(1 << 24, n - i)
        R[i:i + m] = make_logits("normal", m, seed=77 + i // (1 << 24))
    G = torch.empty_like(R).normal_()
    T = capi.birkhoff_proj_n4_tensor(R)
    D = capi.birkhoff_proj_n4_backward_tensor(G, T)
    edge = (1 << 27) - 1000  # matrix index whose elements straddle 2^31
    for a, b in [(0, 4096), (edge, edge + 2000), (n - 3000, n)]:
        Ts = capi.birkhoff_proj_n4_tensor(R[a:b].contiguous())
        assert bitwise_equal(T[a:b], Ts)
        assert bitwise_equal(D[a:b], capi.birkhoff_proj_n4_backward_tensor(G[a:b].contiguous(), Ts))
    del R, G, T, D
    torch.cuda.empty_cache()


def test_multi_gpu_workload_at_full_size(ref):
    """The multi-GPU workload's whole batch on one GPU: N = 2^26 matrices of the
    mixture (50% N(0,1), 25% N(0,9), 25% N(0,1) with +6 on one entry per row),
    tol 1e-6, G ~ N(0,1): T and D equal the reference kernels' bit for bit,
    and every row of T sums to 1 within 1e-5."""
    n = 1 << 26
    free, _ = torch.cuda.mem_get_info()
    if free < 7 * n * 64:
        pytest.skip("needs ~30 GB of free device memory")
    R = torch.empty(n, 4, 4, device="cuda")
    G = torch.empty(n, 4, 4, device="cuda")
    for i in range(0, n, 1 << 24):
        R[i:i + (1 << 24)] = make_logits("mixture", 1 << 24, seed=500 + i // (1 << 24))
        G[i:i + (1 << 24)] = make_logits("normal", 1 << 24, seed=600 + i // (1 << 24))
    T = capi.birkhoff_proj_n4_tensor(R)
    Tr = ref_forward(ref, R)
    torch.cuda.synchronize()
    assert bitwise_equal(T, Tr)
    del Tr
    D = capi.birkhoff_proj_n4_backward_tensor(G, T)
    Dr = ref_backward(ref, G, T)
    torch.cuda.synchronize()
    assert bitwise_equal(D, Dr)
    del Dr, D, G
    assert float((T.sum(2) - 1.0).abs().max()) < TOL
    del R, T
    torch.cuda.empty_cache()


def test_sinkhorn_against_the_newton_path():
    """The Sinkhorn-Knopp workload (N = 2^22, N(0,1), 20 iterations) against the
    Newton path on the same logits.  They are different algorithms -- 20 fixed
    iterations against a converged projection -- so they agree only to SK20's
    convergence: within 1e-5 on all but a fraction of a percent of matrices,
    within 1e-2 everywhere, and the Newton result is the one whose columns
    sum to 1 (SK20 leaves its row sums off instead)."""
    n = 1 << 22
    R = make_logits("normal", n, seed=77)
    Tn = capi.birkhoff_proj_n4_tensor(R)
    Ts = capi.sinkhorn_knopp_n4_logits_tensor(R, 20)
    torch.cuda.synchronize()
    diff = (Tn - Ts).abs().reshape(n, 16).max(1).values
    assert float((diff > TOL).float().mean()) < 0.01
    assert float(diff.max()) < 1e-2
    assert float((Tn.sum(2) - 1).abs().max()) < TOL
    assert float((Ts.sum(1) - 1).abs().max()) < TOL  # SK ends on a column normalisation


# --- the Sinkhorn-Knopp forward with the hardware reciprocal (opt-in) -------

@pytest.mark.parametrize("kind,n", [("normal", 4096), ("normal", 1 << 22), ("sigma_mix", 1 << 20), ("wide", 1 << 20)])
def test_sinkhorn_hw_reciprocal_within_tolerance(kind, n):
    """MHC_SK_HW_RECIPROCAL: within 1e-6 of the correctly rounded forward (the
    reference kernel's bits) on every distribution, and within 1e-5 of the
    vanilla PyTorch Sinkhorn-Knopp (float64) where vanilla's eps semantics
    agree with the kernel's (N(0,1) logits; at N(0,100) vanilla's eps
    dominates tiny rows and the two algorithms differ)."""
    R = make_logits(kind, n, seed=123)
    s = torch.cuda.current_stream().cuda_stream
    T = torch.empty_like(R)
    Ta = torch.empty_like(R)
    capi.sinkhorn_knopp_n4_logits(R.data_ptr(), T.data_ptr(), n, 20, s)
    capi.sinkhorn_knopp_n4_logits_ex(R.data_ptr(), Ta.data_ptr(), n, 20, capi.MHC_SK_HW_RECIPROCAL, s)
    torch.cuda.synchronize()
    assert float((Ta - T).abs().max()) < 1e-6
    if kind == "normal":
        m = min(n, 1 << 16)
        P = oracle.vanilla_sinkhorn(R[:m].double())
        assert float((Ta[:m].double() - P).abs().max()) < 1e-5


def test_sinkhorn_hw_reciprocal_module_and_flags():
    import mhc_proj

    x = make_logits("normal", 4096, seed=123).requires_grad_(True)
    G = make_logits("normal", 4096, seed=124)
    T0 = mhc_proj.MHCSinkhornN4(20)(x)
    (T0 * G).sum().backward()
    g0 = x.grad.clone()
    x.grad = None
    T1 = mhc_proj.MHCSinkhornN4(20, approx_reciprocal=True)(x)
    (T1 * G).sum().backward()
    assert float((T1 - T0).abs().max()) < 1e-6
    assert torch.equal(x.grad, g0)  # the backward recomputes from R either way
    with pytest.raises(capi.MhcError):
        capi.sinkhorn_knopp_n4_logits_ex(x.data_ptr(), T0.data_ptr(), 4096, 20, 2, 0)
