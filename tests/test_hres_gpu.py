"""The projection fused with the mHC layer's H_res producer, on the GPU.

Pins:
  - the reference's producer (fused_h_activations, src/utils.cuh:50-127,
    compiled unmodified into oracle/_ref/libmhcref_hres.so) writes exp(R);
    the shim's restatement of its pre-exponential value R gives those bits
    back through the producer's own __expf, and lies within its three
    roundings of the float64 formula;
  - the fused forward's T equals the reference's Newton kernel on that R,
    bit for bit;
  - the fused backward's gradients equal the float64 chain rule applied to
    the reference's own IFT gradient D (dh within 1e-6 relative per element;
    drms and the batch sums within 4e-6 of the magnitudes of their terms), and
    are deterministic.
"""
import numpy as np
import pytest
import torch

import mhc_proj
import oracle
from mhc_proj import capi

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def ref():
    if not oracle.RefCuda.available():
        pytest.skip("oracle/_ref/libmhcref.so is not built (needs the reference sources)")
    return oracle.RefCuda()


@pytest.fixture(scope="module")
def producer():
    if not oracle.RefHRes.available():
        pytest.skip("oracle/_ref/libmhcref_hres.so is not built (needs the reference sources)")
    return oracle.RefHRes()


def bitwise_equal(a, b):
    return torch.equal(a.contiguous().view(torch.int32), b.contiguous().view(torch.int32))


def stream():
    return torch.cuda.current_stream().cuda_stream


def layer_inputs(n, seed, alpha=1.0, width=24, offset=8):
    """H_proj_concat (n, width) with H_res in columns offset..offset+15, rms,
    alpha (one-element tensor), b_res (16,) with a diagonal bias, on cuda:0."""
    g = torch.Generator(device="cuda").manual_seed(seed)
    H = torch.randn(n, width, device="cuda", generator=g)
    rms = torch.rand(n, device="cuda", generator=g) * 1.5 + 0.5
    b = torch.randn(16, device="cuda", generator=g) + 2.0 * torch.eye(4, device="cuda").reshape(16)
    a = torch.tensor([alpha], device="cuda")
    return H, H[:, offset:offset + 16], rms, a, b


def ref_logits(producer, H, rms, alpha, b):
    n = H.shape[0]
    R = torch.empty(n, 4, 4, device="cuda")
    producer.hres_logits_n4(H.data_ptr(), rms.data_ptr(), alpha, b.data_ptr(), R.data_ptr(), n, stream())
    return R


def test_restated_logits_are_the_producers(producer):
    n = 100003
    H, h, rms, a, b = layer_inputs(n, 1, alpha=0.8)
    pre = torch.empty(n, 4, device="cuda")
    post = torch.empty(n, 4, device="cuda")
    Hres = torch.empty(n, 16, device="cuda")
    bp, bq = torch.randn(4, device="cuda"), torch.randn(4, device="cuda")
    producer.fused_h_activations_n4(pre.data_ptr(), post.data_ptr(), Hres.data_ptr(), H.data_ptr(), rms.data_ptr(),
                                    0.5, 0.5, 0.8, bp.data_ptr(), bq.data_ptr(), b.data_ptr(), n, stream())
    R = ref_logits(producer, H, rms, 0.8, b)
    E = torch.empty(n, 16, device="cuda")
    producer.fast_exp(R.data_ptr(), E.data_ptr(), n * 16, stream())
    torch.cuda.synchronize()
    assert bitwise_equal(E, Hres)
    hn, rn, bn = h.cpu().numpy(), rms.cpu().numpy(), b.cpu().numpy()
    R64 = oracle.hres_logits(hn, rn, 0.8, bn)
    err = np.abs(R.cpu().numpy().astype(np.float64) - R64)
    # three roundings (product, reciprocal, fused multiply-add), each relative to its terms' size
    terms = (np.abs(0.8 * hn.astype(np.float64) / rn.astype(np.float64)[:, None]) + np.abs(bn)).reshape(-1, 4, 4)
    assert (err <= 4 * 2.0 ** -24 * terms + 1e-37).all()


@pytest.mark.parametrize("n", [1, 33, 1000, 65537, (1 << 20) + 3])
@pytest.mark.parametrize("alpha", [0.05, 1.0, 4.0])
def test_fused_forward_is_the_reference_two_step(ref, producer, n, alpha):
    H, h, rms, a, b = layer_inputs(n, 10 + n % 97, alpha=alpha)
    T = capi.birkhoff_proj_n4_hres_tensor(h, rms, a, b)
    R = ref_logits(producer, H, rms, alpha, b)
    Tr = torch.empty_like(R)
    ref.birkhoff_proj_n4(R.data_ptr(), Tr.data_ptr(), 1e-6, n, stream())
    torch.cuda.synchronize()
    assert bitwise_equal(T, Tr)


def test_fused_forward_unaligned_and_dense_layouts(ref, producer):
    n = 40001
    H, h, rms, a, b = layer_inputs(n, 3, alpha=1.5)
    R = ref_logits(producer, H, rms, 1.5, b)
    Tr = torch.empty_like(R)
    ref.birkhoff_proj_n4(R.data_ptr(), Tr.data_ptr(), 1e-6, n, stream())
    # stride 21, offset 5: neither the base nor the stride is 16-byte aligned (scalar path)
    H21 = torch.zeros(n, 21, device="cuda")
    H21[:, 5:21] = h
    T21 = capi.birkhoff_proj_n4_hres_tensor(H21[:, 5:21], rms, a, b)
    # dense (n, 4, 4)
    Td = capi.birkhoff_proj_n4_hres_tensor(h.contiguous().view(n, 4, 4), rms, a, b)
    torch.cuda.synchronize()
    assert bitwise_equal(T21, Tr) and bitwise_equal(Td, Tr)


def run_backward(G, T, h, rms, a, ws_bytes=None, dh=None):
    n = h.shape[0]
    if dh is None:
        dh = torch.empty(n, 16, device="cuda")
    drms = torch.empty(n, device="cuda")
    dalpha = torch.empty((), device="cuda")
    db = torch.empty(4, 4, device="cuda")
    need = capi.birkhoff_proj_n4_hres_backward_workspace(n)
    ws = torch.empty(max(need if ws_bytes is None else ws_bytes, 4) // 4 + 1, device="cuda")
    nbytes = need if ws_bytes is None else ws_bytes
    capi.birkhoff_proj_n4_hres_backward(G.data_ptr(), T.data_ptr(), h.data_ptr(), h.stride(0), rms.data_ptr(),
                                        a.data_ptr(), dh.data_ptr(), dh.stride(0), drms.data_ptr(),
                                        dalpha.data_ptr(), db.data_ptr(), n, ws.data_ptr(), nbytes, stream())
    return dh, drms, dalpha, db


def check_against_chain(D, h, rms, alpha, dh, drms, dalpha, db):
    """Float32 results against the float64 chain rule on the same D.  Bounds:
    dh and drms elementwise (a few roundings of products); the batch sums
    within 4e-6 of the sum of the magnitudes of their terms (fp32
    accumulation over at most a few dozen terms per thread, then trees)."""
    Dn = D.cpu().numpy().reshape(-1, 16).astype(np.float64)
    hn = h.cpu().numpy().astype(np.float64)
    rn = rms.cpu().numpy().astype(np.float64)
    edh, edrms, edalpha, edb = oracle.hres_backward_chain(Dn, hn, rn, alpha)
    assert (np.abs(dh.cpu().numpy() - edh) <= 1e-6 * np.abs(edh) + 1e-37).all()
    mag_q = np.abs(Dn * hn).sum(1)
    assert (np.abs(drms.cpu().numpy() - edrms) <= 4e-6 * abs(alpha) / rn ** 2 * mag_q + 1e-37).all()
    mag_b = np.abs(Dn).sum(axis=0).reshape(4, 4)
    assert (np.abs(db.cpu().numpy() - edb) <= 4e-6 * mag_b + 1e-37).all()
    assert abs(float(dalpha) - edalpha) <= 4e-6 * (mag_q / rn).sum() + 1e-37


@pytest.mark.parametrize("n", [1, 257, 100003, 1 << 21])
def test_fused_backward_against_reference_gradient(ref, producer, n):
    alpha = 0.9
    H, h, rms, a, b = layer_inputs(n, 20 + n % 13, alpha=alpha)
    G = torch.randn(n, 4, 4, device="cuda", generator=torch.Generator(device="cuda").manual_seed(5))
    T = capi.birkhoff_proj_n4_hres_tensor(h, rms, a, b)
    dh, drms, dalpha, db = run_backward(G, T, h, rms, a)
    D = torch.empty_like(G)
    ref.birkhoff_proj_n4_backward(G.data_ptr(), T.data_ptr(), D.data_ptr(), n, stream())
    torch.cuda.synchronize()
    check_against_chain(D, h, rms, alpha, dh, drms, dalpha, db)


def test_fused_backward_is_deterministic_and_layout_free(ref, producer):
    n = 300007
    H, h, rms, a, b = layer_inputs(n, 7, alpha=2.0)
    G = torch.randn(n, 4, 4, device="cuda")
    T = capi.birkhoff_proj_n4_hres_tensor(h, rms, a, b)
    r1 = run_backward(G, T, h, rms, a)
    r2 = run_backward(G, T, h, rms, a)
    # dh written into columns 8..23 of a (n, 24) gradient buffer, h read from a contiguous copy
    buf = torch.full((n, 24), 7.0, device="cuda")
    r3 = run_backward(G, T, h.contiguous(), rms, a, dh=buf[:, 8:24])
    torch.cuda.synchronize()
    for x, y in zip(r1, r2):
        assert bitwise_equal(x, y)
    assert bitwise_equal(r3[0], r1[0]) and bitwise_equal(r3[1], r1[1])
    assert bitwise_equal(r3[2], r1[2]) and bitwise_equal(r3[3], r1[3])
    assert bool((buf[:, :8] == 7.0).all())


def test_fused_backward_small_workspace_and_empty_batch():
    n = 50000
    H, h, rms, a, b = layer_inputs(n, 8)
    G = torch.randn(n, 4, 4, device="cuda")
    T = capi.birkhoff_proj_n4_hres_tensor(h, rms, a, b)
    full = run_backward(G, T, h, rms, a)
    one_row = run_backward(G, T, h, rms, a, ws_bytes=68)  # one block does the whole batch
    torch.cuda.synchronize()
    assert bitwise_equal(full[0], one_row[0]) and bitwise_equal(full[1], one_row[1])
    # one block sums the batch in another order: same values to fp32 accumulation error
    Dabs = (full[0] * (rms / a)[:, None]).abs()  # |D| recovered from dh = D * alpha / rms
    assert bool(((full[3] - one_row[3]).abs().reshape(16) <= 1e-4 * Dabs.sum(0)).all())
    qabs = (Dabs * h.abs()).sum(1) / rms
    assert abs(float(full[2] - one_row[2])) <= 1e-4 * float(qabs.sum())
    with pytest.raises(capi.MhcError):
        run_backward(G, T, h, rms, a, ws_bytes=64)  # smaller than one row of partial sums
    e = torch.empty(0, 24, device="cuda")
    z = run_backward(torch.empty(0, 4, 4, device="cuda"), torch.empty(0, 4, 4, device="cuda"), e[:, 8:24],
                     torch.empty(0, device="cuda"), a)
    torch.cuda.synchronize()
    assert float(z[2]) == 0.0 and bool((z[3] == 0).all())


def test_module_autograd(ref, producer):
    n = 4096
    H, h, rms, a, b = layer_inputs(n, 9, alpha=1.2)
    Hp = H.clone().requires_grad_(True)
    rp = rms.clone().requires_grad_(True)
    ap = torch.nn.Parameter(torch.tensor(1.2, device="cuda"))
    bp = torch.nn.Parameter(b.clone().view(4, 4))
    G = torch.randn(n, 4, 4, device="cuda")
    m = mhc_proj.MHCProjectionN4HRes()
    T = m(Hp[:, 8:24], rp, ap, bp)
    (T * G).sum().backward()
    # the module is the fused kernels: same bits as the C ABI
    T2 = capi.birkhoff_proj_n4_hres_tensor(h, rms, a, b)
    dh, drms, dalpha, db = run_backward(G, T2, h, rms, a)
    torch.cuda.synchronize()
    assert bitwise_equal(T.detach(), T2)
    assert bitwise_equal(Hp.grad[:, 8:24], dh) and bool((Hp.grad[:, :8] == 0).all())
    assert bitwise_equal(rp.grad, drms) and bitwise_equal(ap.grad, dalpha) and bitwise_equal(bp.grad, db)
    # and agrees with autograd through the unfused composition to the projection's tolerance
    Hq = H.clone().requires_grad_(True)
    rq = rms.clone().requires_grad_(True)
    aq = torch.tensor(1.2, device="cuda", requires_grad=True)
    bq = b.clone().view(4, 4).requires_grad_(True)
    Tq = mhc_proj.MHCProjectionN4()(aq * Hq[:, 8:24].reshape(n, 4, 4) / rq[:, None, None] + bq)
    (Tq * G).sum().backward()
    assert torch.allclose(T, Tq, atol=1e-4)
    assert torch.allclose(Hp.grad, Hq.grad, atol=1e-3, rtol=1e-3)
    assert torch.allclose(bp.grad, bq.grad, atol=1e-2, rtol=1e-3)


def test_functional_binding_dtypes_and_number_alpha(ref, producer):
    n = 2048
    H, h, rms, a, b = layer_inputs(n, 11, alpha=0.7)
    out = mhc_proj.torch.birkhoff_proj_n4_hres(h, rms, 0.7, b)["T"]
    T = capi.birkhoff_proj_n4_hres_tensor(h, rms, a, b)
    assert bitwise_equal(out, T)
    G = torch.randn(n, 4, 4, device="cuda")
    g = mhc_proj.torch.birkhoff_proj_n4_hres_backward(G, T, h, rms, 0.7, b_res=b)
    dh, drms, dalpha, db = run_backward(G, T, h, rms, a)
    torch.cuda.synchronize()
    assert g["d_h_res"].shape == h.shape and g["d_b_res"].shape == b.shape and g["d_alpha_res"].dim() == 0
    assert bitwise_equal(g["d_h_res"], dh) and bitwise_equal(g["d_rms"], drms)
    assert bitwise_equal(g["d_alpha_res"], dalpha) and bitwise_equal(g["d_b_res"].view(4, 4), db)
    # bf16 inputs are widened exactly; T returns in h's dtype
    hb = h.to(torch.bfloat16)
    Tb = mhc_proj.torch.birkhoff_proj_n4_hres(hb, rms, 0.7, b)["T"]
    Tf = capi.birkhoff_proj_n4_hres_tensor(hb.float(), rms, a, b)
    assert Tb.dtype == torch.bfloat16 and bitwise_equal(Tb.float(), Tf.to(torch.bfloat16).float())


def test_cuda_graph_capture(producer):
    n = 1 << 15
    H, h, rms, a, b = layer_inputs(n, 12)
    G = torch.randn(n, 4, 4, device="cuda")
    T0 = mhc_proj.torch.birkhoff_proj_n4_hres(h, rms, a, b)["T"]
    g0 = mhc_proj.torch.birkhoff_proj_n4_hres_backward(G, T0, h, rms, a, b_res=b)
    gr = torch.cuda.CUDAGraph()
    with torch.cuda.graph(gr):
        T = mhc_proj.torch.birkhoff_proj_n4_hres(h, rms, a, b)["T"]
        g = mhc_proj.torch.birkhoff_proj_n4_hres_backward(G, T, h, rms, a, b_res=b)
    gr.replay()
    torch.cuda.synchronize()
    assert bitwise_equal(T, T0)
    for k in ("d_h_res", "d_rms", "d_alpha_res", "d_b_res"):
        assert bitwise_equal(g[k], g0[k])


# --- the producer fused with Sinkhorn-Knopp ---------------------------------

def ref_producer_hres(producer, H, rms, alpha, b):
    """The reference producer's H_res (its exp of the pre-activation), (n, 4, 4)."""
    n = H.shape[0]
    pre = torch.empty(n, 4, device="cuda")
    post = torch.empty(n, 4, device="cuda")
    M = torch.empty(n, 4, 4, device="cuda")
    z = torch.zeros(4, device="cuda")
    producer.fused_h_activations_n4(pre.data_ptr(), post.data_ptr(), M.data_ptr(), H.data_ptr(), rms.data_ptr(),
                                    1.0, 1.0, alpha, z.data_ptr(), z.data_ptr(), b.data_ptr(), n, stream())
    return M


@pytest.mark.parametrize("n", [1, 33, 65537, (1 << 20) + 3])
@pytest.mark.parametrize("alpha", [0.05, 1.0])
@pytest.mark.parametrize("iters", [0, 1, 20])
def test_sk_fused_forward_is_the_reference_producer_then_sk(ref, producer, n, alpha, iters):
    H, h, rms, a, b = layer_inputs(n, 30 + n % 89, alpha=alpha)
    T = capi.sinkhorn_knopp_n4_hres_tensor(h, rms, a, b, iters)
    M = ref_producer_hres(producer, H, rms, alpha, b)
    Tr = torch.empty_like(M)
    ref.sinkhorn_knopp_n4(M.data_ptr(), Tr.data_ptr(), n, iters, stream())
    torch.cuda.synchronize()
    assert bitwise_equal(T, Tr)
    if iters == 0:
        assert bitwise_equal(T, M)


def test_sk_fused_forward_layouts(ref, producer):
    n = 40001
    H, h, rms, a, b = layer_inputs(n, 31, alpha=0.7)
    M = ref_producer_hres(producer, H, rms, 0.7, b)
    Tr = torch.empty_like(M)
    ref.sinkhorn_knopp_n4(M.data_ptr(), Tr.data_ptr(), n, 20, stream())
    H21 = torch.zeros(n, 21, device="cuda")
    H21[:, 5:21] = h
    T21 = capi.sinkhorn_knopp_n4_hres_tensor(H21[:, 5:21], rms, a, b)
    Td = capi.sinkhorn_knopp_n4_hres_tensor(h.contiguous().view(n, 4, 4), rms, a, b)
    torch.cuda.synchronize()
    assert bitwise_equal(T21, Tr) and bitwise_equal(Td, Tr)


@pytest.mark.parametrize("n,iters", [(1, 20), (257, 20), (100003, 20), (100003, 5), (1 << 20, 20)])
def test_sk_fused_backward_against_the_unfused_gradient(producer, n, iters):
    alpha = 0.8
    H, h, rms, a, b = layer_inputs(n, 40 + n % 7, alpha=alpha)
    G = torch.randn(n, 4, 4, device="cuda", generator=torch.Generator(device="cuda").manual_seed(6))
    dh, drms, dalpha, db = capi.sinkhorn_knopp_n4_hres_backward_tensor(G, h, rms, a, b, iters)
    M = ref_producer_hres(producer, H, rms, alpha, b)
    dM = capi.sinkhorn_knopp_n4_backward_tensor(G, M, iters)  # the exact VJP of the plain kernel
    dR = dM * M  # what the fused kernel forms, rounded the same way
    torch.cuda.synchronize()
    check_against_chain(dR, h, rms, alpha, dh, drms, dalpha, db)


def test_sk_fused_backward_checks_and_empty_batch(producer):
    n = 1000
    H, h, rms, a, b = layer_inputs(n, 41)
    G = torch.randn(n, 4, 4, device="cuda")
    r1 = capi.sinkhorn_knopp_n4_hres_backward_tensor(G, h, rms, a, b)
    r2 = capi.sinkhorn_knopp_n4_hres_backward_tensor(G, h, rms, a, b)
    torch.cuda.synchronize()
    for x, y in zip(r1, r2):
        assert bitwise_equal(x, y)
    dh, drms, dalpha, db = (torch.empty(n, 16, device="cuda"), torch.empty(n, device="cuda"),
                            torch.empty((), device="cuda"), torch.empty(4, 4, device="cuda"))
    need = capi.sinkhorn_knopp_n4_hres_backward_workspace(n)
    assert need == 8 * 17 * 4  # ceil(1000 / 128) blocks of 17 partial sums
    ws = torch.empty(need // 4, device="cuda")
    args = [G.data_ptr(), h.data_ptr(), 24, rms.data_ptr(), a.data_ptr(), b.data_ptr(), dh.data_ptr(), 16,
            drms.data_ptr(), dalpha.data_ptr(), db.data_ptr(), n]
    with pytest.raises(capi.MhcError) as e:
        capi.sinkhorn_knopp_n4_hres_backward(*args, 20, ws.data_ptr(), need - 4, stream())
    assert e.value.code == capi.MHC_ERR_INVALID_VALUE
    with pytest.raises(capi.MhcError) as e:
        capi.sinkhorn_knopp_n4_hres_backward(*args, 21, ws.data_ptr(), need, stream())
    assert e.value.code == capi.MHC_ERR_ITERS
    with pytest.raises(ValueError):
        mhc_proj.torch.sinkhorn_knopp_n4_hres_backward(G, h, rms, a, b, max_iter=21)
    E = torch.empty(0, 24, device="cuda")
    z = capi.sinkhorn_knopp_n4_hres_backward_tensor(torch.empty(0, 4, 4, device="cuda"), E[:, 8:24],
                                                    torch.empty(0, device="cuda"), a, b)
    torch.cuda.synchronize()
    assert float(z[2]) == 0.0 and bool((z[3] == 0).all())


def test_sk_module_autograd(producer):
    n = 4096
    H, h, rms, a, b = layer_inputs(n, 42, alpha=0.6)
    Hp = H.clone().requires_grad_(True)
    rp = rms.clone().requires_grad_(True)
    ap = torch.nn.Parameter(torch.tensor(0.6, device="cuda"))
    bp = torch.nn.Parameter(b.clone().view(4, 4))
    G = torch.randn(n, 4, 4, device="cuda")
    T = mhc_proj.MHCSinkhornN4HRes(max_iter=20)(Hp[:, 8:24], rp, ap, bp)
    (T * G).sum().backward()
    T2 = capi.sinkhorn_knopp_n4_hres_tensor(h, rms, a, b)
    dh, drms, dalpha, db = capi.sinkhorn_knopp_n4_hres_backward_tensor(G, h, rms, a, b)
    torch.cuda.synchronize()
    assert bitwise_equal(T.detach(), T2)
    assert bitwise_equal(Hp.grad[:, 8:24], dh) and bool((Hp.grad[:, :8] == 0).all())
    assert bitwise_equal(rp.grad, drms) and bitwise_equal(ap.grad, dalpha) and bitwise_equal(bp.grad, db)
    # the vanilla Sinkhorn on the float64 producer output agrees to the kernels' eps semantics
    with torch.enable_grad():
        h64 = h.double().requires_grad_(True)
        P = torch.exp(0.6 * h64.reshape(n, 4, 4) / rms.double()[:, None, None] + b.double().view(4, 4))
        for _ in range(20):
            P = P / P.sum(2, keepdim=True)
            P = P / P.sum(1, keepdim=True)
        (P * G.double()).sum().backward()
    assert torch.allclose(T.double(), P.detach(), atol=1e-5)
    assert torch.allclose(Hp.grad[:, 8:24].double(), h64.grad, atol=1e-4, rtol=1e-4)
