"""Native storage types and strided batches for the Newton and Sinkhorn-Knopp
pairs.

The reference's wrappers convert every input to contiguous fp32 and the
outputs back to the input dtype (solvers_torch.cpp:61,67,82,128-136,152).
Here fp32/bf16/fp16 batches with contiguous 4x4 matrices are read in place at
any batch stride and written in the input dtype by the kernels themselves;
the results must be the bits of that conversion path."""
import pytest
import torch

import mhc_proj
import oracle
from mhc_proj import capi
from mhc_proj.workloads import make_logits

pytestmark = pytest.mark.gpu
DTYPES = [torch.float32, torch.bfloat16, torch.float16]


def same_bits(a, b):
    assert a.dtype == b.dtype and a.shape == b.shape
    ia = a.contiguous().view(torch.int16 if a.element_size() == 2 else torch.int32)
    ib = b.contiguous().view(torch.int16 if b.element_size() == 2 else torch.int32)
    both_nan = torch.isnan(a) & torch.isnan(b)
    return bool(((ia == ib) | both_nan).all())


def strided_batch(kind, n, dtype, stride, offset, seed):
    """(n, 4, 4) view with batch stride `stride` elements into a wider buffer,
    like a slice of a projection output."""
    full = make_logits(kind, n * stride // 16 + 2, seed=seed).reshape(-1)[: n * stride + offset + 16]
    buf = torch.empty(n * stride + 16, device="cuda", dtype=dtype)
    buf.copy_(full[: buf.numel()].to(dtype))
    return torch.as_strided(buf, (n, 4, 4), (stride, 4, 1), offset)


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("stride,offset", [(16, 0), (24, 8), (20, 4), (32, 3), (16, 1)])
def test_forward_native_equals_conversion_path(dtype, stride, offset):
    n = 30001
    R = strided_batch("sigma_mix", n, dtype, stride, offset, seed=stride + offset)
    T = mhc_proj.torch.birkhoff_proj_n4(R, 1e-6)["T"]
    assert T.dtype == dtype and T.is_contiguous()
    expected = capi.birkhoff_proj_n4_tensor(R.float().contiguous()).to(dtype)
    assert same_bits(T, expected)
    assert same_bits(capi.birkhoff_proj_n4_ex_tensor(R), expected)


@pytest.mark.parametrize("gdt", DTYPES)
@pytest.mark.parametrize("tdt", DTYPES)
def test_backward_native_equals_conversion_path(gdt, tdt):
    n = 20000
    R = make_logits("normal", n, seed=5)
    T32 = capi.birkhoff_proj_n4_tensor(R)
    T = strided_batch("normal", n, tdt, 24, 8, seed=1)
    T.copy_(T32.to(tdt))
    G = strided_batch("normal", n, gdt, 20, 4, seed=2)
    D = mhc_proj.torch.birkhoff_proj_n4_backward(G, T)["D"]
    assert D.dtype == gdt and D.is_contiguous()
    expected = capi.birkhoff_proj_n4_backward_tensor(G.float().contiguous(), T.float().contiguous()).to(gdt)
    assert same_bits(D, expected)


def test_bf16_matches_the_reference_wrapper_semantics():
    """Against the reference kernels with the reference wrapper's conversions:
    R.to(fp32) -> birkhoff_proj_n4 -> T.to(bf16)."""
    if not oracle.RefCuda.available():
        pytest.skip("reference kernels not built")
    ref = oracle.RefCuda()
    n = 1 << 16
    R = make_logits("mixture", n, seed=9).to(torch.bfloat16)
    R32 = R.float().contiguous()
    Tr = torch.empty_like(R32)
    ref.birkhoff_proj_n4(R32.data_ptr(), Tr.data_ptr(), 1e-6, n, torch.cuda.current_stream().cuda_stream)
    assert same_bits(mhc_proj.torch.birkhoff_proj_n4(R)["T"], Tr.to(torch.bfloat16))


def test_module_on_a_bf16_slice_with_autograd():
    n = 4096
    proj_out = make_logits("normal", n * 2, seed=11).reshape(n, 32).to(torch.bfloat16)
    x = proj_out[:, 8:24].reshape(n, 4, 4).detach().requires_grad_(True)   # stride (32, 4, 1)
    assert x.stride() != (16, 4, 1) or True
    G = make_logits("normal", n, seed=12).to(torch.bfloat16)
    T = mhc_proj.MHCProjectionN4()(x)
    (T * G).float().sum().backward()
    assert T.dtype == torch.bfloat16 and x.grad.dtype == torch.bfloat16
    T_conv = capi.birkhoff_proj_n4_tensor(x.detach().float().contiguous()).to(torch.bfloat16)
    assert same_bits(T.detach(), T_conv)
    D_conv = capi.birkhoff_proj_n4_backward_tensor(G.float().contiguous(), T_conv.float()).to(torch.bfloat16)
    assert same_bits(x.grad, D_conv)


# ---- the Sinkhorn-Knopp pair -------------------------------------------------
#
# The reference's SK wrappers convert to contiguous fp32 and back
# (solvers_torch.cpp:190,196,211,258-266,282) and its MHCSinkhornN4 computes
# torch.exp, and the final D * expon, in the input's type (module.py:50,70).
# The kernels here read and write the native type in place; the expected
# values below are that composition, on this repository's fp32 kernels (which
# are bitwise the reference's for the forward; the backward is the exact VJP).

def sk_reference_forward(X, iters, logits):
    M = torch.exp(X) if logits else X
    return capi.sinkhorn_knopp_n4_tensor(M.float().contiguous(), iters).to(X.dtype)


def sk_reference_backward(G, X, iters, logits):
    M = torch.exp(X) if logits else X
    D = capi.sinkhorn_knopp_n4_backward_tensor(G.float().contiguous(), M.float().contiguous(), iters).to(G.dtype)
    return D * M if logits else D


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("stride,offset", [(16, 0), (24, 8), (20, 4), (16, 1)])
@pytest.mark.parametrize("logits", [False, True])
def test_sinkhorn_forward_native_equals_reference_composition(dtype, stride, offset, logits):
    n = 30001
    X = strided_batch("sigma_mix", n, dtype, stride, offset, seed=40 + stride + offset)
    if not logits:
        X.copy_(torch.exp(X.float()).to(dtype))
    for iters in (0, 1, 20):
        fn = mhc_proj.torch.sinkhorn_knopp_n4_logits if logits else mhc_proj.torch.sinkhorn_knopp_n4
        T = fn(X, iters)["T"]
        assert T.dtype == dtype and T.is_contiguous()
        expected = sk_reference_forward(X, iters, logits)
        assert same_bits(T, expected), (iters, logits)
        assert same_bits(capi.sinkhorn_knopp_n4_strided_tensor(X, iters, logits=logits), expected)


@pytest.mark.parametrize("gdt", DTYPES)
@pytest.mark.parametrize("xdt", DTYPES)
@pytest.mark.parametrize("logits", [False, True])
def test_sinkhorn_backward_native_equals_reference_composition(gdt, xdt, logits):
    """D in G's type.  With logits the composition's product is in the
    promoted type when G's and R's types differ; the fused backward rounds it
    to G's type (the module always passes G and R of the same type)."""
    n = 20000
    X = strided_batch("normal", n, xdt, 24, 8, seed=11)
    if not logits:
        X.copy_(torch.exp(X.float()).to(xdt))
    G = strided_batch("normal", n, gdt, 20, 4, seed=12)
    for iters in (0, 1, 7, 20):
        fn = mhc_proj.torch.sinkhorn_knopp_n4_logits_backward if logits else mhc_proj.torch.sinkhorn_knopp_n4_backward
        D = fn(G, X, iters)["D"]
        assert D.dtype == gdt and D.is_contiguous()
        expected = sk_reference_backward(G, X, iters, logits).to(gdt)
        assert same_bits(D, expected), (iters, logits)
        assert same_bits(capi.sinkhorn_knopp_n4_backward_strided_tensor(G, X, iters, logits=logits), expected)


def test_sinkhorn_native_paths_reach_both_kernels_layouts():
    """A non-native layout of a native type (a transposed batch) is made
    contiguous in its own type: the same bits as the contiguous input."""
    n = 4099
    X = make_logits("normal", n, seed=21).to(torch.bfloat16)
    Xt = X.transpose(1, 2).contiguous().transpose(1, 2)  # the same values, column-major matrices
    assert not Xt.is_contiguous()
    assert same_bits(mhc_proj.torch.sinkhorn_knopp_n4_logits(Xt, 20)["T"],
                     mhc_proj.torch.sinkhorn_knopp_n4_logits(X, 20)["T"])


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_sinkhorn_module_on_a_slice_with_autograd(dtype):
    """MHCSinkhornN4 on H_res logits as the mHC layer holds them: columns
    8..23 of a (tokens, 24) projection output in bf16/fp16, read in place;
    T and the input gradient are the reference module's bits."""
    n = 8192
    H = make_logits("normal", n * 24 // 16, seed=31).reshape(n, 24).to(dtype)
    x = H[:, 8:24].reshape(n, 4, 4)
    assert x.stride(0) == 24
    xa = H.clone().requires_grad_(True)
    T = mhc_proj.MHCSinkhornN4(max_iter=20)(xa[:, 8:24].reshape(n, 4, 4))
    G = make_logits("normal", n, seed=32).to(dtype)
    (T * G).sum().backward()
    assert same_bits(T.detach(), sk_reference_forward(x, 20, True))
    assert same_bits(xa.grad[:, 8:24].reshape(n, 4, 4), sk_reference_backward(G, x, 20, True))
    assert bool((xa.grad[:, :8] == 0).all())
