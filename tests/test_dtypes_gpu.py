"""Native storage types and strided batches for the Newton pair.

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
