"""Autograd functions and modules over the native kernels.

Same classes, signatures and behaviour as the reference's
mhc_proj/module.py:5-84:
  MHCProjectionN4(tol=1e-6)      forward: Newton projection, saves T;
                                 backward: implicit-function-theorem kernel.
  MHCSinkhornN4(max_iter=20)     forward: exp then fixed-iteration
                                 Sinkhorn-Knopp; backward: the Sinkhorn-Knopp
                                 backward times exp(R).  For fp32 CUDA inputs
                                 both run as one fused kernel each on the
                                 logits (saving R, 320 instead of 640 bytes
                                 of HBM traffic per matrix); other inputs take
                                 the reference's composition (torch.exp in
                                 the input dtype, kernel on exp(R), saves it).
                                 approx_reciprocal=True (not in the
                                 reference) runs the fused forward with the
                                 hardware reciprocal: within 1e-6 of the
                                 reference's bits, ~20% faster; gradients
                                 are unchanged.
Both take any tensor whose last two dimensions are 4 x 4 (ValueError
otherwise) and return a tensor of the input's shape.  A ``None`` incoming
gradient (possible because gradient materialisation is off) yields ``None``.
"""
import torch
import torch.nn as nn

from . import _internal


class MHCProjectionN4Function(torch.autograd.Function):
    @staticmethod
    def forward(ctx, R, tol=1e-6, save_duals=False):
        in_shape = R.shape
        R = R.reshape(-1, 4, 4)
        ctx.save_duals = save_duals
        if save_duals:
            out = _internal.torch.birkhoff_proj_n4(R, tol, return_duals=True)
            T = out["T"]
            ctx.save_for_backward(R, out["beta"])
        else:
            T = _internal.torch.birkhoff_proj_n4(R, tol)["T"]
            ctx.save_for_backward(T)
        ctx.set_materialize_grads(False)
        return T.view(in_shape)

    @staticmethod
    def backward(ctx, grad_output):
        if not ctx.needs_input_grad[0] or grad_output is None:
            return None, None, None
        in_shape = grad_output.shape
        G = grad_output.reshape(-1, 4, 4)
        if ctx.save_duals:
            R, beta = ctx.saved_tensors
            D = _internal.torch.birkhoff_proj_n4_backward_duals(G, R, beta)["D"]
        else:
            (T,) = ctx.saved_tensors
            D = _internal.torch.birkhoff_proj_n4_backward(G, T)["D"]
        return D.view(in_shape), None, None


class MHCProjectionN4(nn.Module):
    """save_duals=True (not in the reference) keeps R and the final duals
    beta (16 bytes per matrix) for the backward instead of T (64), which then
    rebuilds T bit for bit; gradients are identical."""

    def __init__(self, tol=1e-6, save_duals=False):
        super().__init__()
        self.tol = tol
        self.save_duals = save_duals

    def forward(self, x):
        in_shape = x.shape
        if x.ndim < 2 or in_shape[-1] != 4 or in_shape[-2] != 4:
            raise ValueError("x must be a tensor of size B x 4 x 4")
        return MHCProjectionN4Function.apply(x, self.tol, self.save_duals)


class MHCSinkhornN4Function(torch.autograd.Function):
    @staticmethod
    def forward(ctx, R, max_iter=20, approx_reciprocal=False):
        in_shape = R.shape
        R3 = R.reshape(-1, 4, 4)
        ctx.max_iter = max_iter
        # CUDA fp32/bf16/fp16: the kernels form exp(R) (rounded to R's type, as
        # torch.exp in that type) and, backward, the product with it; other
        # inputs take the reference's composition.
        ctx.fused = R3.is_cuda and R3.dtype in (torch.float32, torch.bfloat16, torch.float16)
        if ctx.fused:
            T = _internal.torch.sinkhorn_knopp_n4_logits(R3, max_iter, approx_reciprocal=approx_reciprocal)["T"]
            ctx.save_for_backward(R3)
        else:
            expon = torch.exp(R3)
            T = _internal.torch.sinkhorn_knopp_n4(expon, max_iter)["T"]
            ctx.save_for_backward(expon)
        ctx.set_materialize_grads(False)
        return T.view(in_shape)

    @staticmethod
    def backward(ctx, grad_output):
        if not ctx.needs_input_grad[0] or grad_output is None:
            return None, None, None
        in_shape = grad_output.shape
        G = grad_output.reshape(-1, 4, 4)
        (saved,) = ctx.saved_tensors
        if ctx.fused:
            D = _internal.torch.sinkhorn_knopp_n4_logits_backward(G, saved, ctx.max_iter)["D"]
        else:
            D = _internal.torch.sinkhorn_knopp_n4_backward(G, saved, ctx.max_iter)["D"] * saved
        return D.view(in_shape), None, None


class MHCSinkhornN4(nn.Module):
    """approx_reciprocal=True (not in the reference): the fused forward's
    normalisation factors from the hardware reciprocal."""

    def __init__(self, max_iter=20, approx_reciprocal=False):
        super().__init__()
        self.max_iter = max_iter
        self.approx_reciprocal = approx_reciprocal

    def forward(self, x):
        in_shape = x.shape
        if x.ndim < 2 or in_shape[-1] != 4 or in_shape[-2] != 4:
            raise ValueError("x must be a tensor of size B x 4 x 4")
        return MHCSinkhornN4Function.apply(x, self.max_iter, self.approx_reciprocal)


class MHCProjectionN4HResFunction(torch.autograd.Function):
    """T = birkhoff_proj_n4(alpha_res * h_res / rms + b_res), the H_res
    pre-activation formed in the projection's load; gradients for all four
    inputs from one fused backward kernel plus a deterministic batch
    reduction.  h_res: (..., 16) or (..., 4, 4); rms: (...); alpha_res: a
    one-element tensor; b_res: 16 elements.  Returns (..., 4, 4)."""

    @staticmethod
    def forward(ctx, h_res, rms, alpha_res, b_res, tol=1e-6):
        lead = rms.shape
        h2 = h_res.reshape(-1, 16)
        T = _internal.torch.birkhoff_proj_n4_hres(h2, rms.reshape(-1), alpha_res, b_res, tol)["T"]
        ctx.save_for_backward(T, h2, rms, alpha_res, b_res)
        ctx.h_shape = h_res.shape
        ctx.set_materialize_grads(False)
        return T.view(*lead, 4, 4)

    @staticmethod
    def backward(ctx, grad_output):
        if grad_output is None or not any(ctx.needs_input_grad[:4]):
            return None, None, None, None, None
        T, h2, rms, alpha_res, b_res = ctx.saved_tensors
        g = _internal.torch.birkhoff_proj_n4_hres_backward(grad_output.reshape(-1, 4, 4), T, h2, rms.reshape(-1),
                                                           alpha_res, b_res=b_res)
        need = ctx.needs_input_grad
        return (g["d_h_res"].view(ctx.h_shape) if need[0] else None,
                g["d_rms"].view(rms.shape) if need[1] else None,
                g["d_alpha_res"] if need[2] else None,
                g["d_b_res"] if need[3] else None,
                None)


class MHCProjectionN4HRes(nn.Module):
    """Projection fused with the mHC layer's H_res pre-activation (no
    reference counterpart; the reference's producer is fused_h_activations,
    src/utils.cuh:50-127, a separate kernel that writes exp(R)).

    forward(h_res, rms, alpha_res, b_res) with h_res (..., 16) -- e.g. the
    column slice H_proj_concat[..., 8:24] -- or (..., 4, 4), rms (...),
    alpha_res a number or one-element tensor, b_res 16 elements; returns
    (..., 4, 4), the same T as MHCProjectionN4 applied to
    alpha_res * h_res / rms + b_res computed with the producer's arithmetic."""

    def __init__(self, tol=1e-6):
        super().__init__()
        self.tol = tol

    def forward(self, h_res, rms, alpha_res, b_res):
        _hres_lead(h_res, rms)
        if not torch.is_tensor(alpha_res):
            alpha_res = torch.tensor(float(alpha_res), dtype=torch.float32, device=h_res.device)
        return MHCProjectionN4HResFunction.apply(h_res, rms, alpha_res, b_res, self.tol)


class MHCSinkhornN4HResFunction(torch.autograd.Function):
    """T = sinkhorn_knopp_n4(exp(alpha_res * h_res / rms + b_res)) with the
    producer's own exponential formed in the kernel's load; gradients for
    all four inputs from one fused backward kernel plus the batch fold."""

    @staticmethod
    def forward(ctx, h_res, rms, alpha_res, b_res, max_iter=20):
        lead = rms.shape
        h2 = h_res.reshape(-1, 16)
        T = _internal.torch.sinkhorn_knopp_n4_hres(h2, rms.reshape(-1), alpha_res, b_res, max_iter)["T"]
        ctx.save_for_backward(h2, rms, alpha_res, b_res)
        ctx.h_shape = h_res.shape
        ctx.max_iter = max_iter
        ctx.set_materialize_grads(False)
        return T.view(*lead, 4, 4)

    @staticmethod
    def backward(ctx, grad_output):
        if grad_output is None or not any(ctx.needs_input_grad[:4]):
            return None, None, None, None, None
        h2, rms, alpha_res, b_res = ctx.saved_tensors
        g = _internal.torch.sinkhorn_knopp_n4_hres_backward(grad_output.reshape(-1, 4, 4), h2, rms.reshape(-1),
                                                            alpha_res, b_res, ctx.max_iter)
        need = ctx.needs_input_grad
        return (g["d_h_res"].view(ctx.h_shape) if need[0] else None,
                g["d_rms"].view(rms.shape) if need[1] else None,
                g["d_alpha_res"] if need[2] else None,
                g["d_b_res"] if need[3] else None,
                None)


def _hres_lead(h_res, rms):
    if h_res.shape[-1] == 16:
        lead = h_res.shape[:-1]
    elif h_res.ndim >= 2 and h_res.shape[-2:] == (4, 4):
        lead = h_res.shape[:-2]
    else:
        raise ValueError("h_res must be a tensor of size ... x 16 or ... x 4 x 4")
    if tuple(rms.shape) != tuple(lead):
        raise ValueError("rms must have the leading shape of h_res")


class MHCSinkhornN4HRes(nn.Module):
    """Sinkhorn-Knopp fused with the mHC layer's H_res producer: the same T as
    the reference's producer (fused_h_activations, src/utils.cuh:50-127) writing
    H_res = exp(alpha_res * h_res / rms + b_res) followed by its
    sinkhorn_knopp_n4, without H_res in memory.  forward(h_res, rms,
    alpha_res, b_res) as MHCProjectionN4HRes; returns (..., 4, 4)."""

    def __init__(self, max_iter=20):
        super().__init__()
        self.max_iter = max_iter

    def forward(self, h_res, rms, alpha_res, b_res):
        _hres_lead(h_res, rms)
        if not torch.is_tensor(alpha_res):
            alpha_res = torch.tensor(float(alpha_res), dtype=torch.float32, device=h_res.device)
        return MHCSinkhornN4HResFunction.apply(h_res, rms, alpha_res, b_res, self.max_iter)
