// mhc_proj._internal: the PyTorch face of libmhcproj.so.
//
// Mirrors the reference's pybind11 module (src/bindings.cpp:40-60) and its
// tensor wrappers (src/solvers_torch.cpp): a submodule `torch` with four
// functions of the same names, argument names and defaults, each returning a
// dict.  The conventions are the reference's:
//   - inputs must be 3-D B x 4 x 4, else RuntimeError;
//   - inputs of any dtype/device are converted to fp32 on the CUDA device they
//     are on (the current CUDA device for CPU tensors) and made contiguous;
//   - outputs are new tensors converted back to the (first) input's
//     dtype/device; the backward converts T to G's dtype/device;
//   - sinkhorn_knopp_n4_backward with max_iter > 20 raises ValueError;
//   - extra keyword arguments are accepted and ignored.
// Functions with no reference counterpart: sinkhorn_knopp_n4_logits and its
// backward take the logits R and fuse exp(R) (and, backward, the product with
// exp(R)) into the kernels; birkhoff_proj_n4_hres, sinkhorn_knopp_n4_hres and
// their backwards fuse the mHC layer's H_res producer into the kernels.
// Differences: kernels run on PyTorch's current stream of the target device
// (the reference uses cudaStreamPerThread), batch sizes are 64-bit, B = 0 is
// a no-op, and a failed launch raises RuntimeError.  The Newton pair reads
// fp32/bf16/fp16 CUDA batches with contiguous 4 x 4 matrices in place, at any
// batch stride, instead of copying them to contiguous fp32 and back; the
// results are the same bits.  So do the Sinkhorn-Knopp functions (other
// layouts of those types are made contiguous in their own type first).
#include <stdexcept>
#include <string>

#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <pybind11/pybind11.h>
#include <torch/extension.h>

#include "mhc_proj.h"

namespace py = pybind11;

namespace {

void check_batch(const torch::Tensor& x, const char* name, int64_t batch = -1)
{
    const std::string msg = std::string(name) + " must be a tensor of size B x 4 x 4";
    if (x.dim() != 3) throw std::runtime_error(msg);
    if (x.size(1) != 4 || x.size(2) != 4) throw std::runtime_error(msg);
    if (batch >= 0 && x.size(0) != batch) throw std::runtime_error(msg);
}

// fp32 on the tensor's own CUDA device, or on the current device for
// non-CUDA tensors (solvers_torch.cpp:52-61).
torch::TensorOptions target_options(const torch::Tensor& x)
{
    auto opts = torch::TensorOptions().dtype(torch::kFloat32).device(torch::kCUDA);
    if (x.device().is_cuda()) opts = opts.device(torch::kCUDA, x.device().index());
    return opts;
}

void check_status(int status, const char* what)
{
    if (status != MHC_OK)
        throw std::runtime_error(std::string(what) + " failed: " + mhc_status_string(status));
}

cudaStream_t current_stream() { return at::cuda::getCurrentCUDAStream().stream(); }

// Storage type code of the *_ex entry points, or -1.
int dtype_code(const torch::Tensor& x)
{
    switch (x.scalar_type()) {
        case torch::kFloat32: return MHC_DTYPE_F32;
        case torch::kBFloat16: return MHC_DTYPE_BF16;
        case torch::kFloat16: return MHC_DTYPE_F16;
        default: return -1;
    }
}

// A CUDA batch the kernels read in place: a type they take and contiguous
// 4 x 4 matrices at any non-negative batch stride.
bool native_batch(const torch::Tensor& x)
{
    return x.is_cuda() && dtype_code(x) >= 0 && x.stride(2) == 1 && x.stride(1) == 4 && x.stride(0) >= 0;
}

// The Sinkhorn-Knopp functions read CUDA fp32/bf16/fp16 batches in their own
// type: in place at any batch stride when the 4 x 4 matrices are contiguous,
// else after a copy to contiguous in the same type.  (Converting bf16 logits
// to fp32 first would take exp of the widened values without the rounding to
// bf16 that torch.exp in bf16 -- the reference module's -- performs.)
bool sk_typed(const torch::Tensor& x) { return x.is_cuda() && dtype_code(x) >= 0; }

torch::Tensor sk_layout(const torch::Tensor& x) { return native_batch(x) ? x : x.contiguous(); }

py::dict sk_forward_typed(torch::Tensor X, int max_iter, int flags, const char* what)
{
    const c10::cuda::CUDAGuard guard(X.device());
    X = sk_layout(X);
    const int64_t n = X.size(0);
    torch::Tensor T = torch::empty({n, 4, 4}, X.options().memory_format(at::MemoryFormat::Contiguous));
    check_status(mhc_sinkhorn_knopp_n4_strided(X.data_ptr(), X.stride(0), T.data_ptr(), dtype_code(X), n, max_iter,
                                               flags, current_stream()),
                 what);
    py::dict out;
    out["T"] = T;
    return out;
}

py::dict sk_backward_typed(torch::Tensor G, torch::Tensor X, int max_iter, int flags, const char* what)
{
    const c10::cuda::CUDAGuard guard(G.device());
    G = sk_layout(G);
    X = sk_layout(X);
    const int64_t n = G.size(0);
    torch::Tensor D = torch::empty({n, 4, 4}, G.options().memory_format(at::MemoryFormat::Contiguous));
    check_status(mhc_sinkhorn_knopp_n4_backward_strided(G.data_ptr(), G.stride(0), dtype_code(G), X.data_ptr(),
                                                        X.stride(0), dtype_code(X), D.data_ptr(), n, max_iter, flags,
                                                        current_stream()),
                 what);
    py::dict out;
    out["D"] = D;
    return out;
}

// return_stats=True (an optional keyword, ignored-kwargs compatible) adds
// "iters" (int32, Newton iterations per matrix) and "gnorm" (final gradient
// l1 norm) to the result, computed for fp32 input.
py::dict birkhoff_proj_n4_stats(torch::Tensor R, float tol)
{
    const auto src = R.options();
    const auto opts = target_options(R);
    R = R.to(opts);
    const c10::cuda::CUDAGuard guard(R.device());
    R = R.contiguous();
    const int64_t n = R.size(0);
    torch::Tensor T = torch::empty({n, 4, 4}, opts);
    torch::Tensor it = torch::empty({n}, opts.dtype(torch::kInt32));
    torch::Tensor gn = torch::empty({n}, opts);
    check_status(mhc_birkhoff_proj_n4_stats(R.data_ptr<float>(), T.data_ptr<float>(), tol, n, it.data_ptr<int32_t>(),
                                            gn.data_ptr<float>(), current_stream()),
                 "birkhoff_proj_n4");
    py::dict out;
    out["T"] = T.to(src);
    out["iters"] = it;
    out["gnorm"] = gn;
    return out;
}

// return_duals=True (an optional keyword) adds "beta" (B x 4 fp32: the final
// duals, T = row-softmax(beta + R)), for birkhoff_proj_n4_backward_duals.
py::dict birkhoff_proj_n4_duals(torch::Tensor R, float tol)
{
    const auto src = R.options();
    const auto opts = target_options(R);
    R = R.to(opts);
    const c10::cuda::CUDAGuard guard(R.device());
    R = R.contiguous();
    const int64_t n = R.size(0);
    torch::Tensor T = torch::empty({n, 4, 4}, opts);
    torch::Tensor beta = torch::empty({n, 4}, opts);
    check_status(mhc_birkhoff_proj_n4_duals(R.data_ptr<float>(), T.data_ptr<float>(), beta.data_ptr<float>(), tol, n,
                                            current_stream()),
                 "birkhoff_proj_n4");
    py::dict out;
    out["T"] = T.to(src);
    out["beta"] = beta;
    return out;
}

py::dict birkhoff_proj_n4(torch::Tensor R, float tol, const py::kwargs& kwargs)
{
    check_batch(R, "R");
    if (kwargs.contains("return_stats") && py::cast<bool>(kwargs["return_stats"])) return birkhoff_proj_n4_stats(R, tol);
    if (kwargs.contains("return_duals") && py::cast<bool>(kwargs["return_duals"])) return birkhoff_proj_n4_duals(R, tol);
    if (native_batch(R)) {
        // fp32/bf16/fp16 at any batch stride: read in place, T in R's type
        const c10::cuda::CUDAGuard guard(R.device());
        const int64_t n = R.size(0);
        torch::Tensor T = torch::empty({n, 4, 4}, R.options());
        check_status(mhc_birkhoff_proj_n4_ex(R.data_ptr(), R.stride(0), T.data_ptr(), dtype_code(R), tol, n,
                                             current_stream()),
                     "birkhoff_proj_n4");
        py::dict out;
        out["T"] = T;
        return out;
    }
    const auto src = R.options();
    const auto opts = target_options(R);
    R = R.to(opts);
    const c10::cuda::CUDAGuard guard(R.device());
    R = R.contiguous();
    const int64_t n = R.size(0);
    torch::Tensor T = torch::empty({n, 4, 4}, opts);
    check_status(mhc_birkhoff_proj_n4(R.data_ptr<float>(), T.data_ptr<float>(), tol, n, current_stream()),
                 "birkhoff_proj_n4");
    py::dict out;
    out["T"] = T.to(src);
    return out;
}

py::dict birkhoff_proj_n4_backward(torch::Tensor G, torch::Tensor T, const py::kwargs&)
{
    check_batch(G, "G");
    check_batch(T, "T", G.size(0));
    if (native_batch(G) && native_batch(T) && G.device() == T.device()) {
        const c10::cuda::CUDAGuard guard(G.device());
        const int64_t n = G.size(0);
        torch::Tensor D = torch::empty({n, 4, 4}, G.options());
        check_status(mhc_birkhoff_proj_n4_backward_ex(G.data_ptr(), G.stride(0), dtype_code(G), T.data_ptr(),
                                                      T.stride(0), dtype_code(T), D.data_ptr(), n, current_stream()),
                     "birkhoff_proj_n4_backward");
        py::dict out;
        out["D"] = D;
        return out;
    }
    const auto src = G.options();
    const auto opts = target_options(G);
    G = G.to(opts);
    T = T.to(opts);
    const c10::cuda::CUDAGuard guard(G.device());
    G = G.contiguous();
    T = T.contiguous();
    const int64_t n = G.size(0);
    torch::Tensor D = torch::empty({n, 4, 4}, opts);
    check_status(mhc_birkhoff_proj_n4_backward(G.data_ptr<float>(), T.data_ptr<float>(), D.data_ptr<float>(), n,
                                               current_stream()),
                 "birkhoff_proj_n4_backward");
    py::dict out;
    out["D"] = D.to(src);
    return out;
}

// The IFT backward from the logits R and the duals beta that
// birkhoff_proj_n4(R, return_duals=True) returned, instead of T (no reference
// counterpart).  D is converted to G's dtype/device like the T-based backward.
py::dict birkhoff_proj_n4_backward_duals(torch::Tensor G, torch::Tensor R, torch::Tensor beta, const py::kwargs&)
{
    check_batch(G, "G");
    check_batch(R, "R", G.size(0));
    if (beta.numel() != 4 * G.size(0)) throw std::runtime_error("beta must be a tensor of size B x 4");
    const auto src = G.options();
    const auto opts = target_options(G);
    G = G.to(opts);
    R = R.to(opts);
    beta = beta.to(opts);
    const c10::cuda::CUDAGuard guard(G.device());
    G = G.contiguous();
    R = R.contiguous();
    beta = beta.contiguous();
    const int64_t n = G.size(0);
    torch::Tensor D = torch::empty({n, 4, 4}, opts);
    check_status(mhc_birkhoff_proj_n4_backward_duals(G.data_ptr<float>(), R.data_ptr<float>(), beta.data_ptr<float>(),
                                                     D.data_ptr<float>(), n, current_stream()),
                 "birkhoff_proj_n4_backward_duals");
    py::dict out;
    out["D"] = D.to(src);
    return out;
}

py::dict sinkhorn_knopp_n4(torch::Tensor M, int max_iter, const py::kwargs&)
{
    check_batch(M, "M");
    if (sk_typed(M)) return sk_forward_typed(M, max_iter, 0, "sinkhorn_knopp_n4");
    const auto src = M.options();
    const auto opts = target_options(M);
    M = M.to(opts);
    const c10::cuda::CUDAGuard guard(M.device());
    M = M.contiguous();
    const int64_t n = M.size(0);
    torch::Tensor T = torch::empty({n, 4, 4}, opts);
    check_status(mhc_sinkhorn_knopp_n4(M.data_ptr<float>(), T.data_ptr<float>(), n, max_iter, current_stream()),
                 "sinkhorn_knopp_n4");
    py::dict out;
    out["T"] = T.to(src);
    return out;
}

py::dict sinkhorn_knopp_n4_backward(torch::Tensor G, torch::Tensor M, int max_iter, const py::kwargs&)
{
    check_batch(G, "G");
    check_batch(M, "M", G.size(0));
    if (max_iter > MHC_SK_BACKWARD_MAX_ITERS)
        throw std::invalid_argument("sinkhorn_knopp_n4_backward supports max_iter <= " +
                                    std::to_string(MHC_SK_BACKWARD_MAX_ITERS));
    if (sk_typed(G) && sk_typed(M) && G.device() == M.device())
        return sk_backward_typed(G, M, max_iter, 0, "sinkhorn_knopp_n4_backward");
    const auto src = G.options();
    const auto opts = target_options(G);
    G = G.to(opts);
    M = M.to(opts);
    const c10::cuda::CUDAGuard guard(G.device());
    G = G.contiguous();
    M = M.contiguous();
    const int64_t n = G.size(0);
    torch::Tensor D = torch::empty({n, 4, 4}, opts);
    check_status(mhc_sinkhorn_knopp_n4_backward(G.data_ptr<float>(), M.data_ptr<float>(), D.data_ptr<float>(), n,
                                                max_iter, current_stream()),
                 "sinkhorn_knopp_n4_backward");
    py::dict out;
    out["D"] = D.to(src);
    return out;
}

// Fused exp + Sinkhorn-Knopp on the logits R (no reference counterpart: the
// reference forms exp(R) in Python, mhc_proj/module.py:50,70).
// approx_reciprocal=True (an optional keyword) takes the hardware reciprocal
// (MHC_SK_HW_RECIPROCAL): not the reference kernel's bits, within 1e-6 of them.
py::dict sinkhorn_knopp_n4_logits(torch::Tensor R, int max_iter, const py::kwargs& kwargs)
{
    const bool approx = kwargs.contains("approx_reciprocal") && py::cast<bool>(kwargs["approx_reciprocal"]);
    check_batch(R, "R");
    if (sk_typed(R))
        return sk_forward_typed(R, max_iter, MHC_SK_LOGITS | (approx ? MHC_SK_HW_RECIPROCAL : 0),
                                "sinkhorn_knopp_n4_logits");
    const auto src = R.options();
    const auto opts = target_options(R);
    R = R.to(opts);
    const c10::cuda::CUDAGuard guard(R.device());
    R = R.contiguous();
    const int64_t n = R.size(0);
    torch::Tensor T = torch::empty({n, 4, 4}, opts);
    check_status(mhc_sinkhorn_knopp_n4_logits_ex(R.data_ptr<float>(), T.data_ptr<float>(), n, max_iter,
                                                 approx ? MHC_SK_HW_RECIPROCAL : 0, current_stream()),
                 "sinkhorn_knopp_n4_logits");
    py::dict out;
    out["T"] = T.to(src);
    return out;
}

py::dict sinkhorn_knopp_n4_logits_backward(torch::Tensor G, torch::Tensor R, int max_iter, const py::kwargs&)
{
    check_batch(G, "G");
    check_batch(R, "R", G.size(0));
    if (max_iter > MHC_SK_BACKWARD_MAX_ITERS)
        throw std::invalid_argument("sinkhorn_knopp_n4_logits_backward supports max_iter <= " +
                                    std::to_string(MHC_SK_BACKWARD_MAX_ITERS));
    if (sk_typed(G) && sk_typed(R) && G.device() == R.device())
        return sk_backward_typed(G, R, max_iter, MHC_SK_LOGITS, "sinkhorn_knopp_n4_logits_backward");
    const auto src = G.options();
    const auto opts = target_options(G);
    G = G.to(opts);
    R = R.to(opts);
    const c10::cuda::CUDAGuard guard(G.device());
    G = G.contiguous();
    R = R.contiguous();
    const int64_t n = G.size(0);
    torch::Tensor D = torch::empty({n, 4, 4}, opts);
    check_status(mhc_sinkhorn_knopp_n4_logits_backward(G.data_ptr<float>(), R.data_ptr<float>(),
                                                       D.data_ptr<float>(), n, max_iter, current_stream()),
                 "sinkhorn_knopp_n4_logits_backward");
    py::dict out;
    out["D"] = D.to(src);
    return out;
}

// The projection fused with its producer, the H_res pre-activation of an
// mHC layer, R = alpha_res * h_res / rms + b_res (no reference counterpart:
// the reference's producer, fused_h_activations in src/utils.cuh:50-127,
// writes exp(R) in a kernel of its own and has no backward).
//   h_res: B x 16 or B x 4 x 4, e.g. a column slice H_proj_concat[:, 8:24],
//          read in place when it is fp32 CUDA with contiguous matrices;
//   rms: B elements; alpha_res: a number or a one-element tensor; b_res: 16
//   elements.  Everything is converted to fp32 on h_res's CUDA device (the
//   current device for a CPU h_res); results return in the inputs' dtypes
//   and devices.
struct HResInputs {
    torch::Tensor h, rms, alpha, b;
    int64_t n;
};

HResInputs hres_inputs(torch::Tensor h, torch::Tensor rms, const py::object& alpha, torch::Tensor b)
{
    const bool flat = h.dim() == 2 && h.size(1) == 16;
    const bool mat = h.dim() == 3 && h.size(1) == 4 && h.size(2) == 4;
    if (!flat && !mat) throw std::runtime_error("h_res must be a tensor of size B x 16 or B x 4 x 4");
    const int64_t n = h.size(0);
    if (rms.numel() != n) throw std::runtime_error("rms must have B elements");
    if (b.defined() && b.numel() != 16) throw std::runtime_error("b_res must have 16 elements");
    const bool alpha_number = py::isinstance<py::float_>(alpha) || py::isinstance<py::int_>(alpha);
    if (!alpha_number && py::cast<torch::Tensor>(alpha).numel() != 1)
        throw std::runtime_error("alpha_res must be a number or a one-element tensor");
    const auto opts = target_options(h);
    HResInputs in;
    in.n = n;
    in.h = h.to(opts);
    const bool dense = in.h.stride(-1) == 1 && (flat || in.h.stride(1) == 4) && in.h.stride(0) >= 0;
    if (!dense) in.h = in.h.contiguous();
    in.rms = rms.to(opts).contiguous().reshape({n});
    if (b.defined()) in.b = b.to(opts).contiguous().reshape({16});  // the backward needs no b
    if (alpha_number)
        in.alpha = torch::full({1}, py::cast<double>(alpha), opts);
    else
        in.alpha = py::cast<torch::Tensor>(alpha).to(opts).contiguous().reshape({1});
    return in;
}

py::dict birkhoff_proj_n4_hres(torch::Tensor h_res, torch::Tensor rms, py::object alpha_res, torch::Tensor b_res,
                               float tol, const py::kwargs&)
{
    const auto src = h_res.options();
    HResInputs in = hres_inputs(h_res, rms, alpha_res, b_res);
    const c10::cuda::CUDAGuard guard(in.h.device());
    torch::Tensor T = torch::empty({in.n, 4, 4}, in.h.options());
    check_status(mhc_birkhoff_proj_n4_hres(in.h.data_ptr<float>(), in.h.stride(0), in.rms.data_ptr<float>(),
                                           in.alpha.data_ptr<float>(), in.b.data_ptr<float>(), T.data_ptr<float>(),
                                           tol, in.n, current_stream()),
                 "birkhoff_proj_n4_hres");
    py::dict out;
    out["T"] = T.to(src);
    return out;
}

// The gradient dict of the H_res functions, each gradient shaped and typed
// like its input ("d_alpha_res" 0-d for a number; "d_b_res" 4 x 4 when b_res
// is not given).
py::dict hres_grads(const torch::Tensor& dh, const torch::Tensor& drms, const torch::Tensor& dalpha,
                    const torch::Tensor& db, const torch::Tensor& h_res, const torch::Tensor& rms,
                    const py::object& alpha_res, const torch::Tensor& b_res)
{
    py::dict out;
    out["d_h_res"] = dh.reshape(h_res.sizes()).to(h_res.options());
    out["d_rms"] = drms.reshape(rms.sizes()).to(rms.options());
    if (py::isinstance<py::float_>(alpha_res) || py::isinstance<py::int_>(alpha_res)) {
        out["d_alpha_res"] = dalpha.reshape({});
    } else {
        const torch::Tensor a = py::cast<torch::Tensor>(alpha_res);
        out["d_alpha_res"] = dalpha.reshape(a.sizes()).to(a.options());
    }
    out["d_b_res"] = b_res.defined() ? db.reshape(b_res.sizes()).to(b_res.options()) : db.reshape({4, 4});
    return out;
}

// Gradients of sum(G .* T) with T = birkhoff_proj_n4_hres(h_res, rms,
// alpha_res, b_res): "d_h_res" (shaped like h_res), "d_rms" (like rms),
// "d_alpha_res" (one element; 0-d for a number) and "d_b_res" (like b_res
// when given, else 4 x 4).  T is the forward's output.
py::dict birkhoff_proj_n4_hres_backward(torch::Tensor G, torch::Tensor T, torch::Tensor h_res, torch::Tensor rms,
                                        py::object alpha_res, const py::kwargs& kwargs)
{
    check_batch(G, "G");
    check_batch(T, "T", G.size(0));
    if (h_res.size(0) != G.size(0)) throw std::runtime_error("h_res must have the batch size of G");
    HResInputs in = hres_inputs(h_res, rms, alpha_res, torch::Tensor());
    const auto opts = in.h.options();
    const c10::cuda::CUDAGuard guard(in.h.device());
    G = G.to(opts).contiguous();
    T = T.to(opts).contiguous();
    torch::Tensor dh = torch::empty({in.n, 16}, opts);
    torch::Tensor drms = torch::empty({in.n}, opts);
    torch::Tensor dalpha = torch::empty({1}, opts);
    torch::Tensor db = torch::empty({16}, opts);
    int64_t ws_bytes = 0;
    check_status(mhc_birkhoff_proj_n4_hres_backward_workspace(in.n, &ws_bytes), "birkhoff_proj_n4_hres_backward");
    torch::Tensor ws = torch::empty({(ws_bytes + 3) / 4}, opts);
    check_status(mhc_birkhoff_proj_n4_hres_backward(G.data_ptr<float>(), T.data_ptr<float>(), in.h.data_ptr<float>(),
                                                    in.h.stride(0), in.rms.data_ptr<float>(),
                                                    in.alpha.data_ptr<float>(), dh.data_ptr<float>(), 16,
                                                    drms.data_ptr<float>(), dalpha.data_ptr<float>(),
                                                    db.data_ptr<float>(), in.n, ws.data_ptr(), ws.numel() * 4,
                                                    current_stream()),
                 "birkhoff_proj_n4_hres_backward");
    return hres_grads(dh, drms, dalpha, db, h_res, rms, alpha_res,
                      kwargs.contains("b_res") ? py::cast<torch::Tensor>(kwargs["b_res"]) : torch::Tensor());
}

// Sinkhorn-Knopp on the producer's H_res activation, exp(alpha_res * h_res /
// rms + b_res) with the producer's own exponential (no reference
// counterpart: the reference's producer writes H_res to memory for its
// Sinkhorn-Knopp kernel).  Arguments and conversions as birkhoff_proj_n4_hres.
py::dict sinkhorn_knopp_n4_hres(torch::Tensor h_res, torch::Tensor rms, py::object alpha_res, torch::Tensor b_res,
                                int max_iter, const py::kwargs&)
{
    const auto src = h_res.options();
    HResInputs in = hres_inputs(h_res, rms, alpha_res, b_res);
    const c10::cuda::CUDAGuard guard(in.h.device());
    torch::Tensor T = torch::empty({in.n, 4, 4}, in.h.options());
    check_status(mhc_sinkhorn_knopp_n4_hres(in.h.data_ptr<float>(), in.h.stride(0), in.rms.data_ptr<float>(),
                                            in.alpha.data_ptr<float>(), in.b.data_ptr<float>(), T.data_ptr<float>(),
                                            in.n, max_iter, current_stream()),
                 "sinkhorn_knopp_n4_hres");
    py::dict out;
    out["T"] = T.to(src);
    return out;
}

// Gradients of sum(G .* T) with T = sinkhorn_knopp_n4_hres(...): the keys of
// birkhoff_proj_n4_hres_backward.  max_iter > 20 raises ValueError.
py::dict sinkhorn_knopp_n4_hres_backward(torch::Tensor G, torch::Tensor h_res, torch::Tensor rms,
                                         py::object alpha_res, torch::Tensor b_res, int max_iter, const py::kwargs&)
{
    check_batch(G, "G");
    if (h_res.size(0) != G.size(0)) throw std::runtime_error("h_res must have the batch size of G");
    if (max_iter > MHC_SK_BACKWARD_MAX_ITERS)
        throw std::invalid_argument("sinkhorn_knopp_n4_hres_backward supports max_iter <= " +
                                    std::to_string(MHC_SK_BACKWARD_MAX_ITERS));
    HResInputs in = hres_inputs(h_res, rms, alpha_res, b_res);
    const auto opts = in.h.options();
    const c10::cuda::CUDAGuard guard(in.h.device());
    G = G.to(opts).contiguous();
    torch::Tensor dh = torch::empty({in.n, 16}, opts);
    torch::Tensor drms = torch::empty({in.n}, opts);
    torch::Tensor dalpha = torch::empty({1}, opts);
    torch::Tensor db = torch::empty({16}, opts);
    int64_t ws_bytes = 0;
    check_status(mhc_sinkhorn_knopp_n4_hres_backward_workspace(in.n, &ws_bytes), "sinkhorn_knopp_n4_hres_backward");
    torch::Tensor ws = torch::empty({(ws_bytes + 3) / 4}, opts);
    check_status(mhc_sinkhorn_knopp_n4_hres_backward(G.data_ptr<float>(), in.h.data_ptr<float>(), in.h.stride(0),
                                                     in.rms.data_ptr<float>(), in.alpha.data_ptr<float>(),
                                                     in.b.data_ptr<float>(), dh.data_ptr<float>(), 16,
                                                     drms.data_ptr<float>(), dalpha.data_ptr<float>(),
                                                     db.data_ptr<float>(), in.n, max_iter, ws.data_ptr(),
                                                     ws.numel() * 4, current_stream()),
                 "sinkhorn_knopp_n4_hres_backward");
    return hres_grads(dh, drms, dalpha, db, h_res, rms, alpha_res, b_res);
}

}  // namespace

PYBIND11_MODULE(_internal, m)
{
    m.doc() = "B200 batched n=4 Birkhoff projection for manifold-constrained hyper-connections";
    m.attr("abi_version") = mhc_abi_version();
    py::module m_torch = m.def_submodule("torch", "PyTorch interface");
    m_torch.def("birkhoff_proj_n4", &birkhoff_proj_n4, py::arg("R"), py::arg("tol") = 1e-6,
                "KL projection of 4x4 matrices onto the Birkhoff polytope");
    m_torch.def("birkhoff_proj_n4_backward", &birkhoff_proj_n4_backward, py::arg("G"), py::arg("T"),
                "KL projection of 4x4 matrices onto the Birkhoff polytope, backward pass");
    m_torch.def("birkhoff_proj_n4_backward_duals", &birkhoff_proj_n4_backward_duals, py::arg("G"), py::arg("R"),
                py::arg("beta"), "Backward of birkhoff_proj_n4 from R and its saved duals instead of T");
    m_torch.def("sinkhorn_knopp_n4", &sinkhorn_knopp_n4, py::arg("M"), py::arg("max_iter") = 20,
                "Sinkhorn-Knopp algorithm for 4x4 matrices");
    m_torch.def("sinkhorn_knopp_n4_backward", &sinkhorn_knopp_n4_backward, py::arg("G"), py::arg("M"),
                py::arg("max_iter") = 20, "Sinkhorn-Knopp algorithm for 4x4 matrices, backward pass");
    m_torch.def("sinkhorn_knopp_n4_logits", &sinkhorn_knopp_n4_logits, py::arg("R"), py::arg("max_iter") = 20,
                "Sinkhorn-Knopp on exp(R) in one kernel (R: logits)");
    m_torch.def("sinkhorn_knopp_n4_logits_backward", &sinkhorn_knopp_n4_logits_backward, py::arg("G"),
                py::arg("R"), py::arg("max_iter") = 20,
                "Gradient with respect to R of Sinkhorn-Knopp on exp(R), in one kernel");
    m_torch.def("birkhoff_proj_n4_hres", &birkhoff_proj_n4_hres, py::arg("h_res"), py::arg("rms"),
                py::arg("alpha_res"), py::arg("b_res"), py::arg("tol") = 1e-6,
                "Projection of R = alpha_res * h_res / rms + b_res, formed in the kernel's load");
    m_torch.def("birkhoff_proj_n4_hres_backward", &birkhoff_proj_n4_hres_backward, py::arg("G"), py::arg("T"),
                py::arg("h_res"), py::arg("rms"), py::arg("alpha_res"),
                "Gradients of birkhoff_proj_n4_hres with respect to h_res, rms, alpha_res and b_res");
    m_torch.def("sinkhorn_knopp_n4_hres", &sinkhorn_knopp_n4_hres, py::arg("h_res"), py::arg("rms"),
                py::arg("alpha_res"), py::arg("b_res"), py::arg("max_iter") = 20,
                "Sinkhorn-Knopp on exp(alpha_res * h_res / rms + b_res), formed in the kernel's load");
    m_torch.def("sinkhorn_knopp_n4_hres_backward", &sinkhorn_knopp_n4_hres_backward, py::arg("G"), py::arg("h_res"),
                py::arg("rms"), py::arg("alpha_res"), py::arg("b_res"), py::arg("max_iter") = 20,
                "Gradients of sinkhorn_knopp_n4_hres with respect to h_res, rms, alpha_res and b_res");
}
