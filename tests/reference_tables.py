"""The reference's two benchmark tables, re-measured on this GPU.

    python tests/reference_tables.py > profiles/reference_tables_b200.json

Run time (the reference's benchmark/runtime.py, README.md:181-197): forward,
and forward + backward, per call at batch sizes 128 ... 131072, for
  - this repository's Newton projection (mhc_birkhoff_proj_n4 and its backward),
  - the reference's Newton kernels, compiled from its sources (oracle/_ref),
  - this repository's fused exp + Sinkhorn-Knopp pair (the MHCSinkhornN4 path),
  - the reference's Sinkhorn-Knopp composition (torch.exp, its sinkhorn_knopp_n4,
    its backward times exp(R) -- runtime.py's sk_n4_fwd / sk_n4_bwd),
  - vanilla PyTorch Sinkhorn-Knopp (20 iterations, eps 1e-6; eager -- the
    reference compiles it with torch.compile).
As in runtime.py: inputs x = 10 N(0,1) for the forward table and N(0,1) for
the forward + backward table, G ~ N(0,1), 100 warm-up calls, then CUDA events
around 100 calls, 10 runs, median.  Unlike runtime.py, each call takes a
fresh input from a pool of 8 (runtime.py feeds each output back as the next
input).  Kernels are called through their C entry points on preallocated
device buffers, so both sides pay the same launch path.

Accuracy (the reference's benchmark/accuracy.py, README.md:160-172): the
marginal error |T 1 - 1|_1 + |T^T 1 - 1|_1 (in float64) over N = 10000
matrices (torch.manual_seed(123) on the GPU) for N(0,1), N(0,10^2), U(-1,1)
and U(-10,10): mean, std, median, max.

Test infrastructure: it calls the reference kernels in oracle/_ref.
"""
from __future__ import annotations

import ctypes
import json
import os
import statistics
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
sys.path[:0] = [ROOT, os.path.join(ROOT, "mhc-proj_b200")]

import torch  # noqa: E402

from mhc_proj import capi  # noqa: E402

REF_LIB = os.path.join(ROOT, "oracle", "_ref", "libmhcref.so")
SIZES = [128, 512, 2048, 8192, 32768, 131072]
POOL = 8
WARMUP = 100
ITERS = 100
RUNS = 10


def ref_lib():
    L = ctypes.CDLL(REF_LIB)
    vp, i32, f32 = ctypes.c_void_p, ctypes.c_int, ctypes.c_float
    L.ref_birkhoff_proj_n4.argtypes = [vp, vp, f32, i32, vp]
    L.ref_birkhoff_proj_n4_backward.argtypes = [vp, vp, vp, i32, vp]
    L.ref_sinkhorn_knopp_n4.argtypes = [vp, vp, i32, i32, vp]
    L.ref_sinkhorn_knopp_n4_backward.argtypes = [vp, vp, vp, i32, i32, vp]
    return L


def vanilla(x, iters=20, eps=1e-6):
    P = torch.exp(x)
    for _ in range(iters):
        P = P / (P.sum(dim=2, keepdim=True) + eps)
        P = P / (P.sum(dim=1, keepdim=True) + eps)
    return P


def time_calls(call):
    """Median over RUNS of (CUDA-event time of ITERS calls) / ITERS, in us;
    call(i) uses pool entry i % POOL."""
    for i in range(WARMUP):
        call(i)
    torch.cuda.synchronize()
    per = []
    for _ in range(RUNS):
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record()
        for i in range(ITERS):
            call(i)
        e1.record()
        torch.cuda.synchronize()
        per.append(e0.elapsed_time(e1) * 1e3 / ITERS)
    return statistics.median(per)


def runtime_table(L, backward):
    s = torch.cuda.current_stream().cuda_stream
    rows = []
    for n in SIZES:
        g = torch.Generator(device="cuda").manual_seed(123)
        scale = 1.0 if backward else 10.0
        xs = [scale * torch.randn(n, 4, 4, device="cuda", generator=g) for _ in range(POOL)]
        Gs = [torch.randn(n, 4, 4, device="cuda", generator=g) for _ in range(POOL)]
        T = torch.empty(n, 4, 4, device="cuda")
        D = torch.empty_like(T)

        def ours_newton(i):
            x = xs[i % POOL]
            capi.birkhoff_proj_n4(x.data_ptr(), T.data_ptr(), 1e-6, n, s)
            if backward:
                capi.birkhoff_proj_n4_backward(Gs[i % POOL].data_ptr(), T.data_ptr(), D.data_ptr(), n, s)

        def ref_newton(i):
            x = xs[i % POOL]
            L.ref_birkhoff_proj_n4(x.data_ptr(), T.data_ptr(), 1e-6, n, s)
            if backward:
                L.ref_birkhoff_proj_n4_backward(Gs[i % POOL].data_ptr(), T.data_ptr(), D.data_ptr(), n, s)

        def ours_sk(i):
            x = xs[i % POOL]
            capi.sinkhorn_knopp_n4_logits(x.data_ptr(), T.data_ptr(), n, 20, s)
            if backward:
                capi.sinkhorn_knopp_n4_logits_backward(Gs[i % POOL].data_ptr(), x.data_ptr(), D.data_ptr(), n, 20, s)

        def ref_sk(i):
            M = torch.exp(xs[i % POOL])
            L.ref_sinkhorn_knopp_n4(M.data_ptr(), T.data_ptr(), n, 20, s)
            if backward:
                L.ref_sinkhorn_knopp_n4_backward(Gs[i % POOL].data_ptr(), M.data_ptr(), D.data_ptr(), n, 20, s)
                torch.mul(D, M, out=D)

        def vanilla_sk(i):
            if backward:
                x = xs[i % POOL].detach().requires_grad_(True)
                P = vanilla(x)
                P.backward(Gs[i % POOL])
            else:
                with torch.no_grad():
                    vanilla(xs[i % POOL])

        us = {"ours_newton": time_calls(ours_newton), "reference_newton": time_calls(ref_newton),
              "ours_sinkhorn_fused_exp": time_calls(ours_sk), "reference_sinkhorn_composition": time_calls(ref_sk),
              "vanilla_torch_eager": time_calls(vanilla_sk)}
        base = us["ours_newton"]
        rows.append({"N": n, "us_per_call": us,
                     "normalised_to_ours_newton": {k: v / base for k, v in us.items()},
                     "reference_newton_over_ours_newton": us["reference_newton"] / base,
                     "reference_sinkhorn_over_ours_sinkhorn":
                         us["reference_sinkhorn_composition"] / us["ours_sinkhorn_fused_exp"]})
    return rows


def marginal_error(T):
    T = T.double()
    return (T.sum(-1) - 1).abs().sum(-1) + (T.sum(-2) - 1).abs().sum(-1)


def stats(err):
    return {"mean": float(err.mean()), "std": float(err.std()), "median": float(err.median()),
            "max": float(err.max())}


def accuracy_table(L):
    s = torch.cuda.current_stream().cuda_stream
    n = 10000
    dists = {"N(0,1)": lambda: torch.randn(n, 4, 4, device="cuda"),
             "N(0,10^2)": lambda: 10 * torch.randn(n, 4, 4, device="cuda"),
             "U(-1,1)": lambda: 2 * torch.rand(n, 4, 4, device="cuda") - 1,
             "U(-10,10)": lambda: 20 * torch.rand(n, 4, 4, device="cuda") - 10}
    out = []
    for name, make in dists.items():
        torch.manual_seed(123)
        x = make()
        T_on = torch.empty_like(x)
        capi.birkhoff_proj_n4(x.data_ptr(), T_on.data_ptr(), 1e-6, n, s)
        T_rn = torch.empty_like(x)
        L.ref_birkhoff_proj_n4(x.data_ptr(), T_rn.data_ptr(), 1e-6, n, s)
        T_os = torch.empty_like(x)
        capi.sinkhorn_knopp_n4_logits(x.data_ptr(), T_os.data_ptr(), n, 20, s)
        M = torch.exp(x)
        T_rs = torch.empty_like(x)
        L.ref_sinkhorn_knopp_n4(M.data_ptr(), T_rs.data_ptr(), n, 20, s)
        T_v = vanilla(x)
        torch.cuda.synchronize()
        out.append({"distribution": name, "N": n,
                    "marginal_error": {"vanilla_torch": stats(marginal_error(T_v)),
                                       "reference_sinkhorn_composition": stats(marginal_error(T_rs)),
                                       "ours_sinkhorn_fused_exp": stats(marginal_error(T_os)),
                                       "reference_newton": stats(marginal_error(T_rn)),
                                       "ours_newton": stats(marginal_error(T_on))},
                    "ours_newton_equals_reference_newton_bitwise":
                        bool(torch.equal(T_on.view(torch.int32), T_rn.view(torch.int32)))})
    return out


def main():
    if not os.path.exists(REF_LIB):
        sys.exit(f"{REF_LIB} is not built (make -C oracle REF_SRC=<reference checkout>/src)")
    L = ref_lib()
    result = {"gpu": torch.cuda.get_device_name(0),
              "method": "see tests/reference_tables.py: reference runtime.py / accuracy.py methodology, fresh "
                        "inputs per call, kernels through their C entry points on preallocated buffers",
              "runtime_forward": runtime_table(L, backward=False),
              "runtime_forward_backward": runtime_table(L, backward=True),
              "accuracy": accuracy_table(L)}
    print(json.dumps(result, indent=1))


if __name__ == "__main__":
    main()
