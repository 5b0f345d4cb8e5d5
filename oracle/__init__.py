"""ORACLE -- test infrastructure only.

ctypes bindings over ``liboracle.so`` (the CPU restatement of the reference
algorithms in ``birkhoff_oracle.c``) and over ``_ref/libmhcref.so`` (the
reference's own CUDA kernels compiled unmodified from their source files,
``ref_shim.cu`` giving them extern "C" names), and over
``_ref/libmhcref_hres.so`` (the reference's H_res producer from
src/utils.cuh, ``ref_hres_shim.cu``).

Only the tests, the smoke check and the CPU-baseline leg of the benchmark use
this package, always as the oracle the kernels are compared with or as the timed
baseline, never as a product path.  Build both libraries with ``make -C oracle``.
"""
from __future__ import annotations

import ctypes
import os

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
ORACLE_LIB = os.path.join(_HERE, "liboracle.so")
REF_LIB = os.path.join(_HERE, "_ref", "libmhcref.so")

_f32p = ctypes.POINTER(ctypes.c_float)
_i32p = ctypes.POINTER(ctypes.c_int32)

_lib = None


def _load():
    global _lib
    if _lib is None:
        if not os.path.exists(ORACLE_LIB):
            raise RuntimeError(f"{ORACLE_LIB} is not built; run `make -C oracle`")
        lib = ctypes.CDLL(ORACLE_LIB)
        lib.oracle_max_threads.restype = ctypes.c_int
        lib.oracle_birkhoff_proj_n4.argtypes = [_f32p, _f32p, ctypes.c_float, ctypes.c_int64, _i32p, ctypes.c_int]
        lib.oracle_birkhoff_proj_n4.restype = None
        lib.oracle_birkhoff_proj_n4_line_search.argtypes = [_f32p, _f32p, ctypes.c_float, ctypes.c_int64,
                                                            ctypes.c_int, _i32p, ctypes.c_int]
        lib.oracle_birkhoff_proj_n4_line_search.restype = ctypes.c_int
        lib.oracle_birkhoff_proj_n4_backward.argtypes = [_f32p, _f32p, _f32p, ctypes.c_int64, ctypes.c_int]
        lib.oracle_birkhoff_proj_n4_backward.restype = None
        lib.oracle_sinkhorn_knopp_n4.argtypes = [_f32p, _f32p, ctypes.c_int64, ctypes.c_int, ctypes.c_float, ctypes.c_int]
        lib.oracle_sinkhorn_knopp_n4.restype = None
        lib.oracle_sinkhorn_knopp_n4_backward.argtypes = [
            _f32p, _f32p, _f32p, ctypes.c_int64, ctypes.c_int, ctypes.c_float, ctypes.c_int, ctypes.c_int]
        lib.oracle_sinkhorn_knopp_n4_backward.restype = ctypes.c_int
        _lib = lib
    return _lib


def _as_batch(a: np.ndarray, name: str) -> np.ndarray:
    a = np.ascontiguousarray(a, dtype=np.float32)
    if a.ndim != 3 or a.shape[1:] != (4, 4):
        raise ValueError(f"{name} must have shape (N, 4, 4), got {a.shape}")
    return a


def _p(a: np.ndarray):
    return a.ctypes.data_as(_f32p)


def max_threads() -> int:
    return _load().oracle_max_threads()


def birkhoff_proj_n4(R, tol=1e-6, threads=0, return_evals=False):
    """Newton forward (birkhoff_proj_n4.cu:375-499). Returns T (and the
    number of f/gradient evaluations per matrix if ``return_evals``)."""
    R = _as_batch(R, "R")
    N = R.shape[0]
    T = np.empty_like(R)
    ev = np.empty(N, dtype=np.int32) if return_evals else None
    _load().oracle_birkhoff_proj_n4(_p(R), _p(T), float(tol), N,
                                    ev.ctypes.data_as(_i32p) if ev is not None else None, int(threads))
    return (T, ev) if return_evals else T


def birkhoff_proj_n4_line_search(R, candidates, tol=1e-6, threads=0):
    """The Newton forward with its line search cut to the first `candidates`
    steps of (1, 0.5, 0.1, 0.05, 0.01) before the Sinkhorn fallback (5 = the
    reference, birkhoff_proj_n4.cu:434-487).  Returns (T, Newton iterations
    per matrix).  A study tool: fewer candidates is a different trajectory."""
    R = _as_batch(R, "R")
    N = R.shape[0]
    T = np.empty_like(R)
    it = np.empty(N, dtype=np.int32)
    if _load().oracle_birkhoff_proj_n4_line_search(_p(R), _p(T), float(tol), N, int(candidates),
                                                    it.ctypes.data_as(_i32p), int(threads)) != 0:
        raise ValueError("candidates must be 1..5")
    return T, it


def birkhoff_proj_n4_backward(G, T, threads=0):
    """IFT backward (birkhoff_proj_n4.cu:527-669). Returns D."""
    G = _as_batch(G, "G")
    T = _as_batch(T, "T")
    if G.shape != T.shape:
        raise ValueError("G and T must have the same shape")
    D = np.empty_like(G)
    _load().oracle_birkhoff_proj_n4_backward(_p(G), _p(T), _p(D), G.shape[0], int(threads))
    return D


def sinkhorn_knopp_n4(M, max_iter=20, eps=1e-8, threads=0):
    """Fixed-iteration SK on M = exp(R) (sinkhorn_knopp.cuh:831-912)."""
    M = _as_batch(M, "M")
    T = np.empty_like(M)
    _load().oracle_sinkhorn_knopp_n4(_p(M), _p(T), M.shape[0], int(max_iter), float(eps), int(threads))
    return T


def sinkhorn_knopp_n4_backward(G, M, max_iter=20, eps=1e-8, exact=True, threads=0):
    """Gradient w.r.t. M of sum(G * SK(M)).  ``exact=True`` is the exact VJP;
    ``exact=False`` restates the reference kernel's reverse loop
    (sinkhorn_knopp.cuh:1146-1202), whose row step is not the exact VJP."""
    G = _as_batch(G, "G")
    M = _as_batch(M, "M")
    D = np.empty_like(G)
    rc = _load().oracle_sinkhorn_knopp_n4_backward(_p(G), _p(M), _p(D), G.shape[0], int(max_iter),
                                                   float(eps), 1 if exact else 0, int(threads))
    if rc != 0:
        raise ValueError("max_iter exceeds the oracle's capacity (64)")
    return D


def vanilla_sinkhorn(x, G=None, iters=20, eps=1e-6):
    """The reference's vanilla PyTorch Sinkhorn-Knopp (README.md:37-46,
    benchmark/accuracy.py:7-13): P = exp(x), then `iters` times
    P /= (rowsum + eps); P /= (colsum + eps).  With G, also returns
    d sum(G*P) / dx by autograd.  ``x`` and ``G`` are torch tensors; the
    computation runs on their device."""
    import torch

    with torch.enable_grad():
        xg = x.detach().clone().requires_grad_(G is not None)
        P = torch.exp(xg)
        for _ in range(iters):
            P = P / (P.sum(dim=2, keepdim=True) + eps)
            P = P / (P.sum(dim=1, keepdim=True) + eps)
        if G is None:
            return P.detach()
        (P * G).sum().backward()
        return P.detach(), xg.grad.detach()


class RefCuda:
    """The reference's CUDA kernels, compiled from its own sources.  Calls
    take raw device pointers (ints) and a raw cudaStream_t (int)."""

    def __init__(self, path: str = REF_LIB):
        if not os.path.exists(path):
            raise RuntimeError(f"{path} is not built; run `make -C oracle ref` where the reference sources exist")
        lib = ctypes.CDLL(path)
        vp = ctypes.c_void_p
        lib.ref_birkhoff_proj_n4.argtypes = [vp, vp, ctypes.c_float, ctypes.c_int, vp]
        lib.ref_birkhoff_proj_n4_backward.argtypes = [vp, vp, vp, ctypes.c_int, vp]
        lib.ref_sinkhorn_knopp_n4.argtypes = [vp, vp, ctypes.c_int, ctypes.c_int, vp]
        lib.ref_sinkhorn_knopp_n4_backward.argtypes = [vp, vp, vp, ctypes.c_int, ctypes.c_int, vp]
        for f in ("ref_birkhoff_proj_n4", "ref_birkhoff_proj_n4_backward",
                  "ref_sinkhorn_knopp_n4", "ref_sinkhorn_knopp_n4_backward"):
            getattr(lib, f).restype = ctypes.c_int
        self.lib = lib

    @staticmethod
    def available(path: str = REF_LIB) -> bool:
        return os.path.exists(path)

    def _check(self, rc, what):
        if rc != 0:
            raise RuntimeError(f"reference {what} failed with code {rc}")

    def birkhoff_proj_n4(self, R, T, tol, N, stream):
        self._check(self.lib.ref_birkhoff_proj_n4(R, T, float(tol), int(N), stream), "birkhoff_proj_n4")

    def birkhoff_proj_n4_backward(self, G, T, D, N, stream):
        self._check(self.lib.ref_birkhoff_proj_n4_backward(G, T, D, int(N), stream), "birkhoff_proj_n4_backward")

    def sinkhorn_knopp_n4(self, M, T, N, iters, stream):
        self._check(self.lib.ref_sinkhorn_knopp_n4(M, T, int(N), int(iters), stream), "sinkhorn_knopp_n4")

    def sinkhorn_knopp_n4_backward(self, G, M, D, N, iters, stream):
        self._check(self.lib.ref_sinkhorn_knopp_n4_backward(G, M, D, int(N), int(iters), stream),
                    "sinkhorn_knopp_n4_backward")


# --- the mHC layer's H_res producer ---------------------------------------

REF_HRES_LIB = os.path.join(_HERE, "_ref", "libmhcref_hres.so")


def hres_logits(h, rms, alpha, b):
    """The H_res pre-activation R = alpha * h / rms + b of the reference's
    producer (src/utils.cuh:84-93), in float64 from the float32 inputs: h
    (N, 16), rms (N,), alpha a number, b (16,).  Returns (N, 4, 4) float64.
    The kernels round this to float32 in two steps (the product alpha * h,
    then a fused multiply-add with 1 / rms); the float64 value bounds them."""
    h = np.asarray(h, dtype=np.float64).reshape(-1, 16)
    rms = np.asarray(rms, dtype=np.float64).reshape(-1, 1)
    b = np.asarray(b, dtype=np.float64).reshape(1, 16)
    return (float(alpha) * h / rms + b).reshape(-1, 4, 4)


def hres_backward_chain(D, h, rms, alpha):
    """Chain rule through R = alpha * h / rms + b, in float64: given D = dL/dR
    (N, 4, 4), returns (dh (N, 16), drms (N,), dalpha, db (4, 4)) with
    dh = D alpha / rms, drms = -alpha / rms^2 sum(D h), dalpha =
    sum_k sum(D_k h_k) / rms_k, db = sum_k D_k."""
    D = np.asarray(D, dtype=np.float64).reshape(-1, 16)
    h = np.asarray(h, dtype=np.float64).reshape(-1, 16)
    rms = np.asarray(rms, dtype=np.float64).reshape(-1)
    alpha = float(alpha)
    q = (D * h).sum(axis=1)
    dh = D * (alpha / rms)[:, None]
    drms = -alpha / rms ** 2 * q
    dalpha = float((q / rms).sum())
    db = D.sum(axis=0).reshape(4, 4)
    return dh, drms, dalpha, db


class RefHRes:
    """The reference's H_res producer (fused_h_activations, src/utils.cuh:50-127)
    compiled unmodified from its header (``ref_hres_shim.cu``), plus the
    producer's pre-exponential value restated with the same expression and
    flags.  Calls take raw device pointers (ints) and a raw stream (int)."""

    def __init__(self, path: str = REF_HRES_LIB):
        if not os.path.exists(path):
            raise RuntimeError(f"{path} is not built; run `make -C oracle ref` where the reference sources exist")
        lib = ctypes.CDLL(path)
        vp, f32, i32 = ctypes.c_void_p, ctypes.c_float, ctypes.c_int
        lib.ref_fused_h_activations_n4.argtypes = [vp, vp, vp, vp, vp, f32, f32, f32, vp, vp, vp, i32, vp]
        lib.ref_fused_h_activations_n4.restype = ctypes.c_int
        lib.ref_hres_logits_n4.argtypes = [vp, vp, f32, vp, vp, i32, vp]
        lib.ref_hres_logits_n4.restype = ctypes.c_int
        lib.ref_fast_exp.argtypes = [vp, vp, i32, vp]
        lib.ref_fast_exp.restype = ctypes.c_int
        self.lib = lib

    @staticmethod
    def available(path: str = REF_HRES_LIB) -> bool:
        return os.path.exists(path)

    def fused_h_activations_n4(self, H_pre, H_post, H_res, H_proj_concat, rms, alpha_pre, alpha_post, alpha_res,
                               b_pre, b_post, b_res, B, stream):
        rc = self.lib.ref_fused_h_activations_n4(H_pre, H_post, H_res, H_proj_concat, rms, float(alpha_pre),
                                                 float(alpha_post), float(alpha_res), b_pre, b_post, b_res, int(B),
                                                 stream)
        if rc != 0:
            raise RuntimeError(f"reference fused_h_activations failed with code {rc}")

    def hres_logits_n4(self, H_proj_concat, rms, alpha_res, b_res, R, B, stream):
        rc = self.lib.ref_hres_logits_n4(H_proj_concat, rms, float(alpha_res), b_res, R, int(B), stream)
        if rc != 0:
            raise RuntimeError(f"reference H_res logits failed with code {rc}")

    def fast_exp(self, x, y, n, stream):
        rc = self.lib.ref_fast_exp(x, y, int(n), stream)
        if rc != 0:
            raise RuntimeError(f"reference fast_exp failed with code {rc}")
