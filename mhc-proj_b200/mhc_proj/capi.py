"""ctypes view of the C ABI in include/mhc_proj.h (libmhcproj.so).

For callers that hold raw device pointers instead of tensors.  Each function
mirrors the C entry point; ``stream`` is a raw cudaStream_t (an int, 0 for the
legacy default stream) and every pointer is a device address (an int).  A
non-zero return code raises ``MhcError``.  The ``*_tensor`` helpers take
contiguous fp32 CUDA tensors and launch on PyTorch's current stream.
"""
from __future__ import annotations

import ctypes
import os

_LIB_PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)), "libmhcproj.so")

EXPORTED = (
    "mhc_birkhoff_proj_n4",
    "mhc_birkhoff_proj_n4_backward",
    "mhc_birkhoff_proj_n4_ex",
    "mhc_birkhoff_proj_n4_backward_ex",
    "mhc_birkhoff_proj_n4_stats",
    "mhc_birkhoff_proj_n4_pass_counts",
    "mhc_birkhoff_proj_n4_duals",
    "mhc_birkhoff_proj_n4_backward_duals",
    "mhc_sinkhorn_knopp_n4",
    "mhc_sinkhorn_knopp_n4_backward",
    "mhc_sinkhorn_knopp_n4_logits",
    "mhc_sinkhorn_knopp_n4_logits_ex",
    "mhc_sinkhorn_knopp_n4_logits_backward",
    "mhc_sinkhorn_knopp_n4_strided",
    "mhc_sinkhorn_knopp_n4_backward_strided",
    "mhc_birkhoff_proj_n4_hres",
    "mhc_birkhoff_proj_n4_hres_backward_workspace",
    "mhc_birkhoff_proj_n4_hres_backward",
    "mhc_birkhoff_proj_n4_hres_backward_noalloc",
    "mhc_sinkhorn_knopp_n4_hres",
    "mhc_sinkhorn_knopp_n4_hres_backward_workspace",
    "mhc_sinkhorn_knopp_n4_hres_backward",
    "mhc_status_string",
    "mhc_abi_version",
)
_LAUNCHERS = EXPORTED[:-2]

MHC_OK = 0
MHC_ERR_INVALID_VALUE = -1
MHC_ERR_ITERS = -2
MHC_ERR_CAPTURE = -3
MHC_SK_BACKWARD_MAX_ITERS = 20
MHC_DTYPE_F32, MHC_DTYPE_BF16, MHC_DTYPE_F16 = 0, 1, 2
MHC_SK_HW_RECIPROCAL = 1
MHC_SK_LOGITS = 2


class MhcError(RuntimeError):
    def __init__(self, code: int, what: str):
        self.code = code
        super().__init__(f"{what} failed ({code}): {status_string(code)}")


_lib = None


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        if not os.path.exists(_LIB_PATH):
            raise RuntimeError(f"{_LIB_PATH} is not built (run `python mhc-proj_b200/build.py`)")
        L = ctypes.CDLL(_LIB_PATH)
        vp, i64, f32, i32 = ctypes.c_void_p, ctypes.c_int64, ctypes.c_float, ctypes.c_int
        L.mhc_birkhoff_proj_n4.argtypes = [vp, vp, f32, i64, vp]
        L.mhc_birkhoff_proj_n4_backward.argtypes = [vp, vp, vp, i64, vp]
        L.mhc_sinkhorn_knopp_n4.argtypes = [vp, vp, i64, i32, vp]
        L.mhc_sinkhorn_knopp_n4_backward.argtypes = [vp, vp, vp, i64, i32, vp]
        L.mhc_birkhoff_proj_n4_ex.argtypes = [vp, i64, vp, i32, f32, i64, vp]
        L.mhc_birkhoff_proj_n4_backward_ex.argtypes = [vp, i64, i32, vp, i64, i32, vp, i64, vp]
        L.mhc_birkhoff_proj_n4_stats.argtypes = [vp, vp, f32, i64, vp, vp, vp]
        L.mhc_birkhoff_proj_n4_pass_counts.argtypes = [vp, vp, f32, i64, vp, vp, vp, vp]
        L.mhc_birkhoff_proj_n4_duals.argtypes = [vp, vp, vp, f32, i64, vp]
        L.mhc_birkhoff_proj_n4_backward_duals.argtypes = [vp, vp, vp, vp, i64, vp]
        L.mhc_sinkhorn_knopp_n4_logits.argtypes = [vp, vp, i64, i32, vp]
        L.mhc_sinkhorn_knopp_n4_logits_ex.argtypes = [vp, vp, i64, i32, i32, vp]
        L.mhc_sinkhorn_knopp_n4_logits_backward.argtypes = [vp, vp, vp, i64, i32, vp]
        L.mhc_sinkhorn_knopp_n4_strided.argtypes = [vp, i64, vp, i32, i64, i32, i32, vp]
        L.mhc_sinkhorn_knopp_n4_backward_strided.argtypes = [vp, i64, i32, vp, i64, i32, vp, i64, i32, i32, vp]
        L.mhc_birkhoff_proj_n4_hres.argtypes = [vp, i64, vp, vp, vp, vp, f32, i64, vp]
        L.mhc_birkhoff_proj_n4_hres_backward_workspace.argtypes = [i64, ctypes.POINTER(i64)]
        L.mhc_birkhoff_proj_n4_hres_backward.argtypes = [vp, vp, vp, i64, vp, vp, vp, i64, vp, vp, vp, i64, vp,
                                                         i64, vp]
        L.mhc_birkhoff_proj_n4_hres_backward_noalloc.argtypes = [vp, vp, vp, i64, vp, vp, vp, i64, vp, vp, vp,
                                                                 i64, vp]
        L.mhc_sinkhorn_knopp_n4_hres.argtypes = [vp, i64, vp, vp, vp, vp, i64, i32, vp]
        L.mhc_sinkhorn_knopp_n4_hres_backward_workspace.argtypes = [i64, ctypes.POINTER(i64)]
        L.mhc_sinkhorn_knopp_n4_hres_backward.argtypes = [vp, vp, i64, vp, vp, vp, vp, i64, vp, vp, vp, i64, i32,
                                                          vp, i64, vp]
        for f in _LAUNCHERS:
            getattr(L, f).restype = ctypes.c_int
        L.mhc_status_string.argtypes = [ctypes.c_int]
        L.mhc_status_string.restype = ctypes.c_char_p
        L.mhc_abi_version.argtypes = []
        L.mhc_abi_version.restype = ctypes.c_int
        _lib = L
    return _lib


def status_string(code: int) -> str:
    return lib().mhc_status_string(int(code)).decode()


def abi_version() -> int:
    return lib().mhc_abi_version()


def _check(code: int, what: str) -> None:
    if code != MHC_OK:
        raise MhcError(code, what)


def birkhoff_proj_n4(R: int, T: int, tol: float, N: int, stream: int = 0) -> None:
    _check(lib().mhc_birkhoff_proj_n4(R, T, tol, N, stream), "mhc_birkhoff_proj_n4")


def birkhoff_proj_n4_backward(G: int, T: int, D: int, N: int, stream: int = 0) -> None:
    _check(lib().mhc_birkhoff_proj_n4_backward(G, T, D, N, stream), "mhc_birkhoff_proj_n4_backward")


def birkhoff_proj_n4_stats(R: int, T: int, tol: float, N: int, iters: int, gnorm: int, stream: int = 0) -> None:
    _check(lib().mhc_birkhoff_proj_n4_stats(R, T, tol, N, iters, gnorm, stream), "mhc_birkhoff_proj_n4_stats")


def birkhoff_proj_n4_pass_counts(R: int, T: int, tol: float, N: int, iters: int, gnorm: int, counts: int,
                                 stream: int = 0) -> None:
    _check(lib().mhc_birkhoff_proj_n4_pass_counts(R, T, tol, N, iters, gnorm, counts, stream),
           "mhc_birkhoff_proj_n4_pass_counts")


def birkhoff_proj_n4_duals(R: int, T: int, beta: int, tol: float, N: int, stream: int = 0) -> None:
    _check(lib().mhc_birkhoff_proj_n4_duals(R, T, beta, tol, N, stream), "mhc_birkhoff_proj_n4_duals")


def birkhoff_proj_n4_backward_duals(G: int, R: int, beta: int, D: int, N: int, stream: int = 0) -> None:
    _check(lib().mhc_birkhoff_proj_n4_backward_duals(G, R, beta, D, N, stream), "mhc_birkhoff_proj_n4_backward_duals")


def birkhoff_proj_n4_ex(R: int, r_stride: int, T: int, dtype: int, tol: float, N: int, stream: int = 0) -> None:
    _check(lib().mhc_birkhoff_proj_n4_ex(R, r_stride, T, dtype, tol, N, stream), "mhc_birkhoff_proj_n4_ex")


def birkhoff_proj_n4_backward_ex(G: int, g_stride: int, g_dtype: int, T: int, t_stride: int, t_dtype: int,
                                 D: int, N: int, stream: int = 0) -> None:
    _check(lib().mhc_birkhoff_proj_n4_backward_ex(G, g_stride, g_dtype, T, t_stride, t_dtype, D, N, stream),
           "mhc_birkhoff_proj_n4_backward_ex")


def sinkhorn_knopp_n4(M: int, T: int, N: int, num_iters: int, stream: int = 0) -> None:
    _check(lib().mhc_sinkhorn_knopp_n4(M, T, N, num_iters, stream), "mhc_sinkhorn_knopp_n4")


def sinkhorn_knopp_n4_backward(G: int, M: int, D: int, N: int, num_iters: int, stream: int = 0) -> None:
    _check(lib().mhc_sinkhorn_knopp_n4_backward(G, M, D, N, num_iters, stream), "mhc_sinkhorn_knopp_n4_backward")


def sinkhorn_knopp_n4_logits(R: int, T: int, N: int, num_iters: int, stream: int = 0) -> None:
    _check(lib().mhc_sinkhorn_knopp_n4_logits(R, T, N, num_iters, stream), "mhc_sinkhorn_knopp_n4_logits")


def sinkhorn_knopp_n4_logits_ex(R: int, T: int, N: int, num_iters: int, flags: int, stream: int = 0) -> None:
    _check(lib().mhc_sinkhorn_knopp_n4_logits_ex(R, T, N, num_iters, flags, stream), "mhc_sinkhorn_knopp_n4_logits_ex")


def sinkhorn_knopp_n4_logits_backward(G: int, R: int, D: int, N: int, num_iters: int, stream: int = 0) -> None:
    _check(lib().mhc_sinkhorn_knopp_n4_logits_backward(G, R, D, N, num_iters, stream),
           "mhc_sinkhorn_knopp_n4_logits_backward")


def sinkhorn_knopp_n4_strided(X: int, x_stride: int, T: int, dtype: int, N: int, num_iters: int, flags: int,
                              stream: int = 0) -> None:
    _check(lib().mhc_sinkhorn_knopp_n4_strided(X, x_stride, T, dtype, N, num_iters, flags, stream),
           "mhc_sinkhorn_knopp_n4_strided")


def sinkhorn_knopp_n4_backward_strided(G: int, g_stride: int, g_dtype: int, X: int, x_stride: int, x_dtype: int,
                                       D: int, N: int, num_iters: int, flags: int, stream: int = 0) -> None:
    _check(lib().mhc_sinkhorn_knopp_n4_backward_strided(G, g_stride, g_dtype, X, x_stride, x_dtype, D, N, num_iters,
                                                        flags, stream),
           "mhc_sinkhorn_knopp_n4_backward_strided")


def birkhoff_proj_n4_hres(h: int, h_stride: int, rms: int, alpha: int, b: int, T: int, tol: float, N: int,
                          stream: int = 0) -> None:
    _check(lib().mhc_birkhoff_proj_n4_hres(h, h_stride, rms, alpha, b, T, tol, N, stream),
           "mhc_birkhoff_proj_n4_hres")


def birkhoff_proj_n4_hres_backward_workspace(N: int) -> int:
    """Bytes of workspace mhc_birkhoff_proj_n4_hres_backward uses for N matrices on the current device."""
    out = ctypes.c_int64(0)
    _check(lib().mhc_birkhoff_proj_n4_hres_backward_workspace(N, ctypes.byref(out)),
           "mhc_birkhoff_proj_n4_hres_backward_workspace")
    return out.value


def birkhoff_proj_n4_hres_backward(G: int, T: int, h: int, h_stride: int, rms: int, alpha: int, dh: int,
                                   dh_stride: int, drms: int, dalpha: int, db: int, N: int, workspace: int,
                                   workspace_bytes: int, stream: int = 0) -> None:
    _check(lib().mhc_birkhoff_proj_n4_hres_backward(G, T, h, h_stride, rms, alpha, dh, dh_stride, drms, dalpha, db,
                                                     N, workspace, workspace_bytes, stream),
           "mhc_birkhoff_proj_n4_hres_backward")


def birkhoff_proj_n4_hres_backward_noalloc(G: int, T: int, h: int, h_stride: int, rms: int, alpha: int, dh: int,
                                           dh_stride: int, drms: int, dalpha: int, db: int, N: int,
                                           stream: int = 0) -> None:
    """The backward with the library's fixed device scratch instead of a
    workspace; calls that may overlap on the GPU race (see the header)."""
    _check(lib().mhc_birkhoff_proj_n4_hres_backward_noalloc(G, T, h, h_stride, rms, alpha, dh, dh_stride, drms,
                                                             dalpha, db, N, stream),
           "mhc_birkhoff_proj_n4_hres_backward_noalloc")


def sinkhorn_knopp_n4_hres(h: int, h_stride: int, rms: int, alpha: int, b: int, T: int, N: int, num_iters: int,
                          stream: int = 0) -> None:
    _check(lib().mhc_sinkhorn_knopp_n4_hres(h, h_stride, rms, alpha, b, T, N, num_iters, stream),
           "mhc_sinkhorn_knopp_n4_hres")


def sinkhorn_knopp_n4_hres_backward_workspace(N: int) -> int:
    out = ctypes.c_int64(0)
    _check(lib().mhc_sinkhorn_knopp_n4_hres_backward_workspace(N, ctypes.byref(out)),
           "mhc_sinkhorn_knopp_n4_hres_backward_workspace")
    return out.value


def sinkhorn_knopp_n4_hres_backward(G: int, h: int, h_stride: int, rms: int, alpha: int, b: int, dh: int,
                                    dh_stride: int, drms: int, dalpha: int, db: int, N: int, num_iters: int,
                                    workspace: int, workspace_bytes: int, stream: int = 0) -> None:
    _check(lib().mhc_sinkhorn_knopp_n4_hres_backward(G, h, h_stride, rms, alpha, b, dh, dh_stride, drms, dalpha,
                                                      db, N, num_iters, workspace, workspace_bytes, stream),
           "mhc_sinkhorn_knopp_n4_hres_backward")


# --- tensor conveniences ---------------------------------------------------

def _dev(x, name):
    import torch

    if not (x.is_cuda and x.dtype == torch.float32 and x.is_contiguous() and x.dim() == 3
            and tuple(x.shape[1:]) == (4, 4)):
        raise ValueError(f"{name} must be a contiguous float32 CUDA tensor of shape (N, 4, 4)")
    return x.data_ptr()


def _stream(x) -> int:
    import torch

    return torch.cuda.current_stream(x.device).cuda_stream


def birkhoff_proj_n4_tensor(R, tol: float = 1e-6, out=None):
    import torch

    T = torch.empty_like(R) if out is None else out
    birkhoff_proj_n4(_dev(R, "R"), _dev(T, "T"), tol, R.shape[0], _stream(R))
    return T


def birkhoff_proj_n4_backward_tensor(G, T, out=None):
    import torch

    D = torch.empty_like(G) if out is None else out
    birkhoff_proj_n4_backward(_dev(G, "G"), _dev(T, "T"), _dev(D, "D"), G.shape[0], _stream(G))
    return D


# Order of the counters of mhc_birkhoff_proj_n4_pass_counts (MHC_PASS_* in mhc_proj.h).
PASS_COUNTER_NAMES = ("matrices", "fill", "start", "candidate_0", "candidate_1", "candidate_2", "candidate_3",
                      "candidate_4", "accepted_0", "accepted_1", "accepted_2", "accepted_3", "accepted_4",
                      "sweep_column", "sweep_eval", "at_cap", "lane_slots", "busy_lane_slots")


def birkhoff_proj_n4_pass_counts_tensor(R, tol: float = 1e-6):
    """Forward of a contiguous fp32 CUDA batch R through the counting
    instantiation: returns (T, iters, gnorm, counts) with counts a dict of
    the MHC_PASS_* totals (Python ints)."""
    import torch

    _dev(R, "R")
    n = R.shape[0]
    T = torch.empty_like(R)
    it = torch.empty(n, dtype=torch.int32, device=R.device)
    gn = torch.empty(n, dtype=torch.float32, device=R.device)
    c = torch.zeros(len(PASS_COUNTER_NAMES), dtype=torch.int64, device=R.device)
    birkhoff_proj_n4_pass_counts(R.data_ptr(), T.data_ptr(), tol, n, it.data_ptr(), gn.data_ptr(), c.data_ptr(),
                                 _stream(R))
    return T, it, gn, dict(zip(PASS_COUNTER_NAMES, (int(v) for v in c.tolist())))


def birkhoff_proj_n4_duals_tensor(R, tol: float = 1e-6):
    """(T, beta): the forward and its final duals, beta (N, 4)."""
    import torch

    T = torch.empty_like(R)
    beta = torch.empty(R.shape[0], 4, dtype=torch.float32, device=R.device)
    birkhoff_proj_n4_duals(_dev(R, "R"), _dev(T, "T"), beta.data_ptr(), tol, R.shape[0], _stream(R))
    return T, beta


def birkhoff_proj_n4_backward_duals_tensor(G, R, beta):
    import torch

    D = torch.empty_like(G)
    if not (beta.is_cuda and beta.dtype == torch.float32 and beta.is_contiguous() and beta.numel() == 4 * G.shape[0]):
        raise ValueError("beta must be a contiguous float32 CUDA tensor of N x 4 elements")
    birkhoff_proj_n4_backward_duals(_dev(G, "G"), _dev(R, "R"), beta.data_ptr(), _dev(D, "D"), G.shape[0],
                                    _stream(G))
    return D


def sinkhorn_knopp_n4_tensor(M, num_iters: int = 20, out=None):
    import torch

    T = torch.empty_like(M) if out is None else out
    sinkhorn_knopp_n4(_dev(M, "M"), _dev(T, "T"), M.shape[0], num_iters, _stream(M))
    return T


def sinkhorn_knopp_n4_backward_tensor(G, M, num_iters: int = 20, out=None):
    import torch

    D = torch.empty_like(G) if out is None else out
    sinkhorn_knopp_n4_backward(_dev(G, "G"), _dev(M, "M"), _dev(D, "D"), G.shape[0], num_iters, _stream(G))
    return D


def sinkhorn_knopp_n4_logits_tensor(R, num_iters: int = 20, out=None):
    import torch

    T = torch.empty_like(R) if out is None else out
    sinkhorn_knopp_n4_logits(_dev(R, "R"), _dev(T, "T"), R.shape[0], num_iters, _stream(R))
    return T


def sinkhorn_knopp_n4_logits_backward_tensor(G, R, num_iters: int = 20, out=None):
    import torch

    D = torch.empty_like(G) if out is None else out
    sinkhorn_knopp_n4_logits_backward(_dev(G, "G"), _dev(R, "R"), _dev(D, "D"), G.shape[0], num_iters, _stream(G))
    return D


def _dtype_code(x) -> int:
    import torch

    codes = {torch.float32: MHC_DTYPE_F32, torch.bfloat16: MHC_DTYPE_BF16, torch.float16: MHC_DTYPE_F16}
    if x.dtype not in codes:
        raise ValueError(f"unsupported dtype {x.dtype}")
    return codes[x.dtype]


def _strided(x, name):
    if not (x.is_cuda and x.dim() == 3 and tuple(x.shape[1:]) == (4, 4) and x.stride(2) == 1 and x.stride(1) == 4):
        raise ValueError(f"{name} must be a CUDA (N, 4, 4) tensor with contiguous 4x4 matrices")
    return x.data_ptr(), x.stride(0), _dtype_code(x)


def birkhoff_proj_n4_ex_tensor(R, tol: float = 1e-6):
    """Newton forward on a strided fp32/bf16/fp16 batch; T contiguous in R's dtype."""
    import torch

    ptr, stride, dt = _strided(R, "R")
    T = torch.empty(R.shape, dtype=R.dtype, device=R.device)
    birkhoff_proj_n4_ex(ptr, stride, T.data_ptr(), dt, tol, R.shape[0], _stream(R))
    return T


def birkhoff_proj_n4_backward_ex_tensor(G, T):
    """IFT backward on strided batches; D contiguous in G's dtype."""
    import torch

    gp, gs, gd = _strided(G, "G")
    tp, ts, td = _strided(T, "T")
    D = torch.empty(G.shape, dtype=G.dtype, device=G.device)
    birkhoff_proj_n4_backward_ex(gp, gs, gd, tp, ts, td, D.data_ptr(), G.shape[0], _stream(G))
    return D


def sinkhorn_knopp_n4_strided_tensor(X, num_iters: int = 20, logits: bool = False, approx_reciprocal: bool = False):
    """Sinkhorn-Knopp (logits=True: on exp(X)) of a strided fp32/bf16/fp16
    batch; T contiguous in X's dtype."""
    import torch

    ptr, stride, dt = _strided(X, "X")
    T = torch.empty(X.shape, dtype=X.dtype, device=X.device)
    flags = (MHC_SK_LOGITS if logits else 0) | (MHC_SK_HW_RECIPROCAL if approx_reciprocal else 0)
    sinkhorn_knopp_n4_strided(ptr, stride, T.data_ptr(), dt, X.shape[0], num_iters, flags, _stream(X))
    return T


def sinkhorn_knopp_n4_backward_strided_tensor(G, X, num_iters: int = 20, logits: bool = False):
    """Its backward on strided batches; D contiguous in G's dtype."""
    import torch

    gp, gs, gd = _strided(G, "G")
    xp, xs, xd = _strided(X, "X")
    D = torch.empty(G.shape, dtype=G.dtype, device=G.device)
    sinkhorn_knopp_n4_backward_strided(gp, gs, gd, xp, xs, xd, D.data_ptr(), G.shape[0], num_iters,
                                       MHC_SK_LOGITS if logits else 0, _stream(G))
    return D


def _hres_inputs(h, rms, alpha, b):
    """Pointers and the batch stride of the H_res producer's inputs: h (N, 16)
    or (N, 4, 4) fp32 CUDA with each matrix's 16 entries contiguous (a column
    slice of a wider projection output is fine), rms (N,), alpha one element,
    b 16 elements, all contiguous fp32 on h's device."""
    import torch

    n = h.shape[0]
    flat_ok = h.dim() == 2 and h.shape[1] == 16 and h.stride(1) == 1
    mat_ok = h.dim() == 3 and tuple(h.shape[1:]) == (4, 4) and h.stride(2) == 1 and h.stride(1) == 4
    if not (h.is_cuda and h.dtype == torch.float32 and (flat_ok or mat_ok)):
        raise ValueError("h must be a float32 CUDA tensor of shape (N, 16) or (N, 4, 4) with contiguous matrices")
    for x, name, numel in ((rms, "rms", n), (alpha, "alpha", 1), (b, "b", 16)):
        if not (x.device == h.device and x.dtype == torch.float32 and x.is_contiguous() and x.numel() == numel):
            raise ValueError(f"{name} must be a contiguous float32 tensor of {numel} elements on h's device")
    return h.data_ptr(), h.stride(0), rms.data_ptr(), alpha.data_ptr(), b.data_ptr()


def birkhoff_proj_n4_hres_tensor(h, rms, alpha, b, tol: float = 1e-6):
    """Projection of R = alpha * h / rms + b formed in the kernel's load; T is (N, 4, 4) fp32."""
    import torch

    hp, hs, rp, ap, bp = _hres_inputs(h, rms, alpha, b)
    T = torch.empty(h.shape[0], 4, 4, dtype=torch.float32, device=h.device)
    birkhoff_proj_n4_hres(hp, hs, rp, ap, bp, T.data_ptr(), tol, h.shape[0], _stream(h))
    return T


def birkhoff_proj_n4_hres_backward_tensor(G, T, h, rms, alpha, dh=None):
    """Gradients (dh, drms, dalpha, db) of the fused producer + projection.  dh
    is (N, 16) fp32, or written into the given tensor (same layout rules as h)."""
    import torch

    hp, hs, rp, ap, _ = _hres_inputs(h, rms, alpha, torch.empty(16, device=h.device))
    n = h.shape[0]
    if dh is None:
        dh = torch.empty(n, 16, dtype=torch.float32, device=h.device)
    dhp, dhs, _, _, _ = _hres_inputs(dh, rms, alpha, torch.empty(16, device=h.device))
    drms = torch.empty(n, dtype=torch.float32, device=h.device)
    dalpha = torch.empty((), dtype=torch.float32, device=h.device)
    db = torch.empty(4, 4, dtype=torch.float32, device=h.device)
    with torch.cuda.device(h.device):
        ws = torch.empty(max(birkhoff_proj_n4_hres_backward_workspace(n), 4) // 4, dtype=torch.float32,
                         device=h.device)
    birkhoff_proj_n4_hres_backward(_dev(G, "G"), _dev(T, "T"), hp, hs, rp, ap, dhp, dhs, drms.data_ptr(),
                                   dalpha.data_ptr(), db.data_ptr(), n, ws.data_ptr(), ws.numel() * 4, _stream(h))
    return dh, drms, dalpha, db


def sinkhorn_knopp_n4_hres_tensor(h, rms, alpha, b, num_iters: int = 20):
    """Sinkhorn-Knopp on M = exp(alpha * h / rms + b) (the producer's H_res), formed in the kernel's load."""
    import torch

    hp, hs, rp, ap, bp = _hres_inputs(h, rms, alpha, b)
    T = torch.empty(h.shape[0], 4, 4, dtype=torch.float32, device=h.device)
    sinkhorn_knopp_n4_hres(hp, hs, rp, ap, bp, T.data_ptr(), h.shape[0], num_iters, _stream(h))
    return T


def sinkhorn_knopp_n4_hres_backward_tensor(G, h, rms, alpha, b, num_iters: int = 20, dh=None):
    """Gradients (dh, drms, dalpha, db) of sinkhorn_knopp_n4_hres."""
    import torch

    hp, hs, rp, ap, bp = _hres_inputs(h, rms, alpha, b)
    n = h.shape[0]
    if dh is None:
        dh = torch.empty(n, 16, dtype=torch.float32, device=h.device)
    dhp, dhs, _, _, _ = _hres_inputs(dh, rms, alpha, b)
    drms = torch.empty(n, dtype=torch.float32, device=h.device)
    dalpha = torch.empty((), dtype=torch.float32, device=h.device)
    db = torch.empty(4, 4, dtype=torch.float32, device=h.device)
    ws = torch.empty(sinkhorn_knopp_n4_hres_backward_workspace(n) // 4, dtype=torch.float32, device=h.device)
    sinkhorn_knopp_n4_hres_backward(_dev(G, "G"), hp, hs, rp, ap, bp, dhp, dhs, drms.data_ptr(), dalpha.data_ptr(),
                                    db.data_ptr(), n, num_iters, ws.data_ptr(), ws.numel() * 4, _stream(h))
    return dh, drms, dalpha, db
