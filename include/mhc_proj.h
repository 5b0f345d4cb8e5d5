/*
 * mhc_proj -- batched n=4 Birkhoff projection on B200 (sm_100a).
 *
 * C ABI of libmhcproj.so.  Every entry point takes device pointers to N
 * contiguous row-major 4x4 fp32 matrices (64 bytes each), launches on
 * `stream` and returns without synchronising.  Pointers that are 16-byte
 * aligned take the 128-bit load/store path; any other alignment is accepted
 * and served by a scalar path.  Inputs and outputs must not overlap.
 *
 * Return value: MHC_OK (0), a negative MHC_ERR_* code for a rejected argument
 * (nothing is launched), or a positive cudaError_t from the launch.
 *
 * These entry points replace the reference's C++ launchers, which return
 * void and check nothing; each declaration cites the one it replaces
 * (file:line in the reference project).
 */
#ifndef MHC_PROJ_H
#define MHC_PROJ_H

#include <stdint.h>
#include <cuda_runtime_api.h>

#ifdef __cplusplus
extern "C" {
#endif

#define MHC_PROJ_ABI_VERSION 1

#if defined(__GNUC__)
#define MHC_API __attribute__((visibility("default")))
#else
#define MHC_API
#endif

enum {
    MHC_OK = 0,
    MHC_ERR_INVALID_VALUE = -1, /* N < 0, a null pointer with N > 0, a negative stride or an unknown dtype */
    MHC_ERR_ITERS = -2,         /* iteration count outside the supported range */
    MHC_ERR_CAPTURE = -3        /* a first call in a CUDA context that must look up a device
                                   address was made during stream capture */
};

/* Storage types of the *_ex entry points.  Computation is always fp32: bf16
 * and fp16 inputs widen exactly, outputs round to nearest even -- the same
 * bits as converting to fp32, calling the fp32 entry point and converting
 * back. */
enum {
    MHC_DTYPE_F32 = 0,
    MHC_DTYPE_BF16 = 1,
    MHC_DTYPE_F16 = 2
};

/* Largest iteration count sinkhorn_knopp_n4_backward accepts (the
 * reference's limit, src/sinkhorn_knopp.cuh:1213). */
#define MHC_SK_BACKWARD_MAX_ITERS 20

/* Forward KL projection by dual Newton: T = diag(e^a) exp(R) diag(e^b) with
 * unit row sums and column sums within `tol` (l1 over the first three
 * columns), at most 20 Newton iterations.
 * Replaces: void birkhoff_proj_n4(const float* d_R, float* d_T, float tol,
 *           int N, cudaStream_t) -- src/birkhoff_proj_n4.cu:505 */
MHC_API int mhc_birkhoff_proj_n4(const float* d_R, float* d_T, float tol, int64_t N,
                         cudaStream_t stream);

/* mhc_birkhoff_proj_n4 that also reports, per matrix, the number of Newton
 * iterations taken (0 when the initialisation already meets tol, 20 at the
 * cap) in d_iters[N] and the final gradient l1 norm in d_gnorm[N]; a matrix
 * with d_gnorm >= tol stopped at the iteration cap.  T is the same as from
 * mhc_birkhoff_proj_n4.  No reference counterpart: a convergence report the
 * reference kernel has no way to give. */
MHC_API int mhc_birkhoff_proj_n4_stats(const float* d_R, float* d_T, float tol, int64_t N,
                                       int32_t* d_iters, float* d_gnorm, cudaStream_t stream);

/* Counters of mhc_birkhoff_proj_n4_pass_counts: where the forward's
 * log-sum-exp passes go.  Each matrix costs two passes when it is staged
 * (the beta = 0 objective and the alpha = 0 initialisation,
 * src/birkhoff_proj_n4.cu:402-415), then one pass per step of its state
 * machine: the evaluation at the chosen start (:416-423), line-search
 * candidates k = 0..4 (:450-477), and the two passes of a Sinkhorn sweep
 * after five rejections (:480-486). */
enum {
    MHC_PASS_MATRICES = 0,        /* matrices projected */
    MHC_PASS_FILL = 1,            /* passes made while staging (2 per matrix) */
    MHC_PASS_START = 2,           /* evaluations at the starting point */
    MHC_PASS_CANDIDATE = 3,       /* + k, k = 0..4: candidate evaluations at step gamma_k */
    MHC_PASS_ACCEPTED = 8,        /* + k: candidates accepted at step gamma_k */
    MHC_PASS_SWEEP_COLUMN = 13,   /* column passes of the Sinkhorn fallback sweep */
    MHC_PASS_SWEEP_EVAL = 14,     /* evaluations after the sweep */
    MHC_PASS_AT_CAP = 15,         /* matrices that stopped at the 20-iteration cap */
    MHC_PASS_LANE_SLOTS = 16,     /* state-machine steps x 32 lanes */
    MHC_PASS_BUSY_LANE_SLOTS = 17, /* lane slots that held a matrix (the rest: a warp's tail) */
    MHC_PASS_COUNTERS = 18
};

/* mhc_birkhoff_proj_n4_stats that also adds the forward's pass counts to
 * d_counts[MHC_PASS_COUNTERS] (64-bit, accumulated: zero it first).  A
 * diagnostic of the state machine's work, in an instantiation of its own;
 * T is the same as from mhc_birkhoff_proj_n4.  No reference counterpart. */
MHC_API int mhc_birkhoff_proj_n4_pass_counts(const float* d_R, float* d_T, float tol, int64_t N,
                                             int32_t* d_iters, float* d_gnorm, unsigned long long* d_counts,
                                             cudaStream_t stream);

/* mhc_birkhoff_proj_n4 that also writes, per matrix, the final dual beta
 * (4 floats at d_beta + 4k, beta[3] = 0 up to its sign): T is exactly
 * row-softmax(beta + R), which mhc_birkhoff_proj_n4_backward_duals rebuilds
 * bit for bit, so a caller may keep R and 16 bytes of beta per matrix for the
 * backward instead of T's 64.  T is the same as from mhc_birkhoff_proj_n4.
 * No reference counterpart. */
MHC_API int mhc_birkhoff_proj_n4_duals(const float* d_R, float* d_T, float* d_beta, float tol,
                                       int64_t N, cudaStream_t stream);

/* mhc_birkhoff_proj_n4_backward from R and the saved beta instead of T (T is
 * rebuilt in registers with the forward's arithmetic); D is the same bits.
 * Reads G, R and beta (208 bytes per matrix) instead of G and T (192).  No
 * reference counterpart. */
MHC_API int mhc_birkhoff_proj_n4_backward_duals(const float* d_G, const float* d_R, const float* d_beta,
                                                float* d_D, int64_t N, cudaStream_t stream);

/* mhc_birkhoff_proj_n4 on a strided batch of any storage type: matrix k of R
 * starts at element k * r_stride (its 16 entries row-major and contiguous),
 * T is written contiguous in the same type.  No reference counterpart: the
 * reference's wrapper converts R to contiguous fp32 and T back
 * (solvers_torch.cpp:61,67,82), which this does inside the kernel. */
MHC_API int mhc_birkhoff_proj_n4_ex(const void* d_R, int64_t r_stride, void* d_T, int dtype,
                                    float tol, int64_t N, cudaStream_t stream);

/* Backward by the implicit function theorem: D = dL/dR given G = dL/dT and
 * the forward output T.
 * Replaces: void birkhoff_proj_n4_backward(const float* d_G, const float* d_T,
 *           float* d_D, int N, cudaStream_t) -- src/birkhoff_proj_n4.cu:675 */
MHC_API int mhc_birkhoff_proj_n4_backward(const float* d_G, const float* d_T, float* d_D,
                                  int64_t N, cudaStream_t stream);

/* mhc_birkhoff_proj_n4_backward on strided batches of any storage types:
 * G (g_dtype, stride g_stride elements) and T (t_dtype, stride t_stride); D
 * is written contiguous in G's type.  No reference counterpart: the
 * reference's wrapper converts G and T to contiguous fp32 and D back
 * (solvers_torch.cpp:128-136,152). */
MHC_API int mhc_birkhoff_proj_n4_backward_ex(const void* d_G, int64_t g_stride, int g_dtype,
                                             const void* d_T, int64_t t_stride, int t_dtype,
                                             void* d_D, int64_t N, cudaStream_t stream);

/* Fixed-iteration Sinkhorn-Knopp on M (= exp(R)): `num_iters` row then
 * column normalisations, a sum s <= 1e-8 giving a zero factor.
 * num_iters <= 0 copies M to T.
 * Replaces: void sinkhorn_knopp_n4(const float* d_M, float* d_T, int N,
 *           int num_iters, cudaStream_t) -- src/sinkhorn_knopp_n4.cu:5 */
MHC_API int mhc_sinkhorn_knopp_n4(const float* d_M, float* d_T, int64_t N, int num_iters,
                          cudaStream_t stream);

/* Exact gradient of sum(G .* sinkhorn_knopp_n4(M)) with respect to M.
 * num_iters <= 0 gives D = G; num_iters > MHC_SK_BACKWARD_MAX_ITERS
 * returns MHC_ERR_ITERS.
 * Replaces: void sinkhorn_knopp_n4_backward(const float* d_G, const float* d_M,
 *           float* d_D, int N, int num_iters, cudaStream_t)
 *           -- src/sinkhorn_knopp_n4.cu:13 */
MHC_API int mhc_sinkhorn_knopp_n4_backward(const float* d_G, const float* d_M, float* d_D,
                                   int64_t N, int num_iters, cudaStream_t stream);

/* Sinkhorn-Knopp fused with the exponential: the input is the logits R and
 * the kernel forms M = exp(R) (the accurate expf, as torch.exp computes it)
 * before the normalisations above.  Same result as mhc_sinkhorn_knopp_n4 on
 * M = torch.exp(R), in one pass over HBM (128 B per matrix instead of 256).
 * No reference counterpart: it fuses the torch.exp that the reference's
 * MHCSinkhornN4Function does in Python (mhc_proj/module.py:50) into the
 * kernel. */
MHC_API int mhc_sinkhorn_knopp_n4_logits(const float* d_R, float* d_T, int64_t N, int num_iters,
                                         cudaStream_t stream);

/* Flags of mhc_sinkhorn_knopp_n4_logits_ex and of the strided entry points
 * below. */
enum {
    /* The normalisation factors from the hardware reciprocal (at most one
     * ulp from 1/s) instead of the correctly rounded one: not the reference
     * kernel's bits, but within 1e-6 of them and of the vanilla PyTorch
     * Sinkhorn-Knopp on N(0,1) logits, and about 20% faster. */
    MHC_SK_HW_RECIPROCAL = 1,
    /* (strided entry points) The input is the logits R: M = exp(R), the
     * accurate expf rounded to R's storage type, as torch.exp in that type
     * computes it. */
    MHC_SK_LOGITS = 2
};

/* mhc_sinkhorn_knopp_n4_logits with `flags` (0 or MHC_SK_HW_RECIPROCAL; any
 * other bit returns MHC_ERR_INVALID_VALUE).  No reference counterpart. */
MHC_API int mhc_sinkhorn_knopp_n4_logits_ex(const float* d_R, float* d_T, int64_t N, int num_iters, int flags,
                                            cudaStream_t stream);

/* Gradient with respect to R of sum(G .* sinkhorn_knopp_n4(exp(R))): the
 * backward above times exp(R), in one pass (192 B per matrix instead of
 * 384).  No reference counterpart: it fuses the backward kernel with the
 * D * expon product of the reference's MHCSinkhornN4Function.backward
 * (mhc_proj/module.py:70).  num_iters > MHC_SK_BACKWARD_MAX_ITERS returns
 * MHC_ERR_ITERS. */
MHC_API int mhc_sinkhorn_knopp_n4_logits_backward(const float* d_G, const float* d_R, float* d_D,
                                                  int64_t N, int num_iters, cudaStream_t stream);

/* mhc_sinkhorn_knopp_n4 (or, with MHC_SK_LOGITS, the fused-exponential form)
 * on a strided batch of any storage type: matrix k of X starts at element
 * k * x_stride (its 16 entries row-major and contiguous); T is written
 * contiguous in the same type.  The results are the reference's on such a
 * tensor: its wrapper converts X to contiguous fp32 and T back
 * (solvers_torch.cpp:190,196,211), its module computes torch.exp in X's type
 * (mhc_proj/module.py:50); bf16 and fp16 widen exactly and T is rounded to
 * nearest even.  flags: MHC_SK_LOGITS, MHC_SK_HW_RECIPROCAL.  No reference
 * counterpart. */
MHC_API int mhc_sinkhorn_knopp_n4_strided(const void* d_X, int64_t x_stride, void* d_T, int dtype, int64_t N,
                                          int num_iters, int flags, cudaStream_t stream);

/* The backward of mhc_sinkhorn_knopp_n4_strided: G (g_dtype, stride g_stride
 * elements) and X (x_dtype, stride x_stride: M, or with MHC_SK_LOGITS the
 * logits R); D is written contiguous in G's type.  Without MHC_SK_LOGITS, D is
 * dL/dM rounded to G's type (the reference wrapper's result,
 * solvers_torch.cpp:258-266,282); with it, that rounded dL/dM times M rounded to
 * G's type again -- the reference module's D * expon (mhc_proj/module.py:70)
 * when G and R have the same type.  flags: MHC_SK_LOGITS only.  num_iters >
 * MHC_SK_BACKWARD_MAX_ITERS returns MHC_ERR_ITERS.  No reference
 * counterpart. */
MHC_API int mhc_sinkhorn_knopp_n4_backward_strided(const void* d_G, int64_t g_stride, int g_dtype, const void* d_X,
                                                   int64_t x_stride, int x_dtype, void* d_D, int64_t N,
                                                   int num_iters, int flags, cudaStream_t stream);

/* The projection fused with its producer, the H_res pre-activation of an
 * mHC layer: R[k] = alpha * h[k] / rms[k] + b, formed in the kernel's load
 * with the reference producer's arithmetic before its exponential
 * (src/utils.cuh:84-93: r_inv = 1 / rms, then (alpha * h) * r_inv + b as one
 * multiply and one fused multiply-add).  h[k] is 16 consecutive floats at
 * d_h + k * h_stride -- e.g. columns 8..23 of a [N, 24] projection output,
 * h_stride = 24; d_rms holds N floats; d_alpha one float and d_b sixteen
 * (row-major 4x4), all in device memory so that a call needs no host read.
 * T (contiguous fp32) is the same as mhc_birkhoff_proj_n4 of that R.
 * No reference counterpart: the reference's producer writes exp(R) to
 * memory in a kernel of its own (fused_h_activations, src/utils.cuh:96-127). */
MHC_API int mhc_birkhoff_proj_n4_hres(const float* d_h, int64_t h_stride, const float* d_rms,
                                      const float* d_alpha, const float* d_b, float* d_T, float tol,
                                      int64_t N, cudaStream_t stream);

/* Bytes of device workspace that mhc_birkhoff_proj_n4_hres_backward uses
 * for N matrices on the current device (its per-block partial sums). */
MHC_API int mhc_birkhoff_proj_n4_hres_backward_workspace(int64_t N, int64_t* bytes);

/* Backward of mhc_birkhoff_proj_n4_hres given G = dL/dT and its output T:
 * with D = dL/dR (the same bits as mhc_birkhoff_proj_n4_backward),
 *   dh[k]   = D[k] * alpha / rms[k]        (written at d_dh + k * dh_stride),
 *   drms[k] = -alpha / rms[k]^2 * sum(D[k] .* h[k]),
 *   dalpha  = sum_k sum(D[k] .* h[k]) / rms[k],   db = sum_k D[k].
 * dalpha and db are overwritten (zeros for N = 0), not accumulated.  The
 * batch sums are deterministic: the same N, workspace size and GPU model
 * give the same bits.  d_workspace holds workspace_bytes of scratch (any
 * contents; the size from mhc_birkhoff_proj_n4_hres_backward_workspace, or
 * less at the cost of fewer blocks, but at least 68 bytes when N > 0) that
 * the call owns until it completes on `stream`.  No reference counterpart:
 * the reference has no backward for its producer. */
MHC_API int mhc_birkhoff_proj_n4_hres_backward(const float* d_G, const float* d_T, const float* d_h,
                                               int64_t h_stride, const float* d_rms,
                                               const float* d_alpha, float* d_dh, int64_t dh_stride,
                                               float* d_drms, float* d_dalpha, float* d_db, int64_t N,
                                               void* d_workspace, int64_t workspace_bytes,
                                               cudaStream_t stream);

/* mhc_birkhoff_proj_n4_hres_backward for callers that cannot allocate device
 * memory: code running under a framework or serving engine that has already
 * claimed the device's memory as its own pool and hands this library no
 * allocator, and latency-bound loops that cannot afford cudaMalloc/cudaFree,
 * which can synchronise the whole device.  It takes no workspace and
 * allocates nothing: the per-block partial sums go to a fixed 68 KB array
 * that is part of the library (1024 rows of 17 floats), which every GPU that
 * loads the library holds until the process exits.  The call uses at most
 * 1024 blocks, one row each, so no batch size needs more than the array.
 * The first call in each CUDA context looks the array's address up
 * (cudaGetSymbolAddress) and keeps it for that context: after a device reset,
 * or in a context the caller created, the next call looks it up again.  Make
 * that first call before any stream capture: made during capture it launches
 * nothing and returns MHC_ERR_CAPTURE.  Same results as the workspace form given the size that
 * mhc_birkhoff_proj_n4_hres_backward_workspace reports (on a GPU whose
 * resident-block wave is at most 1024 blocks, B200 included).  The array is
 * shared by every call on a device and keeps the last call's sums: calls
 * whose kernels may overlap on the GPU (different streams without ordering)
 * race and must not be issued.  Nothing in it has to start at zero: each call
 * writes every row it reads first.  No counterpart in the reference. */
MHC_API int mhc_birkhoff_proj_n4_hres_backward_noalloc(const float* d_G, const float* d_T,
                                                       const float* d_h, int64_t h_stride,
                                                       const float* d_rms, const float* d_alpha,
                                                       float* d_dh, int64_t dh_stride, float* d_drms,
                                                       float* d_dalpha, float* d_db, int64_t N,
                                                       cudaStream_t stream);

/* Sinkhorn-Knopp on the mHC layer's H_res activation: M[k] = exp(alpha *
 * h[k] / rms[k] + b) formed in the kernel's load exactly as the reference's
 * producer forms it (fused_h_activations, src/utils.cuh:84-93, with its
 * __expf, utils.cuh:42-44), then the normalisations of mhc_sinkhorn_knopp_n4.
 * h, h_stride, rms, alpha and b as for mhc_birkhoff_proj_n4_hres.  T is the
 * same as the reference's producer followed by its sinkhorn_knopp_n4.  No
 * reference counterpart: there the producer writes H_res to memory. */
MHC_API int mhc_sinkhorn_knopp_n4_hres(const float* d_h, int64_t h_stride, const float* d_rms,
                                       const float* d_alpha, const float* d_b, float* d_T, int64_t N,
                                       int num_iters, cudaStream_t stream);

/* Bytes of device workspace that mhc_sinkhorn_knopp_n4_hres_backward needs for
 * N matrices (68 per block of 128 matrices). */
MHC_API int mhc_sinkhorn_knopp_n4_hres_backward_workspace(int64_t N, int64_t* bytes);

/* Backward of mhc_sinkhorn_knopp_n4_hres given G = dL/dT: with dM the exact
 * gradient with respect to M (mhc_sinkhorn_knopp_n4_backward) and dR = dM .* M,
 * the outputs of mhc_birkhoff_proj_n4_hres_backward (dh, drms per matrix;
 * dalpha and db as deterministic batch sums, overwritten).  The workspace must
 * hold at least the reported bytes; num_iters > MHC_SK_BACKWARD_MAX_ITERS
 * returns MHC_ERR_ITERS.  No reference counterpart. */
MHC_API int mhc_sinkhorn_knopp_n4_hres_backward(const float* d_G, const float* d_h, int64_t h_stride,
                                                const float* d_rms, const float* d_alpha,
                                                const float* d_b, float* d_dh, int64_t dh_stride,
                                                float* d_drms, float* d_dalpha, float* d_db, int64_t N,
                                                int num_iters, void* d_workspace,
                                                int64_t workspace_bytes, cudaStream_t stream);

/* Human-readable text for a return code of the functions above. */
MHC_API const char* mhc_status_string(int status);

/* MHC_PROJ_ABI_VERSION of the loaded library. */
MHC_API int mhc_abi_version(void);

#ifdef __cplusplus
}
#endif

#endif /* MHC_PROJ_H */
