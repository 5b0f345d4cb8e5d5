// Kernels and C-ABI launchers for the fixed-iteration Sinkhorn-Knopp pair, on
// M = exp(R) as the reference takes it, or fused with the exponential on the
// logits R.
//
// This file is built without --use_fast_math (with -ftz=true): the
// Sinkhorn-Knopp arithmetic uses explicit round-to-nearest intrinsics and a
// correctly rounded reciprocal, which that flag does not change, and expf in
// the fused kernels is then the accurate one, the same function PyTorch's
// exp kernel calls, so fused and unfused paths agree.
#include <type_traits>
#include <utility>

#include "sinkhorn_n4.cuh"
#include "partial_sums.cuh"
#include "mhc_proj.h"

namespace mhcp {

constexpr float kSkEps = 1e-8f;  // src/sinkhorn_knopp_n4.cu:10,18
constexpr int kSkBlock = 128;


// exp of every entry (the fused kernels' input is the logits R).
__device__ __forceinline__ void exp_inplace(Mat4& x)
{
#pragma unroll
    for (int e = 0; e < 16; ++e) x.m[e] = expf(x.m[e]);
}

// Where the kernels find M, matrix idx of the batch:
//   MInput     M itself (row-major, contiguous);
//   ExpInput   the logits R, M = exp(R) with the accurate expf (as torch.exp);
//   HResInput  the mHC layer's H_res block, M = exp of the producer's
//              pre-activation alpha * h / rms + b with the producer's own
//              __expf (src/utils.cuh:42-44,84-93), i.e. its H_res output.
struct MInput {
    const float* M;
    template <bool kVec>
    __device__ __forceinline__ void load(int64_t idx, Mat4& x) const { load_mat<kVec>(M, idx, x); }
};

struct ExpInput {
    const float* R;
    template <bool kVec>
    __device__ __forceinline__ void load(int64_t idx, Mat4& x) const
    {
        load_mat<kVec>(R, idx, x);
        exp_inplace(x);
    }
};

struct HResInput {
    const float* h;
    int64_t stride;
    const float* rms;
    const float* alpha;
    const float* b;
    // h[idx] and 1 / rms[idx] (the backward needs both again).
    template <bool kVec>
    __device__ __forceinline__ float load_h(int64_t idx, Mat4& x) const
    {
        load_elems<float, kVec>(h, idx * stride, x);
        return hres_rinv(__ldg(rms + idx));
    }
    __device__ __forceinline__ void activate(const Mat4& hx, float rinv, Mat4& m) const
    {
        const float a = __ldg(alpha);
#pragma unroll
        for (int e = 0; e < 16; ++e) m.m[e] = __expf(hres_logit(a, hx.m[e], rinv, __ldg(b + e)));
    }
    template <bool kVec>
    __device__ __forceinline__ void load(int64_t idx, Mat4& x) const
    {
        Mat4 hx;
        const float rinv = load_h<kVec>(idx, hx);
        activate(hx, rinv, x);
    }
};

// kApprox: the factors from the hardware reciprocal (sk_inv_approx) instead
// of the correctly rounded one.
template <bool kVec, class In, bool kApprox = false>
__global__ void __launch_bounds__(kSkBlock) sk_fwd_kernel(In in, float* __restrict__ T, int64_t N, int iters)
{
    const int64_t idx = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (idx >= N) return;
    Mat4 x0;
    in.template load<kVec>(idx, x0);
    Pairs x = to_pairs(x0);
#pragma unroll 1
    for (int it = 0; it < iters; ++it) sk_iteration<kApprox>(x, kSkEps);
    store_mat<kVec>(T, idx, from_pairs(x));
}

// History rows of a kIters backward (at least one).
template <int kIters>
constexpr int kSkHist = kIters > 0 ? kIters : 1;

// Backward with a compile-time iteration count, in potential form
// (sinkhorn_n4.cuh): D = dL/dM, or with kLogits (ExpInput) the gradient with
// respect to R, dL/dM * exp(R).  v_1 .. v_kIters in shared memory,
// [iteration][thread] so that a warp's 16-byte accesses are conflict-free.
template <int kIters, bool kVec, bool kLogits>
__global__ void __launch_bounds__(kSkBlock) sk_bwd_kernel(const float* __restrict__ G,
                                                          const float* __restrict__ M,
                                                          float* __restrict__ D, int64_t N)
{
    __shared__ float4 vh[kSkHist<kIters>][kSkBlock];
    const int64_t idx = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (idx >= N) return;
    Mat4 x0, g0;
    if constexpr (kLogits)
        ExpInput{M}.load<kVec>(idx, x0);
    else
        MInput{M}.load<kVec>(idx, x0);
    const Pairs m = to_pairs(x0);
    Pairs d;
    if constexpr (kIters > 0) {
        bool mr[4];
        float u[4], v[4];
        pot_forward<kIters, kSkBlock>(m, kSkEps, vh, threadIdx.x, mr, u, v);
        load_mat<kVec>(G, idx, g0);
        pot_reverse<kIters, kSkBlock>(m, to_pairs(g0), vh, threadIdx.x, mr, u, v, d);
    } else {
        load_mat<kVec>(G, idx, g0);
        d = to_pairs(g0);
    }
    if constexpr (kLogits) {
#pragma unroll
        for (int q = 0; q < 8; ++q) d.p[q] = __fmul2_rn(d.p[q], m.p[q]);
    }
    store_mat<kVec>(D, idx, from_pairs(d));
}

// Backward of the producer fused with Sinkhorn-Knopp: dM as above, dR = dM *
// M, then the producer's chain rule (partial_sums.cuh: dh, drms per matrix;
// the per-block partial sums of db and dalpha in column blockIdx.x of
// `partials`).  One matrix per thread; every thread reaches the block fold.
template <int kIters, bool kVec>
__global__ void __launch_bounds__(kSkBlock) sk_hres_bwd_kernel(const float* __restrict__ G, HResInput in,
                                                               float* __restrict__ dh, int64_t dh_stride,
                                                               float* __restrict__ drms,
                                                               float* __restrict__ partials, int64_t N)
{
    __shared__ float4 vh[kSkHist<kIters>][kSkBlock];
    float acc[kHResPartials];
#pragma unroll
    for (int q = 0; q < kHResPartials; ++q) acc[q] = 0.0f;
    const int64_t idx = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (idx < N) {
        Mat4 hx, m, g0, dR, dx;
        const float rinv = in.load_h<kVec>(idx, hx);
        in.activate(hx, rinv, m);
        const Pairs mp = to_pairs(m);
        load_mat<kVec>(G, idx, g0);
        Mat4 dM = g0;
        if constexpr (kIters > 0) {
            bool mr[4];
            float u[4], v[4];
            Pairs d;
            pot_forward<kIters, kSkBlock>(mp, kSkEps, vh, threadIdx.x, mr, u, v);
            pot_reverse<kIters, kSkBlock>(mp, to_pairs(g0), vh, threadIdx.x, mr, u, v, d);
            dM = from_pairs(d);
        }
#pragma unroll
        for (int e = 0; e < 16; ++e) dR.m[e] = __fmul_rn(dM.m[e], m.m[e]);
        drms[idx] = hres_chain(dR, hx, __ldg(in.alpha), rinv, dx, acc);
        store_elems<float, kVec>(dh, idx * dh_stride, dx);
    }
    block_partial_sums<kSkBlock>(acc, partials, gridDim.x, blockIdx.x);
}

template <int kIters, bool kLogits>
static void launch_sk_bwd(bool vec, const float* G, const float* M, float* D, int64_t N, cudaStream_t stream)
{
    const int64_t grid = ceil_div(N, kSkBlock);
    if (vec)
        sk_bwd_kernel<kIters, true, kLogits><<<grid, kSkBlock, 0, stream>>>(G, M, D, N);
    else
        sk_bwd_kernel<kIters, false, kLogits><<<grid, kSkBlock, 0, stream>>>(G, M, D, N);
}

// iters in [0, MHC_SK_BACKWARD_MAX_ITERS] picks the matching instantiation.
template <bool kLogits, int... Is>
static void dispatch_sk_bwd(int iters, bool vec, const float* G, const float* M, float* D, int64_t N,
                            cudaStream_t stream, std::integer_sequence<int, Is...>)
{
    ((iters == Is ? launch_sk_bwd<Is, kLogits>(vec, G, M, D, N, stream) : void()), ...);
}

template <bool kLogits, bool kApprox = false>
static int sk_forward(const float* d_M, float* d_T, int64_t N, int num_iters, cudaStream_t stream)
{
    if (N < 0 || (N > 0 && (!d_M || !d_T))) return MHC_ERR_INVALID_VALUE;
    if (N == 0) return MHC_OK;
    const int iters = num_iters > 0 ? num_iters : 0;
    const int64_t grid = ceil_div(N, kSkBlock);
    using In = std::conditional_t<kLogits, ExpInput, MInput>;
    if (aligned16(d_M) && aligned16(d_T))
        sk_fwd_kernel<true, In, kApprox><<<grid, kSkBlock, 0, stream>>>(In{d_M}, d_T, N, iters);
    else
        sk_fwd_kernel<false, In, kApprox><<<grid, kSkBlock, 0, stream>>>(In{d_M}, d_T, N, iters);
    return static_cast<int>(cudaGetLastError());
}

template <bool kLogits>
static int sk_backward(const float* d_G, const float* d_M, float* d_D, int64_t N, int num_iters,
                       cudaStream_t stream)
{
    if (N < 0 || (N > 0 && (!d_G || !d_M || !d_D))) return MHC_ERR_INVALID_VALUE;
    if (num_iters > MHC_SK_BACKWARD_MAX_ITERS) return MHC_ERR_ITERS;
    if (N == 0) return MHC_OK;
    const bool vec = aligned16(d_G) && aligned16(d_M) && aligned16(d_D);
    dispatch_sk_bwd<kLogits>(num_iters > 0 ? num_iters : 0, vec, d_G, d_M, d_D, N, stream,
                             std::make_integer_sequence<int, MHC_SK_BACKWARD_MAX_ITERS + 1>{});
    return static_cast<int>(cudaGetLastError());
}

template <int kIters>
static void launch_sk_hres_bwd(bool vec, const float* G, const HResInput& in, float* dh, int64_t dh_stride,
                               float* drms, float* partials, int64_t grid, int64_t N, cudaStream_t stream)
{
    if (vec)
        sk_hres_bwd_kernel<kIters, true><<<grid, kSkBlock, 0, stream>>>(G, in, dh, dh_stride, drms, partials, N);
    else
        sk_hres_bwd_kernel<kIters, false><<<grid, kSkBlock, 0, stream>>>(G, in, dh, dh_stride, drms, partials, N);
}

template <int... Is>
static void dispatch_sk_hres_bwd(int iters, bool vec, const float* G, const HResInput& in, float* dh,
                                 int64_t dh_stride, float* drms, float* partials, int64_t grid, int64_t N,
                                 cudaStream_t stream, std::integer_sequence<int, Is...>)
{
    ((iters == Is ? launch_sk_hres_bwd<Is>(vec, G, in, dh, dh_stride, drms, partials, grid, N, stream) : void()),
     ...);
}

}  // namespace mhcp

using namespace mhcp;

extern "C" int mhc_sinkhorn_knopp_n4(const float* d_M, float* d_T, int64_t N, int num_iters, cudaStream_t stream)
{
    return sk_forward<false>(d_M, d_T, N, num_iters, stream);
}

extern "C" int mhc_sinkhorn_knopp_n4_backward(const float* d_G, const float* d_M, float* d_D, int64_t N,
                                              int num_iters, cudaStream_t stream)
{
    return sk_backward<false>(d_G, d_M, d_D, N, num_iters, stream);
}

extern "C" int mhc_sinkhorn_knopp_n4_logits(const float* d_R, float* d_T, int64_t N, int num_iters,
                                            cudaStream_t stream)
{
    return sk_forward<true>(d_R, d_T, N, num_iters, stream);
}

extern "C" int mhc_sinkhorn_knopp_n4_logits_ex(const float* d_R, float* d_T, int64_t N, int num_iters, int flags,
                                               cudaStream_t stream)
{
    if (flags & ~MHC_SK_HW_RECIPROCAL) return MHC_ERR_INVALID_VALUE;
    return (flags & MHC_SK_HW_RECIPROCAL) ? sk_forward<true, true>(d_R, d_T, N, num_iters, stream)
                                          : sk_forward<true>(d_R, d_T, N, num_iters, stream);
}

extern "C" int mhc_sinkhorn_knopp_n4_logits_backward(const float* d_G, const float* d_R, float* d_D, int64_t N,
                                                     int num_iters, cudaStream_t stream)
{
    return sk_backward<true>(d_G, d_R, d_D, N, num_iters, stream);
}

extern "C" int mhc_sinkhorn_knopp_n4_hres(const float* d_h, int64_t h_stride, const float* d_rms,
                                         const float* d_alpha, const float* d_b, float* d_T, int64_t N,
                                         int num_iters, cudaStream_t stream)
{
    if (N < 0 || h_stride < 0 || (N > 0 && (!d_h || !d_rms || !d_alpha || !d_b || !d_T)))
        return MHC_ERR_INVALID_VALUE;
    if (N == 0) return MHC_OK;
    const int iters = num_iters > 0 ? num_iters : 0;
    const int64_t grid = ceil_div(N, kSkBlock);
    const HResInput in{d_h, h_stride, d_rms, d_alpha, d_b};
    if (aligned16(d_h, h_stride, 4) && aligned16(d_T))
        sk_fwd_kernel<true, HResInput><<<grid, kSkBlock, 0, stream>>>(in, d_T, N, iters);
    else
        sk_fwd_kernel<false, HResInput><<<grid, kSkBlock, 0, stream>>>(in, d_T, N, iters);
    return static_cast<int>(cudaGetLastError());
}

extern "C" int mhc_sinkhorn_knopp_n4_hres_backward_workspace(int64_t N, int64_t* bytes)
{
    if (N < 0 || !bytes) return MHC_ERR_INVALID_VALUE;
    *bytes = max(ceil_div(N, kSkBlock), int64_t{1}) * kHResPartials * static_cast<int64_t>(sizeof(float));
    return MHC_OK;
}

extern "C" int mhc_sinkhorn_knopp_n4_hres_backward(const float* d_G, const float* d_h, int64_t h_stride,
                                                  const float* d_rms, const float* d_alpha, const float* d_b,
                                                  float* d_dh, int64_t dh_stride, float* d_drms, float* d_dalpha,
                                                  float* d_db, int64_t N, int num_iters, void* d_workspace,
                                                  int64_t workspace_bytes, cudaStream_t stream)
{
    if (N < 0 || h_stride < 0 || dh_stride < 0 || !d_dalpha || !d_db ||
        (N > 0 && (!d_G || !d_h || !d_rms || !d_alpha || !d_b || !d_dh || !d_drms || !d_workspace)))
        return MHC_ERR_INVALID_VALUE;
    if (num_iters > MHC_SK_BACKWARD_MAX_ITERS) return MHC_ERR_ITERS;
    const int64_t grid = ceil_div(N, kSkBlock);
    if (workspace_bytes < grid * kHResPartials * static_cast<int64_t>(sizeof(float))) return MHC_ERR_INVALID_VALUE;
    float* partials = static_cast<float*>(d_workspace);
    if (N > 0) {
        const HResInput in{d_h, h_stride, d_rms, d_alpha, d_b};
        const bool vec = aligned16(d_G) && aligned16(d_h, h_stride, 4) && aligned16(d_dh, dh_stride, 4);
        dispatch_sk_hres_bwd(num_iters > 0 ? num_iters : 0, vec, d_G, in, d_dh, dh_stride, d_drms, partials, grid, N,
                             stream, std::make_integer_sequence<int, MHC_SK_BACKWARD_MAX_ITERS + 1>{});
    }
    partial_sums_fold_kernel<kHResPartials><<<1, 32 * kHResPartials, 0, stream>>>(partials, grid, d_db, d_dalpha);
    return static_cast<int>(cudaGetLastError());
}
