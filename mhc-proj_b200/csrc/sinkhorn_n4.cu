// Kernels and C-ABI launchers for the fixed-iteration Sinkhorn-Knopp pair, on
// M = exp(R) as the reference takes it, or fused with the exponential on the
// logits R.
//
// This file is built without --use_fast_math (with -ftz=true): the
// Sinkhorn-Knopp arithmetic uses explicit round-to-nearest intrinsics and a
// correctly rounded reciprocal, which that flag does not change, and expf in
// the fused kernels is then the accurate one, the same function PyTorch's
// exp kernel calls, so fused and unfused paths agree.
#include <utility>

#include "sinkhorn_n4.cuh"
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

// kLogits: the input is R and the kernel forms M = exp(R) itself.
template <bool kVec, bool kLogits>
__global__ void __launch_bounds__(kSkBlock) sk_fwd_kernel(const float* __restrict__ M, float* __restrict__ T,
                                                          int64_t N, int iters)
{
    const int64_t idx = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (idx >= N) return;
    Mat4 x0;
    load_mat<kVec>(M, idx, x0);
    if constexpr (kLogits) exp_inplace(x0);
    Pairs x = to_pairs(x0);
#pragma unroll 1
    for (int it = 0; it < iters; ++it) sk_iteration(x, kSkEps, nullptr, nullptr, nullptr);
    store_mat<kVec>(T, idx, from_pairs(x));
}

// Backward with a compile-time iteration count.  Segment starts are kept in
// shared memory, [segment][element][thread] so that a warp's accesses fall in
// distinct banks; each segment is then replayed in registers and reversed.
// kLogits: the input is R; M = exp(R) is formed here and the result is the
// gradient with respect to R, dL/dM * M.
template <int kIters, bool kVec, bool kLogits>
__global__ void __launch_bounds__(kSkBlock) sk_bwd_kernel(const float* __restrict__ G,
                                                          const float* __restrict__ M,
                                                          float* __restrict__ D, int64_t N)
{
    constexpr int kNumSeg = (kIters + kSkSeg - 1) / kSkSeg;
    __shared__ float2 ckpt[kNumSeg > 0 ? kNumSeg : 1][8][kSkBlock];
    const int64_t idx = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (idx >= N) return;
    const int tid = threadIdx.x;

    Mat4 x0;
    load_mat<kVec>(M, idx, x0);
    if constexpr (kLogits) exp_inplace(x0);
    Pairs x = to_pairs(x0);
#pragma unroll
    for (int s = 0; s < kNumSeg; ++s) {
#pragma unroll
        for (int q = 0; q < 8; ++q) ckpt[s][q][tid] = x.p[q];
        if (s + 1 < kNumSeg) {
#pragma unroll
            for (int k = 0; k < kSkSeg; ++k) sk_iteration(x, kSkEps, nullptr, nullptr, nullptr);
        }
    }

    Mat4 g0;
    load_mat<kVec>(G, idx, g0);
    Pairs dy = to_pairs(g0);
#pragma unroll
    for (int s = kNumSeg - 1; s >= 0; --s) {
        constexpr int kFull = kSkSeg;
        const int len = (s == kNumSeg - 1) ? (kIters - s * kSkSeg) : kFull;
        Pairs xr[kSkSeg];
        float ri[kSkSeg][4], ci[kSkSeg][4];
#pragma unroll
        for (int q = 0; q < 8; ++q) x.p[q] = ckpt[s][q][tid];
#pragma unroll
        for (int k = 0; k < kSkSeg; ++k)
            if (k < len) sk_iteration(x, kSkEps, &xr[k], ri[k], ci[k]);
#pragma unroll
        for (int k = kSkSeg - 1; k >= 0; --k)
            if (k < len) sk_iteration_vjp(dy, xr[k], ri[k], ci[k]);
    }
    if constexpr (kLogits) {
        Mat4 m;
        load_mat<kVec>(M, idx, m);
        exp_inplace(m);
        const Pairs mp = to_pairs(m);
#pragma unroll
        for (int q = 0; q < 8; ++q) dy.p[q] = __fmul2_rn(dy.p[q], mp.p[q]);
    }
    store_mat<kVec>(D, idx, from_pairs(dy));
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

template <bool kLogits>
static int sk_forward(const float* d_M, float* d_T, int64_t N, int num_iters, cudaStream_t stream)
{
    if (N < 0 || (N > 0 && (!d_M || !d_T))) return MHC_ERR_INVALID_VALUE;
    if (N == 0) return MHC_OK;
    const int iters = num_iters > 0 ? num_iters : 0;
    const int64_t grid = ceil_div(N, kSkBlock);
    if (aligned16(d_M) && aligned16(d_T))
        sk_fwd_kernel<true, kLogits><<<grid, kSkBlock, 0, stream>>>(d_M, d_T, N, iters);
    else
        sk_fwd_kernel<false, kLogits><<<grid, kSkBlock, 0, stream>>>(d_M, d_T, N, iters);
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

extern "C" int mhc_sinkhorn_knopp_n4_logits_backward(const float* d_G, const float* d_R, float* d_D, int64_t N,
                                                     int num_iters, cudaStream_t stream)
{
    return sk_backward<true>(d_G, d_R, d_D, N, num_iters, stream);
}
