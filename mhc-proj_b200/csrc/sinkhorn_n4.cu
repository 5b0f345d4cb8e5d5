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

// A batch of any storage type at any batch stride: matrix idx of X starts at
// element idx * stride (its 16 entries row-major and contiguous).  kExp: X is
// the logits and M = exp(X) with the accurate expf rounded to Elem -- what
// torch.exp computes in that type (the reference's MHCSinkhornN4Function,
// mhc_proj/module.py:50) -- else M = X.  bf16 and fp16 widen exactly.
template <class Elem, bool kExp>
struct TypedInput {
    const Elem* X;
    int64_t stride;
    template <bool kVec>
    __device__ __forceinline__ void load(int64_t idx, Mat4& x) const
    {
        load_elems<Elem, kVec>(X, idx * stride, x);
        if constexpr (kExp) {
#pragma unroll
            for (int e = 0; e < 16; ++e) x.m[e] = to_f32(from_f32<Elem>(expf(x.m[e])));
        }
    }
};

// kApprox: the factors from the hardware reciprocal (sk_inv_approx) instead
// of the correctly rounded one.  TOut: the storage type of T (contiguous;
// round-to-nearest-even from fp32, as torch's .to()).
template <bool kVec, class In, bool kApprox = false, class TOut = float>
__global__ void __launch_bounds__(kSkBlock) sk_fwd_kernel(In in, TOut* __restrict__ T, int64_t N, int iters)
{
    const int64_t idx = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (idx >= N) return;
    Mat4 x0;
    in.template load<kVec>(idx, x0);
    Pairs x = to_pairs(x0);
#pragma unroll 1
    for (int it = 0; it < iters; ++it) sk_iteration<kApprox>(x, kSkEps);
    store_elems<TOut, kVec>(T, idx * 16, from_pairs(x));
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
        pot_forward<kSkBlock>(m, kSkEps, vh, threadIdx.x, kIters, mr, u, v);
        load_mat<kVec>(G, idx, g0);
        pot_reverse<kSkBlock>(m, to_pairs(g0), vh, threadIdx.x, kIters, mr, u, v, d);
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

// The backward on batches of any storage types at any batch strides, the
// iteration count at run time (1..kSkMaxIters; 0 gives D = G): G of type GE,
// X of type XE (M, or with kLogits the logits R and M = exp(R) rounded to XE
// as TypedInput forms it), D contiguous in GE.  The results are those of the
// reference's wrappers and module on such tensors: D = dL/dM rounded to GE
// (solvers_torch.cpp's D.to(G.dtype)), and with kLogits that rounded D times
// M rounded to GE again (mhc_proj/module.py:70, D * expon in the tensors'
// type).
template <bool kVec, class GE, class XE, bool kLogits>
__global__ void __launch_bounds__(kSkBlock) sk_bwd_typed_kernel(const GE* __restrict__ G, int64_t g_stride,
                                                                TypedInput<XE, kLogits> in, GE* __restrict__ D,
                                                                int64_t N, int iters)
{
    __shared__ float4 vh[kSkMaxIters][kSkBlock];
    const int64_t idx = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (idx >= N) return;
    Mat4 x0, g0;
    in.template load<kVec>(idx, x0);
    const Pairs m = to_pairs(x0);
    Mat4 out;
    if (iters > 0) {
        bool mr[4];
        float u[4], v[4];
        Pairs d;
        pot_forward<kSkBlock>(m, kSkEps, vh, threadIdx.x, iters, mr, u, v);
        load_elems<GE, kVec>(G, idx * g_stride, g0);
        pot_reverse<kSkBlock>(m, to_pairs(g0), vh, threadIdx.x, iters, mr, u, v, d);
        out = from_pairs(d);
    } else {
        load_elems<GE, kVec>(G, idx * g_stride, out);
    }
    if constexpr (kLogits) {
#pragma unroll
        for (int e = 0; e < 16; ++e) out.m[e] = __fmul_rn(to_f32(from_f32<GE>(out.m[e])), x0.m[e]);
    }
    store_elems<GE, kVec>(D, idx * 16, out);
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
            pot_forward<kSkBlock>(mp, kSkEps, vh, threadIdx.x, kIters, mr, u, v);
            pot_reverse<kSkBlock>(mp, to_pairs(g0), vh, threadIdx.x, kIters, mr, u, v, d);
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

static bool sk_valid_dtype(int dt) { return dt == MHC_DTYPE_F32 || dt == MHC_DTYPE_BF16 || dt == MHC_DTYPE_F16; }

template <class Elem, bool kLogits, bool kApprox>
static void sk_forward_typed(const void* X, int64_t x_stride, void* T, int64_t N, int iters, cudaStream_t stream)
{
    using In = TypedInput<Elem, kLogits>;
    const In in{static_cast<const Elem*>(X), x_stride};
    Elem* t = static_cast<Elem*>(T);
    const int64_t grid = ceil_div(N, kSkBlock);
    if (aligned16(X, x_stride, sizeof(Elem)) && aligned16(T))
        sk_fwd_kernel<true, In, kApprox, Elem><<<grid, kSkBlock, 0, stream>>>(in, t, N, iters);
    else
        sk_fwd_kernel<false, In, kApprox, Elem><<<grid, kSkBlock, 0, stream>>>(in, t, N, iters);
}

template <class Elem>
static void sk_forward_typed(const void* X, int64_t x_stride, void* T, int64_t N, int iters, int flags,
                             cudaStream_t stream)
{
    const bool logits = flags & MHC_SK_LOGITS, approx = flags & MHC_SK_HW_RECIPROCAL;
    if (logits)
        approx ? sk_forward_typed<Elem, true, true>(X, x_stride, T, N, iters, stream)
               : sk_forward_typed<Elem, true, false>(X, x_stride, T, N, iters, stream);
    else
        approx ? sk_forward_typed<Elem, false, true>(X, x_stride, T, N, iters, stream)
               : sk_forward_typed<Elem, false, false>(X, x_stride, T, N, iters, stream);
}

template <class GE, class XE, bool kLogits>
static void sk_backward_typed(const void* G, int64_t g_stride, const void* X, int64_t x_stride, void* D, int64_t N,
                              int iters, cudaStream_t stream)
{
    const TypedInput<XE, kLogits> in{static_cast<const XE*>(X), x_stride};
    const GE* g = static_cast<const GE*>(G);
    GE* d = static_cast<GE*>(D);
    const int64_t grid = ceil_div(N, kSkBlock);
    if (aligned16(G, g_stride, sizeof(GE)) && aligned16(X, x_stride, sizeof(XE)) && aligned16(D))
        sk_bwd_typed_kernel<true, GE, XE, kLogits><<<grid, kSkBlock, 0, stream>>>(g, g_stride, in, d, N, iters);
    else
        sk_bwd_typed_kernel<false, GE, XE, kLogits><<<grid, kSkBlock, 0, stream>>>(g, g_stride, in, d, N, iters);
}

template <class GE, bool kLogits>
static void sk_backward_typed(const void* G, int64_t g_stride, const void* X, int64_t x_stride, int x_dtype,
                              void* D, int64_t N, int iters, cudaStream_t stream)
{
    switch (x_dtype) {
        case MHC_DTYPE_BF16:
            return sk_backward_typed<GE, __nv_bfloat16, kLogits>(G, g_stride, X, x_stride, D, N, iters, stream);
        case MHC_DTYPE_F16: return sk_backward_typed<GE, __half, kLogits>(G, g_stride, X, x_stride, D, N, iters, stream);
        default: return sk_backward_typed<GE, float, kLogits>(G, g_stride, X, x_stride, D, N, iters, stream);
    }
}

template <bool kLogits>
static void sk_backward_typed(const void* G, int64_t g_stride, int g_dtype, const void* X, int64_t x_stride,
                              int x_dtype, void* D, int64_t N, int iters, cudaStream_t stream)
{
    switch (g_dtype) {
        case MHC_DTYPE_BF16:
            return sk_backward_typed<__nv_bfloat16, kLogits>(G, g_stride, X, x_stride, x_dtype, D, N, iters, stream);
        case MHC_DTYPE_F16:
            return sk_backward_typed<__half, kLogits>(G, g_stride, X, x_stride, x_dtype, D, N, iters, stream);
        default: return sk_backward_typed<float, kLogits>(G, g_stride, X, x_stride, x_dtype, D, N, iters, stream);
    }
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

extern "C" int mhc_sinkhorn_knopp_n4_strided(const void* d_X, int64_t x_stride, void* d_T, int dtype, int64_t N,
                                             int num_iters, int flags, cudaStream_t stream)
{
    if (N < 0 || x_stride < 0 || !sk_valid_dtype(dtype) || (flags & ~(MHC_SK_HW_RECIPROCAL | MHC_SK_LOGITS)) ||
        (N > 0 && (!d_X || !d_T)))
        return MHC_ERR_INVALID_VALUE;
    if (N == 0) return MHC_OK;
    const int iters = num_iters > 0 ? num_iters : 0;
    switch (dtype) {
        case MHC_DTYPE_BF16: sk_forward_typed<__nv_bfloat16>(d_X, x_stride, d_T, N, iters, flags, stream); break;
        case MHC_DTYPE_F16: sk_forward_typed<__half>(d_X, x_stride, d_T, N, iters, flags, stream); break;
        default:
            if (x_stride == 16)  // the contiguous fp32 kernels
                return (flags & MHC_SK_LOGITS)
                           ? mhc_sinkhorn_knopp_n4_logits_ex(static_cast<const float*>(d_X), static_cast<float*>(d_T),
                                                             N, num_iters, flags & MHC_SK_HW_RECIPROCAL, stream)
                           : ((flags & MHC_SK_HW_RECIPROCAL)
                                  ? sk_forward<false, true>(static_cast<const float*>(d_X), static_cast<float*>(d_T),
                                                            N, num_iters, stream)
                                  : sk_forward<false>(static_cast<const float*>(d_X), static_cast<float*>(d_T), N,
                                                      num_iters, stream));
            sk_forward_typed<float>(d_X, x_stride, d_T, N, iters, flags, stream);
    }
    return static_cast<int>(cudaGetLastError());
}

extern "C" int mhc_sinkhorn_knopp_n4_backward_strided(const void* d_G, int64_t g_stride, int g_dtype, const void* d_X,
                                                      int64_t x_stride, int x_dtype, void* d_D, int64_t N,
                                                      int num_iters, int flags, cudaStream_t stream)
{
    if (N < 0 || g_stride < 0 || x_stride < 0 || !sk_valid_dtype(g_dtype) || !sk_valid_dtype(x_dtype) ||
        (flags & ~MHC_SK_LOGITS) || (N > 0 && (!d_G || !d_X || !d_D)))
        return MHC_ERR_INVALID_VALUE;
    if (num_iters > MHC_SK_BACKWARD_MAX_ITERS) return MHC_ERR_ITERS;
    if (N == 0) return MHC_OK;
    const bool logits = flags & MHC_SK_LOGITS;
    if (g_dtype == MHC_DTYPE_F32 && x_dtype == MHC_DTYPE_F32 && g_stride == 16 && x_stride == 16)
        return logits ? sk_backward<true>(static_cast<const float*>(d_G), static_cast<const float*>(d_X),
                                          static_cast<float*>(d_D), N, num_iters, stream)
                      : sk_backward<false>(static_cast<const float*>(d_G), static_cast<const float*>(d_X),
                                           static_cast<float*>(d_D), N, num_iters, stream);
    const int iters = num_iters > 0 ? num_iters : 0;
    if (logits)
        sk_backward_typed<true>(d_G, g_stride, g_dtype, d_X, x_stride, x_dtype, d_D, N, iters, stream);
    else
        sk_backward_typed<false>(d_G, g_stride, g_dtype, d_X, x_stride, x_dtype, d_D, N, iters, stream);
    return static_cast<int>(cudaGetLastError());
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
