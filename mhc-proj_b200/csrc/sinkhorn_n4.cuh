// Fixed-iteration Sinkhorn-Knopp on 4x4 matrices, one matrix per thread.
//
// Forward (the reference's sinkhorn_knopp_batched_n4_kernel,
// src/sinkhorn_knopp.cuh:831-912): `iters` times
//     r_i = rowsum,  x_i* *= (r_i > eps ? 1/r_i : 0)   (correctly rounded 1/r)
//     c_j = colsum,  x_*j *= (c_j > eps ? 1/c_j : 0)
// on M = exp(R), eps = 1e-8 (src/sinkhorn_knopp_n4.cu:10).
//
// Backward: the exact vector-Jacobian product of that forward with respect to
// M.  Per iteration, with x the row-normalised matrix, rinv/cinv the factors
// and dy the incoming gradient:
//     column step  dx_ij = (dy_ij - cinv_j * sum_k dy_kj x_kj) * cinv_j
//     row step     dz_ij = (dx_ij - sum_l dx_il x_il) * rinv_i
// (The reference's kernel, :1182-1201, subtracts r*rinv in the row step
// instead of r; that is not the derivative of the forward.)
//
// The backward keeps the iteration count at compile time and recomputes the
// forward in segments of kSkSeg iterations from checkpoints held in shared
// memory, so no per-iteration history goes to local memory.
#pragma once

#include "mhc_common.cuh"

namespace mhcp {

constexpr int kSkMaxIters = 20;  // the reference's backward limit, sinkhorn_knopp.cuh:1213
constexpr int kSkSeg = 4;

__device__ __forceinline__ float sk_inv(float s, float eps) { return (s > eps) ? __frcp_rn(s) : 0.0f; }

// One row step then one column step, in place.  Saves the row-normalised
// matrix and both factor vectors when the pointers are non-null.
// Every product and sum is rounded on its own and sums run left to right, as
// in the reference's compiled kernel (there the row-scaled values also feed
// the column scaling, so their multiplies are not contracted into the column
// sums); with the correctly rounded reciprocal the result is the reference's
// bit for bit.
__device__ __forceinline__ void sk_iteration(float x[16], float eps, float* xr_out, float* rinv_out,
                                             float* cinv_out)
{
    float ri[4], ci[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const float s = __fadd_rn(__fadd_rn(__fadd_rn(x[4 * i], x[4 * i + 1]), x[4 * i + 2]), x[4 * i + 3]);
        ri[i] = sk_inv(s, eps);
    }
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) x[4 * i + j] = __fmul_rn(x[4 * i + j], ri[i]);
    if (xr_out) {
#pragma unroll
        for (int e = 0; e < 16; ++e) xr_out[e] = x[e];
    }
#pragma unroll
    for (int j = 0; j < 4; ++j)
        ci[j] = sk_inv(__fadd_rn(__fadd_rn(__fadd_rn(x[j], x[4 + j]), x[8 + j]), x[12 + j]), eps);
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) x[4 * i + j] = __fmul_rn(x[4 * i + j], ci[j]);
    if (rinv_out) {
#pragma unroll
        for (int i = 0; i < 4; ++i) rinv_out[i] = ri[i];
    }
    if (cinv_out) {
#pragma unroll
        for (int j = 0; j < 4; ++j) cinv_out[j] = ci[j];
    }
}

// Reverse of one iteration.  dy holds d/dy on entry and d/dz on exit.
__device__ __forceinline__ void sk_iteration_vjp(float dy[16], const float xr[16], const float rinv[4],
                                                 const float cinv[4])
{
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        float cs = __fmul_rn(dy[j], xr[j]);
        cs = __fmaf_rn(dy[4 + j], xr[4 + j], cs);
        cs = __fmaf_rn(dy[8 + j], xr[8 + j], cs);
        cs = __fmaf_rn(dy[12 + j], xr[12 + j], cs);
#pragma unroll
        for (int i = 0; i < 4; ++i)
            dy[4 * i + j] = __fmul_rn(__fmaf_rn(-cs, cinv[j], dy[4 * i + j]), cinv[j]);
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        float rs = __fmul_rn(dy[4 * i], xr[4 * i]);
        rs = __fmaf_rn(dy[4 * i + 1], xr[4 * i + 1], rs);
        rs = __fmaf_rn(dy[4 * i + 2], xr[4 * i + 2], rs);
        rs = __fmaf_rn(dy[4 * i + 3], xr[4 * i + 3], rs);
#pragma unroll
        for (int j = 0; j < 4; ++j) dy[4 * i + j] = __fmul_rn(__fsub_rn(dy[4 * i + j], rs), rinv[i]);
    }
}

}  // namespace mhcp
