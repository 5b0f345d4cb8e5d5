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


// The correctly rounded reciprocal (round to nearest even, flush-to-zero) from
// the hardware approximation and one Newton step on a fused multiply-add, the
// correction of P. Markstein ("Computation of elementary functions on the IBM
// RISC System/6000 processor", IBM J. Res. Dev. 34(1), 1990): with r0 within
// an ulp of 1/x, the FMA forms e = 1 - x*r0 exactly and r0 + r0*e rounds to
// 1/x.  Where the approximation is exact or the step is undefined (x zero,
// subnormal -- flushed --, infinite or NaN, all giving a NaN e) r0 is the
// answer.  Equal to __frcp_rn for all 2^32 inputs (tests/test_reciprocal_gpu.py)
// in five instructions.
__device__ __forceinline__ float rcp_rn(float x)
{
    float r0;
    asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(r0) : "f"(x));
    const float e = __fmaf_rn(-x, r0, 1.0f);
    const float r1 = __fmaf_rn(r0, e, r0);
    return (e != e) ? r0 : r1;
}

// The Sinkhorn-Knopp factor: s > eps ? 1/s : 0 with the reciprocal correctly
// rounded.  For finite s > eps > 0, rcp_rn's guard never fires (e is finite),
// so the Newton step runs unguarded; s = +inf is clamped to FLT_MAX, whose
// approximate reciprocal flushes to zero and leaves e = 1, so the factor is
// 0 = 1/inf there.  Equal to (s > eps) ? __frcp_rn(s) : 0 for all 2^32 s at
// eps = 1e-8 (tests/test_reciprocal_gpu.py), in one instruction fewer.
__device__ __forceinline__ float sk_inv(float s, float eps)
{
    const float x = fminf(s, 3.40282347e38f);
    float r0;
    asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(r0) : "f"(x));
    const float e = __fmaf_rn(-x, r0, 1.0f);
    return (s > eps) ? __fmaf_rn(r0, e, r0) : 0.0f;
}

// The same factor from the hardware reciprocal (rcp.approx.ftz: at most one
// ulp from 1/s, against the half ulp of __frcp_rn) -- for the backward's
// replay of the forward, which must be close to the forward, not equal to it.
__device__ __forceinline__ float sk_inv_approx(float s, float eps)
{
    float r;
    asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(s));
    return (s > eps) ? r : 0.0f;
}

// A matrix as eight float2 pairs, two per row: P[2i] = (x_i0, x_i1),
// P[2i+1] = (x_i2, x_i3).  Column-wise work then runs on packed fp32x2
// arithmetic (two IEEE round-to-nearest operations per instruction on
// sm_100), so column sums, column scaling and the column step of the
// backward take half the instructions; row sums stay scalar, left to right.
struct Pairs {
    float2 p[8];
};

__device__ __forceinline__ float2 splat(float a) { return make_float2(a, a); }

__device__ __forceinline__ Pairs to_pairs(const Mat4& x)
{
    Pairs r;
#pragma unroll
    for (int q = 0; q < 8; ++q) r.p[q] = make_float2(x.m[2 * q], x.m[2 * q + 1]);
    return r;
}

__device__ __forceinline__ Mat4 from_pairs(const Pairs& r)
{
    Mat4 x;
#pragma unroll
    for (int q = 0; q < 8; ++q) {
        x.m[2 * q] = r.p[q].x;
        x.m[2 * q + 1] = r.p[q].y;
    }
    return x;
}

// One row step then one column step, in place.  Saves the row-normalised
// matrix and both factor vectors when the pointers are non-null.
// Every product and sum is rounded on its own and sums run left to right, as
// in the reference's compiled kernel (there the row-scaled values also feed
// the column scaling, so their multiplies are not contracted into the column
// sums); with the correctly rounded reciprocal the result is the reference's
// bit for bit.
template <bool kApprox = false>
__device__ __forceinline__ void sk_iteration(Pairs& x, float eps, Pairs* xr_out, float* rinv_out,
                                             float* cinv_out)
{
    auto inv = [eps](float v) { return kApprox ? sk_inv_approx(v, eps) : sk_inv(v, eps); };
    float ri[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const float2 a = x.p[2 * i], b = x.p[2 * i + 1];
        ri[i] = inv(__fadd_rn(__fadd_rn(__fadd_rn(a.x, a.y), b.x), b.y));
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        x.p[2 * i] = __fmul2_rn(x.p[2 * i], splat(ri[i]));
        x.p[2 * i + 1] = __fmul2_rn(x.p[2 * i + 1], splat(ri[i]));
    }
    if (xr_out) *xr_out = x;
    // column sums ((x_0j + x_1j) + x_2j) + x_3j, two columns per instruction
    const float2 c01 = __fadd2_rn(__fadd2_rn(__fadd2_rn(x.p[0], x.p[2]), x.p[4]), x.p[6]);
    const float2 c23 = __fadd2_rn(__fadd2_rn(__fadd2_rn(x.p[1], x.p[3]), x.p[5]), x.p[7]);
    const float2 ci01 = make_float2(inv(c01.x), inv(c01.y));
    const float2 ci23 = make_float2(inv(c23.x), inv(c23.y));
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        x.p[2 * i] = __fmul2_rn(x.p[2 * i], ci01);
        x.p[2 * i + 1] = __fmul2_rn(x.p[2 * i + 1], ci23);
    }
    if (rinv_out) {
#pragma unroll
        for (int i = 0; i < 4; ++i) rinv_out[i] = ri[i];
    }
    if (cinv_out) {
        cinv_out[0] = ci01.x;
        cinv_out[1] = ci01.y;
        cinv_out[2] = ci23.x;
        cinv_out[3] = ci23.y;
    }
}

// Reverse of one iteration.  dy holds d/dy on entry and d/dz on exit.
//   column step  dx_ij = (dy_ij - cs_j cinv_j) cinv_j,  cs_j = sum_k dy_kj x_kj
//                (an FMA chain over k = 0..3), formed as
//                fma(dy_ij, cinv_j, -((cs_j cinv_j) cinv_j)): one packed FMA
//                per pair of entries instead of an FMA and a multiply
//   row step     dz_ij = (dx_ij - rs_i) rinv_i,  rs_i = sum_l dx_il x_il
//                (an FMA chain over l = 0..3), formed as
//                fma(dx_ij, rinv_i, -(rs_i rinv_i))
__device__ __forceinline__ void sk_iteration_vjp(Pairs& dy, const Pairs& xr, const float rinv[4],
                                                 const float cinv[4])
{
#pragma unroll
    for (int h = 0; h < 2; ++h) {  // column pairs (0,1) and (2,3)
        float2 cs = __fmul2_rn(dy.p[h], xr.p[h]);
        cs = __ffma2_rn(dy.p[2 + h], xr.p[2 + h], cs);
        cs = __ffma2_rn(dy.p[4 + h], xr.p[4 + h], cs);
        cs = __ffma2_rn(dy.p[6 + h], xr.p[6 + h], cs);
        const float2 ci = make_float2(cinv[2 * h], cinv[2 * h + 1]);
        const float2 t = __fmul2_rn(__fmul2_rn(cs, ci), ci);
        const float2 nt = make_float2(-t.x, -t.y);
#pragma unroll
        for (int i = 0; i < 4; ++i) dy.p[2 * i + h] = __ffma2_rn(dy.p[2 * i + h], ci, nt);
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const float2 a = dy.p[2 * i], b = dy.p[2 * i + 1];
        const float2 u = xr.p[2 * i], w = xr.p[2 * i + 1];
        float rs = __fmul_rn(a.x, u.x);
        rs = __fmaf_rn(a.y, u.y, rs);
        rs = __fmaf_rn(b.x, w.x, rs);
        rs = __fmaf_rn(b.y, w.y, rs);
        const float2 nt = splat(-__fmul_rn(rs, rinv[i]));
        dy.p[2 * i] = __ffma2_rn(a, splat(rinv[i]), nt);
        dy.p[2 * i + 1] = __ffma2_rn(b, splat(rinv[i]), nt);
    }
}

}  // namespace mhcp
