// Fixed-iteration Sinkhorn-Knopp on 4x4 matrices, one matrix per thread.
//
// Forward (the reference's sinkhorn_knopp_batched_n4_kernel,
// src/sinkhorn_knopp.cuh:831-912): `iters` times
//     r_i = rowsum,  x_i* *= (r_i > eps ? 1/r_i : 0)   (correctly rounded 1/r)
//     c_j = colsum,  x_*j *= (c_j > eps ? 1/c_j : 0)
// on M = exp(R), eps = 1e-8 (src/sinkhorn_knopp_n4.cu:10).
//
// Backward: the exact vector-Jacobian product of that forward with respect to
// M, formed from the forward's potentials (below, "the backward in potential
// form").  The reference's kernel (:1146-1202) differentiates the row step as
// (dx - r*rinv)*rinv; that is not the derivative of the forward.
#pragma once

#include "mhc_common.cuh"

namespace mhcp {

constexpr int kSkMaxIters = 20;  // the reference's backward limit, sinkhorn_knopp.cuh:1213


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
// ulp from 1/s, against the half ulp of __frcp_rn), for the opt-in forward
// that need not reproduce the reference's bits.
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

// One row step then one column step, in place.
// Every product and sum is rounded on its own and sums run left to right, as
// in the reference's compiled kernel (there the row-scaled values also feed
// the column scaling, so their multiplies are not contracted into the column
// sums); with the correctly rounded reciprocal the result is the reference's
// bit for bit.
template <bool kApprox = false>
__device__ __forceinline__ void sk_iteration(Pairs& x, float eps)
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
}

// ---- the backward in potential form -----------------------------------------
//
// After k iterations the forward holds diag(u_k) M diag(v_k), where
//     u_k = 1 / (M v_{k-1}),   v_k = 1 / (M^T u_k),   v_0 = 1
// (iteration k's row factors are u_k / u_{k-1}, its column factors
// v_k / v_{k-1}).  The vector-Jacobian product of T = diag(u_K) M diag(v_K)
// with respect to M therefore needs only M and the potentials: with
// G = dL/dT,
//     du = (G o M) v_K,   dv = (G o M)^T u_K,   dM = G o u_K v_K^T,
// then for k = K .. 1
//     dt = -dv o v_k o v_k,    du += M dt,       dM += u_k dt^T,
//     ds = -du o u_k o u_k,    dv  = M^T ds,     dM += ds v_{k-1}^T,   du = 0.
// It is the gradient of the same function as the sequential row/column form
// (sinkhorn_knopp.cuh:851-906), without the per-iteration row-normalised
// matrices: the backward keeps v_1 .. v_K (16 bytes per iteration) and forms
// u_k again from v_{k-1}, by the same operations and hence to the same bits.
//
// eps: in the sequential form a row or column whose sum is at most eps gets a
// zero factor and stays zero.  Only the first iteration can produce one: after
// a column step every entry is at most 1, so a row sum is at most 4 and every
// row factor at least 1/4, which leaves every nonzero column summing to at
// least 1/4; after a row step every entry is at most 1, so every column
// factor is at least 1/4, and a nonzero row keeps at least (1 - 4 eps) / 4 of
// its sum outside the zeroed columns.  So the first iteration's masks (the row
// sums of M, then the column sums after its row step) are those of every
// iteration, and a zero potential zeroes its gradient terms (u_k = 0 gives
// ds = 0) as a zero factor does.

// s_i = ((M_i0 v_0 + M_i1 v_1) + M_i2 v_2) + M_i3 v_3: a multiply and three
// FMAs per row; with v = 1 it is the row sum in the forward's order.
__device__ __forceinline__ void pot_rows(const Pairs& M, const float v[4], float s[4])
{
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const float2 a = M.p[2 * i], b = M.p[2 * i + 1];
        float r = __fmul_rn(a.x, v[0]);
        r = __fmaf_rn(a.y, v[1], r);
        r = __fmaf_rn(b.x, v[2], r);
        s[i] = __fmaf_rn(b.y, v[3], r);
    }
}

// t_j = sum_i M_ij u_i over i = 0..3, column pairs on packed FMAs.
__device__ __forceinline__ void pot_cols(const Pairs& M, const float u[4], float t[4])
{
    float2 t01 = __fmul2_rn(M.p[0], splat(u[0]));
    float2 t23 = __fmul2_rn(M.p[1], splat(u[0]));
#pragma unroll
    for (int i = 1; i < 4; ++i) {
        t01 = __ffma2_rn(M.p[2 * i], splat(u[i]), t01);
        t23 = __ffma2_rn(M.p[2 * i + 1], splat(u[i]), t23);
    }
    t[0] = t01.x;
    t[1] = t01.y;
    t[2] = t23.x;
    t[3] = t23.y;
}

// keep ? 1/x : 0 with the hardware reciprocal (one ulp): the backward must be
// the gradient of the forward within tolerance, not its bits.
__device__ __forceinline__ float pot_inv(float x, bool keep)
{
    float r;
    asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(x));
    return keep ? r : 0.0f;
}

// The forward in potential form, iters >= 1 iterations (at most the rows of
// vh): the first iteration's row masks, u_K and v_K, and v_1 .. v_iters in
// vh[k - 1][tid].  (A compile-time count, as the fixed-count kernels pass,
// folds into the loops.)
template <int kBlock>
__device__ __forceinline__ void pot_forward(const Pairs& M, float eps, float4 (*vh)[kBlock], int tid, int iters,
                                            bool mr[4], float u[4], float v[4])
{
    float s[4], t[4];
    bool mc[4];
    const float one[4] = {1.0f, 1.0f, 1.0f, 1.0f};
    pot_rows(M, one, s);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        mr[i] = s[i] > eps;
        u[i] = pot_inv(s[i], mr[i]);
    }
    pot_cols(M, u, t);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        mc[j] = t[j] > eps;
        v[j] = pot_inv(t[j], mc[j]);
    }
    vh[0][tid] = make_float4(v[0], v[1], v[2], v[3]);
#pragma unroll 4
    for (int k = 1; k < iters; ++k) {
        pot_rows(M, v, s);
#pragma unroll
        for (int i = 0; i < 4; ++i) u[i] = pot_inv(s[i], mr[i]);
        pot_cols(M, u, t);
#pragma unroll
        for (int j = 0; j < 4; ++j) v[j] = pot_inv(t[j], mc[j]);
        vh[k][tid] = make_float4(v[0], v[1], v[2], v[3]);
    }
}

// dL/dM from G, given pot_forward's masks, u_K, v_K and history.
template <int kBlock>
__device__ __forceinline__ void pot_reverse(const Pairs& M, const Pairs& G, const float4 (*vh)[kBlock], int tid,
                                            int iters, const bool mr[4], const float uK[4], const float vK[4],
                                            Pairs& dM)
{
    float du[4], dv[4], v[4];
    {
        Pairs H;
#pragma unroll
        for (int q = 0; q < 8; ++q) H.p[q] = __fmul2_rn(G.p[q], M.p[q]);
        pot_rows(H, vK, du);
        pot_cols(H, uK, dv);
    }
    const float2 v01 = make_float2(vK[0], vK[1]), v23 = make_float2(vK[2], vK[3]);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        dM.p[2 * i] = __fmul2_rn(__fmul2_rn(G.p[2 * i], splat(uK[i])), v01);
        dM.p[2 * i + 1] = __fmul2_rn(__fmul2_rn(G.p[2 * i + 1], splat(uK[i])), v23);
    }
#pragma unroll
    for (int j = 0; j < 4; ++j) v[j] = vK[j];
#pragma unroll 2
    for (int k = iters; k >= 1; --k) {
        float vp[4], s[4], u[4], dt[4], ds[4];
        if (k >= 2) {
            const float4 w = vh[k - 2][tid];
            vp[0] = w.x;
            vp[1] = w.y;
            vp[2] = w.z;
            vp[3] = w.w;
        } else {
#pragma unroll
            for (int j = 0; j < 4; ++j) vp[j] = 1.0f;
        }
        pot_rows(M, vp, s);
#pragma unroll
        for (int i = 0; i < 4; ++i) u[i] = pot_inv(s[i], mr[i]);
        // v_k = 1 / (M^T u_k)
#pragma unroll
        for (int j = 0; j < 4; ++j) dt[j] = __fmul_rn(__fmul_rn(dv[j], v[j]), -v[j]);
        const float2 dt01 = make_float2(dt[0], dt[1]), dt23 = make_float2(dt[2], dt[3]);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const float2 a = M.p[2 * i], b = M.p[2 * i + 1];
            float r = __fmaf_rn(a.x, dt[0], du[i]);
            r = __fmaf_rn(a.y, dt[1], r);
            r = __fmaf_rn(b.x, dt[2], r);
            du[i] = __fmaf_rn(b.y, dt[3], r);
            dM.p[2 * i] = __ffma2_rn(splat(u[i]), dt01, dM.p[2 * i]);
            dM.p[2 * i + 1] = __ffma2_rn(splat(u[i]), dt23, dM.p[2 * i + 1]);
        }
        // u_k = 1 / (M v_{k-1})
#pragma unroll
        for (int i = 0; i < 4; ++i) ds[i] = __fmul_rn(__fmul_rn(du[i], u[i]), -u[i]);
        pot_cols(M, ds, dv);
        const float2 vp01 = make_float2(vp[0], vp[1]), vp23 = make_float2(vp[2], vp[3]);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            dM.p[2 * i] = __ffma2_rn(splat(ds[i]), vp01, dM.p[2 * i]);
            dM.p[2 * i + 1] = __ffma2_rn(splat(ds[i]), vp23, dM.p[2 * i + 1]);
            du[i] = 0.0f;
        }
#pragma unroll
        for (int j = 0; j < 4; ++j) v[j] = vp[j];
    }
}

}  // namespace mhcp
