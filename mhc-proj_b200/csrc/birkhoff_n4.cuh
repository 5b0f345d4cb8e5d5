// Dual-Newton KL projection of 4x4 matrices onto the Birkhoff polytope and its
// implicit-function-theorem backward, one matrix per thread.
//
// Algorithm (the reference's, src/birkhoff_proj_n4.cu):
//   T = diag(e^alpha) exp(R) diag(e^beta) with unit row and column sums.
//   The dual is minimised over beta in R^3 (beta_3 = 0) with alpha eliminated
//   in closed form as a row log-sum-exp, so every iterate has T = row-softmax
//   (beta + R) (rows sum to one) and the gradient is g = colsum(T) - 1.
//
// Mapping.  The reference spreads a matrix over 16 lanes and reduces with
// xor-butterfly shuffles.  Here one thread owns a whole matrix in registers,
// so reductions are register arithmetic with no shuffles, and a warp works on
// 32 matrices.  Every reduction is evaluated in the order the reference's
// butterflies produce, and the multiply-add rounding of the reference build
// is reproduced exactly by the Rounding policy below, so each iterate, each
// line-search decision and the returned T are the reference's, bit for bit.
#pragma once

#include "mhc_common.cuh"

namespace mhcp {

// birkhoff_proj_n4.cu:39-43 and the step list at :434.
constexpr int kNewtonMaxIters = 20;
constexpr int kLineSearchMaxIters = 5;
constexpr float kEpsilon = 1e-8f;

__device__ __forceinline__ float line_step(int k)
{
    // gamma in {1, 0.5, 0.1, 0.05, 0.01}, as selects (no jump table)
    return sel(k == 0, 1.0f, sel(k == 1, 0.5f, sel(k == 2, 0.1f, sel(k == 3, 0.05f, 0.01f))));
}

// ---------------------------------------------------------------------------
// Rounding policies.
//
// A butterfly sum of products p_r = a_r * b_r over r = 0..3 (partners
// (0,1),(2,3) first, then the pair sums) has one multiply feeding each of the
// first-level adds.  Compiled with contraction the lane that owns element r
// gets fma(a_r, b_r, round(a_{r^1} b_{r^1})) at the first level; the lane of
// element 0 (and 2) and the lane of element 1 (and 3) then hold different
// sums.  `prod_sum(view, ...)` returns what lane `view` (0 or 1) holds.
// `Fused` models a contracting build, `Plain` rounds every product.
// ---------------------------------------------------------------------------
struct FusedProducts {
    static __device__ __forceinline__ float prod_sum(int view, float a0, float b0, float a1, float b1,
                                                     float a2, float b2, float a3, float b3)
    {
        if (view == 0)
            return __fadd_rn(__fmaf_rn(a0, b0, __fmul_rn(a1, b1)), __fmaf_rn(a2, b2, __fmul_rn(a3, b3)));
        return __fadd_rn(__fmaf_rn(a1, b1, __fmul_rn(a0, b0)), __fmaf_rn(a3, b3, __fmul_rn(a2, b2)));
    }
};

struct PlainProducts {
    static __device__ __forceinline__ float prod_sum(int, float a0, float b0, float a1, float b1,
                                                     float a2, float b2, float a3, float b3)
    {
        return psum4(__fmul_rn(a0, b0), __fmul_rn(a1, b1), __fmul_rn(a2, b2), __fmul_rn(a3, b3));
    }
};

// Symmetric 3x3 determinant and adjugate-vector product.  H is given by its
// diagonal h00,h11,h22 and off-diagonals h01,h12,h02.  The expression trees
// are the reference's (birkhoff_proj_n4.cu:321-323 and :346-363); the
// policies differ only in which products are contracted.
struct Sym3 {
    float h00, h11, h22, h01, h12, h02;
};

// Contraction as the reference build forms it.  The compiler contracts a
// multiply into an add only when the product has no other use.  det is
// evaluated in the entry block and each adjugate row in its own per-column
// branch (birkhoff_proj_n4.cu:321-363), so:
//   - the cofactors A = h11 h22 - h12^2 and C = h01 h12 - h11 h02 are shared
//     whole by det and the branches and keep their contraction;
//   - the products of B = h01 h22 - h12 h02 also feed the branches'
//     (h02 h12 - h01 h22), so B and that cofactor round every product;
//   - cofactors local to one branch (E, F, K) and the final multiply-adds are
//     contracted.
template <bool kFusedB>
struct AdjRefT {
    static __device__ __forceinline__ float cofA(const Sym3& h) { return __fmaf_rn(h.h11, h.h22, -__fmul_rn(h.h12, h.h12)); }
    static __device__ __forceinline__ float cofC(const Sym3& h) { return __fmaf_rn(h.h01, h.h12, -__fmul_rn(h.h11, h.h02)); }
    static __device__ __forceinline__ float det(const Sym3& h)
    {
        const float A = cofA(h);
        const float B = kFusedB ? __fmaf_rn(h.h01, h.h22, -__fmul_rn(h.h12, h.h02))
                                : __fsub_rn(__fmul_rn(h.h01, h.h22), __fmul_rn(h.h12, h.h02));
        const float C = cofC(h);
        return __fmaf_rn(h.h02, C, __fmaf_rn(h.h00, A, -__fmul_rn(h.h01, B)));
    }
    static __device__ __forceinline__ void adj(const Sym3& h, float r0, float r1, float r2,
                                               float& y0, float& y1, float& y2)
    {
        const float A = cofA(h);
        const float C = cofC(h);
        const float Bq = __fsub_rn(__fmul_rn(h.h02, h.h12), __fmul_rn(h.h01, h.h22));
        const float E = __fmaf_rn(h.h00, h.h22, -__fmul_rn(h.h02, h.h02));
        const float F = __fmaf_rn(h.h01, h.h02, -__fmul_rn(h.h00, h.h12));
        const float K = __fmaf_rn(h.h00, h.h11, -__fmul_rn(h.h01, h.h01));
        y0 = __fmaf_rn(C, r2, __fmaf_rn(A, r0, __fmul_rn(Bq, r1)));
        y1 = __fmaf_rn(F, r2, __fmaf_rn(Bq, r0, __fmul_rn(E, r1)));
        y2 = __fmaf_rn(K, r2, __fmaf_rn(C, r0, __fmul_rn(F, r1)));
    }
};
using AdjRef = AdjRefT<false>;
using AdjBranchFused = AdjRefT<true>;

// Contraction of every cofactor, all in one block.
struct AdjSingleFused {
    static __device__ __forceinline__ float det(const Sym3& h) { return AdjBranchFused::det(h); }
    static __device__ __forceinline__ void adj(const Sym3& h, float r0, float r1, float r2,
                                               float& y0, float& y1, float& y2)
    {
        const float A = __fmaf_rn(h.h11, h.h22, -__fmul_rn(h.h12, h.h12));
        const float C = __fmaf_rn(h.h01, h.h12, -__fmul_rn(h.h11, h.h02));
        const float Bq = __fmaf_rn(h.h02, h.h12, -__fmul_rn(h.h01, h.h22));
        const float E = __fmaf_rn(h.h00, h.h22, -__fmul_rn(h.h02, h.h02));
        const float F = __fmaf_rn(h.h01, h.h02, -__fmul_rn(h.h00, h.h12));
        const float K = __fmaf_rn(h.h00, h.h11, -__fmul_rn(h.h01, h.h01));
        y0 = __fmaf_rn(C, r2, __fmaf_rn(A, r0, __fmul_rn(Bq, r1)));
        y1 = __fmaf_rn(F, r2, __fmaf_rn(Bq, r0, __fmul_rn(E, r1)));
        y2 = __fmaf_rn(K, r2, __fmaf_rn(C, r0, __fmul_rn(F, r1)));
    }
};

// No contraction.
struct AdjPlain {
    static __device__ __forceinline__ float det(const Sym3& h)
    {
        const float A = __fsub_rn(__fmul_rn(h.h11, h.h22), __fmul_rn(h.h12, h.h12));
        const float B = __fsub_rn(__fmul_rn(h.h01, h.h22), __fmul_rn(h.h12, h.h02));
        const float C = __fsub_rn(__fmul_rn(h.h01, h.h12), __fmul_rn(h.h11, h.h02));
        return __fadd_rn(__fsub_rn(__fmul_rn(h.h00, A), __fmul_rn(h.h01, B)), __fmul_rn(h.h02, C));
    }
    static __device__ __forceinline__ void adj(const Sym3& h, float r0, float r1, float r2,
                                               float& y0, float& y1, float& y2)
    {
        const float A = __fsub_rn(__fmul_rn(h.h11, h.h22), __fmul_rn(h.h12, h.h12));
        const float C = __fsub_rn(__fmul_rn(h.h01, h.h12), __fmul_rn(h.h11, h.h02));
        const float Bq = __fsub_rn(__fmul_rn(h.h02, h.h12), __fmul_rn(h.h01, h.h22));
        const float E = __fsub_rn(__fmul_rn(h.h00, h.h22), __fmul_rn(h.h02, h.h02));
        const float F = __fsub_rn(__fmul_rn(h.h01, h.h02), __fmul_rn(h.h00, h.h12));
        const float K = __fsub_rn(__fmul_rn(h.h00, h.h11), __fmul_rn(h.h01, h.h01));
        y0 = __fadd_rn(__fadd_rn(__fmul_rn(A, r0), __fmul_rn(Bq, r1)), __fmul_rn(C, r2));
        y1 = __fadd_rn(__fadd_rn(__fmul_rn(Bq, r0), __fmul_rn(E, r1)), __fmul_rn(F, r2));
        y2 = __fadd_rn(__fadd_rn(__fmul_rn(C, r0), __fmul_rn(F, r1)), __fmul_rn(K, r2));
    }
};

// Source-level expressions, contraction left to the compiler.
struct AdjSource {
    static __device__ __forceinline__ float det(const Sym3& h)
    {
        return h.h00 * (h.h11 * h.h22 - h.h12 * h.h12) - h.h01 * (h.h01 * h.h22 - h.h12 * h.h02) +
               h.h02 * (h.h01 * h.h12 - h.h11 * h.h02);
    }
    static __device__ __forceinline__ void adj(const Sym3& h, float r0, float r1, float r2,
                                               float& y0, float& y1, float& y2)
    {
        y0 = (h.h11 * h.h22 - h.h12 * h.h12) * r0 + (h.h02 * h.h12 - h.h01 * h.h22) * r1 +
             (h.h01 * h.h12 - h.h11 * h.h02) * r2;
        y1 = (h.h02 * h.h12 - h.h01 * h.h22) * r0 + (h.h00 * h.h22 - h.h02 * h.h02) * r1 +
             (h.h01 * h.h02 - h.h00 * h.h12) * r2;
        y2 = (h.h01 * h.h12 - h.h11 * h.h02) * r0 + (h.h01 * h.h02 - h.h00 * h.h12) * r1 +
             (h.h00 * h.h11 - h.h01 * h.h01) * r2;
    }
};

template <class Prod, class Adj>
struct Rounding {
    using P = Prod;
    using A = Adj;
};

// The policy that reproduces the reference build.
using RefRounding = Rounding<PlainProducts, AdjRef>;

// ---------------------------------------------------------------------------
// Newton building blocks (one matrix per thread).
// ---------------------------------------------------------------------------

// Quotient a / b exactly as the reference's fast-math build computes it:
// there a division is div.approx, a * (1/b) with the approximate reciprocal,
// so rows that share a denominator can share one reciprocal.
__device__ __forceinline__ float fast_rcp(float b) { return __fdividef(1.0f, b); }

// One log-sum-exp pass over the four lines of X (X in line-major order):
//   m_l = max_k X_lk,  e_lk = exp(X_lk - m_l),  s_l = sum_k e_lk,
//   lse_l = -m_l - log(s_l).
// With lines = rows of beta + R this is the row part of compute_f_gradient
// (birkhoff_proj_n4.cu:229-234); with lines = columns of R (or of alpha + R)
// it is initialize_beta_alpha0 (:139-141) and the column half of
// sinkhorn_iteration (:168-171).  Reductions run in the butterfly order.
__device__ __forceinline__ void lse_pass(const float X[16], float e[16], float s[4], float lse[4])
{
#pragma unroll
    for (int l = 0; l < 4; ++l) {
        const float* x = X + 4 * l;
        const float mx = pmax4(x[0], x[1], x[2], x[3]);
#pragma unroll
        for (int k = 0; k < 4; ++k) e[4 * l + k] = expf(x[k] - mx);
        s[l] = psum4(e[4 * l], e[4 * l + 1], e[4 * l + 2], e[4 * l + 3]);
        lse[l] = -mx - logf(s[l]);
    }
}

// lse_pass on L lines (the small-batch kernel's lanes take two each).
template <int L>
__device__ __forceinline__ void lse_lines(const float* X, float* e, float* s, float* lse)
{
#pragma unroll
    for (int l = 0; l < L; ++l) {
        const float* x = X + 4 * l;
        const float mx = pmax4(x[0], x[1], x[2], x[3]);
#pragma unroll
        for (int k = 0; k < 4; ++k) e[4 * l + k] = expf(x[k] - mx);
        s[l] = psum4(e[4 * l], e[4 * l + 1], e[4 * l + 2], e[4 * l + 3]);
        lse[l] = -mx - logf(s[l]);
    }
}

// The starting point of the Newton solve (birkhoff_proj_n4.cu:400-423): the
// objective at beta = 0 (rows of 0 + R; the reference's offset is added, so an
// entry -0 becomes +0 as there) and the alpha = 0 initialisation (column
// log-sum-exp of R, :129-147), whose beta -- shifted to beta_3 = 0 -- is the
// start if its objective is strictly lower; beta = 0 otherwise.  The
// f/gradient evaluation at the start is left to the caller.
__device__ __forceinline__ void start_point(const float r[16], float beta[4])
{
    float X[16], e[16], s[4], lse[4];
    float z;  // +0, opaque to the compiler so that 0 + R is not folded to R
    asm("mov.b32 %0, 0;" : "=f"(z));
#pragma unroll
    for (int q = 0; q < 16; ++q) X[q] = z + r[q];
    lse_pass(X, e, s, lse);
    const float f0 = -psum4(lse[0], lse[1], lse[2], lse[3]) - psum4(z, z, z, z);
#pragma unroll
    for (int l = 0; l < 4; ++l)
#pragma unroll
        for (int q = 0; q < 4; ++q) X[4 * l + q] = r[4 * q + l];
    lse_pass(X, e, s, lse);
    const float fa = -psum4(lse[0], lse[1], lse[2], lse[3]);
    const bool take = fa < f0;
#pragma unroll
    for (int j = 0; j < 4; ++j) beta[j] = sel(take, lse[j] - lse[3], z);
}

// Column products of T summed over rows, as the row-0 lanes of the reference
// hold them (they broadcast H, birkhoff_proj_n4.cu:286-309 and :550-573):
// p[0..2] = sum_i T_ij^2 for j = 0,1,2 and p[3..5] = sum_i T_ij T_ik for the
// column pairs (0,1), (1,2), (2,0), the rotation the reference uses.
template <class Prod>
__device__ __forceinline__ void gram_sums(const float* t, float p[6])
{
    p[0] = Prod::prod_sum(0, t[0], t[0], t[4], t[4], t[8], t[8], t[12], t[12]);
    p[1] = Prod::prod_sum(0, t[1], t[1], t[5], t[5], t[9], t[9], t[13], t[13]);
    p[2] = Prod::prod_sum(0, t[2], t[2], t[6], t[6], t[10], t[10], t[14], t[14]);
    p[3] = Prod::prod_sum(0, t[0], t[1], t[4], t[5], t[8], t[9], t[12], t[13]);
    p[4] = Prod::prod_sum(0, t[1], t[2], t[5], t[6], t[9], t[10], t[13], t[14]);
    p[5] = Prod::prod_sum(0, t[2], t[0], t[6], t[4], t[10], t[8], t[14], t[12]);
}

// Leading 3x3 block of diag(c) - T^T T plus `shift` on the diagonal, from
// the sums above.
__device__ __forceinline__ Sym3 gram_matrix(const float p[6], const float c[3], float shift)
{
    Sym3 h;
    h.h00 = __fsub_rn(__fadd_rn(shift, c[0]), p[0]);
    h.h11 = __fsub_rn(__fadd_rn(shift, c[1]), p[1]);
    h.h22 = __fsub_rn(__fadd_rn(shift, c[2]), p[2]);
    h.h01 = -p[3];
    h.h12 = -p[4];
    h.h02 = -p[5];
    return h;
}

template <class Prod>
__device__ __forceinline__ Sym3 gram3(const Mat4& T, const float c[3], float shift)
{
    float p[6];
    gram_sums<Prod>(T.m, p);
    return gram_matrix(p, c, shift);
}

// Newton direction d = -H^{-1} g with H = diag(c) - T^T T + min(|g|^2, 1e-3) I,
// or d = -g when H is near singular or badly conditioned
// (compute_newton_direction, :263-367).  d[3] is the reference's fourth-lane
// value: +0 on the gradient fallback, -0 * (1/det) on the Newton branch.
template <class Rd>
__device__ __forceinline__ void newton_direction(const float p[6], const float c[3], float gnorm, float d[4])
{
    const float shift = fminf(gnorm * gnorm, 1e-3f);
    const Sym3 h = gram_matrix(p, c, shift);
    const float g0 = c[0] - 1.0f;
    const float g1 = c[1] - 1.0f;
    const float g2 = c[2] - 1.0f;
    const float det = Rd::A::det(h);
    const float rdet = fast_rcp(det);
    const float m = (h.h00 + h.h11 + h.h22) / 3.0f;
    const float rho = __fmul_rn(__fmul_rn(__fmul_rn(m, m), m), rdet);
    float y0, y1, y2;
    Rd::A::adj(h, g0, g1, g2, y0, y1, y2);
    // both candidates are computed and one is selected, so the code has no
    // branch for a warp to diverge on
    const bool fallback = det <= kEpsilon || rho > 1000.0f;
    d[0] = sel(fallback, -g0, __fmul_rn(-y0, rdet));
    d[1] = sel(fallback, -g1, __fmul_rn(-y1, rdet));
    d[2] = sel(fallback, -g2, __fmul_rn(-y2, rdet));
    d[3] = sel(fallback, 0.0f, __fmul_rn(-0.0f, rdet));
}

// ---------------------------------------------------------------------------
// IFT backward for one matrix (birkhoff_proj_n4_backward_kernel, :619-669,
// solve_delta_linear_system :527-614):
//   Gamma = G.*T, mu_r = rowsum Gamma, mu_c = colsum Gamma,
//   w = Delta^{-1} (mu_c - T^T mu_r) on the first three columns with
//   Delta = diag(colsum T) - T^T T (det clamped to >= 1e-8), w_3 = 0,
//   v = mu_r - T w,  D = -(v 1^T + 1 w^T - G) .* T.
// Sums of products are taken as the lanes of the reference hold them: the
// right-hand side comes from the row-0 lanes, row sums differ between
// even- and odd-column lanes when products are contracted.
// ---------------------------------------------------------------------------
template <class Rd>
__device__ __forceinline__ void ift_backward(const Mat4& G, const Mat4& T, Mat4& D)
{
    using Prod = typename Rd::P;
    const float* t = T.m;
    const float* g = G.m;

    // row sums of Gamma, even-column view (E) and odd-column view (O)
    float murE[4], murO[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const int o = 4 * i;
        murE[i] = Prod::prod_sum(0, g[o], t[o], g[o + 1], t[o + 1], g[o + 2], t[o + 2], g[o + 3], t[o + 3]);
        murO[i] = Prod::prod_sum(1, g[o], t[o], g[o + 1], t[o + 1], g[o + 2], t[o + 2], g[o + 3], t[o + 3]);
    }
    // rhs_j = mu_c(j) - (T^T mu_r)(j), row-0 view
    float rhs[3];
#pragma unroll
    for (int j = 0; j < 3; ++j) {
        const float muc = Prod::prod_sum(0, g[j], t[j], g[4 + j], t[4 + j], g[8 + j], t[8 + j], g[12 + j], t[12 + j]);
        const float* mr = (j & 1) ? murO : murE;
        const float tm = Prod::prod_sum(0, t[j], mr[0], t[4 + j], mr[1], t[8 + j], mr[2], t[12 + j], mr[3]);
        rhs[j] = __fsub_rn(muc, tm);
    }

    float c[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) c[j] = psum4(t[j], t[4 + j], t[8 + j], t[12 + j]);
    const Sym3 h = gram3<Prod>(T, c, 0.0f);
    float det = Rd::A::det(h);
    det = fmaxf(det, kEpsilon);
    float y0, y1, y2;
    Rd::A::adj(h, rhs[0], rhs[1], rhs[2], y0, y1, y2);
    const float rdet = fast_rcp(det);
    const float w[4] = {__fmul_rn(y0, rdet), __fmul_rn(y1, rdet), __fmul_rn(y2, rdet), 0.0f};

#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const int o = 4 * i;
        const float twE = Prod::prod_sum(0, t[o], w[0], t[o + 1], w[1], t[o + 2], w[2], t[o + 3], w[3]);
        const float twO = Prod::prod_sum(1, t[o], w[0], t[o + 1], w[1], t[o + 2], w[2], t[o + 3], w[3]);
        const float vE = __fsub_rn(murE[i], twE);
        const float vO = __fsub_rn(murO[i], twO);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const float v = (j & 1) ? vO : vE;
            D.m[o + j] = -__fmul_rn(__fsub_rn(__fadd_rn(v, w[j]), g[o + j]), t[o + j]);
        }
    }
}

}  // namespace mhcp
