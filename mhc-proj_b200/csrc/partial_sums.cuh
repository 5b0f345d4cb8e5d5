// Deterministic batch sums of the H_res backward kernels: the gradients of
// the producer's shared parameters (db, 16 floats, and dalpha) are sums over
// the whole batch.  Each block folds its threads' 17 values in a fixed tree
// and writes one row of partial sums; partial_sums_fold_kernel then folds the
// rows in a fixed order.  The rows are stored column-major, partials[q * rows
// + block], so that the fold reads them coalesced however many there are.
#pragma once

#include "mhc_common.cuh"

namespace mhcp {

constexpr int kHResPartials = 17;  // db[0..15], dalpha

// Fold acc[17] over the block (butterflies within each warp, then warp 0
// over the warps) into column `row` of `partials` (rows columns).  Every
// thread of the block must call it.
template <int kBlock>
__device__ __forceinline__ void block_partial_sums(const float (&acc)[kHResPartials], float* __restrict__ partials,
                                                   int64_t rows, int64_t row)
{
    __shared__ float part[kBlock / 32][kHResPartials];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
    for (int q = 0; q < kHResPartials; ++q) {
        float v = acc[q];
#pragma unroll
        for (int m = 16; m > 0; m >>= 1) v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, m));
        if (lane == 0) part[warp][q] = v;
    }
    __syncthreads();
    if (threadIdx.x < kHResPartials) {
        float v = part[0][threadIdx.x];
#pragma unroll
        for (int w = 1; w < kBlock / 32; ++w) v = __fadd_rn(v, part[w][threadIdx.x]);
        partials[static_cast<int64_t>(threadIdx.x) * rows + row] = v;
    }
}

// Folds `rows` rows of partial sums into db[16] and dalpha: warp q takes
// column q, its lanes stride over the rows, then a butterfly.  rows == 0
// writes zeros (the gradient of an empty batch).  A template so that both
// kernel files can instantiate it.
template <int kParts>
__global__ void __launch_bounds__(32 * kParts) partial_sums_fold_kernel(const float* __restrict__ partials,
                                                                        int64_t rows, float* __restrict__ db,
                                                                        float* __restrict__ dalpha)
{
    const int lane = threadIdx.x & 31, q = threadIdx.x >> 5;
    const float* col = partials + static_cast<int64_t>(q) * rows;
    float v = 0.0f;
    for (int64_t b = lane; b < rows; b += 32) v = __fadd_rn(v, col[b]);
#pragma unroll
    for (int m = 16; m > 0; m >>= 1) v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, m));
    if (lane == 0) {
        if (q < kParts - 1)
            db[q] = v;
        else
            *dalpha = v;
    }
}

// The producer's arithmetic (the reference's utils.cuh:84-93 before its
// exponential): r_inv = 1 / rms with the fast-math reciprocal, then
// (alpha * h) * r_inv + b as one multiply and one fused multiply-add.
__device__ __forceinline__ float hres_rinv(float rms) { return __fdividef(1.0f, rms); }
__device__ __forceinline__ float hres_logit(float alpha, float h, float rinv, float b)
{
    return __fmaf_rn(__fmul_rn(alpha, h), rinv, b);
}

// Per matrix, given dR = dL/dR and h: writes dh = dR * alpha / rms into
// dh_out, returns drms, and adds the matrix's terms to acc (db += dR,
// dalpha += sum(dR .* h) / rms).
__device__ __forceinline__ float hres_chain(const Mat4& dR, const Mat4& h, float alpha, float rinv, Mat4& dh_out,
                                            float (&acc)[kHResPartials])
{
    const float s = __fmul_rn(alpha, rinv);
    float rows[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const int o = 4 * i;
        rows[i] = __fmaf_rn(dR.m[o + 3], h.m[o + 3],
                  __fmaf_rn(dR.m[o + 2], h.m[o + 2], __fmaf_rn(dR.m[o + 1], h.m[o + 1], __fmul_rn(dR.m[o], h.m[o]))));
    }
    const float q = psum4(rows[0], rows[1], rows[2], rows[3]);
    acc[16] = __fmaf_rn(rinv, q, acc[16]);
#pragma unroll
    for (int e = 0; e < 16; ++e) {
        acc[e] = __fadd_rn(acc[e], dR.m[e]);
        dh_out.m[e] = __fmul_rn(dR.m[e], s);
    }
    return -__fmul_rn(__fmul_rn(s, rinv), q);
}

}  // namespace mhcp
