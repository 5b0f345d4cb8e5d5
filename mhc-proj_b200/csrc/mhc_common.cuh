// Shared device helpers for the batched n=4 Birkhoff projection kernels.
//
// Data layout in HBM: a batch is N contiguous row-major 4x4 fp32 matrices,
// 64 bytes each (the layout of the reference's [N,4,4] tensors).  With a
// 16-byte aligned base pointer every matrix is four aligned float4 rows, so a
// thread that owns a matrix moves it with four 128-bit loads or stores.
#pragma once

#include <cstdint>
#include <cuda_runtime.h>

namespace mhcp {

// One 4x4 matrix held in registers, row-major: m[4*i + j] = M(i, j).
struct Mat4 {
    float m[16];
};

// 128-bit loads through the read-only path; streaming stores (evict-first)
// because outputs are not re-read by the producing kernel.
template <bool kVec>
__device__ __forceinline__ void load_mat(const float* __restrict__ base, int64_t idx, Mat4& a)
{
    const float* p = base + idx * 16;
    if constexpr (kVec) {
        const float4* q = reinterpret_cast<const float4*>(p);
#pragma unroll
        for (int r = 0; r < 4; ++r) {
            const float4 v = __ldg(q + r);
            a.m[4 * r + 0] = v.x;
            a.m[4 * r + 1] = v.y;
            a.m[4 * r + 2] = v.z;
            a.m[4 * r + 3] = v.w;
        }
    } else {
#pragma unroll
        for (int e = 0; e < 16; ++e) a.m[e] = __ldg(p + e);
    }
}

template <bool kVec>
__device__ __forceinline__ void store_mat(float* __restrict__ base, int64_t idx, const Mat4& a)
{
    float* p = base + idx * 16;
    if constexpr (kVec) {
        float4* q = reinterpret_cast<float4*>(p);
#pragma unroll
        for (int r = 0; r < 4; ++r)
            __stcs(q + r, make_float4(a.m[4 * r + 0], a.m[4 * r + 1], a.m[4 * r + 2], a.m[4 * r + 3]));
    } else {
#pragma unroll
        for (int e = 0; e < 16; ++e) __stcs(p + e, a.m[e]);
    }
}

// Sum of four values in the pairwise order (a + b) + (c + d).  Sixteen lanes
// of a half-warp reducing with xor-butterfly shuffles (offsets 1,2 for rows,
// 4,8 for columns) all end with this value, so a single thread that owns the
// whole matrix reproduces their result bit for bit.
__device__ __forceinline__ float psum4(float a, float b, float c, float d)
{
    return __fadd_rn(__fadd_rn(a, b), __fadd_rn(c, d));
}

__device__ __forceinline__ float pmax4(float a, float b, float c, float d)
{
    return fmaxf(fmaxf(a, b), fmaxf(c, d));
}

__host__ __device__ constexpr int64_t ceil_div(int64_t a, int64_t b) { return (a + b - 1) / b; }

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

}  // namespace mhcp
