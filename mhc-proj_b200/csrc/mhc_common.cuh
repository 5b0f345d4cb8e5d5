// Shared device helpers for the batched n=4 Birkhoff projection kernels.
//
// Data layout in HBM: a batch is N contiguous row-major 4x4 fp32 matrices,
// 64 bytes each (the layout of the reference's [N,4,4] tensors).  With a
// 16-byte aligned base pointer every matrix is four aligned float4 rows, so a
// thread that owns a matrix moves it with four 128-bit loads or stores.
#pragma once

#include <cstdint>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
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

// Four 128-bit streaming stores of a at p (16-byte aligned) when `pred`, as
// predicated instructions rather than a branch around them.
__device__ __forceinline__ void store_mat_if(bool pred, float* p, const Mat4& a)
{
    const unsigned on = pred ? 1u : 0u;
#pragma unroll
    for (int q = 0; q < 4; ++q)
        asm volatile("{ .reg .pred p; setp.ne.u32 p, %0, 0; @p st.global.cs.v4.f32 [%1], {%2, %3, %4, %5}; }"
                     ::"r"(on), "l"(p + 4 * q), "f"(a.m[4 * q]), "f"(a.m[4 * q + 1]), "f"(a.m[4 * q + 2]),
                       "f"(a.m[4 * q + 3])
                     : "memory");
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

// Bitwise select (p ? a : b) as one selp instruction.  Written in PTX so the
// compiler cannot turn it back into a branch around the computation of an
// operand: in the per-lane state machines both operands are always computed
// and lanes must not split over which one is kept.
__device__ __forceinline__ float sel(bool p, float a, float b)
{
    float r;
    asm("{\n\t.reg .pred q;\n\tsetp.ne.u32 q, %3, 0;\n\tselp.f32 %0, %1, %2, q;\n\t}"
        : "=f"(r) : "f"(a), "f"(b), "r"(static_cast<unsigned>(p)));
    return r;
}

__device__ __forceinline__ int sel(bool p, int a, int b)
{
    int r;
    asm("{\n\t.reg .pred q;\n\tsetp.ne.u32 q, %3, 0;\n\tselp.s32 %0, %1, %2, q;\n\t}"
        : "=r"(r) : "r"(a), "r"(b), "r"(static_cast<unsigned>(p)));
    return r;
}

// ---------------------------------------------------------------------------
// Element types other than fp32.  A matrix of `Elem` is loaded into fp32
// registers (bf16 and fp16 widen exactly) and stored back with
// round-to-nearest-even, the conversions torch's .to() performs, so running
// on the native type gives the bits of converting to fp32, computing, and
// converting back.  `off` is the element offset of the matrix's first entry;
// its 16 entries are row-major and contiguous.  kVec: 16-byte aligned.
// ---------------------------------------------------------------------------
__device__ __forceinline__ float to_f32(float x) { return x; }
__device__ __forceinline__ float to_f32(__nv_bfloat16 x) { return __bfloat162float(x); }
__device__ __forceinline__ float to_f32(__half x) { return __half2float(x); }

template <class Elem>
__device__ __forceinline__ Elem from_f32(float x);
template <>
__device__ __forceinline__ float from_f32<float>(float x) { return x; }
template <>
__device__ __forceinline__ __nv_bfloat16 from_f32<__nv_bfloat16>(float x) { return __float2bfloat16_rn(x); }
template <>
__device__ __forceinline__ __half from_f32<__half>(float x) { return __float2half_rn(x); }

template <class Elem, bool kVec>
__device__ __forceinline__ void load_elems(const Elem* __restrict__ base, int64_t off, Mat4& a)
{
    if constexpr (sizeof(Elem) == 4) {
        load_mat<kVec>(reinterpret_cast<const float*>(base) + off, 0, a);
    } else if constexpr (kVec) {
        // 16 half-width values = two 16-byte loads
        const uint4* q = reinterpret_cast<const uint4*>(base + off);
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            const uint4 v = __ldg(q + h);
            const Elem* e = reinterpret_cast<const Elem*>(&v);
#pragma unroll
            for (int k = 0; k < 8; ++k) a.m[8 * h + k] = to_f32(e[k]);
        }
    } else {
#pragma unroll
        for (int k = 0; k < 16; ++k) a.m[k] = to_f32(base[off + k]);
    }
}

template <class Elem, bool kVec>
__device__ __forceinline__ void store_elems(Elem* __restrict__ base, int64_t off, const Mat4& a)
{
    if constexpr (sizeof(Elem) == 4) {
        store_mat<kVec>(reinterpret_cast<float*>(base) + off, 0, a);
    } else if constexpr (kVec) {
        uint4* q = reinterpret_cast<uint4*>(base + off);
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            uint4 v;
            Elem* e = reinterpret_cast<Elem*>(&v);
#pragma unroll
            for (int k = 0; k < 8; ++k) e[k] = from_f32<Elem>(a.m[8 * h + k]);
            __stcs(q + h, v);
        }
    } else {
#pragma unroll
        for (int k = 0; k < 16; ++k) base[off + k] = from_f32<Elem>(a.m[k]);
    }
}

// store_elems when `pred`: predicated 128-bit stores for the 16-byte path
// (no branch), a branch around the scalar path.
template <class Elem, bool kVec>
__device__ __forceinline__ void store_elems_if(bool pred, Elem* __restrict__ base, int64_t off, const Mat4& a)
{
    if constexpr (kVec && sizeof(Elem) == 4) {
        store_mat_if(pred, reinterpret_cast<float*>(base) + off, a);
    } else if constexpr (kVec) {
        const unsigned on = pred ? 1u : 0u;
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            uint4 v;
            Elem* e = reinterpret_cast<Elem*>(&v);
#pragma unroll
            for (int k = 0; k < 8; ++k) e[k] = from_f32<Elem>(a.m[8 * h + k]);
            asm volatile("{ .reg .pred p; setp.ne.u32 p, %0, 0; @p st.global.cs.v4.b32 [%1], {%2, %3, %4, %5}; }"
                         ::"r"(on), "l"(base + off + 8 * h), "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w)
                         : "memory");
        }
    } else {
        if (pred) store_elems<Elem, kVec>(base, off, a);
    }
}

// Two consecutive rows (8 entries) of a matrix at p, stored as Elem: two
// 16-byte stores (fp32) or one (bf16/fp16) on the aligned path.
template <class Elem, bool kVec>
__device__ __forceinline__ void store_rows2(Elem* __restrict__ p, const float (&t)[8])
{
    if constexpr (kVec && sizeof(Elem) == 4) {
        float4* q = reinterpret_cast<float4*>(p);
        __stcs(q, make_float4(t[0], t[1], t[2], t[3]));
        __stcs(q + 1, make_float4(t[4], t[5], t[6], t[7]));
    } else if constexpr (kVec) {
        uint4 v;
        Elem* e = reinterpret_cast<Elem*>(&v);
#pragma unroll
        for (int k = 0; k < 8; ++k) e[k] = from_f32<Elem>(t[k]);
        __stcs(reinterpret_cast<uint4*>(p), v);
    } else {
#pragma unroll
        for (int k = 0; k < 8; ++k) p[k] = from_f32<Elem>(t[k]);
    }
}

__host__ __device__ constexpr int64_t ceil_div(int64_t a, int64_t b) { return (a + b - 1) / b; }

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// A strided batch takes the 16-byte path when its base and every matrix start
// are 16-byte aligned.
inline bool aligned16(const void* p, int64_t stride_elems, int elem_bytes)
{
    return aligned16(p) && ((stride_elems * elem_bytes) & 15) == 0;
}

}  // namespace mhcp
