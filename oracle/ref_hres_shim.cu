// ORACLE -- test infrastructure only.
//
// extern "C" entry points over the reference's H_res producer
// (fused_h_activations, src/utils.cuh:50-127), compiled unmodified from its
// header, so that the fused producer + projection kernels of this repository
// can be compared with the reference's own two-step path on the same device
// buffers.  Built as a library of its own: utils.cuh defines a non-inline
// kernel that sinkhorn_knopp_n4.cu also pulls in, so the two cannot share one
// link.
#include <cuda_runtime.h>

#include "utils.cuh"

namespace {

// The producer's H_res value before its exponential: the expression of
// utils.cuh:84-93 (r_inv = 1 / rms, alpha * h * r_inv + b) restated for the
// n = 4 layout of one [B, 24] row per token, compiled with the reference's
// flags.  The tests check that __expf of this value is the reference
// producer's H_res bit for bit, which pins the restatement.
__global__ void hres_logits_kernel(const float* __restrict__ H_proj_concat, const float* __restrict__ rms,
                                   float alpha_res, const float* __restrict__ b_res, float* __restrict__ R, int B)
{
    const int idx = blockIdx.x * blockDim.x + threadIdx.x;
    if (idx >= B * 16) return;
    const int b = idx / 16, local = idx % 16;
    const float r_inv = 1.0f / rms[b];
    const float val = H_proj_concat[b * 24 + 8 + local];
    R[idx] = alpha_res * val * r_inv + b_res[local];
}

// y = __expf(x), the producer's exponential (utils.cuh:42-44), to check the
// restatement above against the producer's own output.
__global__ void fast_exp_kernel(const float* __restrict__ x, float* __restrict__ y, int n)
{
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) y[i] = mhc::fast_exp(x[i]);
}

}  // namespace

extern "C" {

// H_pre [B,4], H_post [B,4], H_res [B,16] from H_proj_concat [B,24] and rms [B].
int ref_fused_h_activations_n4(float* H_pre, float* H_post, float* H_res, const float* H_proj_concat,
                               const float* rms, float alpha_pre, float alpha_post, float alpha_res,
                               const float* b_pre, const float* b_post, const float* b_res, int B, void* stream)
{
    if (B <= 0) return 0;
    mhc::fused_h_activations(H_pre, H_post, H_res, H_proj_concat, rms, alpha_pre, alpha_post, alpha_res, b_pre,
                             b_post, b_res, B, 4, static_cast<cudaStream_t>(stream));
    return static_cast<int>(cudaGetLastError());
}

int ref_hres_logits_n4(const float* H_proj_concat, const float* rms, float alpha_res, const float* b_res, float* R,
                       int B, void* stream)
{
    if (B <= 0) return 0;
    hres_logits_kernel<<<(B * 16 + 255) / 256, 256, 0, static_cast<cudaStream_t>(stream)>>>(H_proj_concat, rms,
                                                                                          alpha_res, b_res, R, B);
    return static_cast<int>(cudaGetLastError());
}

int ref_fast_exp(const float* x, float* y, int n, void* stream)
{
    if (n <= 0) return 0;
    fast_exp_kernel<<<(n + 255) / 256, 256, 0, static_cast<cudaStream_t>(stream)>>>(x, y, n);
    return static_cast<int>(cudaGetLastError());
}

}  // extern "C"
