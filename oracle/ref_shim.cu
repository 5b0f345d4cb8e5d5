// ORACLE -- test infrastructure only.
//
// extern "C" entry points over the reference's own C++ launchers, so that the
// reference kernels (compiled unmodified from their source files) can be
// called through ctypes and compared with this repository's kernels on the
// same device buffers.  The declarations below restate the launcher
// signatures of the reference:
//   birkhoff_proj_n4           src/birkhoff_proj_n4.cu:505
//   birkhoff_proj_n4_backward  src/birkhoff_proj_n4.cu:675
//   sinkhorn_knopp_n4          src/sinkhorn_knopp_n4.cu:5
//   sinkhorn_knopp_n4_backward src/sinkhorn_knopp_n4.cu:13
#include <cuda_runtime.h>
#include <stdexcept>

void birkhoff_proj_n4(const float* d_R, float* d_T, float tol, int N, cudaStream_t stream);
void birkhoff_proj_n4_backward(const float* d_G, const float* d_T, float* d_D, int N,
                               cudaStream_t stream);
void sinkhorn_knopp_n4(const float* d_M, float* d_T, int N, int num_iters, cudaStream_t stream);
void sinkhorn_knopp_n4_backward(const float* d_G, const float* d_M, float* d_D, int N,
                                int num_iters, cudaStream_t stream);

extern "C" {

int ref_birkhoff_proj_n4(const float* R, float* T, float tol, int N, void* stream)
{
    if (N <= 0) return 0;
    birkhoff_proj_n4(R, T, tol, N, static_cast<cudaStream_t>(stream));
    return static_cast<int>(cudaGetLastError());
}

int ref_birkhoff_proj_n4_backward(const float* G, const float* T, float* D, int N, void* stream)
{
    if (N <= 0) return 0;
    birkhoff_proj_n4_backward(G, T, D, N, static_cast<cudaStream_t>(stream));
    return static_cast<int>(cudaGetLastError());
}

int ref_sinkhorn_knopp_n4(const float* M, float* T, int N, int num_iters, void* stream)
{
    if (N <= 0) return 0;
    sinkhorn_knopp_n4(M, T, N, num_iters, static_cast<cudaStream_t>(stream));
    return static_cast<int>(cudaGetLastError());
}

// Returns -2 when the reference refuses the iteration count (it throws
// std::invalid_argument for num_iters > 20, sinkhorn_knopp.cuh:1213,1220).
int ref_sinkhorn_knopp_n4_backward(const float* G, const float* M, float* D, int N,
                                   int num_iters, void* stream)
{
    if (N <= 0) return 0;
    try {
        sinkhorn_knopp_n4_backward(G, M, D, N, num_iters, static_cast<cudaStream_t>(stream));
    } catch (const std::invalid_argument&) {
        return -2;
    }
    return static_cast<int>(cudaGetLastError());
}

}  // extern "C"
