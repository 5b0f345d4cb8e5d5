// Test infrastructure: compares mhcp::rcp_rn (sinkhorn_n4.cuh) with CUDA's
// __frcp_rn, and the Sinkhorn-Knopp factor mhcp::sk_inv(s, 1e-8) with
// (s > 1e-8 ? __frcp_rn(s) : 0), on all 2^32 float bit patterns, all with
// flush-to-zero (built with the Sinkhorn-Knopp kernels' flags).  Prints the number of inputs whose
// results differ in any bit and exits 0.
#include <cstdint>
#include <cstdio>
#include <cstring>

#include "sinkhorn_n4.cuh"

__global__ void compare_all(unsigned long long* count, unsigned* first)
{
    const uint64_t step = static_cast<uint64_t>(gridDim.x) * blockDim.x;
    unsigned long long local = 0;
    for (uint64_t i = static_cast<uint64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < (1ull << 32); i += step) {
        const float x = __uint_as_float(static_cast<unsigned>(i));
        const float want_inv = (x > 1e-8f) ? __frcp_rn(x) : 0.0f;
        if (__float_as_uint(__frcp_rn(x)) != __float_as_uint(mhcp::rcp_rn(x)) ||
            __float_as_uint(want_inv) != __float_as_uint(mhcp::sk_inv(x, 1e-8f))) {
            ++local;
            const unsigned slot = atomicAdd(first, 1u);
            if (slot < 8) first[1 + slot] = static_cast<unsigned>(i);
        }
    }
    atomicAdd(count, local);
}

int main()
{
    unsigned long long* count = nullptr;
    unsigned* first = nullptr;
    if (cudaMalloc(&count, sizeof(unsigned long long)) != cudaSuccess) return 1;
    if (cudaMalloc(&first, 9 * sizeof(unsigned)) != cudaSuccess) return 1;
    cudaMemset(count, 0, sizeof(unsigned long long));
    cudaMemset(first, 0, 9 * sizeof(unsigned));
    compare_all<<<148 * 16, 256>>>(count, first);
    const cudaError_t err = cudaDeviceSynchronize();
    unsigned long long c = 0;
    unsigned f[9] = {0};
    cudaMemcpy(&c, count, sizeof(c), cudaMemcpyDeviceToHost);
    cudaMemcpy(f, first, sizeof(f), cudaMemcpyDeviceToHost);
    std::printf("status=%s mismatches=%llu\n", cudaGetErrorString(err), c);
    for (unsigned k = 0; k < (f[0] < 8 ? f[0] : 8u); ++k) std::printf("x=0x%08x\n", f[1 + k]);
    cudaFree(count);
    cudaFree(first);
    return err == cudaSuccess ? 0 : 1;
}
