// Kernels and C-ABI launchers for the Newton forward and the IFT backward.
#include "birkhoff_n4.cuh"
#include "mhc_proj.h"

namespace mhcp {

constexpr int kNewtonBlock = 128;
constexpr int kBackwardBlock = 256;
constexpr unsigned kFullMask = 0xffffffffu;

// Stages of the per-lane state machine.  Each stage is one log-sum-exp pass.
enum Stage : int {
    kEval0 = 0,   // f/gradient at beta = 0                           (birkhoff_proj_n4.cu:402-409)
    kAlpha0 = 1,  // column LSE of R: the alpha = 0 initialisation    (:414-415)
    kEvalA = 2,   // f/gradient at the alpha = 0 beta, if it is better (:416-423)
    kCand = 3,    // line-search candidate beta + gamma_k d           (:450-477)
    kSkCol = 4,   // column half of the Sinkhorn fallback sweep       (:480-482)
    kSkEval = 5,  // f/gradient after the sweep                        (:483-486)
    kIdle = 6,
};

// Newton forward, persistent.  Warp w owns matrices [w*per_warp, ...) of the
// batch.  Each lane runs the reference algorithm (birkhoff_proj_n4.cu:375-499)
// for one matrix as a state machine, and a lane that finishes stores its T and
// takes the warp's next matrix, so a warp costs the sum of its matrices' work
// over 32 instead of the maximum over each group of 32 (per-matrix work ranges
// from 4 to ~130 evaluations).
//
// Every step is the same straight-line code for every lane: the Newton
// direction at the lane's current point, one log-sum-exp pass whose lines are
// rows or columns as the stage needs, the row and the column
// post-processing, and the transition, all as selects.  No branch depends on
// a lane's stage, so lanes at different points of the algorithm never split
// the warp; the only branch is the warp-wide refill.
template <class Rd, bool kVec>
__global__ void __launch_bounds__(kNewtonBlock) birkhoff_fwd_kernel(const float* __restrict__ R,
                                                                    float* __restrict__ Tout, float tol,
                                                                    int64_t N, int64_t per_warp)
{
    const int lane = threadIdx.x & 31;
    const int64_t warp = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
    const int64_t begin = warp * per_warp;
    const int64_t end = min(N, begin + per_warp);
    if (begin >= end) return;  // warp-uniform

    Mat4 r;                 // logits of the lane's matrix
    Mat4 T;                 // T at the current point
    float c[4] = {0.0f, 0.0f, 0.0f, 0.0f};  // column sums of T
    float f = 0.0f;         // objective at the current point
    float gn = 0.0f;        // gradient l1 norm at the current point
    float alpha[4] = {0.0f, 0.0f, 0.0f, 0.0f};  // row LSE at the current point
    float beta[4] = {0.0f, 0.0f, 0.0f, 0.0f};
    float d[4] = {0.0f, 0.0f, 0.0f, 0.0f};
    int k = 0, it = 0;
    bool fresh = false;     // a new Newton iteration starts: take the direction now
    int64_t idx = begin + lane;
    int stage = kIdle;
#pragma unroll
    for (int e2 = 0; e2 < 16; ++e2) T.m[e2] = 0.0f;
    if (idx < end) {
        load_mat<kVec>(R, idx, r);
        stage = kEval0;
    } else {
#pragma unroll
        for (int e2 = 0; e2 < 16; ++e2) r.m[e2] = 0.0f;
    }
    int64_t next = min(end, begin + 32);

    while (__any_sync(kFullMask, stage != kIdle)) {
        // Direction at the current point; kept only by lanes starting a new
        // Newton iteration (compute_newton_direction, :443-445).
        {
            float dn[4];
            newton_direction<Rd>(T, c, gn, dn);
#pragma unroll
            for (int j = 0; j < 4; ++j) d[j] = fresh ? dn[j] : d[j];
            k = fresh ? 0 : k;
            fresh = false;
        }
        const bool col = stage == kAlpha0 || stage == kSkCol;
        const float gamma = line_step(k);
        float v[4];  // point of evaluation (rows) or row offsets (columns)
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const float cand = __fmaf_rn(gamma, d[j], beta[j]);
            v[j] = stage == kEval0 ? 0.0f : stage == kCand ? cand : stage == kSkCol ? alpha[j] : beta[j];
        }
        // Line-major input: rows of v + R, columns of R offset by v per row,
        // or raw columns of R for the alpha = 0 initialisation.
        float X[16];
#pragma unroll
        for (int l = 0; l < 4; ++l)
#pragma unroll
            for (int q = 0; q < 4; ++q) {
                const float rv = col ? r.m[4 * q + l] : r.m[4 * l + q];
                const float sum = v[q] + rv;
                X[4 * l + q] = stage == kAlpha0 ? rv : sum;
            }
        float e[16], s[4], lse[4];
        lse_pass(X, e, s, lse);

        // Row post-processing: T, column sums, f and |g| at v
        // (compute_f_gradient, :235-254).
        Mat4 Tn;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const float rs = fast_rcp(s[i]);
#pragma unroll
            for (int j = 0; j < 4; ++j) Tn.m[4 * i + j] = __fmul_rn(e[4 * i + j], rs);
        }
        float cn[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) cn[j] = psum4(Tn.m[j], Tn.m[4 + j], Tn.m[8 + j], Tn.m[12 + j]);
        const float fn = -psum4(lse[0], lse[1], lse[2], lse[3]) - psum4(v[0], v[1], v[2], v[3]);
        const float gnn = __fadd_rn(__fadd_rn(fabsf(cn[0] - 1.0f), fabsf(cn[1] - 1.0f)), fabsf(cn[2] - 1.0f));
        // Column post-processing: b = column LSE, beta' = b - b_3, and the
        // objective at alpha = 0 (:139-146, :168-174).
        const float fa = -psum4(lse[0], lse[1], lse[2], lse[3]);

        // Transition.
        const bool accept = stage == kCand && fn < f && gnn < gn;
        const bool adopt = stage == kEval0 || stage == kEvalA || stage == kSkEval || accept;
        const bool take_a0 = stage == kAlpha0 && fa < f;
        const bool newbeta = take_a0 || stage == kSkCol;
#pragma unroll
        for (int e2 = 0; e2 < 16; ++e2) T.m[e2] = adopt ? Tn.m[e2] : T.m[e2];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            c[j] = adopt ? cn[j] : c[j];
            alpha[j] = adopt ? lse[j] : alpha[j];
            const float bj = lse[j] - lse[3];
            beta[j] = adopt ? v[j] : newbeta ? bj : beta[j];
        }
        f = adopt ? fn : f;
        gn = adopt ? gnn : gn;
        // the first convergence test after initialisation (:426-431), or the
        // test at the end of a Newton iteration (:490-494)
        const bool check_init = stage == kEvalA || (stage == kAlpha0 && !take_a0);
        const bool end_iter = accept || stage == kSkEval;
        const int it_next = check_init ? 0 : end_iter ? it + 1 : it;
        const bool converged = (check_init || end_iter) && gn < tol;
        const bool done = converged || (end_iter && it_next == kNewtonMaxIters);
        const bool next_iter = (check_init || end_iter) && !done;
        it = it_next;
        const bool reject_last = stage == kCand && !accept && k == kLineSearchMaxIters - 1;
        k = (stage == kCand && !accept) ? k + 1 : k;
        fresh = next_iter;
        stage = stage == kIdle ? kIdle
              : done           ? kIdle
              : next_iter      ? kCand
              : stage == kEval0 ? kAlpha0
              : take_a0        ? kEvalA
              : reject_last    ? kSkCol
              : stage == kSkCol ? kSkEval
                               : stage;

        // Retire finished matrices and hand their lanes the warp's next ones.
        const unsigned want = __ballot_sync(kFullMask, done);
        if (want) {
            if (done) {
                store_mat<kVec>(Tout, idx, T);
                idx = next + __popc(want & ((1u << lane) - 1u));
                if (idx < end) {
                    load_mat<kVec>(R, idx, r);
                    stage = kEval0;
                }
            }
            next = min(end, next + __popc(want));
        }
    }
}

template <class Rd, bool kVec>
__global__ void __launch_bounds__(kBackwardBlock) birkhoff_bwd_kernel(const float* __restrict__ G,
                                                                      const float* __restrict__ T,
                                                                      float* __restrict__ D, int64_t N)
{
    const int64_t idx = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (idx >= N) return;
    Mat4 g, t, d;
    load_mat<kVec>(G, idx, g);
    load_mat<kVec>(T, idx, t);
    ift_backward<Rd>(g, t, d);
    store_mat<kVec>(D, idx, d);
}

// Resident warps of the forward kernel on the current device.
static int64_t forward_warp_slots(bool vec)
{
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return 0;
    int sms = 0, blocks = 0;
    if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) return 0;
    const cudaError_t e = vec ? cudaOccupancyMaxActiveBlocksPerMultiprocessor(
                                    &blocks, birkhoff_fwd_kernel<RefRounding, true>, kNewtonBlock, 0)
                              : cudaOccupancyMaxActiveBlocksPerMultiprocessor(
                                    &blocks, birkhoff_fwd_kernel<RefRounding, false>, kNewtonBlock, 0);
    if (e != cudaSuccess || blocks < 1) return 0;
    return static_cast<int64_t>(sms) * blocks * (kNewtonBlock / 32);
}

}  // namespace mhcp

using namespace mhcp;

extern "C" int mhc_birkhoff_proj_n4(const float* d_R, float* d_T, float tol, int64_t N, cudaStream_t stream)
{
    if (N < 0 || (N > 0 && (!d_R || !d_T))) return MHC_ERR_INVALID_VALUE;
    if (N == 0) return MHC_OK;
    const bool vec = aligned16(d_R) && aligned16(d_T);
    const int64_t slots = forward_warp_slots(vec);
    if (slots <= 0) return static_cast<int>(cudaGetLastError() != cudaSuccess ? cudaGetLastError()
                                                                                : cudaErrorUnknown);
    // Enough warps to fill the GPU once; each takes an equal contiguous share.
    const int64_t warps = min(ceil_div(N, 32), slots);
    const int64_t per_warp = ceil_div(N, warps);
    const int64_t used = ceil_div(N, per_warp);
    const int64_t grid = ceil_div(used * 32, kNewtonBlock);
    if (vec)
        birkhoff_fwd_kernel<RefRounding, true><<<grid, kNewtonBlock, 0, stream>>>(d_R, d_T, tol, N, per_warp);
    else
        birkhoff_fwd_kernel<RefRounding, false><<<grid, kNewtonBlock, 0, stream>>>(d_R, d_T, tol, N, per_warp);
    return static_cast<int>(cudaGetLastError());
}

extern "C" int mhc_birkhoff_proj_n4_backward(const float* d_G, const float* d_T, float* d_D, int64_t N,
                                             cudaStream_t stream)
{
    if (N < 0 || (N > 0 && (!d_G || !d_T || !d_D))) return MHC_ERR_INVALID_VALUE;
    if (N == 0) return MHC_OK;
    const int64_t grid = ceil_div(N, kBackwardBlock);
    if (aligned16(d_G) && aligned16(d_T) && aligned16(d_D))
        birkhoff_bwd_kernel<RefRounding, true><<<grid, kBackwardBlock, 0, stream>>>(d_G, d_T, d_D, N);
    else
        birkhoff_bwd_kernel<RefRounding, false><<<grid, kBackwardBlock, 0, stream>>>(d_G, d_T, d_D, N);
    return static_cast<int>(cudaGetLastError());
}

extern "C" const char* mhc_status_string(int status)
{
    switch (status) {
        case MHC_OK: return "success";
        case MHC_ERR_INVALID_VALUE: return "invalid argument (negative N or null pointer)";
        case MHC_ERR_ITERS: return "iteration count outside the supported range";
        default: break;
    }
    if (status > 0) return cudaGetErrorString(static_cast<cudaError_t>(status));
    return "unknown status";
}

extern "C" int mhc_abi_version(void) { return MHC_PROJ_ABI_VERSION; }
