// Kernels and C-ABI launchers for the Newton forward and the IFT backward.
#include <atomic>
#include <mutex>

#include <cuda.h>

#include "birkhoff_n4.cuh"
#include "context_cache.h"
#include "partial_sums.cuh"
#include "mhc_proj.h"

namespace mhcp {

// The persistent forward runs one block per SM whose warps share the SM's
// slice of the batch: 20 warps at 96 registers a thread for batches whose
// steps are still latency-bound, 22 at 80 for the largest (six warps then
// share an SM sub-partition's 16K registers; 21 or 24 warps were slower).
constexpr int kFwdWarpsLatency = 20;
constexpr int kFwdWarpsThroughput = 22;
#ifndef MHC_FWD_WIDE_N
#define MHC_FWD_WIDE_N (int64_t{1} << 21)
#endif
constexpr int64_t kFwdWideN = MHC_FWD_WIDE_N;  // larger batches take the 22-warp block
constexpr int kPairBlock = 128;  // the small-batch kernel's block
// Batches up to this many matrices take the two-lanes-per-matrix kernels.
#ifndef MHC_PAIR_MAX_N
#define MHC_PAIR_MAX_N (int64_t{1} << 13)
#endif
constexpr int64_t kPairMaxN = MHC_PAIR_MAX_N;
// Each forward warp stages its next matrices in a shared-memory ring of
// kRing slots, kRingHalf (one claimed chunk) at a time: 5 KB per warp.
constexpr int kRingHalf = 32;
constexpr int kRing = 2 * kRingHalf;



constexpr int kBackwardBlock = 256;
constexpr unsigned kFullMask = 0xffffffffu;

// Stages of the per-lane state machine.  Each stage is one log-sum-exp pass.
// The two passes that depend on R alone -- the objective at beta = 0
// (birkhoff_proj_n4.cu:402-409) and the alpha = 0 initialisation (:414-415)
// -- are made when the matrix is staged (`start_point`), so a lane starts at
// the better of the two points.
enum Stage : int {
    kStart = 0,   // f/gradient at the starting point, then the first convergence test (:416-431)
    kCand = 1,    // line-search candidate beta + gamma_k d           (:450-477)
    kSkCol = 2,   // column half of the Sinkhorn fallback sweep       (:480-482)
    kSkEval = 3,  // f/gradient after the sweep                        (:483-486)
    kIdle = 4,
};

// Where the forward finds matrix k's logits.  `advance` moves to a block's
// first matrix; `load` reads matrix i of the block's slice (a 32-bit offset).
//
// DenseSource: R[k] at R + k * stride, stored as Elem.
template <class Elem, bool kVec>
struct DenseSource {
    const Elem* R;
    int64_t stride;
    __device__ __forceinline__ void advance(int64_t k) { R += k * stride; }
    __device__ __forceinline__ void load(int i, Mat4& r) const
    {
        load_elems<Elem, kVec>(R, static_cast<int64_t>(i) * stride, r);
    }
};

// HResSource: the H_res pre-activation of the mHC layer formed on load,
// R[k] = alpha * h[k] / rms[k] + b, with the arithmetic of the reference's
// producer before its exponential (utils.cuh:84-93: r_inv = 1 / rms, then
// (alpha * h) * r_inv + b as one multiply and one fused multiply-add).
// h[k] is 16 consecutive floats at h + k * stride (a column slice of the
// projection output); alpha is one float and b sixteen, in device memory.
template <bool kVec>
struct HResSource {
    const float* h;
    int64_t stride;
    const float* rms;
    const float* alpha;
    const float* b;
    int64_t base = 0;  // the warp's first matrix: one live index instead of two moved pointers
    __device__ __forceinline__ void advance(int64_t k) { base = k; }
    __device__ __forceinline__ void load(int i, Mat4& r) const
    {
        const int64_t k = base + i;
        load_elems<float, kVec>(h, k * stride, r);
        const float rinv = hres_rinv(__ldg(rms + k));
        const float a = __ldg(alpha);
#pragma unroll
        for (int e = 0; e < 16; ++e) r.m[e] = hres_logit(a, r.m[e], rinv, __ldg(b + e));
    }
};

// Four floats at p (16-byte aligned when kVec) when `pred`; a predicated
// store on the 16-byte path.
template <bool kVec>
__device__ __forceinline__ void store_vec4_if(bool pred, float* p, const float (&v)[4])
{
    if constexpr (kVec) {
        asm volatile("{ .reg .pred q; setp.ne.u32 q, %0, 0; @q st.global.v4.f32 [%1], {%2, %3, %4, %5}; }"
                     ::"r"(pred ? 1u : 0u), "l"(p), "f"(v[0]), "f"(v[1]), "f"(v[2]), "f"(v[3])
                     : "memory");
    } else if (pred) {
#pragma unroll
        for (int j = 0; j < 4; ++j) p[j] = v[j];
    }
}

// Newton forward, persistent.  Block b (one per SM) owns matrices
// [b*per_block, ...) of the batch, and its kWarps warps take them 32 at a time:
// warp w's first chunk is the w-th, later ones come from a shared counter, so
// the warps of an SM run out of work together instead of each at the end of a
// fixed slice of its own.  Each lane runs the reference algorithm
// (birkhoff_proj_n4.cu:375-499) for one matrix as a state machine, and a lane
// that finishes stores its T and takes the warp's next matrix, so a warp costs
// the sum of its matrices' work over 32 instead of the maximum over each group
// of 32 (per-matrix work ranges from 4 to ~140 evaluations).
//
// Every step is the same straight-line code for every lane: one log-sum-exp
// pass whose lines are rows or columns as the stage needs, the row and the
// column post-processing, the transition, and the Newton direction at the
// point just evaluated (kept by the lanes that adopt that point and start a
// new iteration), all as selects; the store of a finished T and the refill
// of its lane are predicated instructions.  No branch depends on a lane, so
// lanes at different points of the algorithm never split the warp; the only
// branches are warp-uniform (the loop, the ring's fill).
//
// The current point keeps only f, |g|, the row log-sum-exps (the offsets of
// a Sinkhorn sweep) and beta -- not T, whose column and Gram sums give the
// direction in the step that evaluates it: T is written to the output by the
// pass that finishes the matrix.
//
// The warp's next matrices wait in a shared-memory ring: all 32 lanes load
// (and, for HResSource, transform) kRingHalf matrices at once whenever the
// older half of the ring has been handed out, and choose each one's starting
// point there (`start_point`: the beta = 0 objective and the alpha = 0
// initialisation, two passes that depend on R alone, made at full warp width
// instead of as two steps of the state machine).  A refill -- which a few
// lanes of the warp take each step -- is then five predicated shared-memory
// loads (R and the starting beta) instead of global loads and arithmetic
// issued for those few lanes.  The launch bound (32 * kWarps threads, one
// block per SM) caps the registers at what kWarps resident warps allow: 96
// for 20, 80 for 22.
//
// Src supplies the logits (DenseSource or HResSource); Elem is the storage
// type of T (fp32, bf16 or fp16; computation is fp32), which is contiguous.
// kStats: also write, per matrix, the number of Newton iterations taken and
// the final gradient l1 norm, and, when `counts` is given, add the warp's
// pass counts by stage to it (MHC_PASS_* in mhc_proj.h); kDuals: also write
// the final beta (4 floats, the point whose T is the output: T =
// row-softmax(beta + R)).  Separate instantiations; the plain one carries no
// cost for either.
template <class Rd, class Src, class Elem, bool kVec, bool kStats, bool kDuals, int kWarps>
__global__ void __launch_bounds__(32 * kWarps, 1) birkhoff_fwd_kernel(Src src, Elem* __restrict__ Tout, float tol,
                                                                    int64_t N, int64_t per_block,
                                                                    int32_t* __restrict__ iters_out = nullptr,
                                                                    float* __restrict__ gnorm_out = nullptr,
                                                                    float* __restrict__ beta_out = nullptr,
                                                                    unsigned long long* __restrict__ counts = nullptr)
{
    using Prod = typename Rd::P;
    const int lane = threadIdx.x & 31;
    const int64_t begin = static_cast<int64_t>(blockIdx.x) * per_block;
    if (begin >= N) return;  // block-uniform
    // The block's slice, addressed by 32-bit offsets from its first matrix
    // (per_block is at most ceil(N / blocks) and below 2^31).  Its warps take
    // 32 matrices at a time from it through a shared counter.
    const int blk_cnt = static_cast<int>(min(N - begin, per_block));
    // Warp w's first chunk is the w-th (so that the warps holding a small
    // pool's matrices sit on different SM sub-partitions); later chunks are
    // claimed through the shared counter.
    __shared__ int pool_next;
    if (threadIdx.x == 0) pool_next = 32 * kWarps;
    __syncthreads();
    int cnt = 0;  // matrices this warp has claimed (positions [0, cnt) of its sequence)
    src.advance(begin);
    Tout += begin * 16;
    if constexpr (kStats) {
        iters_out += begin;
        gnorm_out += begin;
    }

    Mat4 r = {};            // logits of the lane's matrix
    float f = 0.0f;         // objective at the current point
    float gn = 0.0f;        // gradient l1 norm at the current point
    float alpha[4] = {0.0f, 0.0f, 0.0f, 0.0f};  // row LSE at the current point
    float beta[4] = {0.0f, 0.0f, 0.0f, 0.0f};
    float d[4] = {0.0f, 0.0f, 0.0f, 0.0f};
    int k = 0, it = 0;
    int idx = 0;  // the lane's matrix, offset in the block's slice
    int stage = kIdle;
    // A ring slot is five 16-byte entries: the four rows of R and the
    // starting beta.  One more entry per warp after the ring holds the warp's
    // output pointer (below).
    constexpr int kSlot = 5;
    extern __shared__ float4 ring_dyn[];
    float4 (*ring_all)[kRing * kSlot + 1] = reinterpret_cast<float4 (*)[kRing * kSlot + 1]>(ring_dyn);
    // the block offsets of the two chunks in the warp's ring
    __shared__ int chunk_all[kWarps][2];
    int* chunk = chunk_all[threadIdx.x >> 5];
    // The line-search steps gamma_k as a per-warp table: one shared load per
    // step instead of a chain of compares and selects.
    __shared__ float gtab_all[kWarps][8];
    float* gtab = gtab_all[threadIdx.x >> 5];
    if (lane < 8) gtab[lane] = line_step(lane);
    __syncwarp();
    float4* ring = ring_all[threadIdx.x >> 5];
    // One output pointer of the warp lives in shared memory at a fixed offset
    // from the ring instead of in two registers, and is loaded where it is
    // stored through: beta's for kDuals (as two more registers it made that
    // instantiation spill at a 96-register cap: 3.31 ms at 2^24 instead of
    // 3.17), T's otherwise (3.08 -> 3.05 ms).  The fills'
    // __syncwarp below orders this store before every lane's load.
    if (lane == 0) {
        if constexpr (kDuals)
            *reinterpret_cast<float**>(ring + kRing * kSlot) = beta_out + begin * 4;
        else
            *reinterpret_cast<Elem**>(ring + kRing * kSlot) = Tout;
    }
    // The pointer, by a volatile load so that it is not hoisted into registers.
    auto warp_pointer = [&]() {
        unsigned long long v;
        asm volatile("ld.shared.u64 %0, [%1];" : "=l"(v)
                     : "r"(static_cast<unsigned>(__cvta_generic_to_shared(ring + kRing * kSlot))));
        return v;
    };
    auto fill = [&](int first) {  // the next 32 matrices of the pool into positions [first, first + 32)
        int c = 32 * static_cast<int>(threadIdx.x >> 5);
        if (first > 0) {
            if (lane == 0) c = atomicAdd(&pool_next, 32);
            c = __shfl_sync(kFullMask, c, 0);
        }
        const int valid = max(0, min(32, blk_cnt - c));
        if (lane == 0) chunk[(first >> 5) & 1] = c;
        cnt += valid;
        {
            const int i = first + lane;
            if (lane < valid) {
                Mat4 m;
                src.load(c + lane, m);
                float b[4];
                start_point(m.m, b);
                float4* slot = ring + (i & (kRing - 1)) * kSlot;
#pragma unroll
                for (int j = 0; j < 4; ++j)
                    slot[j] = make_float4(m.m[4 * j], m.m[4 * j + 1], m.m[4 * j + 2], m.m[4 * j + 3]);
                slot[4] = make_float4(b[0], b[1], b[2], b[3]);
            }
        }
    };
    // R and the starting beta of slot i into the lane's registers as
    // predicated shared loads: they keep their values where !get.
    auto take_if = [&](bool get, int i) {
        const unsigned on = get ? 1u : 0u;
        const unsigned addr =
            static_cast<unsigned>(__cvta_generic_to_shared(ring + ((i & (kRing - 1)) * kSlot)));
#pragma unroll
        for (int j = 0; j < 4; ++j)
            asm volatile("{ .reg .pred p; setp.ne.u32 p, %4, 0; @p ld.shared.v4.f32 {%0, %1, %2, %3}, [%5]; }"
                         : "+f"(r.m[4 * j]), "+f"(r.m[4 * j + 1]), "+f"(r.m[4 * j + 2]), "+f"(r.m[4 * j + 3])
                         : "r"(on), "r"(addr + 16u * j)
                         : "memory");
        asm volatile("{ .reg .pred p; setp.ne.u32 p, %4, 0; @p ld.shared.v4.f32 {%0, %1, %2, %3}, [%5]; }"
                     : "+f"(beta[0]), "+f"(beta[1]), "+f"(beta[2]), "+f"(beta[3])
                     : "r"(on), "r"(addr + 64u)
                     : "memory");
    };
    fill(0);
    fill(kRingHalf);
    __syncwarp();
    int base = 0;  // the ring holds positions [base, base + kRing)
    take_if(lane < cnt, lane);
    if (lane < cnt) stage = kStart;
    idx = chunk[0] + lane;
    int next = min(cnt, 32);
    // kStats with counts: the warp's pass counts, the same in every lane
    unsigned tally[MHC_PASS_COUNTERS] = {};

    // gamma_k of the next step, loaded where k is updated (ahead of the
    // step that uses it)
    float gamma_next = gtab[k];
    while (__any_sync(kFullMask, stage != kIdle)) {
        const bool s_start = stage == kStart, s_cand = stage == kCand;
        const bool s_skcol = stage == kSkCol, s_skeval = stage == kSkEval;

        const float gamma = gamma_next;
        // Point of evaluation (rows) or per-row offsets (columns).
        float v[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const float base = sel(s_skcol, alpha[j], beta[j]);
            const float cand = __fmaf_rn(gamma, d[j], beta[j]);
            v[j] = sel(s_cand, cand, base);
        }
        float X[16];
#pragma unroll
        for (int l = 0; l < 4; ++l)
#pragma unroll
            for (int q = 0; q < 4; ++q)
                X[4 * l + q] = v[q] + (l == q ? r.m[4 * l + q] : sel(s_skcol, r.m[4 * q + l], r.m[4 * l + q]));
        float e[16], s[4], lse[4];
        lse_pass(X, e, s, lse);

        // Row post-processing: T, column sums, f and |g| at v
        // (compute_f_gradient, :235-254), and the Gram sums of T.
        Mat4 Tn;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const float rs = fast_rcp(s[i]);
#pragma unroll
            for (int j = 0; j < 4; ++j) Tn.m[4 * i + j] = __fmul_rn(e[4 * i + j], rs);
        }
        float cn[3];
#pragma unroll
        for (int j = 0; j < 3; ++j) cn[j] = psum4(Tn.m[j], Tn.m[4 + j], Tn.m[8 + j], Tn.m[12 + j]);
        const float fn = -psum4(lse[0], lse[1], lse[2], lse[3]) - psum4(v[0], v[1], v[2], v[3]);
        const float gnn = __fadd_rn(__fadd_rn(fabsf(cn[0] - 1.0f), fabsf(cn[1] - 1.0f)), fabsf(cn[2] - 1.0f));
        float pn[6];
        gram_sums<Prod>(Tn.m, pn);

        // Transition.
        const bool accept = s_cand && fn < f && gnn < gn;
        const bool adopt = s_start || s_skeval || accept;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            alpha[j] = sel(adopt, lse[j], alpha[j]);
            // the column half of the sweep gives beta = b - b_3 (:168-174)
            beta[j] = sel(adopt, v[j], sel(s_skcol, lse[j] - lse[3], beta[j]));
        }
        f = sel(adopt, fn, f);
        gn = sel(adopt, gnn, gn);
        // the first convergence test after initialisation (:426-431), or the
        // test at the end of a Newton iteration (:490-494)
        const bool end_iter = accept || s_skeval;
        const int it_next = sel(s_start, 0, sel(end_iter, it + 1, it));
        const bool tested = s_start || end_iter;
        const bool converged = tested && gn < tol;
        const bool done = converged || (end_iter && it_next == kNewtonMaxIters);
        const bool next_iter = tested && !done;
        it = it_next;
        const bool reject_last = s_cand && !accept && k == kLineSearchMaxIters - 1;
        if constexpr (kStats) {
            if (counts) {
                auto add = [&](int q, bool b) { tally[q] += __popc(__ballot_sync(kFullMask, b)); };
                const bool busy = stage != kIdle;
                tally[MHC_PASS_LANE_SLOTS] += 32;
                add(MHC_PASS_BUSY_LANE_SLOTS, busy);
                add(MHC_PASS_START, s_start);
#pragma unroll
                for (int q = 0; q < kLineSearchMaxIters; ++q) {
                    add(MHC_PASS_CANDIDATE + q, s_cand && k == q);
                    add(MHC_PASS_ACCEPTED + q, accept && k == q);
                }
                add(MHC_PASS_SWEEP_COLUMN, s_skcol);
                add(MHC_PASS_SWEEP_EVAL, s_skeval);
                add(MHC_PASS_AT_CAP, busy && done && !converged);
            }
        }
        // Direction at the adopted point, kept by lanes that start a new
        // Newton iteration (compute_newton_direction, :443-445).
        {
            float dn[4];
            newton_direction<Rd>(pn, cn, gnn, dn);
#pragma unroll
            for (int j = 0; j < 4; ++j) d[j] = sel(next_iter, dn[j], d[j]);
        }
        k = sel(next_iter, 0, sel(s_cand && !accept, k + 1, k));
        gamma_next = gtab[k];
        stage = sel(stage == kIdle || done, static_cast<int>(kIdle),
                sel(next_iter, static_cast<int>(kCand),
                sel(reject_last, static_cast<int>(kSkCol),
                sel(s_skcol, static_cast<int>(kSkEval), stage))));

        // T leaves with the pass that produced it (a row pass: no column pass
        // ends a matrix): predicated stores on the 16-byte path, so that no
        // branch splits the warp here.
        Elem* t_at = Tout;
        if constexpr (!kDuals) t_at = reinterpret_cast<Elem*>(warp_pointer());
        store_elems_if<Elem, kVec>(done, t_at, static_cast<int64_t>(idx) * 16, Tn);
        if constexpr (kStats) {
            if (done) {
                iters_out[idx] = it;
                gnorm_out[idx] = gn;
            }
        }
        if constexpr (kDuals) {
            // beta of the output's point, the adopted one
            store_vec4_if<kVec>(done, reinterpret_cast<float*>(warp_pointer()) + static_cast<int64_t>(idx) * 4,
                                beta);
        }
        // Finished lanes take the warp's next matrices in lane order.  No
        // branch, not even on `want`: with no finished lane nothing changes.
        const unsigned want = __ballot_sync(kFullMask, done);
        const int cand = next + __popc(want & ((1u << lane) - 1u));
        const bool get = done && cand < cnt;
        idx = sel(get, chunk[(cand >> 5) & 1] + (cand & 31), idx);
        take_if(get, cand);
        stage = sel(get, static_cast<int>(kStart), stage);
        next = min(cnt, next + __popc(want));
        if (next > base + kRingHalf) {  // the older half is all handed out: stage the next one
            __syncwarp();
            fill(base + kRing);
            __syncwarp();
            base += kRingHalf;
        }
    }
    if constexpr (kStats) {
        if (counts && lane == 0) {
            tally[MHC_PASS_MATRICES] = static_cast<unsigned>(cnt);
            tally[MHC_PASS_FILL] = 2u * static_cast<unsigned>(cnt);  // this warp's claimed matrices
            for (int q = 0; q < MHC_PASS_COUNTERS; ++q)
                if (tally[q]) atomicAdd(counts + q, static_cast<unsigned long long>(tally[q]));
        }
    }
}

// Small batches: two lanes per matrix.  A batch that fills only a fraction
// of one wave leaves each warp alone on its SM sub-partition, and the kernel
// lasts as long as its slowest matrix's passes times the latency of one step
// of a lone warp.  Here the two lanes of a pair each take two of the four
// lines of every pass -- rows 2h, 2h+1 of a row pass, columns 2h, 2h+1 of a
// column pass -- and exchange their half of each sum over the matrix with
// one shuffle: the reference's order (r0 + r1) + (r2 + r3) is kept, because
// lane 0 holds the first pair's sum and lane 1 the second's, and an IEEE sum
// of the two is the same in either order.  Both lanes then hold the same
// column sums, Gram sums, f and |g|, and compute the same direction.  The
// state machine is the persistent kernel's without the ring: each pair owns
// one matrix, which it stores (its two rows each) when it finishes.
template <class Rd, class Src, class Elem, bool kVec>
__global__ void __launch_bounds__(kPairBlock) birkhoff_fwd_pair_kernel(Src src, Elem* __restrict__ Tout, float tol,
                                                                         int64_t N)
{
    const int64_t m = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 1;
    const bool h = (threadIdx.x & 1) != 0;  // second lane of the pair: lines 2, 3
    const bool live = m < N;
    float rows[8], cols[8];  // this lane's two rows and two columns of R
    {
        Mat4 r = {};
        if (live) {
            src.advance(m);
            src.load(0, r);
        }
#pragma unroll
        for (int l = 0; l < 2; ++l)
#pragma unroll
            for (int q = 0; q < 4; ++q) {
                rows[4 * l + q] = sel(h, r.m[4 * (2 + l) + q], r.m[4 * l + q]);
                cols[4 * l + q] = sel(h, r.m[4 * q + 2 + l], r.m[4 * q + l]);
            }
    }
    auto other = [](float x) { return __shfl_xor_sync(kFullMask, x, 1); };
    // The four lines' values from this lane's two: lines 0, 1 from lane 0.
    auto all4 = [&](const float (&mine)[2], float (&a)[4]) {
#pragma unroll
        for (int l = 0; l < 2; ++l) {
            const float t = other(mine[l]);
            a[l] = sel(h, t, mine[l]);
            a[2 + l] = sel(h, mine[l], t);
        }
    };
    auto half_sum = [&](float mine) { return __fadd_rn(mine, other(mine)); };

    float X[8], e[8], s[2], ls[2], lse[4];
    float beta[4];
    {
        // the starting point (birkhoff_proj_n4.cu:400-423), as start_point
        float z;
        asm("mov.b32 %0, 0;" : "=f"(z));
#pragma unroll
        for (int q = 0; q < 8; ++q) X[q] = z + rows[q];
        lse_lines<2>(X, e, s, ls);
        all4(ls, lse);
        const float f0 = -psum4(lse[0], lse[1], lse[2], lse[3]) - psum4(z, z, z, z);
        lse_lines<2>(cols, e, s, ls);
        all4(ls, lse);
        const float fa = -psum4(lse[0], lse[1], lse[2], lse[3]);
        const bool take = fa < f0;
#pragma unroll
        for (int j = 0; j < 4; ++j) beta[j] = sel(take, lse[j] - lse[3], z);
    }

    float f = 0.0f, gn = 0.0f;
    float alpha[4] = {0.0f, 0.0f, 0.0f, 0.0f};
    float d[4] = {0.0f, 0.0f, 0.0f, 0.0f};
    int k = 0, it = 0;
    int stage = live ? kStart : kIdle;
    while (__any_sync(kFullMask, stage != kIdle)) {
        const bool s_start = stage == kStart, s_cand = stage == kCand;
        const bool s_skcol = stage == kSkCol, s_skeval = stage == kSkEval;
        const float gamma = line_step(k);
        float v[4];
#pragma unroll
        for (int j = 0; j < 4; ++j)
            v[j] = sel(s_cand, __fmaf_rn(gamma, d[j], beta[j]), sel(s_skcol, alpha[j], beta[j]));
#pragma unroll
        for (int q = 0; q < 8; ++q) X[q] = v[q & 3] + sel(s_skcol, cols[q], rows[q]);
        lse_lines<2>(X, e, s, ls);
        all4(ls, lse);

        // this lane's two rows of T, then the sums over all four rows
        float t[8];
#pragma unroll
        for (int l = 0; l < 2; ++l) {
            const float rs = fast_rcp(s[l]);
#pragma unroll
            for (int q = 0; q < 4; ++q) t[4 * l + q] = __fmul_rn(e[4 * l + q], rs);
        }
        float cn[3];
#pragma unroll
        for (int j = 0; j < 3; ++j) cn[j] = half_sum(__fadd_rn(t[j], t[4 + j]));
        // (l0 + l1) + (l2 + l3) from one exchange of the pair's half sums
        const float fn = -half_sum(__fadd_rn(ls[0], ls[1])) - psum4(v[0], v[1], v[2], v[3]);
        const float gnn = __fadd_rn(__fadd_rn(fabsf(cn[0] - 1.0f), fabsf(cn[1] - 1.0f)), fabsf(cn[2] - 1.0f));
        float pn[6];
        {
            constexpr int J[6] = {0, 1, 2, 0, 1, 2};
            constexpr int K[6] = {0, 1, 2, 1, 2, 0};
#pragma unroll
            for (int q = 0; q < 6; ++q)
                pn[q] = half_sum(__fadd_rn(__fmul_rn(t[J[q]], t[K[q]]), __fmul_rn(t[4 + J[q]], t[4 + K[q]])));
        }

        // Transition, as in birkhoff_fwd_kernel.
        const bool accept = s_cand && fn < f && gnn < gn;
        const bool adopt = s_start || s_skeval || accept;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            alpha[j] = sel(adopt, lse[j], alpha[j]);
            beta[j] = sel(adopt, v[j], sel(s_skcol, lse[j] - lse[3], beta[j]));
        }
        f = sel(adopt, fn, f);
        gn = sel(adopt, gnn, gn);
        const bool end_iter = accept || s_skeval;
        const int it_next = sel(s_start, 0, sel(end_iter, it + 1, it));
        const bool tested = s_start || end_iter;
        const bool converged = tested && gn < tol;
        const bool done = converged || (end_iter && it_next == kNewtonMaxIters);
        const bool next_iter = tested && !done;
        it = it_next;
        const bool reject_last = s_cand && !accept && k == kLineSearchMaxIters - 1;
        {
            float dn[4];
            newton_direction<Rd>(pn, cn, gnn, dn);
#pragma unroll
            for (int j = 0; j < 4; ++j) d[j] = sel(next_iter, dn[j], d[j]);
        }
        k = sel(next_iter, 0, sel(s_cand && !accept, k + 1, k));
        stage = sel(stage == kIdle || done, static_cast<int>(kIdle),
                sel(next_iter, static_cast<int>(kCand),
                sel(reject_last, static_cast<int>(kSkCol),
                sel(s_skcol, static_cast<int>(kSkEval), stage))));
        if (done) store_rows2<Elem, kVec>(Tout + m * 16 + (h ? 8 : 0), t);
    }
}

// T = row-softmax(beta + R) with the forward's arithmetic, so that a T
// rebuilt from the saved beta is the forward's output bit for bit.
__device__ __forceinline__ void rebuild_t(const Mat4& r, const float (&beta)[4], Mat4& T)
{
    float X[16], e[16], s[4], lse[4];
#pragma unroll
    for (int l = 0; l < 4; ++l)
#pragma unroll
        for (int q = 0; q < 4; ++q) X[4 * l + q] = beta[q] + r.m[4 * l + q];
    lse_pass(X, e, s, lse);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const float rs = fast_rcp(s[i]);
#pragma unroll
        for (int j = 0; j < 4; ++j) T.m[4 * i + j] = __fmul_rn(e[4 * i + j], rs);
    }
}

// The IFT backward from the saved duals instead of T: T is rebuilt from R and
// beta (16 bytes per matrix saved instead of 64), then D as from T.
template <class Rd, bool kVec>
__global__ void __launch_bounds__(kBackwardBlock) birkhoff_bwd_duals_kernel(const float* __restrict__ G,
                                                                            const float* __restrict__ R,
                                                                            const float* __restrict__ beta,
                                                                            float* __restrict__ D, int64_t N)
{
    const int64_t idx = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (idx >= N) return;
    Mat4 g, r, t, d;
    float b[4];
    load_mat<kVec>(R, idx, r);
    if constexpr (kVec) {
        const float4 v = __ldg(reinterpret_cast<const float4*>(beta) + idx);
        b[0] = v.x, b[1] = v.y, b[2] = v.z, b[3] = v.w;
    } else {
#pragma unroll
        for (int j = 0; j < 4; ++j) b[j] = __ldg(beta + idx * 4 + j);
    }
    rebuild_t(r, b, t);
    load_mat<kVec>(G, idx, g);
    ift_backward<Rd>(g, t, d);
    store_mat<kVec>(D, idx, d);
}

// One thread per matrix.  G and T may have different storage types and batch
// strides; D is contiguous in G's type (the reference returns D in G's
// dtype, solvers_torch.cpp:152).
template <class Rd, class GE, class TE, bool kVec>
__global__ void __launch_bounds__(kBackwardBlock) birkhoff_bwd_kernel(const GE* __restrict__ G, int64_t g_stride,
                                                                      const TE* __restrict__ T, int64_t t_stride,
                                                                      GE* __restrict__ D, int64_t N)
{
    const int64_t idx = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (idx >= N) return;
    Mat4 g, t, d;
    load_elems<GE, kVec>(G, idx * g_stride, g);
    load_elems<TE, kVec>(T, idx * t_stride, t);
    ift_backward<Rd>(g, t, d);
    store_elems<GE, kVec>(D, idx * 16, d);
}

// The IFT backward of a small batch with two lanes per matrix, as the
// small-batch forward: lane h takes rows 2h and 2h+1, and every sum over the
// four rows (the column sums of G.*T and of T, T^T mu_r, the Gram sums) is
// exchanged as two half sums in the reference's order (r0 + r1) + (r2 + r3);
// both lanes then solve the same 3x3 system and write their two rows of D.
// The same bits as birkhoff_bwd_kernel, which leaves a batch that is a
// fraction of one wave waiting on one thread's whole chain per matrix.
template <class GE, class TE, bool kVec>
__global__ void __launch_bounds__(kPairBlock) birkhoff_bwd_pair_kernel(const GE* __restrict__ G, int64_t g_stride,
                                                                       const TE* __restrict__ T, int64_t t_stride,
                                                                       GE* __restrict__ D, int64_t N)
{
    const int64_t m = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 1;
    const bool h = (threadIdx.x & 1) != 0;
    if (m >= N) return;  // both lanes of a pair leave together
    float g[8], t[8];    // this lane's two rows
    {
        Mat4 gm, tm;
        load_elems<GE, kVec>(G, m * g_stride, gm);
        load_elems<TE, kVec>(T, m * t_stride, tm);
#pragma unroll
        for (int q = 0; q < 8; ++q) {
            g[q] = sel(h, gm.m[8 + q], gm.m[q]);
            t[q] = sel(h, tm.m[8 + q], tm.m[q]);
        }
    }
    const unsigned pair = 3u << (threadIdx.x & 30);
    auto half_sum = [&](float mine) { return __fadd_rn(mine, __shfl_xor_sync(pair, mine, 1)); };
    float mr[2];
#pragma unroll
    for (int l = 0; l < 2; ++l)
        mr[l] = psum4(__fmul_rn(g[4 * l], t[4 * l]), __fmul_rn(g[4 * l + 1], t[4 * l + 1]),
                      __fmul_rn(g[4 * l + 2], t[4 * l + 2]), __fmul_rn(g[4 * l + 3], t[4 * l + 3]));
    float rhs[3], c[3];
#pragma unroll
    for (int j = 0; j < 3; ++j) {
        const float muc = half_sum(__fadd_rn(__fmul_rn(g[j], t[j]), __fmul_rn(g[4 + j], t[4 + j])));
        const float tmu = half_sum(__fadd_rn(__fmul_rn(t[j], mr[0]), __fmul_rn(t[4 + j], mr[1])));
        rhs[j] = __fsub_rn(muc, tmu);
        c[j] = half_sum(__fadd_rn(t[j], t[4 + j]));
    }
    float p[6];
    {
        constexpr int J[6] = {0, 1, 2, 0, 1, 2};
        constexpr int K[6] = {0, 1, 2, 1, 2, 0};
#pragma unroll
        for (int q = 0; q < 6; ++q)
            p[q] = half_sum(__fadd_rn(__fmul_rn(t[J[q]], t[K[q]]), __fmul_rn(t[4 + J[q]], t[4 + K[q]])));
    }
    const Sym3 hm = gram_matrix(p, c, 0.0f);
    const float det = fmaxf(RefRounding::A::det(hm), kEpsilon);
    float y0, y1, y2;
    RefRounding::A::adj(hm, rhs[0], rhs[1], rhs[2], y0, y1, y2);
    const float rdet = fast_rcp(det);
    const float w[4] = {__fmul_rn(y0, rdet), __fmul_rn(y1, rdet), __fmul_rn(y2, rdet), 0.0f};
    float d[8];
#pragma unroll
    for (int l = 0; l < 2; ++l) {
        const float* tr = t + 4 * l;
        const float tw = psum4(__fmul_rn(tr[0], w[0]), __fmul_rn(tr[1], w[1]), __fmul_rn(tr[2], w[2]),
                               __fmul_rn(tr[3], w[3]));
        const float v = __fsub_rn(mr[l], tw);
#pragma unroll
        for (int j = 0; j < 4; ++j) d[4 * l + j] = -__fmul_rn(__fsub_rn(__fadd_rn(v, w[j]), g[4 * l + j]), tr[j]);
    }
    store_rows2<GE, kVec>(D + m * 16 + (h ? 8 : 0), d);
}

// The H_res backward: the IFT gradient D = dL/dR of each matrix, carried
// through R = alpha * h / rms + b.  Per matrix, dh = D * (alpha / rms) and
// drms = -(alpha / rms^2) * sum(D .* h); over the batch, dalpha =
// sum_k sum(D_k .* h_k) / rms_k and db = sum_k D_k.  The batch sums are
// deterministic (partial_sums.cuh): each thread accumulates a fixed set of
// matrices (grid-stride order), each block folds its threads in a fixed tree
// into one row of `partials`, and partial_sums_fold_kernel folds the rows in
// a fixed order.  The same N on the same GPU model therefore always gives the
// same bits.
constexpr int kHResBlock = 256;

template <bool kVec>
__global__ void __launch_bounds__(kHResBlock) birkhoff_hres_bwd_kernel(
    const float* __restrict__ G, const float* __restrict__ T, const float* __restrict__ h, int64_t h_stride,
    const float* __restrict__ rms, const float* __restrict__ alpha, float* __restrict__ dh, int64_t dh_stride,
    float* __restrict__ drms, float* __restrict__ partials, int64_t N)
{
    float acc[kHResPartials];
#pragma unroll
    for (int q = 0; q < kHResPartials; ++q) acc[q] = 0.0f;
    const float a = __ldg(alpha);
    const int64_t step = static_cast<int64_t>(gridDim.x) * blockDim.x;
    for (int64_t idx = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; idx < N; idx += step) {
        Mat4 g, t, d, x, dx;
        load_elems<float, kVec>(G, idx * 16, g);
        load_elems<float, kVec>(T, idx * 16, t);
        ift_backward<RefRounding>(g, t, d);
        load_elems<float, kVec>(h, idx * h_stride, x);
        drms[idx] = hres_chain(d, x, a, hres_rinv(__ldg(rms + idx)), dx, acc);
        store_elems<float, kVec>(dh, idx * dh_stride, dx);
    }
    block_partial_sums<kHResBlock>(acc, partials, gridDim.x, blockIdx.x);
}

// Resident blocks of a forward kernel instantiation on the current device,
// queried once per device and instantiation (so later launches make no extra
// runtime calls, which also keeps them legal inside stream capture).
constexpr int kMaxDevices = 64;
// Dynamic shared memory of a forward block of kWarps warps: each warp's ring
// (64 slots of five 16-byte entries) and its output pointer.
constexpr int fwd_ring_bytes(int warps) { return warps * (kRing * 5 + 1) * 16; }

template <auto kKernel, int kWarps>
static int64_t forward_block_slots()
{
    static std::atomic<int64_t> cache[kMaxDevices];  // per instantiation; 0 = not queried yet
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return 0;
    if (dev >= 0 && dev < kMaxDevices) {
        const int64_t hit = cache[dev].load(std::memory_order_relaxed);
        if (hit > 0) return hit;
    }
    int sms = 0, blocks = 0;
    if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) return 0;
    if (cudaFuncSetAttribute(kKernel, cudaFuncAttributeMaxDynamicSharedMemorySize, fwd_ring_bytes(kWarps)) !=
        cudaSuccess)
        return 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&blocks, kKernel, 32 * kWarps, fwd_ring_bytes(kWarps)) !=
            cudaSuccess ||
        blocks < 1)
        return 0;
    const int64_t slots = static_cast<int64_t>(sms) * blocks;  // resident blocks
    if (dev >= 0 && dev < kMaxDevices) cache[dev].store(slots, std::memory_order_relaxed);
    return slots;
}

template <class Src, class Elem, bool kVec, bool kStats, bool kDuals, int kWarps>
static int launch_forward_warps(Src src, void* T, float tol, int64_t N, cudaStream_t stream, int32_t* iters,
                                float* gnorm, float* beta, unsigned long long* counts)
{
    constexpr auto kernel = birkhoff_fwd_kernel<RefRounding, Src, Elem, kVec, kStats, kDuals, kWarps>;
    constexpr int kBlock = 32 * kWarps;
    constexpr int kSmem = fwd_ring_bytes(kWarps);
    const int64_t slots = forward_block_slots<kernel, kWarps>();
    if (slots <= 0) {
        const cudaError_t e = cudaGetLastError();
        return static_cast<int>(e != cudaSuccess ? e : cudaErrorUnknown);
    }
    // Enough blocks to fill the GPU once, each an equal contiguous share that
    // its warps take 32 matrices at a time, small enough for 32-bit offsets.
    const int64_t blocks = max(min(ceil_div(N, 32), slots), ceil_div(N, int64_t{1} << 30));
    const int64_t per_block = ceil_div(N, blocks);
    const int64_t grid = ceil_div(N, per_block);
    kernel<<<grid, kBlock, kSmem, stream>>>(src, static_cast<Elem*>(T), tol, N, per_block, iters, gnorm, beta,
                                            counts);
    cudaError_t e = cudaGetLastError();
    if (e == cudaErrorInvalidValue &&
        cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmem) == cudaSuccess) {
        // The shared-memory attribute belongs to the CUDA context: after a
        // device reset the cached launch shape is still right but the
        // attribute is gone, so set it again and launch once more.
        kernel<<<grid, kBlock, kSmem, stream>>>(src, static_cast<Elem*>(T), tol, N, per_block, iters, gnorm, beta,
                                                counts);
        e = cudaGetLastError();
    }
    return static_cast<int>(e);
}

template <class Src, class Elem, bool kVec, bool kStats = false, bool kDuals = false>
static int launch_forward(Src src, void* T, float tol, int64_t N, cudaStream_t stream, int32_t* iters = nullptr,
                          float* gnorm = nullptr, float* beta = nullptr, unsigned long long* counts = nullptr)
{
    if (N > kFwdWideN)
        return launch_forward_warps<Src, Elem, kVec, kStats, kDuals, kFwdWarpsThroughput>(src, T, tol, N, stream,
                                                                                          iters, gnorm, beta, counts);
    return launch_forward_warps<Src, Elem, kVec, kStats, kDuals, kFwdWarpsLatency>(src, T, tol, N, stream, iters,
                                                                                   gnorm, beta, counts);
}


template <class Src, class Elem, bool kVec>
static int launch_forward_pairs(Src src, void* T, float tol, int64_t N, cudaStream_t stream)
{
    const int64_t grid = ceil_div(2 * N, kPairBlock);
    birkhoff_fwd_pair_kernel<RefRounding, Src, Elem, kVec>
        <<<grid, kPairBlock, 0, stream>>>(src, static_cast<Elem*>(T), tol, N);
    return static_cast<int>(cudaGetLastError());
}

template <class Elem>
static int forward_typed(const void* R, int64_t r_stride, void* T, float tol, int64_t N, cudaStream_t stream)
{
    const Elem* r = static_cast<const Elem*>(R);
    const bool vec = aligned16(R, r_stride, sizeof(Elem)) && aligned16(T);
    if (N <= kPairMaxN)
        return vec ? launch_forward_pairs<DenseSource<Elem, true>, Elem, true>({r, r_stride}, T, tol, N, stream)
                   : launch_forward_pairs<DenseSource<Elem, false>, Elem, false>({r, r_stride}, T, tol, N, stream);
    return vec ? launch_forward<DenseSource<Elem, true>, Elem, true>({r, r_stride}, T, tol, N, stream)
               : launch_forward<DenseSource<Elem, false>, Elem, false>({r, r_stride}, T, tol, N, stream);
}

template <class GE, class TE>
static int backward_typed(const void* G, int64_t g_stride, const void* T, int64_t t_stride, void* D, int64_t N,
                          cudaStream_t stream)
{
    const int64_t grid = ceil_div(N, kBackwardBlock);
    const bool vec = aligned16(G, g_stride, sizeof(GE)) && aligned16(T, t_stride, sizeof(TE)) && aligned16(D);
    const GE* g = static_cast<const GE*>(G);
    const TE* t = static_cast<const TE*>(T);
    GE* d = static_cast<GE*>(D);
    if (N <= kPairMaxN) {  // two lanes per matrix, as the small-batch forward
        const int64_t pgrid = ceil_div(2 * N, kPairBlock);
        if (vec)
            birkhoff_bwd_pair_kernel<GE, TE, true><<<pgrid, kPairBlock, 0, stream>>>(g, g_stride, t, t_stride, d, N);
        else
            birkhoff_bwd_pair_kernel<GE, TE, false><<<pgrid, kPairBlock, 0, stream>>>(g, g_stride, t, t_stride, d, N);
        return static_cast<int>(cudaGetLastError());
    }
    if (vec)
        birkhoff_bwd_kernel<RefRounding, GE, TE, true><<<grid, kBackwardBlock, 0, stream>>>(g, g_stride, t, t_stride,
                                                                                            d, N);
    else
        birkhoff_bwd_kernel<RefRounding, GE, TE, false><<<grid, kBackwardBlock, 0, stream>>>(g, g_stride, t,
                                                                                             t_stride, d, N);
    return static_cast<int>(cudaGetLastError());
}

template <class GE>
static int backward_t(const void* G, int64_t g_stride, const void* T, int64_t t_stride, int t_dtype, void* D,
                      int64_t N, cudaStream_t stream)
{
    switch (t_dtype) {
        case MHC_DTYPE_F32: return backward_typed<GE, float>(G, g_stride, T, t_stride, D, N, stream);
        case MHC_DTYPE_BF16: return backward_typed<GE, __nv_bfloat16>(G, g_stride, T, t_stride, D, N, stream);
        case MHC_DTYPE_F16: return backward_typed<GE, __half>(G, g_stride, T, t_stride, D, N, stream);
        default: return MHC_ERR_INVALID_VALUE;
    }
}

// Blocks of the H_res backward: one wave of resident blocks, at most one per
// 256 matrices, and at most `cap` (the rows the caller's partial-sum
// storage holds).
static int hres_backward_blocks(int64_t N, int64_t cap)
{
    static std::atomic<int64_t> cache[kMaxDevices];
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return -1;
    int64_t wave = (dev >= 0 && dev < kMaxDevices) ? cache[dev].load(std::memory_order_relaxed) : 0;
    if (wave <= 0) {
        int sms = 0, per_sm = 0;
        if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) return -1;
        if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, birkhoff_hres_bwd_kernel<true>, kHResBlock, 0) !=
                cudaSuccess ||
            per_sm < 1)
            return -1;
        wave = static_cast<int64_t>(sms) * per_sm;
        if (dev >= 0 && dev < kMaxDevices) cache[dev].store(wave, std::memory_order_relaxed);
    }
    return static_cast<int>(max(int64_t{0}, min(min(ceil_div(N, kHResBlock), wave), cap)));
}

static int hres_backward_launch(const float* G, const float* T, const float* h, int64_t h_stride, const float* rms,
                                const float* alpha, float* dh, int64_t dh_stride, float* drms, float* dalpha,
                                float* db, int64_t N, float* partials, int blocks, cudaStream_t stream)
{
    if (blocks > 0) {
        const bool vec = aligned16(G) && aligned16(T) && aligned16(h, h_stride, 4) && aligned16(dh, dh_stride, 4);
        if (vec)
            birkhoff_hres_bwd_kernel<true><<<blocks, kHResBlock, 0, stream>>>(G, T, h, h_stride, rms, alpha, dh,
                                                                              dh_stride, drms, partials, N);
        else
            birkhoff_hres_bwd_kernel<false><<<blocks, kHResBlock, 0, stream>>>(G, T, h, h_stride, rms, alpha, dh,
                                                                               dh_stride, drms, partials, N);
    }
    partial_sums_fold_kernel<kHResPartials><<<1, 32 * kHResPartials, 0, stream>>>(partials, blocks, db, dalpha);
    return static_cast<int>(cudaGetLastError());
}

// Scratch of mhc_birkhoff_proj_n4_hres_backward_noalloc, for callers that
// cannot allocate device memory: partial sums for up to kNoAllocRows blocks
// (68 KB), part of the library's own image, so every GPU that loads the
// library holds it until the process exits.  Every call writes each row it
// reads before reading it, so nothing in it has to start at zero; calls
// whose kernels overlap on the GPU share it and race.
constexpr int kNoAllocRows = 1024;
static __device__ __align__(256) float g_hres_partials[kNoAllocRows * kHResPartials];

// The driver's cuCtxGetCurrent and cuCtxGetId, reached through the
// runtime's driver entry points so that the library needs no link to
// libcuda.  Resolved once, outside any stream capture.
struct ContextIdApi {
    using GetCurrent = CUresult (*)(CUcontext*);
    using GetId = CUresult (*)(CUcontext, unsigned long long*);
    GetCurrent get_current = nullptr;
    GetId get_id = nullptr;
};
static std::once_flag g_ctx_api_once;
static std::atomic<bool> g_ctx_api_ready{false};
static ContextIdApi g_ctx_api;

static void resolve_context_id_api()
{
    std::call_once(g_ctx_api_once, [] {
        void* f = nullptr;
        cudaDriverEntryPointQueryResult q = cudaDriverEntryPointSymbolNotFound;
        if (cudaGetDriverEntryPointByVersion("cuCtxGetCurrent", &f, 12000, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            g_ctx_api.get_current = reinterpret_cast<ContextIdApi::GetCurrent>(f);
        f = nullptr;
        if (cudaGetDriverEntryPointByVersion("cuCtxGetId", &f, 12000, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            g_ctx_api.get_id = reinterpret_cast<ContextIdApi::GetId>(f);
        cudaGetLastError();  // a missing entry point leaves no error behind
        g_ctx_api_ready.store(true, std::memory_order_release);
    });
}

// The process-unique id of the current CUDA context, or 0 when there is none
// yet or the driver cannot tell.  Needs resolve_context_id_api() first.
static unsigned long long current_context_id()
{
    if (!g_ctx_api.get_current || !g_ctx_api.get_id) return 0;
    CUcontext ctx = nullptr;
    unsigned long long id = 0;
    if (g_ctx_api.get_current(&ctx) != CUDA_SUCCESS || !ctx || g_ctx_api.get_id(ctx, &id) != CUDA_SUCCESS) return 0;
    return id;
}

// Device address of g_hres_partials in the current context.  In host code
// the array's name is only a host-side stand-in, so the address is looked
// up (cudaGetSymbolAddress, with the device current) on the first call in
// each context and kept for that context: a device reset or another context
// on the same device places the array elsewhere and is looked up again.  A
// call during stream capture uses only a kept address; one that would have
// to look it up (or, the first time, find the driver's context calls)
// returns MHC_ERR_CAPTURE instead of doing that inside the capture.
static int noalloc_partials(cudaStream_t stream, float** out)
{
    static ContextCache<kMaxDevices> cache;
    cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
    const cudaError_t ce = cudaStreamIsCapturing(stream, &cap);
    if (ce != cudaSuccess) return static_cast<int>(ce);
    const bool capturing = cap != cudaStreamCaptureStatusNone;
    if (!g_ctx_api_ready.load(std::memory_order_acquire)) {
        if (capturing) return MHC_ERR_CAPTURE;
        resolve_context_id_api();
    }
    int dev = 0;
    const cudaError_t de = cudaGetDevice(&dev);
    if (de != cudaSuccess) return static_cast<int>(de);
    void* addr = nullptr;
    const int status = cache.get(dev, current_context_id(), [&](void** v) -> int {
        if (capturing) return MHC_ERR_CAPTURE;
        return static_cast<int>(cudaGetSymbolAddress(v, g_hres_partials));
    }, &addr);
    if (status != 0) return status;
    *out = static_cast<float*>(addr);
    return MHC_OK;
}

static bool valid_dtype(int dt) { return dt == MHC_DTYPE_F32 || dt == MHC_DTYPE_BF16 || dt == MHC_DTYPE_F16; }

}  // namespace mhcp

using namespace mhcp;

extern "C" int mhc_birkhoff_proj_n4_ex(const void* d_R, int64_t r_stride, void* d_T, int dtype, float tol, int64_t N,
                                       cudaStream_t stream)
{
    if (N < 0 || r_stride < 0 || !valid_dtype(dtype) || (N > 0 && (!d_R || !d_T))) return MHC_ERR_INVALID_VALUE;
    if (N == 0) return MHC_OK;
    switch (dtype) {
        case MHC_DTYPE_BF16: return forward_typed<__nv_bfloat16>(d_R, r_stride, d_T, tol, N, stream);
        case MHC_DTYPE_F16: return forward_typed<__half>(d_R, r_stride, d_T, tol, N, stream);
        default: return forward_typed<float>(d_R, r_stride, d_T, tol, N, stream);
    }
}

extern "C" int mhc_birkhoff_proj_n4(const float* d_R, float* d_T, float tol, int64_t N, cudaStream_t stream)
{
    return mhc_birkhoff_proj_n4_ex(d_R, 16, d_T, MHC_DTYPE_F32, tol, N, stream);
}

extern "C" int mhc_birkhoff_proj_n4_stats(const float* d_R, float* d_T, float tol, int64_t N, int32_t* d_iters,
                                          float* d_gnorm, cudaStream_t stream)
{
    if (N < 0 || (N > 0 && (!d_R || !d_T || !d_iters || !d_gnorm))) return MHC_ERR_INVALID_VALUE;
    if (N == 0) return MHC_OK;
    return aligned16(d_R) && aligned16(d_T)
               ? launch_forward<DenseSource<float, true>, float, true, true>({d_R, 16}, d_T, tol, N, stream, d_iters,
                                                                             d_gnorm)
               : launch_forward<DenseSource<float, false>, float, false, true>({d_R, 16}, d_T, tol, N, stream,
                                                                               d_iters, d_gnorm);
}

extern "C" int mhc_birkhoff_proj_n4_pass_counts(const float* d_R, float* d_T, float tol, int64_t N,
                                                int32_t* d_iters, float* d_gnorm, unsigned long long* d_counts,
                                                cudaStream_t stream)
{
    if (N < 0 || (N > 0 && (!d_R || !d_T || !d_iters || !d_gnorm || !d_counts))) return MHC_ERR_INVALID_VALUE;
    if (N == 0) return MHC_OK;
    return aligned16(d_R) && aligned16(d_T)
               ? launch_forward<DenseSource<float, true>, float, true, true>({d_R, 16}, d_T, tol, N, stream, d_iters,
                                                                             d_gnorm, nullptr, d_counts)
               : launch_forward<DenseSource<float, false>, float, false, true>({d_R, 16}, d_T, tol, N, stream,
                                                                               d_iters, d_gnorm, nullptr, d_counts);
}

extern "C" int mhc_birkhoff_proj_n4_backward_ex(const void* d_G, int64_t g_stride, int g_dtype, const void* d_T,
                                                int64_t t_stride, int t_dtype, void* d_D, int64_t N,
                                                cudaStream_t stream)
{
    if (N < 0 || g_stride < 0 || t_stride < 0 || !valid_dtype(g_dtype) || !valid_dtype(t_dtype) ||
        (N > 0 && (!d_G || !d_T || !d_D)))
        return MHC_ERR_INVALID_VALUE;
    if (N == 0) return MHC_OK;
    switch (g_dtype) {
        case MHC_DTYPE_BF16:
            return backward_t<__nv_bfloat16>(d_G, g_stride, d_T, t_stride, t_dtype, d_D, N, stream);
        case MHC_DTYPE_F16: return backward_t<__half>(d_G, g_stride, d_T, t_stride, t_dtype, d_D, N, stream);
        default: return backward_t<float>(d_G, g_stride, d_T, t_stride, t_dtype, d_D, N, stream);
    }
}

extern "C" int mhc_birkhoff_proj_n4_backward(const float* d_G, const float* d_T, float* d_D, int64_t N,
                                             cudaStream_t stream)
{
    return mhc_birkhoff_proj_n4_backward_ex(d_G, 16, MHC_DTYPE_F32, d_T, 16, MHC_DTYPE_F32, d_D, N, stream);
}

extern "C" int mhc_birkhoff_proj_n4_hres(const float* d_h, int64_t h_stride, const float* d_rms,
                                         const float* d_alpha, const float* d_b, float* d_T, float tol, int64_t N,
                                         cudaStream_t stream)
{
    if (N < 0 || h_stride < 0 || (N > 0 && (!d_h || !d_rms || !d_alpha || !d_b || !d_T)))
        return MHC_ERR_INVALID_VALUE;
    if (N == 0) return MHC_OK;
    const HResSource<true> vs{d_h, h_stride, d_rms, d_alpha, d_b};
    const HResSource<false> ss{d_h, h_stride, d_rms, d_alpha, d_b};
    return aligned16(d_h, h_stride, 4) && aligned16(d_T)
               ? launch_forward<HResSource<true>, float, true>(vs, d_T, tol, N, stream)
               : launch_forward<HResSource<false>, float, false>(ss, d_T, tol, N, stream);
}

extern "C" int mhc_birkhoff_proj_n4_hres_backward_workspace(int64_t N, int64_t* bytes)
{
    if (N < 0 || !bytes) return MHC_ERR_INVALID_VALUE;
    const int blocks = hres_backward_blocks(N, int64_t{1} << 30);
    if (blocks < 0) {
        const cudaError_t e = cudaGetLastError();
        return static_cast<int>(e != cudaSuccess ? e : cudaErrorUnknown);
    }
    *bytes = static_cast<int64_t>(max(blocks, 1)) * kHResPartials * static_cast<int64_t>(sizeof(float));
    return MHC_OK;
}

extern "C" int mhc_birkhoff_proj_n4_hres_backward(const float* d_G, const float* d_T, const float* d_h,
                                                  int64_t h_stride, const float* d_rms, const float* d_alpha,
                                                  float* d_dh, int64_t dh_stride, float* d_drms, float* d_dalpha,
                                                  float* d_db, int64_t N, void* d_workspace,
                                                  int64_t workspace_bytes, cudaStream_t stream)
{
    if (N < 0 || h_stride < 0 || dh_stride < 0 || !d_dalpha || !d_db || workspace_bytes < 0 ||
        (N > 0 && (!d_G || !d_T || !d_h || !d_rms || !d_alpha || !d_dh || !d_drms || !d_workspace)))
        return MHC_ERR_INVALID_VALUE;
    const int64_t rows = workspace_bytes / (kHResPartials * static_cast<int64_t>(sizeof(float)));
    const int blocks = hres_backward_blocks(N, rows);
    if (blocks < 0) {
        const cudaError_t e = cudaGetLastError();
        return static_cast<int>(e != cudaSuccess ? e : cudaErrorUnknown);
    }
    if (N > 0 && blocks == 0) return MHC_ERR_INVALID_VALUE;  // workspace smaller than one row
    return hres_backward_launch(d_G, d_T, d_h, h_stride, d_rms, d_alpha, d_dh, dh_stride, d_drms, d_dalpha, d_db, N,
                                static_cast<float*>(d_workspace), blocks, stream);
}

extern "C" int mhc_birkhoff_proj_n4_hres_backward_noalloc(const float* d_G, const float* d_T, const float* d_h,
                                                          int64_t h_stride, const float* d_rms, const float* d_alpha,
                                                          float* d_dh, int64_t dh_stride, float* d_drms,
                                                          float* d_dalpha, float* d_db, int64_t N,
                                                          cudaStream_t stream)
{
    if (N < 0 || h_stride < 0 || dh_stride < 0 || !d_dalpha || !d_db ||
        (N > 0 && (!d_G || !d_T || !d_h || !d_rms || !d_alpha || !d_dh || !d_drms)))
        return MHC_ERR_INVALID_VALUE;
    float* partials = nullptr;
    const int se = noalloc_partials(stream, &partials);
    if (se != MHC_OK) return se;
    // at most kNoAllocRows blocks, each row of the array one block's sums:
    // no batch size needs more scratch than the array holds
    const int blocks = hres_backward_blocks(N, kNoAllocRows);
    if (blocks < 0) {
        const cudaError_t e = cudaGetLastError();
        return static_cast<int>(e != cudaSuccess ? e : cudaErrorUnknown);
    }
    return hres_backward_launch(d_G, d_T, d_h, h_stride, d_rms, d_alpha, d_dh, dh_stride, d_drms, d_dalpha, d_db, N,
                                partials, blocks, stream);
}

extern "C" int mhc_birkhoff_proj_n4_duals(const float* d_R, float* d_T, float* d_beta, float tol, int64_t N,
                                          cudaStream_t stream)
{
    if (N < 0 || (N > 0 && (!d_R || !d_T || !d_beta))) return MHC_ERR_INVALID_VALUE;
    if (N == 0) return MHC_OK;
    return aligned16(d_R) && aligned16(d_T) && aligned16(d_beta)
               ? launch_forward<DenseSource<float, true>, float, true, false, true>({d_R, 16}, d_T, tol, N, stream,
                                                                                    nullptr, nullptr, d_beta)
               : launch_forward<DenseSource<float, false>, float, false, false, true>({d_R, 16}, d_T, tol, N, stream,
                                                                                      nullptr, nullptr, d_beta);
}

extern "C" int mhc_birkhoff_proj_n4_backward_duals(const float* d_G, const float* d_R, const float* d_beta,
                                                   float* d_D, int64_t N, cudaStream_t stream)
{
    if (N < 0 || (N > 0 && (!d_G || !d_R || !d_beta || !d_D))) return MHC_ERR_INVALID_VALUE;
    if (N == 0) return MHC_OK;
    const int64_t grid = ceil_div(N, kBackwardBlock);
    if (aligned16(d_G) && aligned16(d_R) && aligned16(d_beta) && aligned16(d_D))
        birkhoff_bwd_duals_kernel<RefRounding, true><<<grid, kBackwardBlock, 0, stream>>>(d_G, d_R, d_beta, d_D, N);
    else
        birkhoff_bwd_duals_kernel<RefRounding, false><<<grid, kBackwardBlock, 0, stream>>>(d_G, d_R, d_beta, d_D, N);
    return static_cast<int>(cudaGetLastError());
}

extern "C" const char* mhc_status_string(int status)
{
    switch (status) {
        case MHC_OK: return "success";
        case MHC_ERR_INVALID_VALUE: return "invalid argument (negative N or stride, null pointer or unknown dtype)";
        case MHC_ERR_ITERS: return "iteration count outside the supported range";
        case MHC_ERR_CAPTURE:
            return "first call in this CUDA context made during stream capture; make one call outside capture first";
        default: break;
    }
    if (status > 0) return cudaGetErrorString(static_cast<cudaError_t>(status));
    return "unknown status";
}

extern "C" int mhc_abi_version(void) { return MHC_PROJ_ABI_VERSION; }
