/*
 * ORACLE -- test infrastructure only.
 *
 * CPU restatement of the reference mHC-proj algorithms for the batched n=4
 * Birkhoff projection.  It is the oracle the CUDA kernels of this repository
 * are compared with, and the timed CPU baseline; no product code path calls it.
 *
 * What it restates (file:line in the reference project):
 *   - the dual-Newton forward        src/birkhoff_proj_n4.cu:375-499
 *       helpers initialize_beta_alpha0 :129-147, sinkhorn_iteration :150-175,
 *       compute_f_gradient :222-255, compute_newton_direction :263-367,
 *       constants :39-43 and the step list :434
 *   - the implicit-function-theorem backward
 *                                    src/birkhoff_proj_n4.cu:527-669
 *   - the fixed-iteration Sinkhorn-Knopp n4 forward
 *                                    src/sinkhorn_knopp.cuh:831-912
 *       (eps passed by src/sinkhorn_knopp_n4.cu:10)
 *   - the Sinkhorn-Knopp n4 backward, two versions (sk_backward_one):
 *       * exact: the exact vector-Jacobian product of the forward (what
 *         PyTorch autograd of the same forward gives), differentiated step by
 *         step through the row/column form (sums as left-to-right FMA
 *         chains, each update as one fused multiply-add) -- an independent
 *         statement of the gradient that the GPU kernel forms from the
 *         forward's potentials;
 *       * reference row step: the reference kernel's reverse loop
 *         src/sinkhorn_knopp.cuh:1146-1202 including its row step
 *         (d - r*rinv)*rinv at :1182-1201, which differs from the exact VJP
 *         (d - r)*rinv, rounded as the reference's build contracts it.  Kept
 *         only so tests can show that difference.
 *
 * Arithmetic: IEEE fp32 with flush-to-zero and denormals-are-zero set per
 * worker thread (the reference builds with --use_fast_math, which flushes
 * denormals), libm expf/logf, and no implicit FMA contraction (built with
 * -ffp-contract=off).  The multiply-adds that the reference's build does
 * contract -- in the 3x3 determinant and adjugate of the Newton direction and
 * of the backward solve, where a product with a single use feeds an add, and
 * in the line-search step beta + gamma*d -- are written as fmaf, so the
 * rounding follows the reference's compiled code.  Reductions are evaluated
 * in the pairwise order that the reference's xor-butterfly shuffles produce
 * in every lane: (x0 + x1) + (x2 + x3).  Because the GPU's fast exp/log/divide
 * are approximations, this oracle agrees with the GPU to tolerance, not bit
 * for bit; exact agreement with the reference GPU kernels is checked on the
 * GPU against the reference built from its own sources.
 */
#include <math.h>
#include <stdint.h>
#include <string.h>
#include <xmmintrin.h>
#include <pmmintrin.h>
#include <pthread.h>
#include <unistd.h>

/* birkhoff_proj_n4.cu:39-43 */
#define NEWTON_MAX_ITERS 20
#define LINE_SEARCH_MAX_ITERS 5
#define EPSILON 1e-8f

static void set_ftz_daz(void)
{
    _MM_SET_FLUSH_ZERO_MODE(_MM_FLUSH_ZERO_ON);
    _MM_SET_DENORMALS_ZERO_MODE(_MM_DENORMALS_ZERO_ON);
}

static inline float sum4(float a, float b, float c, float d) { return (a + b) + (c + d); }
static inline float max4(float a, float b, float c, float d) { return fmaxf(fmaxf(a, b), fmaxf(c, d)); }

/* State of one matrix during the Newton solve. */
typedef struct {
    float T[16];
    float c[4];
    float f;
    float gnorm;
} fg_state;

/* compute_f_gradient, birkhoff_proj_n4.cu:222-255.
 * T = row-softmax(beta + R), c = colsum(T), f = -sum(alpha) - sum(beta),
 * gnorm = |c0-1| + |c1-1| + |c2-1|. */
static void eval_f_grad(const float beta[4], const float R[16], fg_state* s)
{
    float alpha[4];
    for (int i = 0; i < 4; i++) {
        float u[4], e[4];
        for (int j = 0; j < 4; j++) u[j] = beta[j] + R[4 * i + j];
        const float m = max4(u[0], u[1], u[2], u[3]);
        for (int j = 0; j < 4; j++) e[j] = expf(u[j] - m);
        const float se = sum4(e[0], e[1], e[2], e[3]);
        alpha[i] = -m - logf(se);
        for (int j = 0; j < 4; j++) s->T[4 * i + j] = e[j] / se;
    }
    for (int j = 0; j < 4; j++)
        s->c[j] = sum4(s->T[j], s->T[4 + j], s->T[8 + j], s->T[12 + j]);
    s->f = -sum4(alpha[0], alpha[1], alpha[2], alpha[3]) - sum4(beta[0], beta[1], beta[2], beta[3]);
    const float g0 = s->c[0] - 1.0f, g1 = s->c[1] - 1.0f, g2 = s->c[2] - 1.0f;
    s->gnorm = (fabsf(g0) + fabsf(g1)) + (fabsf(g2) + 0.0f);
}

/* initialize_beta_alpha0, birkhoff_proj_n4.cu:129-147: one column
 * log-sum-exp at alpha = 0, then beta shifted so that beta[3] = 0. */
static float init_beta_alpha0(const float R[16], float beta[4])
{
    float b[4];
    for (int j = 0; j < 4; j++) {
        const float nu = max4(R[j], R[4 + j], R[8 + j], R[12 + j]);
        const float se = sum4(expf(R[j] - nu), expf(R[4 + j] - nu),
                              expf(R[8 + j] - nu), expf(R[12 + j] - nu));
        b[j] = -nu - logf(se);
    }
    const float f = -sum4(b[0], b[1], b[2], b[3]);
    for (int j = 0; j < 4; j++) beta[j] = b[j] - b[3];
    return f;
}

/* sinkhorn_iteration, birkhoff_proj_n4.cu:150-175: one log-domain row sweep
 * then column sweep on beta, then beta[3] shifted to 0. */
static void sinkhorn_sweep(float beta[4], const float R[16])
{
    float alpha[4], b[4];
    for (int i = 0; i < 4; i++) {
        float u[4];
        for (int j = 0; j < 4; j++) u[j] = beta[j] + R[4 * i + j];
        const float m = max4(u[0], u[1], u[2], u[3]);
        const float se = sum4(expf(u[0] - m), expf(u[1] - m), expf(u[2] - m), expf(u[3] - m));
        alpha[i] = -m - logf(se);
    }
    for (int j = 0; j < 4; j++) {
        float v[4];
        for (int i = 0; i < 4; i++) v[i] = alpha[i] + R[4 * i + j];
        const float nu = max4(v[0], v[1], v[2], v[3]);
        const float se = sum4(expf(v[0] - nu), expf(v[1] - nu), expf(v[2] - nu), expf(v[3] - nu));
        b[j] = -nu - logf(se);
    }
    for (int j = 0; j < 4; j++) beta[j] = b[j] - b[3];
}

/* Leading 3x3 block of H = diag(c) - T^T T (column products summed over rows).
 * hd[j] = c_j - sum_i T_ij^2; ho = {h01, h12, h02}. */
static void gram3(const float T[16], const float c[4], float diag, float hd[3], float ho[3])
{
    for (int j = 0; j < 3; j++) {
        const float p = sum4(T[j] * T[j], T[4 + j] * T[4 + j], T[8 + j] * T[8 + j], T[12 + j] * T[12 + j]);
        hd[j] = (diag + c[j]) - p;
    }
    /* the reference pairs column j with column (j+1 mod 3): (0,1), (1,2), (2,0) */
    for (int j = 0; j < 3; j++) {
        const int k = (j == 2) ? 0 : j + 1;
        ho[j] = -sum4(T[j] * T[k], T[4 + j] * T[4 + k], T[8 + j] * T[8 + k], T[12 + j] * T[12 + k]);
    }
}

/* Cofactors of the symmetric 3x3 H.  In the reference's compiled code det is
 * evaluated once and each adjugate row in its own per-column branch; a
 * product is contracted into the add it feeds only when it has no other use.
 * So A = h11 h22 - h12^2 and C = h01 h12 - h11 h02 (shared whole with the
 * branches) are contracted, B = h01 h22 - h12 h02 and the branches'
 * h02 h12 - h01 h22 (whose products are shared) are not, and the cofactors
 * local to one branch are. */
static float cof_fused(float a, float b, float c, float d) { return fmaf(a, b, -(c * d)); }
static float cof_plain(float a, float b, float c, float d) { return a * b - c * d; }

/* Adjugate product y = adj(H) r, birkhoff_proj_n4.cu:346-363. */
static void adj3(float h00, float h11, float h22, float h01, float h12, float h02,
                 const float r[3], float y[3])
{
    const float A = cof_fused(h11, h22, h12, h12);
    const float C = cof_fused(h01, h12, h11, h02);
    const float Bq = cof_plain(h02, h12, h01, h22);
    const float E = cof_fused(h00, h22, h02, h02);
    const float F = cof_fused(h01, h02, h00, h12);
    const float K = cof_fused(h00, h11, h01, h01);
    y[0] = fmaf(C, r[2], fmaf(A, r[0], Bq * r[1]));
    y[1] = fmaf(F, r[2], fmaf(Bq, r[0], E * r[1]));
    y[2] = fmaf(K, r[2], fmaf(C, r[0], F * r[1]));
}

/* det(H), birkhoff_proj_n4.cu:321-323. */
static float det3(float h00, float h11, float h22, float h01, float h12, float h02)
{
    const float A = cof_fused(h11, h22, h12, h12);
    const float B = cof_plain(h01, h22, h12, h02);
    const float C = cof_fused(h01, h12, h11, h02);
    return fmaf(h02, C, fmaf(h00, A, -(h01 * B)));
}

/* compute_newton_direction, birkhoff_proj_n4.cu:263-367. d[3] is always 0. */
static void newton_direction(const fg_state* s, float d[4])
{
    const float diag = fminf(s->gnorm * s->gnorm, 1e-3f);
    float hd[3], ho[3];
    gram3(s->T, s->c, diag, hd, ho);
    const float h00 = hd[0], h11 = hd[1], h22 = hd[2];
    const float h01 = ho[0], h12 = ho[1], h02 = ho[2];
    const float g[3] = {s->c[0] - 1.0f, s->c[1] - 1.0f, s->c[2] - 1.0f};
    const float det = det3(h00, h11, h22, h01, h12, h02);
    const float m = (h00 + h11 + h22) / 3.0f;
    const float rho = m * m * m / det;
    d[3] = 0.0f;
    if (det <= EPSILON || rho > 1000.0f) {
        for (int j = 0; j < 3; j++) d[j] = -g[j];
        return;
    }
    float y[3];
    adj3(h00, h11, h22, h01, h12, h02, g, y);
    for (int j = 0; j < 3; j++) d[j] = -y[j] / det;
}

/* birkhoff_proj_n4_kernel, birkhoff_proj_n4.cu:375-499, for one matrix, with
 * the line search cut to its first `candidates` steps (5 = the reference;
 * fewer gives the shortened trajectories a study compares with it).  Returns
 * the number of f/gradient evaluations spent (a cost measure); *iters_out,
 * when given, receives the Newton iterations taken. */
static int newton_one_ls(const float R[16], float T[16], float tol, int candidates, int* iters_out)
{
    static const float gamma_list[LINE_SEARCH_MAX_ITERS] = {1.0f, 0.5f, 0.1f, 0.05f, 0.01f};
    float beta[4] = {0.0f, 0.0f, 0.0f, 0.0f};
    fg_state cur, cand;
    int evals = 1;
    eval_f_grad(beta, R, &cur);

    float beta_a[4];
    const float f_a = init_beta_alpha0(R, beta_a);
    evals++;
    if (f_a < cur.f) {
        memcpy(beta, beta_a, sizeof(beta));
        eval_f_grad(beta, R, &cur);
        evals++;
    }
    int iters = 0;
    if (!(cur.gnorm < tol)) {
        for (int it = 0; it < NEWTON_MAX_ITERS; it++) {
            float d[4];
            iters = it + 1;
            newton_direction(&cur, d);
            for (int k = 0; k < candidates; k++) {
                const float gamma = gamma_list[k];
                float bc[4];
                for (int j = 0; j < 4; j++) bc[j] = fmaf(gamma, d[j], beta[j]);
                eval_f_grad(bc, R, &cand);
                evals++;
                if (cand.f < cur.f && cand.gnorm < cur.gnorm) {
                    memcpy(beta, bc, sizeof(beta));
                    cur = cand;
                    break;
                }
                if (k == candidates - 1) {
                    sinkhorn_sweep(beta, R);
                    eval_f_grad(beta, R, &cur);
                    evals += 2;
                }
            }
            if (cur.gnorm < tol) break;
        }
    }
    memcpy(T, cur.T, sizeof(cur.T));
    if (iters_out) *iters_out = iters;
    return evals;
}

static int newton_one(const float R[16], float T[16], float tol)
{
    return newton_one_ls(R, T, tol, LINE_SEARCH_MAX_ITERS, NULL);
}

/* birkhoff_proj_n4_backward_kernel, birkhoff_proj_n4.cu:619-669 with
 * solve_delta_linear_system :527-614, for one matrix. */
static void ift_one(const float G[16], const float T[16], float D[16])
{
    float gam[16];
    for (int e = 0; e < 16; e++) gam[e] = G[e] * T[e];
    float muc[4], mur[4], rhs[3];
    for (int j = 0; j < 4; j++) muc[j] = sum4(gam[j], gam[4 + j], gam[8 + j], gam[12 + j]);
    for (int i = 0; i < 4; i++) mur[i] = sum4(gam[4 * i], gam[4 * i + 1], gam[4 * i + 2], gam[4 * i + 3]);
    for (int j = 0; j < 3; j++)
        rhs[j] = muc[j] - sum4(T[j] * mur[0], T[4 + j] * mur[1], T[8 + j] * mur[2], T[12 + j] * mur[3]);
    float c[4];
    for (int j = 0; j < 4; j++) c[j] = sum4(T[j], T[4 + j], T[8 + j], T[12 + j]);
    float hd[3], ho[3];
    gram3(T, c, 0.0f, hd, ho);
    /* hii = c_i - p_ii (no shift): gram3 with diag 0 gives (0 + c) - p = c - p */
    float det = det3(hd[0], hd[1], hd[2], ho[0], ho[1], ho[2]);
    det = fmaxf(det, EPSILON);
    float y[3], w[4];
    adj3(hd[0], hd[1], hd[2], ho[0], ho[1], ho[2], rhs, y);
    for (int j = 0; j < 3; j++) w[j] = y[j] / det;
    w[3] = 0.0f;
    for (int i = 0; i < 4; i++) {
        const float tw = sum4(T[4 * i] * w[0], T[4 * i + 1] * w[1], T[4 * i + 2] * w[2], T[4 * i + 3] * w[3]);
        const float v = mur[i] - tw;
        for (int j = 0; j < 4; j++) {
            const float dd = (v + w[j] - G[4 * i + j]) * T[4 * i + j];
            D[4 * i + j] = -dd;
        }
    }
}

/* One Sinkhorn-Knopp n4 normalisation step pair, sinkhorn_knopp.cuh:851-906:
 * rows then columns, x *= (s > eps ? 1/s : 0) with a correctly rounded 1/s. */
static void sk_row_step(float x[16], float rinv[4], float eps)
{
    for (int i = 0; i < 4; i++) {
        const float s = ((x[4 * i] + x[4 * i + 1]) + x[4 * i + 2]) + x[4 * i + 3];
        rinv[i] = (s > eps) ? 1.0f / s : 0.0f;
        for (int j = 0; j < 4; j++) x[4 * i + j] *= rinv[i];
    }
}

static void sk_col_step(float x[16], float cinv[4], float eps)
{
    for (int j = 0; j < 4; j++) {
        const float s = ((x[j] + x[4 + j]) + x[8 + j]) + x[12 + j];
        cinv[j] = (s > eps) ? 1.0f / s : 0.0f;
    }
    for (int i = 0; i < 4; i++)
        for (int j = 0; j < 4; j++) x[4 * i + j] *= cinv[j];
}

static void sk_forward_one(const float M[16], float T[16], int iters, float eps)
{
    float x[16], ri[4], ci[4];
    memcpy(x, M, sizeof(x));
    for (int it = 0; it < iters; it++) {
        sk_row_step(x, ri, eps);
        sk_col_step(x, ci, eps);
    }
    memcpy(T, x, sizeof(x));
}

/* Backward through `iters` row/column steps w.r.t. M.  exact != 0 gives the
 * exact VJP; exact == 0 gives the reference kernel's row step. */
#define SK_MAX_ITERS 64
static void sk_backward_one(const float G[16], const float M[16], float D[16],
                            int iters, float eps, int exact)
{
    float xs[SK_MAX_ITERS][16];  /* row-normalised matrix of each iteration */
    float ri[SK_MAX_ITERS][4], ci[SK_MAX_ITERS][4];
    float x[16], dx[16];
    memcpy(x, M, sizeof(x));
    for (int it = 0; it < iters; it++) {
        sk_row_step(x, ri[it], eps);
        memcpy(xs[it], x, sizeof(x));
        sk_col_step(x, ci[it], eps);
    }
    memcpy(dx, G, sizeof(dx));
    for (int it = iters - 1; it >= 0; it--) {
        const float* xr = xs[it];
        /* column step y = x * cinv: dx = (dy - cinv_j sum_k dy_kj x_kj) cinv_j */
        for (int j = 0; j < 4; j++) {
            float cs;
            if (exact) { /* a left-to-right FMA chain */
                cs = dx[j] * xr[j];
                cs = fmaf(dx[4 + j], xr[4 + j], cs);
                cs = fmaf(dx[8 + j], xr[8 + j], cs);
                cs = fmaf(dx[12 + j], xr[12 + j], cs);
            } else {     /* as the reference's build contracts ((a+b)+c)+d of products */
                cs = fmaf(dx[12 + j], xr[12 + j], fmaf(dx[8 + j], xr[8 + j], fmaf(dx[j], xr[j], dx[4 + j] * xr[4 + j])));
            }
            if (exact) { /* fma(dy, cinv, -((cs cinv) cinv)) */
                const float t = (cs * ci[it][j]) * ci[it][j];
                for (int i = 0; i < 4; i++) dx[4 * i + j] = fmaf(dx[4 * i + j], ci[it][j], -t);
            } else {
                for (int i = 0; i < 4; i++) dx[4 * i + j] = fmaf(-cs, ci[it][j], dx[4 * i + j]) * ci[it][j];
            }
        }
        /* row step x = z * rinv: dz = (dx - sum_l dx_il x_il) rinv_i (exact), or
         * the reference's (dx - r rinv) rinv (sinkhorn_knopp.cuh:1182-1201) */
        for (int i = 0; i < 4; i++) {
            const float* d4 = dx + 4 * i;
            const float* x4 = xr + 4 * i;
            float rs;
            if (exact) {
                rs = d4[0] * x4[0];
                rs = fmaf(d4[1], x4[1], rs);
                rs = fmaf(d4[2], x4[2], rs);
                rs = fmaf(d4[3], x4[3], rs);
            } else {
                rs = fmaf(d4[3], x4[3], fmaf(d4[2], x4[2], fmaf(d4[0], x4[0], d4[1] * x4[1])));
            }
            if (exact) { /* fma(dx, rinv, -(rs rinv)) */
                const float t = rs * ri[it][i];
                for (int j = 0; j < 4; j++) dx[4 * i + j] = fmaf(dx[4 * i + j], ri[it][i], -t);
            } else {
                const float sub = rs * ri[it][i];
                for (int j = 0; j < 4; j++) dx[4 * i + j] = (dx[4 * i + j] - sub) * ri[it][i];
            }
        }
    }
    memcpy(D, dx, sizeof(dx));
}

/* ---------------------------------------------------------------------------
 * Exported batch entry points.  nthreads <= 0 uses one thread per online CPU.
 * The batch is cut into contiguous slices, one per pthread.
 * ------------------------------------------------------------------------ */

typedef void (*batch_fn)(void* ctx, int64_t begin, int64_t end);

typedef struct {
    batch_fn fn;
    void* ctx;
    int64_t begin, end;
} slice_arg;

static void* slice_main(void* p)
{
    slice_arg* a = (slice_arg*)p;
    const unsigned int saved = _mm_getcsr();
    set_ftz_daz();
    a->fn(a->ctx, a->begin, a->end);
    _mm_setcsr(saved); /* the calling thread runs a slice too: leave its mode as found */
    return NULL;
}

#define ORACLE_MAX_THREADS 512

int oracle_max_threads(void)
{
    long n = sysconf(_SC_NPROCESSORS_ONLN);
    if (n < 1) n = 1;
    if (n > ORACLE_MAX_THREADS) n = ORACLE_MAX_THREADS;
    return (int)n;
}

static void run_batch(batch_fn fn, void* ctx, int64_t N, int nthreads)
{
    int nt = nthreads > 0 ? nthreads : oracle_max_threads();
    if (nt > ORACLE_MAX_THREADS) nt = ORACLE_MAX_THREADS;
    if ((int64_t)nt > N) nt = (int)(N > 0 ? N : 1);
    slice_arg args[ORACLE_MAX_THREADS];
    pthread_t tids[ORACLE_MAX_THREADS];
    int started[ORACLE_MAX_THREADS];
    for (int t = 0; t < nt; t++) {
        args[t].fn = fn;
        args[t].ctx = ctx;
        args[t].begin = N * t / nt;
        args[t].end = N * (t + 1) / nt;
        started[t] = 0;
    }
    for (int t = 1; t < nt; t++)
        started[t] = pthread_create(&tids[t], NULL, slice_main, &args[t]) == 0;
    /* the calling thread does slice 0, and any slice whose thread failed to start */
    slice_main(&args[0]);
    for (int t = 1; t < nt; t++) {
        if (started[t]) pthread_join(tids[t], NULL);
        else slice_main(&args[t]);
    }
}

typedef struct { const float* R; float* T; float tol; int32_t* evals; } newton_ctx;
static void newton_range(void* p, int64_t b0, int64_t b1)
{
    newton_ctx* c = (newton_ctx*)p;
    for (int64_t b = b0; b < b1; b++) {
        const int e = newton_one(c->R + 16 * b, c->T + 16 * b, c->tol);
        if (c->evals) c->evals[b] = e;
    }
}

void oracle_birkhoff_proj_n4(const float* R, float* T, float tol, int64_t N,
                             int32_t* evals, int nthreads)
{
    newton_ctx c = {R, T, tol, evals};
    run_batch(newton_range, &c, N, nthreads);
}

typedef struct { const float* R; float* T; float tol; int candidates; int32_t* iters; } newton_ls_ctx;
static void newton_ls_range(void* p, int64_t b0, int64_t b1)
{
    newton_ls_ctx* c = (newton_ls_ctx*)p;
    for (int64_t b = b0; b < b1; b++) {
        int it = 0;
        newton_one_ls(c->R + 16 * b, c->T + 16 * b, c->tol, c->candidates, &it);
        if (c->iters) c->iters[b] = it;
    }
}

/* The forward with the line search cut to `candidates` steps (1..5; 5 is
 * the reference).  Returns -1 for a count outside 1..5. */
int oracle_birkhoff_proj_n4_line_search(const float* R, float* T, float tol, int64_t N, int candidates,
                                        int32_t* iters, int nthreads)
{
    if (candidates < 1 || candidates > LINE_SEARCH_MAX_ITERS) return -1;
    newton_ls_ctx c = {R, T, tol, candidates, iters};
    run_batch(newton_ls_range, &c, N, nthreads);
    return 0;
}

typedef struct { const float* G; const float* T; float* D; } ift_ctx;
static void ift_range(void* p, int64_t b0, int64_t b1)
{
    ift_ctx* c = (ift_ctx*)p;
    for (int64_t b = b0; b < b1; b++) ift_one(c->G + 16 * b, c->T + 16 * b, c->D + 16 * b);
}

void oracle_birkhoff_proj_n4_backward(const float* G, const float* T, float* D,
                                      int64_t N, int nthreads)
{
    ift_ctx c = {G, T, D};
    run_batch(ift_range, &c, N, nthreads);
}

typedef struct { const float* M; float* T; int iters; float eps; } skf_ctx;
static void skf_range(void* p, int64_t b0, int64_t b1)
{
    skf_ctx* c = (skf_ctx*)p;
    for (int64_t b = b0; b < b1; b++) sk_forward_one(c->M + 16 * b, c->T + 16 * b, c->iters, c->eps);
}

void oracle_sinkhorn_knopp_n4(const float* M, float* T, int64_t N, int iters,
                              float eps, int nthreads)
{
    skf_ctx c = {M, T, iters, eps};
    run_batch(skf_range, &c, N, nthreads);
}

typedef struct { const float* G; const float* M; float* D; int iters; float eps; int exact; } skb_ctx;
static void skb_range(void* p, int64_t b0, int64_t b1)
{
    skb_ctx* c = (skb_ctx*)p;
    for (int64_t b = b0; b < b1; b++)
        sk_backward_one(c->G + 16 * b, c->M + 16 * b, c->D + 16 * b, c->iters, c->eps, c->exact);
}

/* Returns -1 when iters exceeds the oracle's checkpoint capacity. */
int oracle_sinkhorn_knopp_n4_backward(const float* G, const float* M, float* D,
                                      int64_t N, int iters, float eps, int exact,
                                      int nthreads)
{
    if (iters < 0 || iters > SK_MAX_ITERS) return -1;
    skb_ctx c = {G, M, D, iters, eps, exact};
    run_batch(skb_range, &c, N, nthreads);
    return 0;
}
