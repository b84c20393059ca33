/*
 * dtw_oracle.c -- CPU restatement of d2p's soft dynamic time warping (softmin
 * over the three predecessors, optional Sakoe-Chiba band).
 *
 * TEST INFRASTRUCTURE ONLY.  Nothing in the d2p_b200 product path links,
 * loads or calls this file; it is the checker used by tests/.
 *
 * It restates, cell for cell, the reference's CPU algorithm
 * src/dtw/kernels_cpu.cpp:
 *   band test, softmin weights  :23-52    forward  :58-128
 *   backward (posteriors = beta, dS/dT) :134-230
 *   hvp                         :236-375   param grad (temperature) :381-534
 *   numerics: src/common/numerics.h (PINF = 1e30, safe_exp clamp at +-88,
 *   Kahan-summed softmin3 :97-105)
 * alpha[0,0] = 0, every other cell +inf until reached; alpha[i,j] = c_ij +
 * softmin_T(alpha diag, up, left) for cells inside the band; the value is
 * alpha[L1, L2] and the marginals are the visit probabilities beta.
 *
 * Compiled twice (REAL=float -> *_f32, REAL=double -> *_f64): the f32 build
 * follows the reference's float arithmetic and operation order, the f64 build
 * is the noise-floor reference.  Planes [B][(L1+1)(L2+1)] row-major over
 * (i, j); cells visited by anti-diagonal, i ascending.
 */
#include <math.h>
#include <stddef.h>
#include <stdint.h>
#include <string.h>

#ifdef ORACLE_F64
#define REAL double
#define SFX(name) name##_f64
#define R_EXP exp
#define R_LOG log
#else
#define REAL float
#define SFX(name) name##_f32
#define R_EXP expf
#define R_LOG logf
#endif

#define D_PINF ((REAL)1e30)

typedef struct {
    REAL sum, c;
} dk_t;

static inline void dk_add(dk_t *k, REAL v) {
    REAL y = v - k->c;
    REAL t = k->sum + y;
    k->c = (t - k->sum) - y;
    k->sum = t;
}

static inline REAL d_exp(REAL x) {
    if (x < (REAL)-88) return (REAL)0;
    if (x > (REAL)88) x = (REAL)88;
    return R_EXP(x);
}

static inline REAL d_min3(REAL a, REAL b, REAL c) {
    REAL m = a < b ? a : b;
    return m < c ? m : c;
}

/* the band test is float arithmetic in the reference, in both builds here */
static inline int d_in_band(int i, int j, int L1, int L2, int64_t bw) {
    if (bw < 0) return 1;
    if (L1 == 0 || L2 == 0) return 1;
    float e = (float)((int64_t)i * L2) / (float)L1;
    return fabsf((float)j - e) <= (float)bw;
}

/* numerics.h:97-105 */
static inline REAL d_softmin3(REAL a, REAL b, REAL c, REAL T) {
    REAL m = d_min3(a, b, c);
    if (m >= D_PINF) return D_PINF;
    dk_t k = {0, 0};
    dk_add(&k, d_exp((m - a) / T));
    dk_add(&k, d_exp((m - b) / T));
    dk_add(&k, d_exp((m - c) / T));
    return m - T * R_LOG(k.sum);
}

/* kernels_cpu.cpp:31-52 */
static inline void d_w3(REAL a, REAL b, REAL c, REAL T, REAL *wa, REAL *wb, REAL *wc) {
    REAL m = d_min3(a, b, c);
    if (m >= D_PINF) {
        *wa = *wb = *wc = 0;
        return;
    }
    REAL ea = a < D_PINF ? d_exp((m - a) / T) : (REAL)0;
    REAL eb = b < D_PINF ? d_exp((m - b) / T) : (REAL)0;
    REAL ec = c < D_PINF ? d_exp((m - c) / T) : (REAL)0;
    REAL tot = ea + eb + ec;
    if (tot > 0) {
        *wa = ea / tot;
        *wb = eb / tot;
        *wc = ec / tot;
    } else {
        *wa = *wb = *wc = 0;
    }
}

#define DA(i, j) ((size_t)(i) * cols + (size_t)(j))
#define DS(i, j) ((size_t)((i) - 1) * (size_t)L2max + (size_t)((j) - 1))
#define D_FWD(L1, L2)                                               \
    for (int k = 2; k <= (L1) + (L2); ++k)                          \
        for (int i = (k - (L2) > 1 ? k - (L2) : 1), j;              \
             i <= ((L1) < k - 1 ? (L1) : k - 1) && (j = k - i, 1); ++i)
#define D_REV(L1, L2)                                               \
    for (int k = (L1) + (L2); k >= 2; --k)                          \
        for (int i = (k - (L2) > 1 ? k - (L2) : 1), j;              \
             i <= ((L1) < k - 1 ? (L1) : k - 1) && (j = k - i, 1); ++i)

/* the predecessors' alphas, +inf outside the band */
#define PREDS(a, i, j, bw)                                                     \
    REAL a_d = a[DA(i - 1, j - 1)], a_u = a[DA(i - 1, j)], a_l = a[DA(i, j - 1)]; \
    const int b_d = d_in_band(i - 1, j - 1, L1, L2, bw), b_u = d_in_band(i - 1, j, L1, L2, bw), \
              b_l = d_in_band(i, j - 1, L1, L2, bw);                          \
    if (!b_d) a_d = D_PINF;                                                    \
    if (!b_u) a_u = D_PINF;                                                    \
    if (!b_l) a_l = D_PINF

/* :58-128 */
static REAL dtw_forward_one(const REAL *c, REAL *a, int L1, int L2, int L1max, int L2max, REAL T, int64_t bw) {
    const size_t cols = (size_t)L2max + 1, n = ((size_t)L1max + 1) * cols;
    for (size_t q = 0; q < n; ++q) a[q] = D_PINF;
    a[0] = 0;
    D_FWD(L1, L2) {
        if (!d_in_band(i, j, L1, L2, bw)) continue;
        PREDS(a, i, j, bw);
        (void)b_d;
        (void)b_u;
        (void)b_l;
        a[DA(i, j)] = c[DS(i, j)] + d_softmin3(a_d, a_u, a_l, T);
    }
    return a[DA(L1, L2)];
}

/* :134-230 */
static void dtw_backward_one(const REAL *c, const REAL *a, REAL *be, REAL *post, REAL *gT, int L1, int L2,
                             int L1max, int L2max, REAL T, int64_t bw) {
    const size_t cols = (size_t)L2max + 1, n = ((size_t)L1max + 1) * cols;
    memset(post, 0, sizeof(REAL) * (size_t)L1max * L2max);
    memset(be, 0, sizeof(REAL) * n);
    be[DA(L1, L2)] = 1;
    REAL st = 0;
    D_REV(L1, L2) {
        if (!d_in_band(i, j, L1, L2, bw)) continue;
        REAL b = be[DA(i, j)];
        if (b == 0) continue;
        post[DS(i, j)] = b;
        PREDS(a, i, j, bw);
        REAL wd, wu, wl;
        d_w3(a_d, a_u, a_l, T, &wd, &wu, &wl);
        if (b_d && wd > 0) be[DA(i - 1, j - 1)] += b * wd;
        if (b_u && wu > 0) be[DA(i - 1, j)] += b * wu;
        if (b_l && wl > 0) be[DA(i, j - 1)] += b * wl;
        REAL sv = a[DA(i, j)] - c[DS(i, j)];
        if (sv < D_PINF) {
            REAL Ea = wd * a_d + wu * a_u + wl * a_l;
            st += b * (sv - Ea) / T;
        }
    }
    *gT = st;
}

/* :236-375 */
static void dtw_hvp_one(const REAL *c, const REAL *v, const REAL *a, REAL *da, REAL *be, REAL *dbe, REAL *H, int L1,
                        int L2, int L1max, int L2max, REAL T, int64_t bw) {
    const size_t cols = (size_t)L2max + 1, n = ((size_t)L1max + 1) * cols;
    (void)c;
    memset(da, 0, sizeof(REAL) * n);
    memset(be, 0, sizeof(REAL) * n);
    memset(dbe, 0, sizeof(REAL) * n);
    memset(H, 0, sizeof(REAL) * (size_t)L1max * L2max);
    D_FWD(L1, L2) {
        if (!d_in_band(i, j, L1, L2, bw)) continue;
        PREDS(a, i, j, bw);
        REAL wd, wu, wl;
        d_w3(a_d, a_u, a_l, T, &wd, &wu, &wl);
        REAL dd = b_d ? da[DA(i - 1, j - 1)] : (REAL)0, du = b_u ? da[DA(i - 1, j)] : (REAL)0,
             dl = b_l ? da[DA(i, j - 1)] : (REAL)0;
        da[DA(i, j)] = v[DS(i, j)] + wd * dd + wu * du + wl * dl;
    }
    be[DA(L1, L2)] = 1;
    dbe[DA(L1, L2)] = 0;
    D_REV(L1, L2) {
        if (!d_in_band(i, j, L1, L2, bw)) continue;
        REAL b = be[DA(i, j)], db = dbe[DA(i, j)];
        if (b == 0) continue;
        PREDS(a, i, j, bw);
        REAL wd, wu, wl;
        d_w3(a_d, a_u, a_l, T, &wd, &wu, &wl);
        REAL dd = b_d ? da[DA(i - 1, j - 1)] : (REAL)0, du = b_u ? da[DA(i - 1, j)] : (REAL)0,
             dl = b_l ? da[DA(i, j - 1)] : (REAL)0;
        REAL E = wd * dd + wu * du + wl * dl;
        REAL ed = wd * (-dd + E) / T, eu = wu * (-du + E) / T, el = wl * (-dl + E) / T;
        H[DS(i, j)] = db;
        if (b_d && wd > 0) { be[DA(i - 1, j - 1)] += b * wd; dbe[DA(i - 1, j - 1)] += db * wd + b * ed; }
        if (b_u && wu > 0) { be[DA(i - 1, j)] += b * wu; dbe[DA(i - 1, j)] += db * wu + b * eu; }
        if (b_l && wl > 0) { be[DA(i, j - 1)] += b * wl; dbe[DA(i, j - 1)] += db * wl + b * el; }
    }
}

/* :381-534: dP/dT */
static void dtw_param_one(const REAL *c, const REAL *a, REAL *u, REAL *be, REAL *w, REAL *dP, int L1, int L2,
                          int L1max, int L2max, REAL T, int64_t bw) {
    const size_t cols = (size_t)L2max + 1, n = ((size_t)L1max + 1) * cols;
    memset(u, 0, sizeof(REAL) * n);
    memset(be, 0, sizeof(REAL) * n);
    memset(w, 0, sizeof(REAL) * n);
    memset(dP, 0, sizeof(REAL) * (size_t)L1max * L2max);
    D_FWD(L1, L2) {
        if (!d_in_band(i, j, L1, L2, bw)) continue;
        PREDS(a, i, j, bw);
        REAL wd, wu, wl;
        d_w3(a_d, a_u, a_l, T, &wd, &wu, &wl);
        REAL ud = b_d ? u[DA(i - 1, j - 1)] : (REAL)0, uu = b_u ? u[DA(i - 1, j)] : (REAL)0,
             ul = b_l ? u[DA(i, j - 1)] : (REAL)0;
        REAL sv = a[DA(i, j)] - c[DS(i, j)];
        REAL Ea = wd * a_d + wu * a_u + wl * a_l;
        u[DA(i, j)] = (sv - Ea) / T + wd * ud + wu * uu + wl * ul;
    }
    be[DA(L1, L2)] = 1;
    w[DA(L1, L2)] = 0;
    D_REV(L1, L2) {
        if (!d_in_band(i, j, L1, L2, bw)) continue;
        REAL b = be[DA(i, j)], W = w[DA(i, j)];
        if (b == 0 && fabs((double)W) < (double)1e-20f) continue;
        dP[DS(i, j)] = W;
        PREDS(a, i, j, bw);
        REAL wd, wu, wl;
        d_w3(a_d, a_u, a_l, T, &wd, &wu, &wl);
        REAL ud = b_d ? u[DA(i - 1, j - 1)] : (REAL)0, uu = b_u ? u[DA(i - 1, j)] : (REAL)0,
             ul = b_l ? u[DA(i, j - 1)] : (REAL)0;
        REAL Ea = wd * a_d + wu * a_u + wl * a_l;
        REAL Eu = wd * ud + wu * uu + wl * ul;
        REAL iT = (REAL)1 / T;
        REAL iT2 = iT * iT;
        REAL ed = wd * ((Eu - ud) * iT + (a_d - Ea) * iT2);
        REAL eu = wu * ((Eu - uu) * iT + (a_u - Ea) * iT2);
        REAL el = wl * ((Eu - ul) * iT + (a_l - Ea) * iT2);
        if (b_d && wd > 0) { be[DA(i - 1, j - 1)] += b * wd; w[DA(i - 1, j - 1)] += W * wd + b * ed; }
        if (b_u && wu > 0) { be[DA(i - 1, j)] += b * wu; w[DA(i - 1, j)] += W * wu + b * eu; }
        if (b_l && wl > 0) { be[DA(i, j - 1)] += b * wl; w[DA(i, j - 1)] += W * wl + b * el; }
    }
}

/* ------------------------------------------------------------------ batch API
 * lengths [B, 2] is required, as in the reference's kernels. */
void SFX(oracle_dtw_forward)(const REAL *costs, const int *lengths, int B, int L1max, int L2max, REAL T, int64_t bw,
                             REAL *alpha, REAL *value) {
    const size_t sp = (size_t)L1max * L2max, ap = ((size_t)L1max + 1) * ((size_t)L2max + 1);
#pragma omp parallel for schedule(dynamic, 1)
    for (int b = 0; b < B; ++b)
        value[b] = dtw_forward_one(costs + b * sp, alpha + b * ap, lengths[2 * b], lengths[2 * b + 1], L1max, L2max,
                                   T, bw);
}

void SFX(oracle_dtw_backward)(const REAL *costs, const int *lengths, int B, int L1max, int L2max, REAL T, int64_t bw,
                              const REAL *alpha, REAL *beta, REAL *post, REAL *grad_T) {
    const size_t sp = (size_t)L1max * L2max, ap = ((size_t)L1max + 1) * ((size_t)L2max + 1);
#pragma omp parallel for schedule(dynamic, 1)
    for (int b = 0; b < B; ++b)
        dtw_backward_one(costs + b * sp, alpha + b * ap, beta + b * ap, post + b * sp, grad_T + b, lengths[2 * b],
                         lengths[2 * b + 1], L1max, L2max, T, bw);
}

void SFX(oracle_dtw_hvp)(const REAL *costs, const REAL *V, const int *lengths, int B, int L1max, int L2max, REAL T,
                         int64_t bw, const REAL *alpha, REAL *d_alpha, REAL *beta, REAL *d_beta, REAL *H) {
    const size_t sp = (size_t)L1max * L2max, ap = ((size_t)L1max + 1) * ((size_t)L2max + 1);
#pragma omp parallel for schedule(dynamic, 1)
    for (int b = 0; b < B; ++b)
        dtw_hvp_one(costs + b * sp, V + b * sp, alpha + b * ap, d_alpha + b * ap, beta + b * ap, d_beta + b * ap,
                    H + b * sp, lengths[2 * b], lengths[2 * b + 1], L1max, L2max, T, bw);
}

void SFX(oracle_dtw_param_grad)(const REAL *costs, const int *lengths, int B, int L1max, int L2max, REAL T,
                                int64_t bw, const REAL *alpha, REAL *U, REAL *beta, REAL *W, REAL *dP) {
    const size_t sp = (size_t)L1max * L2max, ap = ((size_t)L1max + 1) * ((size_t)L2max + 1);
#pragma omp parallel for schedule(dynamic, 1)
    for (int b = 0; b < B; ++b)
        dtw_param_one(costs + b * sp, alpha + b * ap, U + b * ap, beta + b * ap, W + b * ap, dP + b * sp,
                      lengths[2 * b], lengths[2 * b + 1], L1max, L2max, T, bw);
}
