/*
 * nw_oracle.c -- CPU restatement of d2p's soft Needleman-Wunsch (global
 * alignment, linear gap penalty).
 *
 * TEST INFRASTRUCTURE ONLY.  Nothing in the d2p_b200 product path links,
 * loads or calls this file; it is the checker used by tests/ and by
 * bench-side CPU baselines.
 *
 * It restates, cell for cell, the reference's CPU algorithm
 * src/nw/kernels_cpu.cpp:
 *   3-option softmax weights  :43-64   forward   :79-155
 *   backward (posteriors,     :161-262 hvp       :271-441
 *     dS/dgap, dS/dT)                  param grad:450-642
 *   numerics                  : src/common/numerics.h:23-80 (NINF=-1e30,
 *                               safe_exp clamp at +-88, Kahan-summed
 *                               logsumexp)
 * The file is compiled twice (REAL=float -> *_f32, REAL=double -> *_f64):
 * the f32 build follows the reference's float arithmetic, the f64 build is
 * the noise-floor reference.
 *
 * Layout is the reference's: scores [B,L1,L2] row-major, lengths [B,2]
 * int32, DP planes [B,(L1+1)*(L2+1)] row-major over (i, j).  Cells are
 * visited by anti-diagonal k = i + j, i ascending, as the reference does.
 */
#include <math.h>
#include <stddef.h>
#include <string.h>

#ifdef ORACLE_F64
#define REAL double
#define SFX(name) name##_f64
#define R_EXP exp
#define R_LOG log
#else
#define REAL float
#define SFX(name) name##_f32
/* float exp / log as the reference calls them (std::exp, std::log on float) */
#define R_EXP expf
#define R_LOG logf
#endif

#define N_NINF ((REAL)-1e30)

typedef struct {
    REAL sum, c;
} nk_t;

static inline void nk_add(nk_t *k, REAL v) {
    REAL y = v - k->c;
    REAL t = k->sum + y;
    k->c = (t - k->sum) - y;
    k->sum = t;
}

static inline REAL n_exp(REAL x) {
    if (x < (REAL)-88) return (REAL)0;
    if (x > (REAL)88) x = (REAL)88;
    return R_EXP(x);
}

static inline REAL n_max3(REAL a, REAL b, REAL c) {
    REAL m = a > b ? a : b;
    return m > c ? m : c;
}

/* numerics.h:72-80 */
static inline REAL n_lse3(REAL a, REAL b, REAL c, REAL T) {
    REAL m = n_max3(a, b, c);
    if (m <= N_NINF) return N_NINF;
    nk_t k = {0, 0};
    nk_add(&k, n_exp((a - m) / T));
    nk_add(&k, n_exp((b - m) / T));
    nk_add(&k, n_exp((c - m) / T));
    return m + T * R_LOG(k.sum);
}

/* kernels_cpu.cpp:43-64: normalised weights, 0 for -inf options */
static void n_softmax3(REAL a, REAL b, REAL c, REAL T, REAL *wa, REAL *wb, REAL *wc) {
    REAL m = n_max3(a, b, c);
    if (m <= N_NINF) {
        *wa = *wb = *wc = 0;
        return;
    }
    nk_t k = {0, 0};
    if (a > N_NINF) { *wa = n_exp((a - m) / T); nk_add(&k, *wa); } else { *wa = 0; }
    if (b > N_NINF) { *wb = n_exp((b - m) / T); nk_add(&k, *wb); } else { *wb = 0; }
    if (c > N_NINF) { *wc = n_exp((c - m) / T); nk_add(&k, *wc); } else { *wc = 0; }
    if (k.sum > 0) {
        *wa /= k.sum;
        *wb /= k.sum;
        *wc /= k.sum;
    }
}

#define NA(i, j) ((size_t)(i) * cols + (size_t)(j))
#define NS(i, j) ((size_t)((i) - 1) * (size_t)L2max + (size_t)((j) - 1))

/* iterate the interior cells of a problem by anti-diagonal, i ascending */
#define FOR_CELLS_FWD(L1, L2)                                      \
    for (int k = 2; k <= (L1) + (L2); ++k)                         \
        for (int i = (k - (L2) > 1 ? k - (L2) : 1), j;             \
             i <= ((L1) < k - 1 ? (L1) : k - 1) && (j = k - i, 1); ++i)
#define FOR_CELLS_REV(L1, L2)                                      \
    for (int k = (L1) + (L2); k >= 2; --k)                         \
        for (int i = (k - (L2) > 1 ? k - (L2) : 1), j;             \
             i <= ((L1) < k - 1 ? (L1) : k - 1) && (j = k - i, 1); ++i)

/* kernels_cpu.cpp:79-155 */
static REAL nw_forward_one(const REAL *s, REAL *a, int L1, int L2, int L1max, int L2max, REAL gap, REAL T) {
    const size_t cols = (size_t)L2max + 1;
    const size_t n = ((size_t)L1max + 1) * cols;
    for (size_t q = 0; q < n; ++q) a[q] = N_NINF;
    a[0] = 0;
    for (int i = 1; i <= L1; ++i) a[NA(i, 0)] = (REAL)i * gap;
    for (int j = 1; j <= L2; ++j) a[NA(0, j)] = (REAL)j * gap;
    FOR_CELLS_FWD(L1, L2) {
        REAL sc = s[NS(i, j)];
        a[NA(i, j)] = n_lse3(a[NA(i - 1, j - 1)] + sc, a[NA(i - 1, j)] + gap, a[NA(i, j - 1)] + gap, T);
    }
    return a[NA(L1, L2)];
}

/* kernels_cpu.cpp:161-262 */
static void nw_backward_one(const REAL *s, const REAL *a, REAL S, REAL *be, REAL *post, REAL *gg, REAL *gT,
                            int L1, int L2, int L1max, int L2max, REAL gap, REAL T) {
    const size_t cols = (size_t)L2max + 1;
    const size_t n = ((size_t)L1max + 1) * cols;
    memset(post, 0, sizeof(REAL) * (size_t)L1max * L2max);
    memset(be, 0, sizeof(REAL) * n);
    be[NA(L1, L2)] = 1;
    nk_t gsum = {0, 0}, msum = {0, 0};
    FOR_CELLS_REV(L1, L2) {
        REAL b = be[NA(i, j)];
        if (b == 0) continue;
        REAL sc = s[NS(i, j)];
        REAL wd, wu, wl;
        n_softmax3(a[NA(i - 1, j - 1)] + sc, a[NA(i - 1, j)] + gap, a[NA(i, j - 1)] + gap, T, &wd, &wu, &wl);
        REAL p = b * wd;
        post[NS(i, j)] = p;
        nk_add(&msum, p * sc);
        nk_add(&gsum, b * (wu + wl));
        if (wd > 0) be[NA(i - 1, j - 1)] += b * wd;
        if (wu > 0) be[NA(i - 1, j)] += b * wu;
        if (wl > 0) be[NA(i, j - 1)] += b * wl;
    }
    /* a path that reaches the boundary at (i,0) or (0,j) takes i or j more gaps */
    for (int i = 1; i <= L1; ++i) nk_add(&gsum, be[NA(i, 0)] * (REAL)i);
    for (int j = 1; j <= L2; ++j) nk_add(&gsum, be[NA(0, j)] * (REAL)j);
    *gg = gsum.sum;
    *gT = (S - (msum.sum + gsum.sum * gap)) / T;
}

/* kernels_cpu.cpp:271-441: forward tangent d alpha along V, then beta and
 * d beta in reverse; H = d beta w_diag + beta dw_diag */
static void nw_hvp_one(const REAL *s, const REAL *v, const REAL *a, REAL *da, REAL *be, REAL *dbe, REAL *H,
                       int L1, int L2, int L1max, int L2max, REAL gap, REAL T) {
    const size_t cols = (size_t)L2max + 1;
    const size_t n = ((size_t)L1max + 1) * cols;
    memset(da, 0, sizeof(REAL) * n);
    memset(be, 0, sizeof(REAL) * n);
    memset(dbe, 0, sizeof(REAL) * n);
    memset(H, 0, sizeof(REAL) * (size_t)L1max * L2max);
    FOR_CELLS_FWD(L1, L2) {
        REAL sc = s[NS(i, j)];
        REAL wd, wu, wl;
        n_softmax3(a[NA(i - 1, j - 1)] + sc, a[NA(i - 1, j)] + gap, a[NA(i, j - 1)] + gap, T, &wd, &wu, &wl);
        da[NA(i, j)] = wd * (da[NA(i - 1, j - 1)] + v[NS(i, j)]) + wu * da[NA(i - 1, j)] + wl * da[NA(i, j - 1)];
    }
    be[NA(L1, L2)] = 1;
    FOR_CELLS_REV(L1, L2) {
        REAL b = be[NA(i, j)], db = dbe[NA(i, j)];
        if (b == 0 && fabs((double)db) < 1e-20) continue;
        REAL sc = s[NS(i, j)];
        REAL wd, wu, wl;
        n_softmax3(a[NA(i - 1, j - 1)] + sc, a[NA(i - 1, j)] + gap, a[NA(i, j - 1)] + gap, T, &wd, &wu, &wl);
        REAL dvd = da[NA(i - 1, j - 1)] + v[NS(i, j)], dvu = da[NA(i - 1, j)], dvl = da[NA(i, j - 1)];
        REAL E = wd * dvd + wu * dvu + wl * dvl;
        REAL dwd = wd * (dvd - E) / T, dwu = wu * (dvu - E) / T, dwl = wl * (dvl - E) / T;
        H[NS(i, j)] = db * wd + b * dwd;
        if (wd > 0) { be[NA(i - 1, j - 1)] += b * wd; dbe[NA(i - 1, j - 1)] += db * wd + b * dwd; }
        if (wu > 0) { be[NA(i - 1, j)] += b * wu; dbe[NA(i - 1, j)] += db * wu + b * dwu; }
        if (wl > 0) { be[NA(i, j - 1)] += b * wl; dbe[NA(i, j - 1)] += db * wl + b * dwl; }
    }
}

/* kernels_cpu.cpp:450-642: U = d alpha / d theta forward (the gap tangent
 * starts at i or j on the boundary), beta and W = d beta / d theta in reverse,
 * dP/dtheta = W w_diag + beta dw_diag.  param_type 0 = gap, 1 = temperature. */
static void nw_param_one(const REAL *s, const REAL *a, REAL *u, REAL *be, REAL *w, REAL *dP, int L1, int L2,
                         int L1max, int L2max, REAL gap, REAL T, int param_type) {
    const size_t cols = (size_t)L2max + 1;
    const size_t n = ((size_t)L1max + 1) * cols;
    memset(u, 0, sizeof(REAL) * n);
    memset(be, 0, sizeof(REAL) * n);
    memset(w, 0, sizeof(REAL) * n);
    memset(dP, 0, sizeof(REAL) * (size_t)L1max * L2max);
    if (param_type == 0) {
        for (int i = 1; i <= L1; ++i) u[NA(i, 0)] = (REAL)i;
        for (int j = 1; j <= L2; ++j) u[NA(0, j)] = (REAL)j;
    }
    const REAL g1 = param_type == 0 ? (REAL)1 : (REAL)0;
    FOR_CELLS_FWD(L1, L2) {
        REAL sc = s[NS(i, j)];
        REAL vd = a[NA(i - 1, j - 1)] + sc, vu = a[NA(i - 1, j)] + gap, vl = a[NA(i, j - 1)] + gap;
        REAL wd, wu, wl;
        n_softmax3(vd, vu, vl, T, &wd, &wu, &wl);
        REAL U = wd * u[NA(i - 1, j - 1)] + wu * (u[NA(i - 1, j)] + g1) + wl * (u[NA(i, j - 1)] + g1);
        if (param_type == 1) U += (a[NA(i, j)] - (wd * vd + wu * vu + wl * vl)) / T;
        u[NA(i, j)] = U;
    }
    be[NA(L1, L2)] = 1;
    FOR_CELLS_REV(L1, L2) {
        REAL b = be[NA(i, j)], W = w[NA(i, j)];
        if (b == 0 && fabs((double)W) < 1e-20) continue;
        REAL sc = s[NS(i, j)];
        REAL vd = a[NA(i - 1, j - 1)] + sc, vu = a[NA(i - 1, j)] + gap, vl = a[NA(i, j - 1)] + gap;
        REAL wd, wu, wl;
        n_softmax3(vd, vu, vl, T, &wd, &wu, &wl);
        REAL ud = u[NA(i - 1, j - 1)], uu = u[NA(i - 1, j)] + g1, ul = u[NA(i, j - 1)] + g1;
        REAL E = wd * ud + wu * uu + wl * ul;
        REAL dwd = wd * (ud - E) / T, dwu = wu * (uu - E) / T, dwl = wl * (ul - E) / T;
        if (param_type == 1) {
            REAL Ev = wd * vd + wu * vu + wl * vl;
            REAL iT2 = (REAL)1 / (T * T);
            dwd += wd * (Ev - vd) * iT2;
            dwu += wu * (Ev - vu) * iT2;
            dwl += wl * (Ev - vl) * iT2;
        }
        dP[NS(i, j)] = W * wd + b * dwd;
        if (wd > 0) { be[NA(i - 1, j - 1)] += b * wd; w[NA(i - 1, j - 1)] += W * wd + b * dwd; }
        if (wu > 0) { be[NA(i - 1, j)] += b * wu; w[NA(i - 1, j)] += W * wu + b * dwu; }
        if (wl > 0) { be[NA(i, j - 1)] += b * wl; w[NA(i, j - 1)] += W * wl + b * dwl; }
    }
}

/* ------------------------------------------------------------------ batch API */
static inline void n_lens(const int *lengths, int b, int L1max, int L2max, int *L1, int *L2) {
    *L1 = lengths ? lengths[2 * b] : L1max;
    *L2 = lengths ? lengths[2 * b + 1] : L2max;
}

void SFX(oracle_nw_forward)(const REAL *scores, const int *lengths, int B, int L1max, int L2max, REAL gap,
                            REAL T, REAL *alpha, REAL *value) {
    const size_t sp = (size_t)L1max * L2max, ap = ((size_t)L1max + 1) * ((size_t)L2max + 1);
#pragma omp parallel for schedule(dynamic, 1)
    for (int b = 0; b < B; ++b) {
        int L1, L2;
        n_lens(lengths, b, L1max, L2max, &L1, &L2);
        value[b] = nw_forward_one(scores + b * sp, alpha + b * ap, L1, L2, L1max, L2max, gap, T);
    }
}

void SFX(oracle_nw_backward)(const REAL *scores, const int *lengths, int B, int L1max, int L2max, REAL gap,
                             REAL T, const REAL *alpha, const REAL *value, REAL *beta, REAL *post, REAL *grad_gap,
                             REAL *grad_T) {
    const size_t sp = (size_t)L1max * L2max, ap = ((size_t)L1max + 1) * ((size_t)L2max + 1);
#pragma omp parallel for schedule(dynamic, 1)
    for (int b = 0; b < B; ++b) {
        int L1, L2;
        n_lens(lengths, b, L1max, L2max, &L1, &L2);
        nw_backward_one(scores + b * sp, alpha + b * ap, value[b], beta + b * ap, post + b * sp, grad_gap + b,
                        grad_T + b, L1, L2, L1max, L2max, gap, T);
    }
}

void SFX(oracle_nw_hvp)(const REAL *scores, const REAL *V, const int *lengths, int B, int L1max, int L2max,
                        REAL gap, REAL T, const REAL *alpha, REAL *d_alpha, REAL *beta, REAL *d_beta, REAL *H) {
    const size_t sp = (size_t)L1max * L2max, ap = ((size_t)L1max + 1) * ((size_t)L2max + 1);
#pragma omp parallel for schedule(dynamic, 1)
    for (int b = 0; b < B; ++b) {
        int L1, L2;
        n_lens(lengths, b, L1max, L2max, &L1, &L2);
        nw_hvp_one(scores + b * sp, V + b * sp, alpha + b * ap, d_alpha + b * ap, beta + b * ap, d_beta + b * ap,
                   H + b * sp, L1, L2, L1max, L2max, gap, T);
    }
}

void SFX(oracle_nw_param_grad)(const REAL *scores, const int *lengths, int B, int L1max, int L2max, REAL gap,
                               REAL T, const REAL *alpha, REAL *U, REAL *beta, REAL *W, REAL *dP, int param_type) {
    const size_t sp = (size_t)L1max * L2max, ap = ((size_t)L1max + 1) * ((size_t)L2max + 1);
#pragma omp parallel for schedule(dynamic, 1)
    for (int b = 0; b < B; ++b) {
        int L1, L2;
        n_lens(lengths, b, L1max, L2max, &L1, &L2);
        nw_param_one(scores + b * sp, alpha + b * ap, U + b * ap, beta + b * ap, W + b * ap, dP + b * sp, L1, L2,
                     L1max, L2max, gap, T, param_type);
    }
}
