/*
 * sw_oracle.c -- CPU restatement of d2p's soft Smith-Waterman algorithms.
 *
 * TEST INFRASTRUCTURE ONLY.  Nothing in the d2p_b200 product path links,
 * loads or calls this file; it is the checker used by tests/, by
 * __graft_entry__.smoke() and by bench.py's cpu_baseline leg.
 *
 * It restates, cell for cell, the CPU algorithms of the reference:
 *   linear gap : src/sw/kernels_cpu.cpp        (forward :70-150,
 *                backward :156-279, hvp :288-485, param grad :500-710)
 *   affine gap : src/sw_affine/kernels_cpu.cpp (forward :94-193,
 *                backward :199-346, hvp :352-620, param grad :630-921)
 *   numerics   : src/common/numerics.h:20-84  (NINF=-1e30, safe_exp clamp
 *                at +-88, Kahan-summed logsumexp)
 * The file is compiled twice (REAL=float -> *_f32, REAL=double -> *_f64).
 * The f32 build follows the reference's float arithmetic; the f64 build is
 * the same algorithm in double precision and serves as the noise-floor
 * reference ("truth") when fp32 implementations are compared.
 *
 * Layout conventions are the reference's: scores [B,L1,L2] row-major,
 * lengths [B,2] int32, DP planes [B, S*(L1+1)*(L2+1)] (S = 1 linear, 3
 * affine: planes M|I|D).  Cells are visited in anti-diagonal order exactly
 * as the reference does, so the order of floating-point accumulation is
 * the same as the reference CPU path.
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

#define O_NINF ((REAL)-1e30)

typedef struct {
    REAL sum, c;
} kahan_t;

static inline void kahan_add(kahan_t *k, REAL v) {
    REAL y = v - k->c;
    REAL t = k->sum + y;
    k->c = (t - k->sum) - y;
    k->sum = t;
}

/* numerics.h:30-34 */
static inline REAL o_safe_exp(REAL x) {
    if (x < (REAL)-88) return (REAL)0;
    if (x > (REAL)88) x = (REAL)88;
    return R_EXP(x);
}

static inline REAL o_max2(REAL a, REAL b) { return a > b ? a : b; }
static inline REAL o_min2(REAL a, REAL b) { return a < b ? a : b; }
static inline REAL o_max4(REAL a, REAL b, REAL c, REAL d) {
    return o_max2(o_max2(a, b), o_max2(c, d));
}

/* numerics.h:62-71 / :84-95 : T*log(sum exp(x/T)) with Kahan summation */
static inline REAL o_lse2(REAL a, REAL b, REAL T) {
    REAL m = o_max2(a, b);
    if (m <= O_NINF) return O_NINF;
    kahan_t k = {0, 0};
    kahan_add(&k, o_safe_exp((a - m) / T));
    kahan_add(&k, o_safe_exp((b - m) / T));
    return m + T * R_LOG(k.sum);
}

static inline REAL o_lse4(REAL a, REAL b, REAL c, REAL d, REAL T) {
    REAL m = o_max4(a, b, c, d);
    if (m <= O_NINF) return O_NINF;
    kahan_t k = {0, 0};
    kahan_add(&k, o_safe_exp((a - m) / T));
    kahan_add(&k, o_safe_exp((b - m) / T));
    kahan_add(&k, o_safe_exp((c - m) / T));
    kahan_add(&k, o_safe_exp((d - m) / T));
    return m + T * R_LOG(k.sum);
}

/* softmax weights with -inf options forced to 0
 * (src/sw/kernels_cpu.cpp:41-62, src/sw_affine/kernels_cpu.cpp:53-87) */
static void o_softmax(const REAL *v, int n, REAL T, REAL *w) {
    REAL m = v[0];
    for (int q = 1; q < n; ++q) m = o_max2(m, v[q]);
    if (m <= O_NINF) {
        for (int q = 0; q < n; ++q) w[q] = 0;
        return;
    }
    kahan_t k = {0, 0};
    for (int q = 0; q < n; ++q) {
        if (v[q] > O_NINF) {
            w[q] = o_safe_exp((v[q] - m) / T);
            kahan_add(&k, w[q]);
        } else {
            w[q] = 0;
        }
    }
    if (k.sum > 0)
        for (int q = 0; q < n; ++q) w[q] /= k.sum;
}

/* param-grad style weights (src/sw/kernels_cpu.cpp:575-590): plain sum,
 * 1e-20 guard, no -inf special casing beyond safe_exp. */
static void o_softmax_plain4(const REAL *v, REAL T, REAL *w, REAL m) {
    REAL s = 0;
    for (int q = 0; q < 4; ++q) {
        w[q] = o_safe_exp((v[q] - m) / T);
    }
    s = w[0] + w[1] + w[2] + w[3];
    REAL inv = (s > (REAL)1e-20) ? (REAL)1 / s : (REAL)0;
    for (int q = 0; q < 4; ++q) w[q] *= inv;
}

static inline REAL o_post_weight(REAL a, REAL S, REAL T) {
    /* exp(min((a-S)/T, 0)) : kernels_cpu.cpp:200-203 */
    return o_safe_exp(o_min2((a - S) / T, (REAL)0));
}

#define AIDX(i, j) ((size_t)(i) * cols + (size_t)(j))
#define SIDX(i, j) ((size_t)((i) - 1) * (size_t)L2max + (size_t)((j) - 1))

/* ======================================================================
 * LINEAR GAP
 * ==================================================================== */

/* Forward for one problem: src/sw/kernels_cpu.cpp:70-150. */
static REAL lin_forward_one(const REAL *s, REAL *a, int L1, int L2, int L1max,
                            int L2max, REAL gap, REAL T) {
    const size_t cols = (size_t)L2max + 1;
    const size_t n = (size_t)(L1max + 1) * cols;
    for (size_t q = 0; q < n; ++q) a[q] = O_NINF;
    a[0] = 0;
    for (int k = 2; k <= L1 + L2; ++k) {
        int i0 = k - L2 > 1 ? k - L2 : 1;
        int i1 = L1 < k - 1 ? L1 : k - 1;
        for (int i = i0; i <= i1; ++i) {
            int j = k - i;
            REAL sc = s[SIDX(i, j)];
            REAL va = (i > 1 && j > 1) ? a[AIDX(i - 1, j - 1)] + sc : O_NINF;
            REAL vu = (i > 1) ? a[AIDX(i - 1, j)] + gap : O_NINF;
            REAL vl = (j > 1) ? a[AIDX(i, j - 1)] + gap : O_NINF;
            a[AIDX(i, j)] = o_lse4(va, vu, vl, sc, T);
        }
    }
    REAL m = O_NINF;
    for (int i = 0; i <= L1; ++i)
        for (int j = 0; j <= L2; ++j) m = o_max2(m, a[AIDX(i, j)]);
    kahan_t z = {0, 0};
    for (int i = 0; i <= L1; ++i)
        for (int j = 0; j <= L2; ++j)
            if (a[AIDX(i, j)] > O_NINF) kahan_add(&z, o_safe_exp((a[AIDX(i, j)] - m) / T));
    return m + T * R_LOG(z.sum);
}

/* Backward for one problem: src/sw/kernels_cpu.cpp:156-279. */
static void lin_backward_one(const REAL *s, const REAL *a, REAL S, REAL *be, REAL *post,
                             REAL *ggap, REAL *gT, int L1, int L2, int L1max, int L2max,
                             REAL gap, REAL T) {
    const size_t cols = (size_t)L2max + 1;
    const size_t n = (size_t)(L1max + 1) * cols;
    const size_t ns = (size_t)L1max * L2max;
    for (size_t q = 0; q < ns; ++q) post[q] = 0;
    for (size_t q = 0; q < n; ++q) be[q] = O_NINF;
    for (int i = 0; i <= L1; ++i)
        for (int j = 0; j <= L2; ++j) be[AIDX(i, j)] = o_post_weight(a[AIDX(i, j)], S, T);
    REAL gsum = 0;
    for (int k = L1 + L2; k >= 2; --k) {
        int i0 = k - L2 > 1 ? k - L2 : 1;
        int i1 = L1 < k - 1 ? L1 : k - 1;
        for (int i = i0; i <= i1; ++i) {
            int j = k - i;
            REAL b = be[AIDX(i, j)];
            if (isinf((double)b) || isnan((double)b) || b == 0) continue;
            REAL sc = s[SIDX(i, j)];
            REAL v[4], w[4];
            v[0] = (i > 1 && j > 1) ? a[AIDX(i - 1, j - 1)] + sc : O_NINF;
            v[1] = (i > 1) ? a[AIDX(i - 1, j)] + gap : O_NINF;
            v[2] = (j > 1) ? a[AIDX(i, j - 1)] + gap : O_NINF;
            v[3] = sc;
            o_softmax(v, 4, T, w);
            post[SIDX(i, j)] += b * (w[0] + w[3]);
            if (i > 1 && j > 1 && w[0] > 0) be[AIDX(i - 1, j - 1)] += b * w[0];
            if (i > 1 && w[1] > 0) {
                be[AIDX(i - 1, j)] += b * w[1];
                gsum += b * w[1];
            }
            if (j > 1 && w[2] > 0) {
                be[AIDX(i, j - 1)] += b * w[2];
                gsum += b * w[2];
            }
        }
    }
    kahan_t ms = {0, 0};
    for (size_t q = 0; q < ns; ++q) kahan_add(&ms, post[q] * s[q]);
    *ggap = gsum;
    *gT = (S - (ms.sum + gsum * gap)) / T;
}

/* HVP for one problem: src/sw/kernels_cpu.cpp:288-485. */
static void lin_hvp_one(const REAL *s, const REAL *v, const REAL *a, REAL S, REAL *da, REAL *be,
                        REAL *dbe, REAL *H, int L1, int L2, int L1max, int L2max, REAL gap,
                        REAL T) {
    const size_t cols = (size_t)L2max + 1;
    const size_t n = (size_t)(L1max + 1) * cols;
    const size_t ns = (size_t)L1max * L2max;
    for (size_t q = 0; q < n; ++q) da[q] = be[q] = dbe[q] = 0;
    for (size_t q = 0; q < ns; ++q) H[q] = 0;
    for (int k = 2; k <= L1 + L2; ++k) {
        int i0 = k - L2 > 1 ? k - L2 : 1;
        int i1 = L1 < k - 1 ? L1 : k - 1;
        for (int i = i0; i <= i1; ++i) {
            int j = k - i;
            REAL sc = s[SIDX(i, j)], vij = v[SIDX(i, j)];
            REAL x[4], w[4];
            x[0] = (i > 1 && j > 1) ? a[AIDX(i - 1, j - 1)] + sc : O_NINF;
            x[1] = (i > 1) ? a[AIDX(i - 1, j)] + gap : O_NINF;
            x[2] = (j > 1) ? a[AIDX(i, j - 1)] + gap : O_NINF;
            x[3] = sc;
            o_softmax(x, 4, T, w);
            REAL dva = (i > 1 && j > 1) ? da[AIDX(i - 1, j - 1)] + vij : 0;
            REAL dvu = (i > 1) ? da[AIDX(i - 1, j)] : 0;
            REAL dvl = (j > 1) ? da[AIDX(i, j - 1)] : 0;
            da[AIDX(i, j)] = w[0] * dva + w[1] * dvu + w[2] * dvl + w[3] * vij;
        }
    }
    kahan_t acc = {0, 0};
    for (int i = 0; i <= L1; ++i)
        for (int j = 0; j <= L2; ++j)
            kahan_add(&acc, o_post_weight(a[AIDX(i, j)], S, T) * da[AIDX(i, j)]);
    REAL dS = acc.sum;
    for (int i = 0; i <= L1; ++i)
        for (int j = 0; j <= L2; ++j) {
            be[AIDX(i, j)] = o_post_weight(a[AIDX(i, j)], S, T);
            dbe[AIDX(i, j)] = be[AIDX(i, j)] * (da[AIDX(i, j)] - dS) / T;
        }
    for (int k = L1 + L2; k >= 2; --k) {
        int i0 = k - L2 > 1 ? k - L2 : 1;
        int i1 = L1 < k - 1 ? L1 : k - 1;
        for (int i = i0; i <= i1; ++i) {
            int j = k - i;
            REAL b = be[AIDX(i, j)], db = dbe[AIDX(i, j)];
            if (isinf((double)b) || isnan((double)b) || b == 0) continue;
            REAL sc = s[SIDX(i, j)], vij = v[SIDX(i, j)];
            REAL x[4], w[4];
            x[0] = (i > 1 && j > 1) ? a[AIDX(i - 1, j - 1)] + sc : O_NINF;
            x[1] = (i > 1) ? a[AIDX(i - 1, j)] + gap : O_NINF;
            x[2] = (j > 1) ? a[AIDX(i, j - 1)] + gap : O_NINF;
            x[3] = sc;
            o_softmax(x, 4, T, w);
            REAL dv[4];
            dv[0] = (i > 1 && j > 1) ? da[AIDX(i - 1, j - 1)] + vij : 0;
            dv[1] = (i > 1) ? da[AIDX(i - 1, j)] : 0;
            dv[2] = (j > 1) ? da[AIDX(i, j - 1)] : 0;
            dv[3] = vij;
            REAL swdv = w[0] * dv[0] + w[1] * dv[1] + w[2] * dv[2] + w[3] * dv[3];
            REAL dw[4];
            for (int q = 0; q < 4; ++q) dw[q] = w[q] * (dv[q] - swdv) / T;
            H[SIDX(i, j)] += db * (w[0] + w[3]) + b * (dw[0] + dw[3]);
            if (i > 1 && j > 1 && w[0] > 0) be[AIDX(i - 1, j - 1)] += b * w[0];
            if (i > 1 && w[1] > 0) be[AIDX(i - 1, j)] += b * w[1];
            if (j > 1 && w[2] > 0) be[AIDX(i, j - 1)] += b * w[2];
            if (i > 1 && j > 1 && w[0] > 0) dbe[AIDX(i - 1, j - 1)] += db * w[0] + b * dw[0];
            if (i > 1 && w[1] > 0) dbe[AIDX(i - 1, j)] += db * w[1] + b * dw[1];
            if (j > 1 && w[2] > 0) dbe[AIDX(i, j - 1)] += db * w[2] + b * dw[2];
        }
    }
}

/* Param gradient dP/dtheta, theta in {gap (0), T (1)}:
 * src/sw/kernels_cpu.cpp:500-710. */
static void lin_param_one(const REAL *s, const REAL *a, REAL S, REAL dSdt, REAL *u, REAL *be,
                          REAL *w, REAL *dP, int L1, int L2, int L1max, int L2max, REAL gap,
                          REAL T, int ptype) {
    const size_t cols = (size_t)L2max + 1;
    const size_t n = (size_t)(L1max + 1) * cols;
    const size_t ns = (size_t)L1max * L2max;
    for (size_t q = 0; q < n; ++q) u[q] = be[q] = w[q] = 0;
    for (size_t q = 0; q < ns; ++q) dP[q] = 0;
    for (int k = 2; k <= L1 + L2; ++k) {
        int i0 = k - L2 > 1 ? k - L2 : 1;
        int i1 = L1 < k - 1 ? L1 : k - 1;
        for (int i = i0; i <= i1; ++i) {
            int j = k - i;
            REAL sc = s[SIDX(i, j)];
            REAL x[4], wt[4];
            x[0] = (i > 1 && j > 1) ? a[AIDX(i - 1, j - 1)] + sc : O_NINF;
            x[1] = (i > 1) ? a[AIDX(i - 1, j)] + gap : O_NINF;
            x[2] = (j > 1) ? a[AIDX(i, j - 1)] + gap : O_NINF;
            x[3] = sc;
            REAL m = o_max4(x[0], x[1], x[2], x[3]);
            if (m <= O_NINF) {
                u[AIDX(i, j)] = 0;
                continue;
            }
            o_softmax_plain4(x, T, wt, m);
            REAL du[4];
            du[0] = (i > 1 && j > 1) ? u[AIDX(i - 1, j - 1)] : 0;
            du[1] = (i > 1) ? u[AIDX(i - 1, j)] : 0;
            du[2] = (j > 1) ? u[AIDX(i, j - 1)] : 0;
            du[3] = 0;
            if (ptype == 0) {
                du[1] += 1;
                du[2] += 1;
            }
            REAL uv = wt[0] * du[0] + wt[1] * du[1] + wt[2] * du[2] + wt[3] * du[3];
            if (ptype == 1) {
                REAL mv = wt[0] * x[0] + wt[1] * x[1] + wt[2] * x[2] + wt[3] * x[3];
                uv += (a[AIDX(i, j)] - mv) / T;
            }
            u[AIDX(i, j)] = uv;
        }
    }
    for (int i = 0; i <= L1; ++i)
        for (int j = 0; j <= L2; ++j) be[AIDX(i, j)] = o_post_weight(a[AIDX(i, j)], S, T);
    for (int k = L1 + L2; k >= 2; --k) {
        int i0 = k - L2 > 1 ? k - L2 : 1;
        int i1 = L1 < k - 1 ? L1 : k - 1;
        for (int i = i0; i <= i1; ++i) {
            int j = k - i;
            REAL bc = be[AIDX(i, j)];
            REAL binit = 0;
            if (a[AIDX(i, j)] > O_NINF) binit = o_post_weight(a[AIDX(i, j)], S, T);
            REAL dWi = binit * (u[AIDX(i, j)] - dSdt) / T;
            if (ptype == 1 && a[AIDX(i, j)] > O_NINF) dWi -= binit * (a[AIDX(i, j)] - S) / (T * T);
            REAL wc = w[AIDX(i, j)] + dWi;
            if (bc <= (REAL)1e-20 && fabs((double)wc) <= 1e-20) continue;
            REAL sc = s[SIDX(i, j)];
            REAL x[4], wt[4];
            x[0] = (i > 1 && j > 1) ? a[AIDX(i - 1, j - 1)] + sc : O_NINF;
            x[1] = (i > 1) ? a[AIDX(i - 1, j)] + gap : O_NINF;
            x[2] = (j > 1) ? a[AIDX(i, j - 1)] + gap : O_NINF;
            x[3] = sc;
            REAL m = o_max4(x[0], x[1], x[2], x[3]);
            if (m <= O_NINF) continue;
            o_softmax_plain4(x, T, wt, m);
            REAL du[4];
            du[0] = (i > 1 && j > 1) ? u[AIDX(i - 1, j - 1)] : 0;
            du[1] = (i > 1) ? u[AIDX(i - 1, j)] : 0;
            du[2] = (j > 1) ? u[AIDX(i, j - 1)] : 0;
            du[3] = 0;
            if (ptype == 0) {
                du[1] += 1;
                du[2] += 1;
            }
            REAL mdu = wt[0] * du[0] + wt[1] * du[1] + wt[2] * du[2] + wt[3] * du[3];
            REAL dw[4];
            for (int q = 0; q < 4; ++q) dw[q] = wt[q] * (du[q] - mdu) / T;
            if (ptype == 1) {
                REAL mv = wt[0] * x[0] + wt[1] * x[1] + wt[2] * x[2] + wt[3] * x[3];
                REAL it2 = (REAL)1 / (T * T);
                for (int q = 0; q < 4; ++q) dw[q] += wt[q] * (mv - x[q]) * it2;
            }
            dP[SIDX(i, j)] += wc * (wt[0] + wt[3]) + bc * (dw[0] + dw[3]);
            if (x[0] > O_NINF) {
                be[AIDX(i - 1, j - 1)] += bc * wt[0];
                w[AIDX(i - 1, j - 1)] += wc * wt[0] + bc * dw[0];
            }
            if (x[1] > O_NINF) {
                be[AIDX(i - 1, j)] += bc * wt[1];
                w[AIDX(i - 1, j)] += wc * wt[1] + bc * dw[1];
            }
            if (x[2] > O_NINF) {
                be[AIDX(i, j - 1)] += bc * wt[2];
                w[AIDX(i, j - 1)] += wc * wt[2] + bc * dw[2];
            }
        }
    }
}

/* ======================================================================
 * AFFINE GAP (3 states M, I, D; planes stacked M|I|D)
 * ==================================================================== */
#define PM(i, j) (a[0 * plane + AIDX(i, j)])
#define PI(i, j) (a[1 * plane + AIDX(i, j)])
#define PD(i, j) (a[2 * plane + AIDX(i, j)])

/* src/sw_affine/kernels_cpu.cpp:94-193 */
static REAL aff_forward_one(const REAL *s, REAL *a, int L1, int L2, int L1max, int L2max,
                            REAL go, REAL ge, REAL T) {
    const size_t cols = (size_t)L2max + 1;
    const size_t plane = (size_t)(L1max + 1) * cols;
    for (size_t q = 0; q < 3 * plane; ++q) a[q] = O_NINF;
    a[0] = 0;
    for (int k = 2; k <= L1 + L2; ++k) {
        int i0 = k - L2 > 1 ? k - L2 : 1;
        int i1 = L1 < k - 1 ? L1 : k - 1;
        for (int i = i0; i <= i1; ++i) {
            int j = k - i;
            REAL sc = s[SIDX(i, j)];
            int dg = (i > 1 && j > 1);
            PM(i, j) = o_lse4(dg ? PM(i - 1, j - 1) + sc : O_NINF,
                              dg ? PI(i - 1, j - 1) + sc : O_NINF,
                              dg ? PD(i - 1, j - 1) + sc : O_NINF, sc, T);
            PI(i, j) = o_lse2(i > 1 ? PM(i - 1, j) + go : O_NINF,
                              i > 1 ? PI(i - 1, j) + ge : O_NINF, T);
            PD(i, j) = o_lse2(j > 1 ? PM(i, j - 1) + go : O_NINF,
                              j > 1 ? PD(i, j - 1) + ge : O_NINF, T);
        }
    }
    REAL m = O_NINF;
    for (int i = 0; i <= L1; ++i)
        for (int j = 0; j <= L2; ++j)
            for (int st = 0; st < 3; ++st) m = o_max2(m, a[st * plane + AIDX(i, j)]);
    kahan_t z = {0, 0};
    for (int i = 0; i <= L1; ++i)
        for (int j = 0; j <= L2; ++j)
            for (int st = 0; st < 3; ++st) {
                REAL val = a[st * plane + AIDX(i, j)];
                if (val > O_NINF) kahan_add(&z, o_safe_exp((val - m) / T));
            }
    return m + T * R_LOG(z.sum);
}

/* src/sw_affine/kernels_cpu.cpp:199-346 */
static void aff_backward_one(const REAL *s, const REAL *a, REAL S, REAL *be, REAL *post,
                             REAL *gopen, REAL *gext, REAL *gT, int L1, int L2, int L1max,
                             int L2max, REAL go, REAL ge, REAL T) {
    const size_t cols = (size_t)L2max + 1;
    const size_t plane = (size_t)(L1max + 1) * cols;
    const size_t ns = (size_t)L1max * L2max;
    for (size_t q = 0; q < ns; ++q) post[q] = 0;
    for (size_t q = 0; q < 3 * plane; ++q) be[q] = 0;
    for (int i = 0; i <= L1; ++i)
        for (int j = 0; j <= L2; ++j)
            for (int st = 0; st < 3; ++st)
                be[st * plane + AIDX(i, j)] = o_post_weight(a[st * plane + AIDX(i, j)], S, T);
    REAL so = 0, se = 0;
    for (int k = L1 + L2; k >= 2; --k) {
        int i0 = k - L2 > 1 ? k - L2 : 1;
        int i1 = L1 < k - 1 ? L1 : k - 1;
        for (int i = i0; i <= i1; ++i) {
            int j = k - i;
            REAL sc = s[SIDX(i, j)];
            int dg = (i > 1 && j > 1);
            REAL bM = be[AIDX(i, j)];
            if (!isinf((double)bM) && !isnan((double)bM) && bM != 0) {
                REAL v[4] = {dg ? PM(i - 1, j - 1) + sc : O_NINF, dg ? PI(i - 1, j - 1) + sc : O_NINF,
                             dg ? PD(i - 1, j - 1) + sc : O_NINF, sc};
                REAL w[4];
                o_softmax(v, 4, T, w);
                post[SIDX(i, j)] += bM * (w[0] + w[1] + w[2] + w[3]);
                if (dg) {
                    if (w[0] > 0) be[0 * plane + AIDX(i - 1, j - 1)] += bM * w[0];
                    if (w[1] > 0) be[1 * plane + AIDX(i - 1, j - 1)] += bM * w[1];
                    if (w[2] > 0) be[2 * plane + AIDX(i - 1, j - 1)] += bM * w[2];
                }
            }
            REAL bI = be[plane + AIDX(i, j)];
            if (!isinf((double)bI) && !isnan((double)bI) && bI != 0) {
                REAL v[2] = {i > 1 ? PM(i - 1, j) + go : O_NINF, i > 1 ? PI(i - 1, j) + ge : O_NINF};
                REAL w[2];
                o_softmax(v, 2, T, w);
                if (i > 1) {
                    if (w[0] > 0) {
                        be[0 * plane + AIDX(i - 1, j)] += bI * w[0];
                        so += bI * w[0];
                    }
                    if (w[1] > 0) {
                        be[1 * plane + AIDX(i - 1, j)] += bI * w[1];
                        se += bI * w[1];
                    }
                }
            }
            REAL bD = be[2 * plane + AIDX(i, j)];
            if (!isinf((double)bD) && !isnan((double)bD) && bD != 0) {
                REAL v[2] = {j > 1 ? PM(i, j - 1) + go : O_NINF, j > 1 ? PD(i, j - 1) + ge : O_NINF};
                REAL w[2];
                o_softmax(v, 2, T, w);
                if (j > 1) {
                    if (w[0] > 0) {
                        be[0 * plane + AIDX(i, j - 1)] += bD * w[0];
                        so += bD * w[0];
                    }
                    if (w[1] > 0) {
                        be[2 * plane + AIDX(i, j - 1)] += bD * w[1];
                        se += bD * w[1];
                    }
                }
            }
        }
    }
    kahan_t ms = {0, 0};
    for (size_t q = 0; q < ns; ++q) kahan_add(&ms, post[q] * s[q]);
    *gopen = so;
    *gext = se;
    *gT = (S - (ms.sum + so * go + se * ge)) / T;
}

/* src/sw_affine/kernels_cpu.cpp:352-620 */
static void aff_hvp_one(const REAL *s, const REAL *v, const REAL *a, REAL S, REAL *da, REAL *be,
                        REAL *dbe, REAL *H, int L1, int L2, int L1max, int L2max, REAL go,
                        REAL ge, REAL T) {
    const size_t cols = (size_t)L2max + 1;
    const size_t plane = (size_t)(L1max + 1) * cols;
    const size_t ns = (size_t)L1max * L2max;
    for (size_t q = 0; q < 3 * plane; ++q) da[q] = dbe[q] = be[q] = 0;
    for (size_t q = 0; q < ns; ++q) H[q] = 0;
#define DM(i, j) (da[0 * plane + AIDX(i, j)])
#define DI(i, j) (da[1 * plane + AIDX(i, j)])
#define DD(i, j) (da[2 * plane + AIDX(i, j)])
    for (int k = 2; k <= L1 + L2; ++k) {
        int i0 = k - L2 > 1 ? k - L2 : 1;
        int i1 = L1 < k - 1 ? L1 : k - 1;
        for (int i = i0; i <= i1; ++i) {
            int j = k - i;
            REAL sc = s[SIDX(i, j)], vij = v[SIDX(i, j)];
            int dg = (i > 1 && j > 1);
            REAL xm[4] = {dg ? PM(i - 1, j - 1) + sc : O_NINF, dg ? PI(i - 1, j - 1) + sc : O_NINF,
                          dg ? PD(i - 1, j - 1) + sc : O_NINF, sc};
            REAL wm[4];
            o_softmax(xm, 4, T, wm);
            DM(i, j) = wm[0] * (dg ? DM(i - 1, j - 1) + vij : 0) + wm[1] * (dg ? DI(i - 1, j - 1) + vij : 0) +
                       wm[2] * (dg ? DD(i - 1, j - 1) + vij : 0) + wm[3] * vij;
            REAL xi[2] = {i > 1 ? PM(i - 1, j) + go : O_NINF, i > 1 ? PI(i - 1, j) + ge : O_NINF};
            REAL wi[2];
            o_softmax(xi, 2, T, wi);
            DI(i, j) = wi[0] * (i > 1 ? DM(i - 1, j) : 0) + wi[1] * (i > 1 ? DI(i - 1, j) : 0);
            REAL xd[2] = {j > 1 ? PM(i, j - 1) + go : O_NINF, j > 1 ? PD(i, j - 1) + ge : O_NINF};
            REAL wd[2];
            o_softmax(xd, 2, T, wd);
            DD(i, j) = wd[0] * (j > 1 ? DM(i, j - 1) : 0) + wd[1] * (j > 1 ? DD(i, j - 1) : 0);
        }
    }
    kahan_t acc = {0, 0};
    for (int i = 0; i <= L1; ++i)
        for (int j = 0; j <= L2; ++j)
            for (int st = 0; st < 3; ++st)
                kahan_add(&acc, o_post_weight(a[st * plane + AIDX(i, j)], S, T) * da[st * plane + AIDX(i, j)]);
    REAL dS = acc.sum;
    for (int i = 0; i <= L1; ++i)
        for (int j = 0; j <= L2; ++j)
            for (int st = 0; st < 3; ++st) {
                size_t q = st * plane + AIDX(i, j);
                be[q] = o_post_weight(a[q], S, T);
                dbe[q] = be[q] * (da[q] - dS) / T;
            }
    for (int k = L1 + L2; k >= 2; --k) {
        int i0 = k - L2 > 1 ? k - L2 : 1;
        int i1 = L1 < k - 1 ? L1 : k - 1;
        for (int i = i0; i <= i1; ++i) {
            int j = k - i;
            REAL sc = s[SIDX(i, j)], vij = v[SIDX(i, j)];
            int dg = (i > 1 && j > 1);
            /* M */
            {
                REAL bM = be[AIDX(i, j)], dbM = dbe[AIDX(i, j)];
                REAL xm[4] = {dg ? PM(i - 1, j - 1) + sc : O_NINF, dg ? PI(i - 1, j - 1) + sc : O_NINF,
                              dg ? PD(i - 1, j - 1) + sc : O_NINF, sc};
                REAL wm[4];
                o_softmax(xm, 4, T, wm);
                REAL dv[4] = {dg ? DM(i - 1, j - 1) + vij : 0, dg ? DI(i - 1, j - 1) + vij : 0,
                              dg ? DD(i - 1, j - 1) + vij : 0, vij};
                REAL sw = wm[0] * dv[0] + wm[1] * dv[1] + wm[2] * dv[2] + wm[3] * dv[3];
                REAL dw[4];
                for (int q = 0; q < 4; ++q) dw[q] = wm[q] * (dv[q] - sw) / T;
                H[SIDX(i, j)] += dbM * (wm[0] + wm[1] + wm[2] + wm[3]) + bM * (dw[0] + dw[1] + dw[2] + dw[3]);
                if (dg) {
                    be[0 * plane + AIDX(i - 1, j - 1)] += bM * wm[0];
                    be[1 * plane + AIDX(i - 1, j - 1)] += bM * wm[1];
                    be[2 * plane + AIDX(i - 1, j - 1)] += bM * wm[2];
                    dbe[0 * plane + AIDX(i - 1, j - 1)] += dbM * wm[0] + bM * dw[0];
                    dbe[1 * plane + AIDX(i - 1, j - 1)] += dbM * wm[1] + bM * dw[1];
                    dbe[2 * plane + AIDX(i - 1, j - 1)] += dbM * wm[2] + bM * dw[2];
                }
            }
            /* I */
            {
                REAL bI = be[plane + AIDX(i, j)], dbI = dbe[plane + AIDX(i, j)];
                REAL xi[2] = {i > 1 ? PM(i - 1, j) + go : O_NINF, i > 1 ? PI(i - 1, j) + ge : O_NINF};
                REAL wi[2];
                o_softmax(xi, 2, T, wi);
                REAL d0 = i > 1 ? DM(i - 1, j) : 0, d1 = i > 1 ? DI(i - 1, j) : 0;
                REAL sw = wi[0] * d0 + wi[1] * d1;
                REAL dw0 = wi[0] * (d0 - sw) / T, dw1 = wi[1] * (d1 - sw) / T;
                if (i > 1) {
                    be[0 * plane + AIDX(i - 1, j)] += bI * wi[0];
                    be[1 * plane + AIDX(i - 1, j)] += bI * wi[1];
                    dbe[0 * plane + AIDX(i - 1, j)] += dbI * wi[0] + bI * dw0;
                    dbe[1 * plane + AIDX(i - 1, j)] += dbI * wi[1] + bI * dw1;
                }
            }
            /* D */
            {
                REAL bD = be[2 * plane + AIDX(i, j)], dbD = dbe[2 * plane + AIDX(i, j)];
                REAL xd[2] = {j > 1 ? PM(i, j - 1) + go : O_NINF, j > 1 ? PD(i, j - 1) + ge : O_NINF};
                REAL wd[2];
                o_softmax(xd, 2, T, wd);
                REAL d0 = j > 1 ? DM(i, j - 1) : 0, d1 = j > 1 ? DD(i, j - 1) : 0;
                REAL sw = wd[0] * d0 + wd[1] * d1;
                REAL dw0 = wd[0] * (d0 - sw) / T, dw1 = wd[1] * (d1 - sw) / T;
                if (j > 1) {
                    be[0 * plane + AIDX(i, j - 1)] += bD * wd[0];
                    be[2 * plane + AIDX(i, j - 1)] += bD * wd[1];
                    dbe[0 * plane + AIDX(i, j - 1)] += dbD * wd[0] + bD * dw0;
                    dbe[2 * plane + AIDX(i, j - 1)] += dbD * wd[1] + bD * dw1;
                }
            }
        }
    }
#undef DM
#undef DI
#undef DD
}

/* src/sw_affine/kernels_cpu.cpp:630-921, ptype 0=open 1=ext 2=T */
static void aff_param_one(const REAL *s, const REAL *a, REAL S, REAL dSdt, REAL *u, REAL *be,
                          REAL *w, REAL *dP, int L1, int L2, int L1max, int L2max, REAL go,
                          REAL ge, REAL T, int ptype) {
    const size_t cols = (size_t)L2max + 1;
    const size_t plane = (size_t)(L1max + 1) * cols;
    const size_t ns = (size_t)L1max * L2max;
    for (size_t q = 0; q < 3 * plane; ++q) u[q] = be[q] = w[q] = 0;
    for (size_t q = 0; q < ns; ++q) dP[q] = 0;
#define UM(i, j) (u[0 * plane + AIDX(i, j)])
#define UI(i, j) (u[1 * plane + AIDX(i, j)])
#define UD(i, j) (u[2 * plane + AIDX(i, j)])
    const REAL it2 = (REAL)1 / (T * T);
    for (int k = 2; k <= L1 + L2; ++k) {
        int i0 = k - L2 > 1 ? k - L2 : 1;
        int i1 = L1 < k - 1 ? L1 : k - 1;
        for (int i = i0; i <= i1; ++i) {
            int j = k - i;
            REAL sc = s[SIDX(i, j)];
            int dg = (i > 1 && j > 1);
            REAL xm[4] = {dg ? PM(i - 1, j - 1) + sc : O_NINF, dg ? PI(i - 1, j - 1) + sc : O_NINF,
                          dg ? PD(i - 1, j - 1) + sc : O_NINF, sc};
            REAL wm[4];
            o_softmax(xm, 4, T, wm);
            REAL dUM = wm[0] * (dg ? UM(i - 1, j - 1) : 0) + wm[1] * (dg ? UI(i - 1, j - 1) : 0) +
                       wm[2] * (dg ? UD(i - 1, j - 1) : 0);
            if (ptype == 2) {
                REAL E = wm[0] * xm[0] + wm[1] * xm[1] + wm[2] * xm[2] + wm[3] * xm[3];
                dUM += (PM(i, j) - E) / T;
            }
            UM(i, j) = dUM;
            REAL xi[2] = {i > 1 ? PM(i - 1, j) + go : O_NINF, i > 1 ? PI(i - 1, j) + ge : O_NINF};
            REAL wi[2];
            o_softmax(xi, 2, T, wi);
            REAL d0 = i > 1 ? UM(i - 1, j) : 0, d1 = i > 1 ? UI(i - 1, j) : 0;
            if (ptype == 0) d0 += 1;
            if (ptype == 1) d1 += 1;
            REAL dUI = wi[0] * d0 + wi[1] * d1;
            if (ptype == 2) dUI += (PI(i, j) - (wi[0] * xi[0] + wi[1] * xi[1])) / T;
            UI(i, j) = dUI;
            REAL xd[2] = {j > 1 ? PM(i, j - 1) + go : O_NINF, j > 1 ? PD(i, j - 1) + ge : O_NINF};
            REAL wd[2];
            o_softmax(xd, 2, T, wd);
            REAL e0 = j > 1 ? UM(i, j - 1) : 0, e1 = j > 1 ? UD(i, j - 1) : 0;
            if (ptype == 0) e0 += 1;
            if (ptype == 1) e1 += 1;
            REAL dUD = wd[0] * e0 + wd[1] * e1;
            if (ptype == 2) dUD += (PD(i, j) - (wd[0] * xd[0] + wd[1] * xd[1])) / T;
            UD(i, j) = dUD;
        }
    }
    for (int i = 0; i <= L1; ++i)
        for (int j = 0; j <= L2; ++j)
            for (int st = 0; st < 3; ++st) {
                size_t q = st * plane + AIDX(i, j);
                be[q] = a[q] <= O_NINF ? 0 : o_post_weight(a[q], S, T);
            }
    for (int k = L1 + L2; k >= 2; --k) {
        int i0 = k - L2 > 1 ? k - L2 : 1;
        int i1 = L1 < k - 1 ? L1 : k - 1;
        for (int i = i0; i <= i1; ++i) {
            int j = k - i;
            REAL sc = s[SIDX(i, j)];
            int dg = (i > 1 && j > 1);
            size_t qM = AIDX(i, j), qI = plane + AIDX(i, j), qD = 2 * plane + AIDX(i, j);
            /* M */
            {
                REAL bM = be[qM];
                REAL bi = a[qM] <= O_NINF ? 0 : o_post_weight(a[qM], S, T);
                REAL WM = w[qM] + bi * (u[qM] - dSdt) / T;
                if (ptype == 2 && a[qM] > O_NINF) WM -= bi * (a[qM] - S) / (T * T);
                REAL xm[4] = {dg ? PM(i - 1, j - 1) + sc : O_NINF, dg ? PI(i - 1, j - 1) + sc : O_NINF,
                              dg ? PD(i - 1, j - 1) + sc : O_NINF, sc};
                REAL wm[4];
                o_softmax(xm, 4, T, wm);
                REAL du[4] = {dg ? UM(i - 1, j - 1) : 0, dg ? UI(i - 1, j - 1) : 0, dg ? UD(i - 1, j - 1) : 0, 0};
                REAL sw = wm[0] * du[0] + wm[1] * du[1] + wm[2] * du[2] + wm[3] * du[3];
                REAL dw[4];
                for (int q = 0; q < 4; ++q) dw[q] = wm[q] * (du[q] - sw) / T;
                if (ptype == 2) {
                    REAL E = wm[0] * xm[0] + wm[1] * xm[1] + wm[2] * xm[2] + wm[3] * xm[3];
                    for (int q = 0; q < 4; ++q) dw[q] += wm[q] * (E - xm[q]) * it2;
                }
                dP[SIDX(i, j)] += WM;
                if (dg) {
                    be[AIDX(i - 1, j - 1)] += bM * wm[0];
                    be[plane + AIDX(i - 1, j - 1)] += bM * wm[1];
                    be[2 * plane + AIDX(i - 1, j - 1)] += bM * wm[2];
                    w[AIDX(i - 1, j - 1)] += WM * wm[0] + bM * dw[0];
                    w[plane + AIDX(i - 1, j - 1)] += WM * wm[1] + bM * dw[1];
                    w[2 * plane + AIDX(i - 1, j - 1)] += WM * wm[2] + bM * dw[2];
                }
            }
            /* I */
            {
                REAL bI = be[qI];
                REAL bi = a[qI] <= O_NINF ? 0 : o_post_weight(a[qI], S, T);
                REAL WI = w[qI] + bi * (u[qI] - dSdt) / T;
                if (ptype == 2 && a[qI] > O_NINF) WI -= bi * (a[qI] - S) / (T * T);
                if (i > 1) {
                    REAL xi[2] = {PM(i - 1, j) + go, PI(i - 1, j) + ge};
                    REAL wi[2];
                    o_softmax(xi, 2, T, wi);
                    REAL d0 = UM(i - 1, j), d1 = UI(i - 1, j);
                    if (ptype == 0) d0 += 1;
                    if (ptype == 1) d1 += 1;
                    REAL sw = wi[0] * d0 + wi[1] * d1;
                    REAL dw0 = wi[0] * (d0 - sw) / T, dw1 = wi[1] * (d1 - sw) / T;
                    if (ptype == 2) {
                        REAL E = wi[0] * xi[0] + wi[1] * xi[1];
                        dw0 += wi[0] * (E - xi[0]) * it2;
                        dw1 += wi[1] * (E - xi[1]) * it2;
                    }
                    be[AIDX(i - 1, j)] += bI * wi[0];
                    be[plane + AIDX(i - 1, j)] += bI * wi[1];
                    w[AIDX(i - 1, j)] += WI * wi[0] + bI * dw0;
                    w[plane + AIDX(i - 1, j)] += WI * wi[1] + bI * dw1;
                }
            }
            /* D */
            {
                REAL bD = be[qD];
                REAL bi = a[qD] <= O_NINF ? 0 : o_post_weight(a[qD], S, T);
                REAL WD = w[qD] + bi * (u[qD] - dSdt) / T;
                if (ptype == 2 && a[qD] > O_NINF) WD -= bi * (a[qD] - S) / (T * T);
                if (j > 1) {
                    REAL xd[2] = {PM(i, j - 1) + go, PD(i, j - 1) + ge};
                    REAL wd[2];
                    o_softmax(xd, 2, T, wd);
                    REAL d0 = UM(i, j - 1), d1 = UD(i, j - 1);
                    if (ptype == 0) d0 += 1;
                    if (ptype == 1) d1 += 1;
                    REAL sw = wd[0] * d0 + wd[1] * d1;
                    REAL dw0 = wd[0] * (d0 - sw) / T, dw1 = wd[1] * (d1 - sw) / T;
                    if (ptype == 2) {
                        REAL E = wd[0] * xd[0] + wd[1] * xd[1];
                        dw0 += wd[0] * (E - xd[0]) * it2;
                        dw1 += wd[1] * (E - xd[1]) * it2;
                    }
                    be[AIDX(i, j - 1)] += bD * wd[0];
                    be[2 * plane + AIDX(i, j - 1)] += bD * wd[1];
                    w[AIDX(i, j - 1)] += WD * wd[0] + bD * dw0;
                    w[2 * plane + AIDX(i, j - 1)] += WD * wd[1] + bD * dw1;
                }
            }
        }
    }
#undef UM
#undef UI
#undef UD
}

/* ======================================================================
 * Batched entry points (OpenMP over the batch; each problem is serial).
 * All buffers are caller-allocated; planes are [B, S*(L1+1)*(L2+1)].
 * ==================================================================== */

void SFX(oracle_sw_forward)(const REAL *scores, const int *lengths, int B, int L1max, int L2max,
                            REAL gap, REAL T, REAL *alpha, REAL *value) {
    const size_t n = (size_t)(L1max + 1) * (L2max + 1), ns = (size_t)L1max * L2max;
#pragma omp parallel for schedule(dynamic, 1)
    for (int b = 0; b < B; ++b)
        value[b] = lin_forward_one(scores + b * ns, alpha + b * n, lengths[2 * b], lengths[2 * b + 1],
                                   L1max, L2max, gap, T);
}

void SFX(oracle_sw_backward)(const REAL *scores, const int *lengths, int B, int L1max, int L2max,
                             REAL gap, REAL T, const REAL *alpha, const REAL *value, REAL *beta,
                             REAL *marginals, REAL *grad_gap, REAL *grad_T) {
    const size_t n = (size_t)(L1max + 1) * (L2max + 1), ns = (size_t)L1max * L2max;
#pragma omp parallel for schedule(dynamic, 1)
    for (int b = 0; b < B; ++b)
        lin_backward_one(scores + b * ns, alpha + b * n, value[b], beta + b * n, marginals + b * ns,
                         grad_gap + b, grad_T + b, lengths[2 * b], lengths[2 * b + 1], L1max, L2max,
                         gap, T);
}

void SFX(oracle_sw_hvp)(const REAL *scores, const REAL *V, const int *lengths, int B, int L1max,
                        int L2max, REAL gap, REAL T, const REAL *alpha, const REAL *value,
                        REAL *ws1, REAL *ws2, REAL *ws3, REAL *H) {
    const size_t n = (size_t)(L1max + 1) * (L2max + 1), ns = (size_t)L1max * L2max;
#pragma omp parallel for schedule(dynamic, 1)
    for (int b = 0; b < B; ++b)
        lin_hvp_one(scores + b * ns, V + b * ns, alpha + b * n, value[b], ws1 + b * n, ws2 + b * n,
                    ws3 + b * n, H + b * ns, lengths[2 * b], lengths[2 * b + 1], L1max, L2max, gap, T);
}

void SFX(oracle_sw_param_grad)(const REAL *scores, const int *lengths, int B, int L1max,
                               int L2max, REAL gap, REAL T, const REAL *alpha, const REAL *value,
                               const REAL *dS_dtheta, REAL *ws1, REAL *ws2, REAL *ws3, REAL *dP,
                               int param_type) {
    const size_t n = (size_t)(L1max + 1) * (L2max + 1), ns = (size_t)L1max * L2max;
#pragma omp parallel for schedule(dynamic, 1)
    for (int b = 0; b < B; ++b)
        lin_param_one(scores + b * ns, alpha + b * n, value[b], dS_dtheta[b], ws1 + b * n, ws2 + b * n,
                      ws3 + b * n, dP + b * ns, lengths[2 * b], lengths[2 * b + 1], L1max, L2max, gap,
                      T, param_type);
}

void SFX(oracle_sw_affine_forward)(const REAL *scores, const int *lengths, int B, int L1max,
                                   int L2max, REAL go, REAL ge, REAL T, REAL *alpha, REAL *value) {
    const size_t n = 3 * (size_t)(L1max + 1) * (L2max + 1), ns = (size_t)L1max * L2max;
#pragma omp parallel for schedule(dynamic, 1)
    for (int b = 0; b < B; ++b)
        value[b] = aff_forward_one(scores + b * ns, alpha + b * n, lengths[2 * b], lengths[2 * b + 1],
                                   L1max, L2max, go, ge, T);
}

void SFX(oracle_sw_affine_backward)(const REAL *scores, const int *lengths, int B, int L1max,
                                    int L2max, REAL go, REAL ge, REAL T, const REAL *alpha,
                                    const REAL *value, REAL *beta, REAL *marginals, REAL *grad_open,
                                    REAL *grad_ext, REAL *grad_T) {
    const size_t n = 3 * (size_t)(L1max + 1) * (L2max + 1), ns = (size_t)L1max * L2max;
#pragma omp parallel for schedule(dynamic, 1)
    for (int b = 0; b < B; ++b)
        aff_backward_one(scores + b * ns, alpha + b * n, value[b], beta + b * n, marginals + b * ns,
                         grad_open + b, grad_ext + b, grad_T + b, lengths[2 * b], lengths[2 * b + 1],
                         L1max, L2max, go, ge, T);
}

void SFX(oracle_sw_affine_hvp)(const REAL *scores, const REAL *V, const int *lengths, int B,
                               int L1max, int L2max, REAL go, REAL ge, REAL T, const REAL *alpha,
                               const REAL *value, REAL *ws1, REAL *ws2, REAL *ws3, REAL *H) {
    const size_t n = 3 * (size_t)(L1max + 1) * (L2max + 1), ns = (size_t)L1max * L2max;
#pragma omp parallel for schedule(dynamic, 1)
    for (int b = 0; b < B; ++b)
        aff_hvp_one(scores + b * ns, V + b * ns, alpha + b * n, value[b], ws1 + b * n, ws2 + b * n,
                    ws3 + b * n, H + b * ns, lengths[2 * b], lengths[2 * b + 1], L1max, L2max, go, ge,
                    T);
}

void SFX(oracle_sw_affine_param_grad)(const REAL *scores, const int *lengths, int B, int L1max,
                                      int L2max, REAL go, REAL ge, REAL T, const REAL *alpha,
                                      const REAL *value, const REAL *dS_dtheta, REAL *ws1,
                                      REAL *ws2, REAL *ws3, REAL *dP, int param_type) {
    const size_t n = 3 * (size_t)(L1max + 1) * (L2max + 1), ns = (size_t)L1max * L2max;
#pragma omp parallel for schedule(dynamic, 1)
    for (int b = 0; b < B; ++b)
        aff_param_one(scores + b * ns, alpha + b * n, value[b], dS_dtheta[b], ws1 + b * n, ws2 + b * n,
                      ws3 + b * n, dP + b * ns, lengths[2 * b], lengths[2 * b + 1], L1max, L2max, go,
                      ge, T, param_type);
}
