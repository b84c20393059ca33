/*
 * nw_affine_oracle.c -- CPU restatement of d2p's soft Needleman-Wunsch with
 * affine gaps (three states: M match, I gap in the second sequence, D gap in
 * the first).
 *
 * TEST INFRASTRUCTURE ONLY.  Nothing in the d2p_b200 product path links,
 * loads or calls this file; it is the checker used by tests/ and by
 * bench-side CPU baselines.
 *
 * It restates, cell for cell, the reference's CPU algorithm
 * src/nw_affine/kernels_cpu.cpp:
 *   numerics (safe_exp, Kahan-summed 3-way logsumexp, 3-way softmax
 *   weights)                     :37-95
 *   forward                      :101-185   backward (posteriors,
 *   hvp                          :362-650     dS/dopen, dS/dext, dS/dT) :191-356
 *   param grad                   :656-1000
 * Boundaries: M(0,0) = 0, I(i,0) = open + (i-1) ext, D(0,j) = open + (j-1) ext,
 * every other boundary state NINF; the value is the logsumexp of the three
 * states at (L1, L2).  M takes the diagonal predecessor's three states, I the
 * upper cell's (M, D open a gap, I extends it), D the left cell's.
 *
 * The file is compiled twice (REAL=float -> *_f32, REAL=double -> *_f64): the
 * f32 build follows the reference's float arithmetic (the same operation
 * order, Kahan sums where it has them, its 1e-20 skip thresholds), the f64
 * build is the noise-floor reference.  Planes are [B][3][(L1+1)(L2+1)]
 * (M, I, D), row-major over (i, j); cells are visited by anti-diagonal,
 * i ascending, as the reference does.
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
#define R_EXP expf
#define R_LOG logf
#endif

#define A_NINF ((REAL)-1e30)
#define A_SKIP ((REAL)1e-20f)

typedef struct {
    REAL sum, c;
} ak_t;

static inline void ak_add(ak_t *k, REAL v) {
    REAL y = v - k->c;
    REAL t = k->sum + y;
    k->c = (t - k->sum) - y;
    k->sum = t;
}

static inline REAL a_exp(REAL x) {
    if (x < (REAL)-88) return (REAL)0;
    if (x > (REAL)88) x = (REAL)88;
    return R_EXP(x);
}

static inline REAL a_max3(REAL a, REAL b, REAL c) {
    REAL m = a > b ? a : b;
    return m > c ? m : c;
}

/* :59-72 */
static inline REAL a_lse3(REAL a, REAL b, REAL c, REAL T) {
    REAL m = a_max3(a, b, c);
    if (m <= A_NINF) return A_NINF;
    ak_t k = {0, 0};
    if (a > A_NINF) ak_add(&k, a_exp((a - m) / T));
    if (b > A_NINF) ak_add(&k, a_exp((b - m) / T));
    if (c > A_NINF) ak_add(&k, a_exp((c - m) / T));
    if (k.sum <= 0) return A_NINF;
    return m + T * R_LOG(k.sum);
}

/* :74-95 */
static inline void a_w3(REAL a, REAL b, REAL c, REAL T, REAL *wa, REAL *wb, REAL *wc) {
    REAL m = a_max3(a, b, c);
    if (m <= A_NINF) {
        *wa = *wb = *wc = 0;
        return;
    }
    REAL ea = a > A_NINF ? a_exp((a - m) / T) : (REAL)0;
    REAL eb = b > A_NINF ? a_exp((b - m) / T) : (REAL)0;
    REAL ec = c > A_NINF ? a_exp((c - m) / T) : (REAL)0;
    REAL tot = ea + eb + ec;
    if (tot > 0) {
        *wa = ea / tot;
        *wb = eb / tot;
        *wc = ec / tot;
    } else {
        *wa = *wb = *wc = 0;
    }
}

/* per-problem views */
typedef struct {
    REAL *M, *I, *D;
} st3_t;

static inline st3_t st3(REAL *base, size_t stride) {
    st3_t s = {base, base + stride, base + 2 * stride};
    return s;
}

#define XA(i, j) ((size_t)(i) * cols + (size_t)(j))
#define XS(i, j) ((size_t)((i) - 1) * (size_t)L2max + (size_t)((j) - 1))
#define FOR_FWD(L1, L2)                                             \
    for (int k = 2; k <= (L1) + (L2); ++k)                          \
        for (int i = (k - (L2) > 1 ? k - (L2) : 1), j;              \
             i <= ((L1) < k - 1 ? (L1) : k - 1) && (j = k - i, 1); ++i)
#define FOR_REV(L1, L2)                                             \
    for (int k = (L1) + (L2); k >= 2; --k)                          \
        for (int i = (k - (L2) > 1 ? k - (L2) : 1), j;              \
             i <= ((L1) < k - 1 ? (L1) : k - 1) && (j = k - i, 1); ++i)

/* the options of each state at (i, j), as the reference forms them */
#define OPT_M(A, i, j) A.M[XA(i - 1, j - 1)], A.I[XA(i - 1, j - 1)], A.D[XA(i - 1, j - 1)]
#define OPT_I(A, i, j) A.M[XA(i - 1, j)] + go, A.I[XA(i - 1, j)] + ge, A.D[XA(i - 1, j)] + go
#define OPT_D(A, i, j) A.M[XA(i, j - 1)] + go, A.I[XA(i, j - 1)] + go, A.D[XA(i, j - 1)] + ge

/* :101-185 */
static REAL nwa_forward_one(const REAL *s, REAL *alpha, int L1, int L2, int L1max, int L2max, REAL go, REAL ge,
                            REAL T) {
    const size_t cols = (size_t)L2max + 1, n = ((size_t)L1max + 1) * cols;
    st3_t A = st3(alpha, n);
    for (size_t q = 0; q < n; ++q) A.M[q] = A.I[q] = A.D[q] = A_NINF;
    A.M[0] = 0;
    for (int i = 1; i <= L1; ++i) A.I[XA(i, 0)] = go + (REAL)(i - 1) * ge;
    for (int j = 1; j <= L2; ++j) A.D[XA(0, j)] = go + (REAL)(j - 1) * ge;
    FOR_FWD(L1, L2) {
        REAL sc = s[XS(i, j)];
        A.M[XA(i, j)] = sc + a_lse3(OPT_M(A, i, j), T);
        A.I[XA(i, j)] = a_lse3(OPT_I(A, i, j), T);
        A.D[XA(i, j)] = a_lse3(OPT_D(A, i, j), T);
    }
    const size_t f = XA(L1, L2);
    return a_lse3(A.M[f], A.I[f], A.D[f], T);
}

/* :191-356 */
static void nwa_backward_one(const REAL *s, const REAL *alpha, REAL S, REAL *beta, REAL *post, REAL *g_open,
                             REAL *g_ext, REAL *g_T, int L1, int L2, int L1max, int L2max, REAL go, REAL ge,
                             REAL T) {
    const size_t cols = (size_t)L2max + 1, n = ((size_t)L1max + 1) * cols;
    st3_t A = st3((REAL *)alpha, n), Bt = st3(beta, n);
    memset(beta, 0, sizeof(REAL) * 3 * n);
    memset(post, 0, sizeof(REAL) * (size_t)L1max * L2max);
    const size_t f = XA(L1, L2);
    REAL wm, wi, wd;
    a_w3(A.M[f], A.I[f], A.D[f], T, &wm, &wi, &wd);
    Bt.M[f] = wm;
    Bt.I[f] = wi;
    Bt.D[f] = wd;
    REAL so = 0, se = 0;
    ak_t ms = {0, 0};
    FOR_REV(L1, L2) {
        const size_t c = XA(i, j), cd = XA(i - 1, j - 1), cu = XA(i - 1, j), cl = XA(i, j - 1);
        REAL sc = s[XS(i, j)];
        REAL bM = Bt.M[c], bI = Bt.I[c], bD = Bt.D[c];
        REAL w1, w2, w3;
        if (bM > A_SKIP && a_lse3(OPT_M(A, i, j), T) > A_NINF) {
            a_w3(OPT_M(A, i, j), T, &w1, &w2, &w3);
            if (A.M[cd] > A_NINF) Bt.M[cd] += bM * w1;
            if (A.I[cd] > A_NINF) Bt.I[cd] += bM * w2;
            if (A.D[cd] > A_NINF) Bt.D[cd] += bM * w3;
            post[XS(i, j)] += bM;
            ak_add(&ms, bM * sc);
        }
        if (bI > A_SKIP && a_lse3(OPT_I(A, i, j), T) > A_NINF) {
            a_w3(OPT_I(A, i, j), T, &w1, &w2, &w3);
            Bt.M[cu] += bI * w1;
            Bt.I[cu] += bI * w2;
            Bt.D[cu] += bI * w3;
            so += bI * (w1 + w3);
            se += bI * w2;
        }
        if (bD > A_SKIP && a_lse3(OPT_D(A, i, j), T) > A_NINF) {
            a_w3(OPT_D(A, i, j), T, &w1, &w2, &w3);
            Bt.M[cl] += bD * w1;
            Bt.I[cl] += bD * w2;
            Bt.D[cl] += bD * w3;
            so += bD * (w1 + w2);
            se += bD * w3;
        }
    }
    /* leading gaps: boundary states set from open / ext directly */
    for (int i = 1; i <= L1; ++i) {
        REAL bb = Bt.I[XA(i, 0)];
        if (bb > A_SKIP) {
            so += bb;
            se += bb * (REAL)(i - 1);
        }
    }
    for (int j = 1; j <= L2; ++j) {
        REAL bb = Bt.D[XA(0, j)];
        if (bb > A_SKIP) {
            so += bb;
            se += bb * (REAL)(j - 1);
        }
    }
    *g_open = so;
    *g_ext = se;
    REAL expected = ms.sum + so * go + se * ge;
    *g_T = (S - expected) / T;
}

/* :362-650: tangent along V (H = d beta_M) */
static void nwa_hvp_one(const REAL *s, const REAL *v, const REAL *alpha, REAL *dalpha, REAL *beta, REAL *dbeta,
                        REAL *H, int L1, int L2, int L1max, int L2max, REAL go, REAL ge, REAL T) {
    const size_t cols = (size_t)L2max + 1, n = ((size_t)L1max + 1) * cols;
    st3_t A = st3((REAL *)alpha, n), dA = st3(dalpha, n), Bt = st3(beta, n), dB = st3(dbeta, n);
    memset(dalpha, 0, sizeof(REAL) * 3 * n);
    memset(beta, 0, sizeof(REAL) * 3 * n);
    memset(dbeta, 0, sizeof(REAL) * 3 * n);
    memset(H, 0, sizeof(REAL) * (size_t)L1max * L2max);
    (void)s;
    REAL w1, w2, w3;
    FOR_FWD(L1, L2) {
        const size_t c = XA(i, j), cd = XA(i - 1, j - 1), cu = XA(i - 1, j), cl = XA(i, j - 1);
        REAL Vs = v[XS(i, j)];
        if (a_lse3(OPT_M(A, i, j), T) > A_NINF) {
            a_w3(OPT_M(A, i, j), T, &w1, &w2, &w3);
            dA.M[c] = Vs + w1 * dA.M[cd] + w2 * dA.I[cd] + w3 * dA.D[cd];
        } else {
            dA.M[c] = 0;
        }
        if (a_lse3(OPT_I(A, i, j), T) > A_NINF) {
            a_w3(OPT_I(A, i, j), T, &w1, &w2, &w3);
            dA.I[c] = w1 * dA.M[cu] + w2 * dA.I[cu] + w3 * dA.D[cu];
        } else {
            dA.I[c] = 0;
        }
        if (a_lse3(OPT_D(A, i, j), T) > A_NINF) {
            a_w3(OPT_D(A, i, j), T, &w1, &w2, &w3);
            dA.D[c] = w1 * dA.M[cl] + w2 * dA.I[cl] + w3 * dA.D[cl];
        } else {
            dA.D[c] = 0;
        }
    }
    const size_t f = XA(L1, L2);
    REAL wm, wi, wd;
    a_w3(A.M[f], A.I[f], A.D[f], T, &wm, &wi, &wd);
    Bt.M[f] = wm;
    Bt.I[f] = wi;
    Bt.D[f] = wd;
    {
        REAL dm = dA.M[f], di = dA.I[f], dd = dA.D[f];
        REAL E = wm * dm + wi * di + wd * dd;
        dB.M[f] = wm * (dm - E) / T;
        dB.I[f] = wi * (di - E) / T;
        dB.D[f] = wd * (dd - E) / T;
    }
    FOR_REV(L1, L2) {
        const size_t c = XA(i, j), cd = XA(i - 1, j - 1), cu = XA(i - 1, j), cl = XA(i, j - 1);
        REAL bM = Bt.M[c], bI = Bt.I[c], bD = Bt.D[c];
        REAL dbM = dB.M[c], dbI = dB.I[c], dbD = dB.D[c];
        if (bM > A_SKIP || fabs((double)dbM) > (double)A_SKIP) {
            if (a_lse3(OPT_M(A, i, j), T) > A_NINF) {
                a_w3(OPT_M(A, i, j), T, &w1, &w2, &w3);
                REAL d1 = dA.M[cd], d2 = dA.I[cd], d3 = dA.D[cd];
                REAL E = w1 * d1 + w2 * d2 + w3 * d3;
                REAL e1 = w1 * (d1 - E) / T, e2 = w2 * (d2 - E) / T, e3 = w3 * (d3 - E) / T;
                if (A.M[cd] > A_NINF) { Bt.M[cd] += bM * w1; dB.M[cd] += dbM * w1 + bM * e1; }
                if (A.I[cd] > A_NINF) { Bt.I[cd] += bM * w2; dB.I[cd] += dbM * w2 + bM * e2; }
                if (A.D[cd] > A_NINF) { Bt.D[cd] += bM * w3; dB.D[cd] += dbM * w3 + bM * e3; }
                H[XS(i, j)] += dbM;
            }
        }
        if (bI > A_SKIP || fabs((double)dbI) > (double)A_SKIP) {
            if (a_lse3(OPT_I(A, i, j), T) > A_NINF) {
                a_w3(OPT_I(A, i, j), T, &w1, &w2, &w3);
                REAL d1 = dA.M[cu], d2 = dA.I[cu], d3 = dA.D[cu];
                REAL E = w1 * d1 + w2 * d2 + w3 * d3;
                REAL e1 = w1 * (d1 - E) / T, e2 = w2 * (d2 - E) / T, e3 = w3 * (d3 - E) / T;
                Bt.M[cu] += bI * w1; dB.M[cu] += dbI * w1 + bI * e1;
                Bt.I[cu] += bI * w2; dB.I[cu] += dbI * w2 + bI * e2;
                Bt.D[cu] += bI * w3; dB.D[cu] += dbI * w3 + bI * e3;
            }
        }
        if (bD > A_SKIP || fabs((double)dbD) > (double)A_SKIP) {
            if (a_lse3(OPT_D(A, i, j), T) > A_NINF) {
                a_w3(OPT_D(A, i, j), T, &w1, &w2, &w3);
                REAL d1 = dA.M[cl], d2 = dA.I[cl], d3 = dA.D[cl];
                REAL E = w1 * d1 + w2 * d2 + w3 * d3;
                REAL e1 = w1 * (d1 - E) / T, e2 = w2 * (d2 - E) / T, e3 = w3 * (d3 - E) / T;
                Bt.M[cl] += bD * w1; dB.M[cl] += dbD * w1 + bD * e1;
                Bt.I[cl] += bD * w2; dB.I[cl] += dbD * w2 + bD * e2;
                Bt.D[cl] += bD * w3; dB.D[cl] += dbD * w3 + bD * e3;
            }
        }
    }
}

/* :656-1000: U = d alpha / d theta forward, W = d beta / d theta reverse,
 * dP/dtheta = W_M.  param_type 0 = gap_open, 1 = gap_ext, 2 = temperature. */
static void nwa_param_one(const REAL *s, const REAL *alpha, REAL *U, REAL *beta, REAL *W, REAL *dP, int L1, int L2,
                          int L1max, int L2max, REAL go, REAL ge, REAL T, int pt) {
    const size_t cols = (size_t)L2max + 1, n = ((size_t)L1max + 1) * cols;
    st3_t A = st3((REAL *)alpha, n), u = st3(U, n), Bt = st3(beta, n), w = st3(W, n);
    memset(U, 0, sizeof(REAL) * 3 * n);
    memset(beta, 0, sizeof(REAL) * 3 * n);
    memset(W, 0, sizeof(REAL) * 3 * n);
    memset(dP, 0, sizeof(REAL) * (size_t)L1max * L2max);
    if (pt == 0) {
        for (int i = 1; i <= L1; ++i) u.I[XA(i, 0)] = 1;
        for (int j = 1; j <= L2; ++j) u.D[XA(0, j)] = 1;
    } else if (pt == 1) {
        for (int i = 1; i <= L1; ++i) u.I[XA(i, 0)] = (REAL)(i - 1);
        for (int j = 1; j <= L2; ++j) u.D[XA(0, j)] = (REAL)(j - 1);
    }
    /* the direct derivative of each option's gap term */
    const REAL oI1 = pt == 0 ? 1 : 0, oI2 = pt == 1 ? 1 : 0, oI3 = pt == 0 ? 1 : 0;
    const REAL oD1 = pt == 0 ? 1 : 0, oD2 = pt == 0 ? 1 : 0, oD3 = pt == 1 ? 1 : 0;
    REAL w1, w2, w3;
    FOR_FWD(L1, L2) {
        const size_t c = XA(i, j), cd = XA(i - 1, j - 1), cu = XA(i - 1, j), cl = XA(i, j - 1);
        REAL m1 = A.M[cd], m2 = A.I[cd], m3 = A.D[cd];
        if (a_lse3(m1, m2, m3, T) > A_NINF) {
            a_w3(m1, m2, m3, T, &w1, &w2, &w3);
            REAL x = w1 * u.M[cd] + w2 * u.I[cd] + w3 * u.D[cd];
            if (pt == 2) {
                REAL Ev = w1 * m1 + w2 * m2 + w3 * m3;
                REAL sc = s[XS(i, j)];
                x += (A.M[c] - (Ev + sc)) / T;
            }
            u.M[c] = x;
        }
        REAL i1 = A.M[cu] + go, i2 = A.I[cu] + ge, i3 = A.D[cu] + go;
        if (a_lse3(i1, i2, i3, T) > A_NINF) {
            a_w3(i1, i2, i3, T, &w1, &w2, &w3);
            REAL x = w1 * (u.M[cu] + oI1) + w2 * (u.I[cu] + oI2) + w3 * (u.D[cu] + oI3);
            if (pt == 2) {
                REAL Ev = w1 * i1 + w2 * i2 + w3 * i3;
                x += (A.I[c] - Ev) / T;
            }
            u.I[c] = x;
        }
        REAL d1 = A.M[cl] + go, d2 = A.I[cl] + go, d3 = A.D[cl] + ge;
        if (a_lse3(d1, d2, d3, T) > A_NINF) {
            a_w3(d1, d2, d3, T, &w1, &w2, &w3);
            REAL x = w1 * (u.M[cl] + oD1) + w2 * (u.I[cl] + oD2) + w3 * (u.D[cl] + oD3);
            if (pt == 2) {
                REAL Ev = w1 * d1 + w2 * d2 + w3 * d3;
                x += (A.D[c] - Ev) / T;
            }
            u.D[c] = x;
        }
    }
    const size_t f = XA(L1, L2);
    REAL wm, wi, wd;
    a_w3(A.M[f], A.I[f], A.D[f], T, &wm, &wi, &wd);
    Bt.M[f] = wm;
    Bt.I[f] = wi;
    Bt.D[f] = wd;
    {
        REAL um = u.M[f], ui = u.I[f], ud = u.D[f];
        REAL E = wm * um + wi * ui + wd * ud;
        REAL em = wm * (um - E) / T, ei = wi * (ui - E) / T, ed = wd * (ud - E) / T;
        if (pt == 2) {
            REAL Ev = wm * A.M[f] + wi * A.I[f] + wd * A.D[f];
            REAL iT2 = (REAL)1 / (T * T);
            em += wm * (Ev - A.M[f]) * iT2;
            ei += wi * (Ev - A.I[f]) * iT2;
            ed += wd * (Ev - A.D[f]) * iT2;
        }
        w.M[f] = em;
        w.I[f] = ei;
        w.D[f] = ed;
    }
    FOR_REV(L1, L2) {
        const size_t c = XA(i, j), cd = XA(i - 1, j - 1), cu = XA(i - 1, j), cl = XA(i, j - 1);
        REAL bM = Bt.M[c], bI = Bt.I[c], bD = Bt.D[c];
        REAL wM = w.M[c], wI = w.I[c], wD = w.D[c];
        if (bM > A_SKIP || fabs((double)wM) > (double)A_SKIP) {
            REAL m1 = A.M[cd], m2 = A.I[cd], m3 = A.D[cd];
            if (a_lse3(m1, m2, m3, T) > A_NINF) {
                a_w3(m1, m2, m3, T, &w1, &w2, &w3);
                REAL u1 = u.M[cd], u2 = u.I[cd], u3 = u.D[cd];
                REAL E = w1 * u1 + w2 * u2 + w3 * u3;
                REAL e1 = w1 * (u1 - E) / T, e2 = w2 * (u2 - E) / T, e3 = w3 * (u3 - E) / T;
                if (pt == 2) {
                    REAL Ev = w1 * m1 + w2 * m2 + w3 * m3;
                    REAL iT2 = (REAL)1 / (T * T);
                    e1 += w1 * (Ev - m1) * iT2;
                    e2 += w2 * (Ev - m2) * iT2;
                    e3 += w3 * (Ev - m3) * iT2;
                }
                if (m1 > A_NINF) { Bt.M[cd] += bM * w1; w.M[cd] += wM * w1 + bM * e1; }
                if (m2 > A_NINF) { Bt.I[cd] += bM * w2; w.I[cd] += wM * w2 + bM * e2; }
                if (m3 > A_NINF) { Bt.D[cd] += bM * w3; w.D[cd] += wM * w3 + bM * e3; }
                dP[XS(i, j)] += wM;
            }
        }
        if (bI > A_SKIP || fabs((double)wI) > (double)A_SKIP) {
            REAL i1 = A.M[cu] + go, i2 = A.I[cu] + ge, i3 = A.D[cu] + go;
            if (a_lse3(i1, i2, i3, T) > A_NINF) {
                a_w3(i1, i2, i3, T, &w1, &w2, &w3);
                REAL u1 = u.M[cu] + oI1, u2 = u.I[cu] + oI2, u3 = u.D[cu] + oI3;
                REAL E = w1 * u1 + w2 * u2 + w3 * u3;
                REAL e1 = w1 * (u1 - E) / T, e2 = w2 * (u2 - E) / T, e3 = w3 * (u3 - E) / T;
                if (pt == 2) {
                    REAL Ev = w1 * i1 + w2 * i2 + w3 * i3;
                    REAL iT2 = (REAL)1 / (T * T);
                    e1 += w1 * (Ev - i1) * iT2;
                    e2 += w2 * (Ev - i2) * iT2;
                    e3 += w3 * (Ev - i3) * iT2;
                }
                Bt.M[cu] += bI * w1; w.M[cu] += wI * w1 + bI * e1;
                Bt.I[cu] += bI * w2; w.I[cu] += wI * w2 + bI * e2;
                Bt.D[cu] += bI * w3; w.D[cu] += wI * w3 + bI * e3;
            }
        }
        if (bD > A_SKIP || fabs((double)wD) > (double)A_SKIP) {
            REAL d1 = A.M[cl] + go, d2 = A.I[cl] + go, d3 = A.D[cl] + ge;
            if (a_lse3(d1, d2, d3, T) > A_NINF) {
                a_w3(d1, d2, d3, T, &w1, &w2, &w3);
                REAL u1 = u.M[cl] + oD1, u2 = u.I[cl] + oD2, u3 = u.D[cl] + oD3;
                REAL E = w1 * u1 + w2 * u2 + w3 * u3;
                REAL e1 = w1 * (u1 - E) / T, e2 = w2 * (u2 - E) / T, e3 = w3 * (u3 - E) / T;
                if (pt == 2) {
                    REAL Ev = w1 * d1 + w2 * d2 + w3 * d3;
                    REAL iT2 = (REAL)1 / (T * T);
                    e1 += w1 * (Ev - d1) * iT2;
                    e2 += w2 * (Ev - d2) * iT2;
                    e3 += w3 * (Ev - d3) * iT2;
                }
                Bt.M[cl] += bD * w1; w.M[cl] += wD * w1 + bD * e1;
                Bt.I[cl] += bD * w2; w.I[cl] += wD * w2 + bD * e2;
                Bt.D[cl] += bD * w3; w.D[cl] += wD * w3 + bD * e3;
            }
        }
    }
}

/* ------------------------------------------------------------------ batch API */
static inline void a_lens(const int *lengths, int b, int L1max, int L2max, int *L1, int *L2) {
    *L1 = lengths ? lengths[2 * b] : L1max;
    *L2 = lengths ? lengths[2 * b + 1] : L2max;
}

void SFX(oracle_nwa_forward)(const REAL *scores, const int *lengths, int B, int L1max, int L2max, REAL go, REAL ge,
                             REAL T, REAL *alpha, REAL *value) {
    const size_t sp = (size_t)L1max * L2max, ap = 3 * ((size_t)L1max + 1) * ((size_t)L2max + 1);
#pragma omp parallel for schedule(dynamic, 1)
    for (int b = 0; b < B; ++b) {
        int L1, L2;
        a_lens(lengths, b, L1max, L2max, &L1, &L2);
        value[b] = nwa_forward_one(scores + b * sp, alpha + b * ap, L1, L2, L1max, L2max, go, ge, T);
    }
}

void SFX(oracle_nwa_backward)(const REAL *scores, const int *lengths, int B, int L1max, int L2max, REAL go,
                              REAL ge, REAL T, const REAL *alpha, const REAL *value, REAL *beta, REAL *post,
                              REAL *g_open, REAL *g_ext, REAL *g_T) {
    const size_t sp = (size_t)L1max * L2max, ap = 3 * ((size_t)L1max + 1) * ((size_t)L2max + 1);
#pragma omp parallel for schedule(dynamic, 1)
    for (int b = 0; b < B; ++b) {
        int L1, L2;
        a_lens(lengths, b, L1max, L2max, &L1, &L2);
        nwa_backward_one(scores + b * sp, alpha + b * ap, value[b], beta + b * ap, post + b * sp, g_open + b,
                         g_ext + b, g_T + b, L1, L2, L1max, L2max, go, ge, T);
    }
}

void SFX(oracle_nwa_hvp)(const REAL *scores, const REAL *V, const int *lengths, int B, int L1max, int L2max,
                         REAL go, REAL ge, REAL T, const REAL *alpha, REAL *dalpha, REAL *beta, REAL *dbeta,
                         REAL *H) {
    const size_t sp = (size_t)L1max * L2max, ap = 3 * ((size_t)L1max + 1) * ((size_t)L2max + 1);
#pragma omp parallel for schedule(dynamic, 1)
    for (int b = 0; b < B; ++b) {
        int L1, L2;
        a_lens(lengths, b, L1max, L2max, &L1, &L2);
        nwa_hvp_one(scores + b * sp, V + b * sp, alpha + b * ap, dalpha + b * ap, beta + b * ap, dbeta + b * ap,
                    H + b * sp, L1, L2, L1max, L2max, go, ge, T);
    }
}

void SFX(oracle_nwa_param_grad)(const REAL *scores, const int *lengths, int B, int L1max, int L2max, REAL go,
                                REAL ge, REAL T, const REAL *alpha, REAL *U, REAL *beta, REAL *W, REAL *dP,
                                int param_type) {
    const size_t sp = (size_t)L1max * L2max, ap = 3 * ((size_t)L1max + 1) * ((size_t)L2max + 1);
#pragma omp parallel for schedule(dynamic, 1)
    for (int b = 0; b < B; ++b) {
        int L1, L2;
        a_lens(lengths, b, L1max, L2max, &L1, &L2);
        nwa_param_one(scores + b * sp, alpha + b * ap, U + b * ap, beta + b * ap, W + b * ap, dP + b * sp, L1, L2,
                      L1max, L2max, go, ge, T, param_type);
    }
}
