// sw_plane.cu -- "plane" engine: one CTA per problem, DP planes in a caller
// workspace, anti-diagonal sweeps inside a single launch.
//
// This engine implements every mode of the soft Smith-Waterman operator family
// (linear and affine gap): value + marginals + parameter gradients, the
// Hessian-vector product, and the parameter Jacobians dP/dtheta.  It replaces
// the reference's per-anti-diagonal launch loops (src/sw/kernels.cu:1144-1421,
// src/sw_affine/kernels.cu:1291-1511) with one launch per operator: the
// anti-diagonal loop runs on the device with a CTA barrier per diagonal, and the
// reverse pass is written in *gather* form (each cell pulls beta from its three
// successors) so there are no float atomics and results are bitwise
// deterministic run to run.
//
// Recurrences (natural units, reference src/sw/kernels_cpu.cpp:70-279 and
// src/sw_affine/kernels_cpu.cpp:94-346); this file evaluates them in the base-2
// scaled domain described in sw_common.cuh:
//   linear : a_ij = LSE(a_{i-1,j-1}+s [i>1,j>1], a_{i-1,j}+g [i>1], a_{i,j-1}+g [j>1], s)
//   affine : M = LSE(M_d+s, I_d+s, D_d+s [i>1,j>1], s);  I = LSE(M_u+go, I_u+ge) [i>1];
//            D = LSE(M_l+go, D_l+ge) [j>1]
//   value  : S = LSE over all valid cells and states, including alpha[0,0] = 0.
//
// The fast path for value+marginals (sw_wavefront.cu) supersedes this engine for
// MODE_MARG when shapes allow; this engine remains the general implementation.
#include "sw_common.cuh"
#include "sw_internal.h"

namespace d2pb {

constexpr int kPlaneThreads = 512;

// --------------------------------------------------------------------------
// helpers
// --------------------------------------------------------------------------
__device__ __forceinline__ float read_param(const float* dev, float host) {
    return dev ? __ldg(dev) : host;
}

// Zero the padded (masked) part of an output plane [L1max, L2max] for a problem
// whose valid region is [L1, L2].
__device__ void zero_padding(float* out, int L1max, int L2max, int L1, int L2) {
    if (!out) return;
    if (L1 == L1max && L2 == L2max) return;
    const int n = L1max * L2max;
    for (int q = threadIdx.x; q < n; q += blockDim.x) {
        int i = q / L2max, j = q - i * L2max;
        if (i >= L1 || j >= L2) out[q] = 0.f;
    }
}

// ==========================================================================
// LINEAR GAP
// ==========================================================================
// workspace planes per problem (each L1max*L2max floats):
//   0: a (scaled alpha)  1: beta  2: tangent forward (dalpha or U)
//   3: tangent backward (dbeta or W)  4: R = (alpha - E[v]) / T  (PT mode)
template <int MODE>
__global__ void __launch_bounds__(kPlaneThreads) lin_plane_kernel(SwArgs p) {
    __shared__ __align__(16) float red[4 * 32];
    __shared__ float sh_aS, sh_dS;

    const int b = blockIdx.x;
    const int L1m = p.L1, L2m = p.L2;
    // lengths are validated by the caller; clamp so a bad value can never index
    // outside the padded problem
    const int L1 = p.lengths ? min(max(p.lengths[2 * b], 0), L1m) : L1m;
    const int L2 = p.lengths ? min(max(p.lengths[2 * b + 1], 0), L2m) : L2m;
    const float gapn = read_param(p.gap_dev, p.gap);
    const float T = read_param(p.temp_dev, p.temp);
    const float c = kLog2e / T;     // natural -> scaled
    const float ic = 1.f / c;       // scaled -> natural
    const float iT = 1.f / T;
    const float g = gapn * c;

    const size_t plane = (size_t)L1m * L2m;
    const float* __restrict__ s = p.scores + (size_t)b * plane;
    const float* __restrict__ V = (MODE == MODE_HVP) ? p.tangent + (size_t)b * plane : nullptr;
    float* ws = p.ws + (size_t)b * plane * lin_planes(MODE);
    float* __restrict__ A = ws;
    float* __restrict__ Bt = ws + plane;
    float* __restrict__ TG = ws + 2 * plane;
    float* __restrict__ TB = ws + 3 * plane;
    float* __restrict__ RR = ws + 4 * plane;
    float* __restrict__ out = p.out ? p.out + (size_t)b * plane : nullptr;

    zero_padding(out, L1m, L2m, L1, L2);
    const int W = L2m;  // row stride

    // ---------------- forward sweep ----------------
    OnlineLse acc;
    acc.init();
    if (threadIdx.x == 0) acc.add(0.f, 0.f, 0.f);  // alpha[0,0] = 0 (d alpha = 0)
    for (int k = 2; k <= L1 + L2; ++k) {
        const int ilo = max(1, k - L2), ihi = min(L1, k - 1);
        for (int i = ilo + threadIdx.x; i <= ihi; i += blockDim.x) {
            const int j = k - i;
            const size_t q = (size_t)(i - 1) * W + (j - 1);
            const float x = s[q] * c;
            const bool up = i > 1, lf = j > 1, dg = up && lf;
            const float v0 = dg ? A[q - W - 1] + x : kNeg;
            const float v1 = up ? A[q - W] + g : kNeg;
            const float v2 = lf ? A[q - 1] + g : kNeg;
            const Lse4 r = lse4(v0, v1, v2, x);
            A[q] = r.a;
            float ya = 0.f, yb = 0.f;
            if (MODE != MODE_MARG) {
                const float inv = 1.f / r.sum;
                const float w0 = r.t0 * inv, w1 = r.t1 * inv, w2 = r.t2 * inv, w3 = r.t3 * inv;
                float tg;
                if (MODE == MODE_HVP) {
                    const float vv = V[q];
                    const float d0 = dg ? TG[q - W - 1] + vv : 0.f;
                    const float d1 = up ? TG[q - W] : 0.f;
                    const float d2 = lf ? TG[q - 1] : 0.f;
                    tg = w0 * d0 + w1 * d1 + w2 * d2 + w3 * vv;
                } else {
                    const float pg = (MODE == MODE_PGAP) ? 1.f : 0.f;
                    const float d0 = dg ? TG[q - W - 1] : 0.f;
                    const float d1 = (up ? TG[q - W] : 0.f) + pg;
                    const float d2 = (lf ? TG[q - 1] : 0.f) + pg;
                    tg = w0 * d0 + w1 * d1 + w2 * d2;
                    if (MODE == MODE_PT) {
                        // (alpha - E[v]) / T, E[v] over the four logits (natural units)
                        const float ev = (w0 * (dg ? v0 : 0.f) + w1 * (up ? v1 : 0.f) +
                                          w2 * (lf ? v2 : 0.f) + w3 * x);
                        const float rt = (r.a - ev) * ic * iT;
                        RR[q] = rt;
                        tg += rt;
                        yb = r.a * ic;  // alpha (natural), for sum p*alpha
                    }
                }
                TG[q] = tg;
                ya = tg;
            }
            acc.add(r.a, ya, yb);
        }
        __syncthreads();
    }
    const OnlineLse tot = block_lse(acc, red);
    if (threadIdx.x == 0) {
        const float aS = tot.m + lg2f(tot.s);
        sh_aS = aS;
        float dS = 0.f;
        if (MODE == MODE_HVP || MODE == MODE_PGAP) dS = tot.y1 / tot.s;
        if (MODE == MODE_PT) {
            const float Snat = aS * ic;
            dS = tot.y1 / tot.s + (Snat - tot.y2 / tot.s) * iT;
        }
        sh_dS = dS;
        if (p.value) p.value[b] = aS * ic;
    }
    __syncthreads();
    const float aS = sh_aS;
    const float dS = sh_dS;
    const float Snat = aS * ic;

    // ---------------- reverse sweep (gather form) ----------------
    double gsum = 0.0, msum = 0.0;
    float dsum = 0.f;
    for (int k = L1 + L2; k >= 2; --k) {
        const int ilo = max(1, k - L2), ihi = min(L1, k - 1);
        for (int i = ilo + threadIdx.x; i <= ihi; i += blockDim.x) {
            const int j = k - i;
            const size_t q = (size_t)(i - 1) * W + (j - 1);
            const float a = A[q];
            const float sc = s[q];
            const float x = sc * c;
            const bool up = i > 1, lf = j > 1, dg = up && lf;
            const bool hasD = (i < L1) && (j < L2), hasU = i < L1, hasL = j < L2;
            const float binit = ex2f(fminf(a - aS, 0.f));
            float beta = binit;
            // successor weights: transitions (i,j) -> succ
            float wD = 0.f, wU = 0.f, wL = 0.f;
            if (hasD) { wD = ex2f(a + s[q + W + 1] * c - A[q + W + 1]); beta += Bt[q + W + 1] * wD; }
            if (hasU) { wU = ex2f(a + g - A[q + W]); beta += Bt[q + W] * wU; }
            if (hasL) { wL = ex2f(a + g - A[q + 1]); beta += Bt[q + 1] * wL; }
            Bt[q] = beta;
            // own incoming weights
            const float wa = dg ? ex2f(A[q - W - 1] + x - a) : 0.f;
            const float wsk = ex2f(x - a);
            if (MODE == MODE_MARG) {
                const float vu = up ? A[q - W] + g : kNeg, vl = lf ? A[q - 1] + g : kNeg;
                const float va = dg ? A[q - W - 1] + x : kNeg;
                const float wu = up ? ex2f(vu - a) : 0.f;
                const float wl = lf ? ex2f(vl - a) : 0.f;
                const float mu = beta * (wa + wsk);
                if (out) out[q] = mu;
                gsum += (double)(beta * (wu + wl));
                // dS/dT = entropy of the path distribution (see the note at the
                // end of the kernel): visit probability x local choice entropy
                // + end-cell entropy; all terms are >= 0 (no cancellation).
                const float hloc = (dg ? wa * (a - va) : 0.f) + (up ? wu * (a - vu) : 0.f) +
                                   (lf ? wl * (a - vl) : 0.f) + wsk * (a - x);
                msum += (double)beta * (double)hloc + (double)binit * (double)(aS - a);
            } else if (MODE == MODE_HVP) {
                const float da = TG[q];
                const float vv = V[q];
                float db = binit * (da - dS) * iT;
                if (hasD) {
                    const size_t qs = q + W + 1;
                    const float dw = wD * (da + V[qs] - TG[qs]) * iT;
                    db += TB[qs] * wD + Bt[qs] * dw;
                }
                if (hasU) {
                    const size_t qs = q + W;
                    const float dw = wU * (da - TG[qs]) * iT;
                    db += TB[qs] * wU + Bt[qs] * dw;
                }
                if (hasL) {
                    const size_t qs = q + 1;
                    const float dw = wL * (da - TG[qs]) * iT;
                    db += TB[qs] * wL + Bt[qs] * dw;
                }
                TB[q] = db;
                const float dva = dg ? TG[q - W - 1] + vv : 0.f;
                const float dwa = wa * (dva - da) * iT;
                const float dws = wsk * (vv - da) * iT;
                if (out) out[q] = db * (wa + wsk) + beta * (dwa + dws);
            } else {  // parameter Jacobian
                const bool PT = (MODE == MODE_PT);
                const float pg = (MODE == MODE_PGAP) ? 1.f : 0.f;
                const float u = TG[q];
                float Wv = binit * (u - dS) * iT;
                if (PT) Wv -= binit * ((a - aS) * ic) * iT * iT;
                const float an = a * ic;  // alpha (natural)
                if (hasD) {
                    const size_t qs = q + W + 1;
                    const float rs = PT ? RR[qs] : 0.f;
                    const float Edu = TG[qs] - rs;
                    float dw = wD * (u - Edu) * iT;
                    if (PT) {
                        const float Ev = A[qs] * ic - T * rs;
                        const float vtr = an + s[qs];  // logit of the align transition (natural)
                        dw += wD * (Ev - vtr) * iT * iT;
                    }
                    Wv += TB[qs] * wD + Bt[qs] * dw;
                }
                if (hasU) {
                    const size_t qs = q + W;
                    const float rs = PT ? RR[qs] : 0.f;
                    const float Edu = TG[qs] - rs;
                    float dw = wU * (u + pg - Edu) * iT;
                    if (PT) {
                        const float Ev = A[qs] * ic - T * rs;
                        dw += wU * (Ev - (an + gapn)) * iT * iT;
                    }
                    Wv += TB[qs] * wU + Bt[qs] * dw;
                }
                if (hasL) {
                    const size_t qs = q + 1;
                    const float rs = PT ? RR[qs] : 0.f;
                    const float Edu = TG[qs] - rs;
                    float dw = wL * (u + pg - Edu) * iT;
                    if (PT) {
                        const float Ev = A[qs] * ic - T * rs;
                        dw += wL * (Ev - (an + gapn)) * iT * iT;
                    }
                    Wv += TB[qs] * wL + Bt[qs] * dw;
                }
                TB[q] = Wv;
                const float r0 = PT ? RR[q] : 0.f;
                const float Edu = u - r0;
                const float dua = dg ? TG[q - W - 1] : 0.f;
                float dwa = wa * (dua - Edu) * iT;
                float dws = wsk * (0.f - Edu) * iT;
                if (PT) {
                    const float Ev = an - T * r0;
                    const float va = dg ? A[q - W - 1] * ic + sc : 0.f;
                    dwa += wa * (Ev - va) * iT * iT;
                    dws += wsk * (Ev - sc) * iT * iT;
                }
                const float dPv = Wv * (wa + wsk) + beta * (dwa + dws);
                if (out) out[q] = dPv;
                if (p.dot_with) dsum += p.dot_with[(size_t)b * plane + q] * dPv;
            }
        }
        __syncthreads();
    }
    if (MODE >= MODE_PGAP && p.dot_with && p.dot_out) {
        const float D = block_sum(dsum, red);
        if (threadIdx.x == 0) p.dot_out[b] = D;
    }
    if (MODE == MODE_MARG && (p.grad_gap || p.grad_T)) {
        // The origin alpha[0,0] = 0 is a possible end state (empty alignment).
        if (threadIdx.x == 0) msum += (double)ex2f(-aS) * (double)aS;
        const double G = block_sum_d(gsum, reinterpret_cast<double*>(red));
        const double H = block_sum_d(msum, reinterpret_cast<double*>(red));
        if (threadIdx.x == 0) {
            if (p.grad_gap) p.grad_gap[b] = (float)G;
            // dS/dT = (S - E[path score]) / T  (reference kernels_cpu.cpp:274-276)
            //       = H[path]  (entropy of the Gibbs path distribution, nats),
            // evaluated as a sum of non-negative terms in base-2 units.
            if (p.grad_T) p.grad_T[b] = (float)(H * (double)kLn2);
        }
    }
}

// ==========================================================================
// AFFINE GAP
// ==========================================================================
// planes per problem: alpha M,I,D (0-2), beta M,I,D (3-5), tangent fwd M,I,D
// (6-8), tangent bwd M,I,D (9-11), R M,I,D (12-14).
template <int MODE>
__global__ void __launch_bounds__(kPlaneThreads) aff_plane_kernel(SwArgs p) {
    __shared__ __align__(16) float red[4 * 32];
    __shared__ float sh_aS, sh_dS;

    const int b = blockIdx.x;
    const int L1m = p.L1, L2m = p.L2;
    // lengths are validated by the caller; clamp so a bad value can never index
    // outside the padded problem
    const int L1 = p.lengths ? min(max(p.lengths[2 * b], 0), L1m) : L1m;
    const int L2 = p.lengths ? min(max(p.lengths[2 * b + 1], 0), L2m) : L2m;
    const float gon = read_param(p.gap_dev, p.gap);
    const float gen = read_param(p.gap2_dev, p.gap2);
    const float T = read_param(p.temp_dev, p.temp);
    const float c = kLog2e / T, ic = 1.f / c, iT = 1.f / T;
    const float go = gon * c, ge = gen * c;

    const size_t plane = (size_t)L1m * L2m;
    const float* __restrict__ s = p.scores + (size_t)b * plane;
    const __nv_bfloat16* __restrict__ sbf = p.scores_bf16 ? p.scores_bf16 + (size_t)b * plane : nullptr;
    const float* __restrict__ V = (MODE == MODE_HVP) ? p.tangent + (size_t)b * plane : nullptr;
    float* ws = p.ws + (size_t)b * plane * aff_planes(MODE);
    float* AM = ws;
    float* AI = ws + plane;
    float* AD = ws + 2 * plane;
    float* BM = ws + 3 * plane;
    float* BI = ws + 4 * plane;
    float* BD = ws + 5 * plane;
    float* TM = ws + 6 * plane;
    float* TI = ws + 7 * plane;
    float* TD = ws + 8 * plane;
    float* XM = ws + 9 * plane;
    float* XI = ws + 10 * plane;
    float* XD = ws + 11 * plane;
    float* RM = ws + 12 * plane;
    float* RI = ws + 13 * plane;
    float* RD = ws + 14 * plane;
    float* __restrict__ out = p.out ? p.out + (size_t)b * plane : nullptr;
    zero_padding(out, L1m, L2m, L1, L2);
    const int W = L2m;
    auto score = [&](size_t q) -> float { return sbf ? __bfloat162float(sbf[q]) : s[q]; };

    OnlineLse acc;
    acc.init();
    if (threadIdx.x == 0) acc.add(0.f, 0.f, 0.f);
    const float pgo = (MODE == MODE_PGAP) ? 1.f : 0.f;   // param 0: gap_open
    const float pge = (MODE == MODE_PGE) ? 1.f : 0.f;    // param 1: gap_ext
    const bool PT = (MODE == MODE_PT);

    for (int k = 2; k <= L1 + L2; ++k) {
        const int ilo = max(1, k - L2), ihi = min(L1, k - 1);
        for (int i = ilo + threadIdx.x; i <= ihi; i += blockDim.x) {
            const int j = k - i;
            const size_t q = (size_t)(i - 1) * W + (j - 1);
            const float sc = score(q);
            const float x = sc * c;
            const bool up = i > 1, lf = j > 1, dg = up && lf;
            const float m0 = dg ? AM[q - W - 1] + x : kNeg;
            const float m1 = dg ? AI[q - W - 1] + x : kNeg;
            const float m2 = dg ? AD[q - W - 1] + x : kNeg;
            const Lse4 rm = lse4(m0, m1, m2, x);
            const float i0 = up ? AM[q - W] + go : kNeg;
            const float i1 = up ? AI[q - W] + ge : kNeg;
            const Lse2 ri = lse2(i0, i1);
            const float d0 = lf ? AM[q - 1] + go : kNeg;
            const float d1 = lf ? AD[q - 1] + ge : kNeg;
            const Lse2 rd = lse2(d0, d1);
            AM[q] = rm.a;
            AI[q] = ri.a;
            AD[q] = rd.a;
            if (MODE == MODE_MARG) {
                acc.add(rm.a);
                acc.add(ri.a);
                acc.add(rd.a);
            } else {
                const float im = 1.f / rm.sum, ii = 1.f / ri.sum, id = 1.f / rd.sum;
                const float wm0 = rm.t0 * im, wm1 = rm.t1 * im, wm2 = rm.t2 * im, wm3 = rm.t3 * im;
                const float wi0 = ri.t0 * ii, wi1 = ri.t1 * ii;
                const float wd0 = rd.t0 * id, wd1 = rd.t1 * id;
                float tm, ti, td;
                if (MODE == MODE_HVP) {
                    const float vv = V[q];
                    tm = wm0 * (dg ? TM[q - W - 1] + vv : 0.f) + wm1 * (dg ? TI[q - W - 1] + vv : 0.f) +
                         wm2 * (dg ? TD[q - W - 1] + vv : 0.f) + wm3 * vv;
                    ti = up ? wi0 * TM[q - W] + wi1 * TI[q - W] : 0.f;
                    td = lf ? wd0 * TM[q - 1] + wd1 * TD[q - 1] : 0.f;
                } else {
                    tm = dg ? wm0 * TM[q - W - 1] + wm1 * TI[q - W - 1] + wm2 * TD[q - W - 1] : 0.f;
                    ti = wi0 * ((up ? TM[q - W] : 0.f) + pgo) + wi1 * ((up ? TI[q - W] : 0.f) + pge);
                    td = wd0 * ((lf ? TM[q - 1] : 0.f) + pgo) + wd1 * ((lf ? TD[q - 1] : 0.f) + pge);
                    if (PT) {
                        const float evm = wm0 * (dg ? m0 : 0.f) + wm1 * (dg ? m1 : 0.f) +
                                          wm2 * (dg ? m2 : 0.f) + wm3 * x;
                        const float rmv = (rm.a - evm) * ic * iT;
                        float riv = 0.f, rdv = 0.f;
                        if (ri.a > kNegThresh) riv = (ri.a - (wi0 * i0 + wi1 * i1)) * ic * iT;
                        if (rd.a > kNegThresh) rdv = (rd.a - (wd0 * d0 + wd1 * d1)) * ic * iT;
                        RM[q] = rmv;
                        RI[q] = riv;
                        RD[q] = rdv;
                        tm += rmv;
                        ti += riv;
                        td += rdv;
                    }
                }
                TM[q] = tm;
                TI[q] = ti;
                TD[q] = td;
                acc.add(rm.a, tm, PT ? rm.a * ic : 0.f);
                acc.add(ri.a, ti, PT ? ri.a * ic : 0.f);
                acc.add(rd.a, td, PT ? rd.a * ic : 0.f);
            }
        }
        __syncthreads();
    }
    const OnlineLse tot = block_lse(acc, red);
    if (threadIdx.x == 0) {
        const float aS = tot.m + lg2f(tot.s);
        sh_aS = aS;
        float dS = 0.f;
        if (MODE == MODE_HVP || MODE == MODE_PGAP || MODE == MODE_PGE) dS = tot.y1 / tot.s;
        if (PT) dS = tot.y1 / tot.s + (aS * ic - tot.y2 / tot.s) * iT;
        sh_dS = dS;
        if (p.value) p.value[b] = aS * ic;
    }
    __syncthreads();
    const float aS = sh_aS, dS = sh_dS, Snat = aS * ic;

    double so = 0.0, se = 0.0, msum = 0.0;
    float dsum = 0.f;
    for (int k = L1 + L2; k >= 2; --k) {
        const int ilo = max(1, k - L2), ihi = min(L1, k - 1);
        for (int i = ilo + threadIdx.x; i <= ihi; i += blockDim.x) {
            const int j = k - i;
            const size_t q = (size_t)(i - 1) * W + (j - 1);
            const float sc = score(q);
            const bool up = i > 1, lf = j > 1;
            const bool hasD = (i < L1) && (j < L2), hasU = i < L1, hasL = j < L2;
            const float am = AM[q], ai = AI[q], ad = AD[q];
            const float bim = ex2f(fminf(am - aS, 0.f));
            const float bii = ex2f(fminf(ai - aS, 0.f));
            const float bid = ex2f(fminf(ad - aS, 0.f));
            float bm = bim, bi = bii, bd = bid;
            // successor transition weights
            float xs = 0.f, wMM = 0.f, wIM = 0.f, wDM = 0.f, wMI = 0.f, wII = 0.f, wMD = 0.f, wDD = 0.f;
            size_t qD = q + W + 1, qU = q + W, qL = q + 1;
            if (hasD) {
                xs = score(qD) * c;
                const float amD = AM[qD];
                wMM = ex2f(am + xs - amD);   // M(ij) -> M(D)
                wIM = ex2f(ai + xs - amD);   // I(ij) -> M(D)
                wDM = ex2f(ad + xs - amD);   // D(ij) -> M(D)
                const float bMD = BM[qD];
                bm += bMD * wMM;
                bi += bMD * wIM;
                bd += bMD * wDM;
            }
            if (hasU) {
                const float aiU = AI[qU];
                wMI = ex2f(am + go - aiU);   // M(ij) -> I(U)
                wII = ex2f(ai + ge - aiU);   // I(ij) -> I(U)
                const float bIU = BI[qU];
                bm += bIU * wMI;
                bi += bIU * wII;
            }
            if (hasL) {
                const float adL = AD[qL];
                wMD = ex2f(am + go - adL);   // M(ij) -> D(L)
                wDD = ex2f(ad + ge - adL);   // D(ij) -> D(L)
                const float bDL = BD[qL];
                bm += bDL * wMD;
                bd += bDL * wDD;
            }
            BM[q] = bm;
            BI[q] = bi;
            BD[q] = bd;
            if (MODE == MODE_MARG) {
                if (out) out[q] = bm;
                // path entropy (dS/dT): end-state terms for M, I, D ...
                double hs = (double)bim * (double)(aS - am);
                if (ai > kNegThresh) hs += (double)bii * (double)(aS - ai);
                if (ad > kNegThresh) hs += (double)bid * (double)(aS - ad);
                // ... plus visit probability x local choice entropy
                {
                    const bool dg = up && lf;
                    const float x = sc * c;
                    float hm = ex2f(x - am) * (am - x);
                    if (dg) {
                        const float v0 = AM[q - W - 1] + x, v1 = AI[q - W - 1] + x, v2 = AD[q - W - 1] + x;
                        hm += ex2f(v0 - am) * (am - v0);
                        if (v1 > kNegThresh) hm += ex2f(v1 - am) * (am - v1);
                        if (v2 > kNegThresh) hm += ex2f(v2 - am) * (am - v2);
                    }
                    hs += (double)bm * (double)hm;
                }
                // incoming gap transitions of I(ij), D(ij)
                if (up) {
                    const float v0 = AM[q - W] + go, v1 = AI[q - W] + ge;
                    const float w0 = ex2f(v0 - ai), w1 = ex2f(v1 - ai);
                    so += (double)(bi * w0);
                    se += (double)(bi * w1);
                    float hi = w0 * (ai - v0);
                    if (v1 > kNegThresh) hi += w1 * (ai - v1);
                    hs += (double)bi * (double)hi;
                }
                if (lf) {
                    const float v0 = AM[q - 1] + go, v1 = AD[q - 1] + ge;
                    const float w0 = ex2f(v0 - ad), w1 = ex2f(v1 - ad);
                    so += (double)(bd * w0);
                    se += (double)(bd * w1);
                    float hd = w0 * (ad - v0);
                    if (v1 > kNegThresh) hd += w1 * (ad - v1);
                    hs += (double)bd * (double)hd;
                }
                msum += hs;
            } else if (MODE == MODE_HVP) {
                const float dm = TM[q], di = TI[q], dd = TD[q];
                float dbm = bim * (dm - dS) * iT;
                float dbi = bii * (di - dS) * iT;
                float dbd = bid * (dd - dS) * iT;
                if (hasD) {
                    const float vD = V[qD], dmD = TM[qD], xbD = XM[qD], bMD = BM[qD];
                    dbm += xbD * wMM + bMD * (wMM * (dm + vD - dmD) * iT);
                    dbi += xbD * wIM + bMD * (wIM * (di + vD - dmD) * iT);
                    dbd += xbD * wDM + bMD * (wDM * (dd + vD - dmD) * iT);
                }
                if (hasU) {
                    const float diU = TI[qU], xbU = XI[qU], bIU = BI[qU];
                    dbm += xbU * wMI + bIU * (wMI * (dm - diU) * iT);
                    dbi += xbU * wII + bIU * (wII * (di - diU) * iT);
                }
                if (hasL) {
                    const float ddL = TD[qL], xbL = XD[qL], bDL = BD[qL];
                    dbm += xbL * wMD + bDL * (wMD * (dm - ddL) * iT);
                    dbd += xbL * wDD + bDL * (wDD * (dd - ddL) * iT);
                }
                XM[q] = dbm;
                XI[q] = dbi;
                XD[q] = dbd;
                if (out) out[q] = dbm;
            } else {
                const float um = TM[q], ui = TI[q], ud = TD[q];
                float Wm = bim * (um - dS) * iT, Wi = bii * (ui - dS) * iT, Wd = bid * (ud - dS) * iT;
                if (PT) {
                    if (am > kNegThresh) Wm -= bim * ((am - aS) * ic) * iT * iT;
                    if (ai > kNegThresh) Wi -= bii * ((ai - aS) * ic) * iT * iT;
                    if (ad > kNegThresh) Wd -= bid * ((ad - aS) * ic) * iT * iT;
                }
                const float amn = am * ic, ain = ai * ic, adn = ad * ic;
                if (hasD) {
                    const float rs = PT ? RM[qD] : 0.f;
                    const float Edu = TM[qD] - rs;
                    const float Ev = AM[qD] * ic - T * rs;
                    const float scD = xs * ic;
                    const float xbD = XM[qD], bMD = BM[qD];
                    float dw;
                    dw = wMM * (um - Edu) * iT + (PT ? wMM * (Ev - (amn + scD)) * iT * iT : 0.f);
                    Wm += xbD * wMM + bMD * dw;
                    dw = wIM * (ui - Edu) * iT + (PT ? wIM * (Ev - (ain + scD)) * iT * iT : 0.f);
                    Wi += xbD * wIM + bMD * dw;
                    dw = wDM * (ud - Edu) * iT + (PT ? wDM * (Ev - (adn + scD)) * iT * iT : 0.f);
                    Wd += xbD * wDM + bMD * dw;
                }
                if (hasU) {
                    const float rs = PT ? RI[qU] : 0.f;
                    const float Edu = TI[qU] - rs;
                    const float Ev = AI[qU] * ic - T * rs;
                    const float xbU = XI[qU], bIU = BI[qU];
                    float dw;
                    dw = wMI * (um + pgo - Edu) * iT + (PT ? wMI * (Ev - (amn + gon)) * iT * iT : 0.f);
                    Wm += xbU * wMI + bIU * dw;
                    dw = wII * (ui + pge - Edu) * iT + (PT ? wII * (Ev - (ain + gen)) * iT * iT : 0.f);
                    Wi += xbU * wII + bIU * dw;
                }
                if (hasL) {
                    const float rs = PT ? RD[qL] : 0.f;
                    const float Edu = TD[qL] - rs;
                    const float Ev = AD[qL] * ic - T * rs;
                    const float xbL = XD[qL], bDL = BD[qL];
                    float dw;
                    dw = wMD * (um + pgo - Edu) * iT + (PT ? wMD * (Ev - (amn + gon)) * iT * iT : 0.f);
                    Wm += xbL * wMD + bDL * dw;
                    dw = wDD * (ud + pge - Edu) * iT + (PT ? wDD * (Ev - (adn + gen)) * iT * iT : 0.f);
                    Wd += xbL * wDD + bDL * dw;
                }
                XM[q] = Wm;
                XI[q] = Wi;
                XD[q] = Wd;
                if (out) out[q] = Wm;
                if (p.dot_with) dsum += p.dot_with[(size_t)b * plane + q] * Wm;
            }
        }
        __syncthreads();
    }
    if (MODE >= MODE_PGAP && p.dot_with && p.dot_out) {
        const float D = block_sum(dsum, red);
        if (threadIdx.x == 0) p.dot_out[b] = D;
    }
    if (MODE == MODE_MARG && (p.grad_gap || p.grad_gap2 || p.grad_T)) {
        if (threadIdx.x == 0) msum += (double)ex2f(-aS) * (double)aS;  // origin M[0,0] = 0
        const double O = block_sum_d(so, reinterpret_cast<double*>(red));
        const double E = block_sum_d(se, reinterpret_cast<double*>(red));
        const double H = block_sum_d(msum, reinterpret_cast<double*>(red));
        if (threadIdx.x == 0) {
            if (p.grad_gap) p.grad_gap[b] = (float)O;
            if (p.grad_gap2) p.grad_gap2[b] = (float)E;
            // dS/dT = (S - E[path score]) / T (reference sw_affine kernels_cpu.cpp:336-344)
            //       = entropy of the path distribution (non-negative terms only)
            if (p.grad_T) p.grad_T[b] = (float)(H * (double)kLn2);
        }
    }
}

// --------------------------------------------------------------------------
// host launchers
// --------------------------------------------------------------------------
int launch_lin_plane(const SwArgs& a, cudaStream_t st) {
    dim3 grid(a.B), block(kPlaneThreads);
    switch (a.mode) {
        case MODE_MARG: lin_plane_kernel<MODE_MARG><<<grid, block, 0, st>>>(a); break;
        case MODE_HVP: lin_plane_kernel<MODE_HVP><<<grid, block, 0, st>>>(a); break;
        case MODE_PGAP: lin_plane_kernel<MODE_PGAP><<<grid, block, 0, st>>>(a); break;
        case MODE_PT: lin_plane_kernel<MODE_PT><<<grid, block, 0, st>>>(a); break;
        default: return kErrInvalid;
    }
    return (int)cudaGetLastError();
}

int launch_aff_plane(const SwArgs& a, cudaStream_t st) {
    dim3 grid(a.B), block(kPlaneThreads);
    switch (a.mode) {
        case MODE_MARG: aff_plane_kernel<MODE_MARG><<<grid, block, 0, st>>>(a); break;
        case MODE_HVP: aff_plane_kernel<MODE_HVP><<<grid, block, 0, st>>>(a); break;
        case MODE_PGAP: aff_plane_kernel<MODE_PGAP><<<grid, block, 0, st>>>(a); break;
        case MODE_PGE: aff_plane_kernel<MODE_PGE><<<grid, block, 0, st>>>(a); break;
        case MODE_PT: aff_plane_kernel<MODE_PT><<<grid, block, 0, st>>>(a); break;
        default: return kErrInvalid;
    }
    return (int)cudaGetLastError();
}

}  // namespace d2pb
