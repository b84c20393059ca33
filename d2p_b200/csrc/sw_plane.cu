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
// Frames.  Log-domain values grow along the matrix (alpha ~ 10^3 after a few
// hundred anti-diagonals); stored raw in fp32 they lose absolute precision, and
// every exponential of a difference inherits that loss.  Each anti-diagonal k
// therefore has an integer frame F[k] (chosen from the middle cell of diagonal
// k-1) and the planes store a - F[k].  Differences of frames are exact, so every
// weight 2^(v - a) is formed from small numbers.  S is kept as integer + fraction.
//
// The value + marginals modes are the fix-up of every problem the
// linear-domain kernels flag (low temperatures, extreme scores), so their
// reverse passes follow the reference's arithmetic: each cell's (each state's)
// incoming weights are divided by their own sum, like the reference's softmax,
// and every exponent is formed with the large values cancelling first.  The
// rounding of a large stored alpha then cancels out of the flow through the
// cell instead of accumulating along the paths.  The linear mode also keeps
// alpha in score units, as the reference does.
//
// The linear-domain kernels (sw_linear.cu, sw_affine_fast.cu, sw_tangent.cu,
// sw_affine_tangent.cu) supersede this engine where their range allows; this
// engine remains the general implementation.
#include "sw_common.cuh"
#include "sw_internal.h"

namespace d2pb {

constexpr int kPlaneThreads = 512;

// problems this engine computed, linear and affine (cumulative on the device;
// d2p_engine_counts reads them)
__device__ unsigned long long g_plane_problems[2];

int plane_problem_counts(unsigned long long* n2) {
    return (int)cudaMemcpyFromSymbol(n2, g_plane_problems, 2 * sizeof(unsigned long long));
}

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

// Online log-sum-exp over framed values with an integer base R:
//   sum_k 2^(R + m) * s  with companion sums
//   y1 = sum e_k * ya_k,   y2 = sum e_k * (v_k - m)        (e_k = 2^(v_k - m))
// y2 gives E_p[v] - m without forming differences of large numbers.
struct FrameLse {
    float R, m, s, y1, y2;
    bool any;
    __device__ __forceinline__ void init() { R = 0.f; m = 0.f; s = 0.f; y1 = 0.f; y2 = 0.f; any = false; }
    __device__ __forceinline__ void add(float at, float F, float ya = 0.f) {
        if (at <= kNegThresh) return;
        if (!any) {
            R = F;
            m = at;
            s = 1.f;
            y1 = ya;
            y2 = 0.f;
            any = true;
            return;
        }
        const float v = at + (F - R);
        if (v > m) {
            const float d = m - v, f = ex2f(d);
            y2 = f * (y2 + s * d);
            s = s * f + 1.f;
            y1 = y1 * f + ya;
            m = v;
        } else {
            const float d = v - m, e = ex2f(d);
            s += e;
            y1 += e * ya;
            y2 += e * d;
        }
        if (m > 64.f) {  // keep m small: move its integer part into R (exact)
            const float fl = floorf(m);
            R += fl;
            m -= fl;
        }
    }
    __device__ __forceinline__ void merge(const FrameLse& o) {
        if (!o.any) return;
        if (!any) {
            *this = o;
            return;
        }
        const float Rn = fmaxf(R, o.R);
        const float ma = m + (R - Rn), mb = o.m + (o.R - Rn);
        if (mb > ma) {
            const float d = ma - mb, f = ex2f(d);
            y2 = f * (y2 + s * d) + o.y2;
            s = s * f + o.s;
            y1 = y1 * f + o.y1;
            m = mb;
        } else {
            const float d = mb - ma, f = ex2f(d);
            y2 += f * (o.y2 + o.s * d);
            s += o.s * f;
            y1 += o.y1 * f;
            m = ma;
        }
        R = Rn;
    }
};

__device__ FrameLse block_frame_lse(FrameLse v, float* scratch) {
    const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5, nw = (blockDim.x + 31) >> 5;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        FrameLse q;
        q.R = __shfl_xor_sync(0xffffffffu, v.R, o);
        q.m = __shfl_xor_sync(0xffffffffu, v.m, o);
        q.s = __shfl_xor_sync(0xffffffffu, v.s, o);
        q.y1 = __shfl_xor_sync(0xffffffffu, v.y1, o);
        q.y2 = __shfl_xor_sync(0xffffffffu, v.y2, o);
        q.any = __shfl_xor_sync(0xffffffffu, (int)v.any, o) != 0;
        v.merge(q);
    }
    if (lane == 0) {
        scratch[6 * wid + 0] = v.R;
        scratch[6 * wid + 1] = v.m;
        scratch[6 * wid + 2] = v.s;
        scratch[6 * wid + 3] = v.y1;
        scratch[6 * wid + 4] = v.y2;
        scratch[6 * wid + 5] = v.any ? 1.f : 0.f;
    }
    __syncthreads();
    FrameLse r;
    r.init();
    for (int w = 0; w < nw; ++w) {
        FrameLse q;
        q.R = scratch[6 * w + 0];
        q.m = scratch[6 * w + 1];
        q.s = scratch[6 * w + 2];
        q.y1 = scratch[6 * w + 3];
        q.y2 = scratch[6 * w + 4];
        q.any = scratch[6 * w + 5] != 0.f;
        r.merge(q);
    }
    __syncthreads();
    return r;
}

// Forward bookkeeping shared by both families: at the start of diagonal k the
// frame F[k] is read from the double-buffered shared slot written by the middle
// cell of diagonal k-1.
struct FrameWin {
    float Fk, Fk1, Fk2;  // F[k], F[k-1], F[k-2]
};

// ==========================================================================
// LINEAR GAP
// ==========================================================================
// workspace planes per problem (each L1max*L2max floats):
//   0: a - F (framed scaled alpha; value + marginals: alpha, score units)
//   1: beta (value + marginals: beta / N)  2: tangent forward (dalpha or U)
//   3: tangent backward (dbeta or W)  4: R = (alpha - E[v]) / T  (PT mode)
template <int MODE>
__global__ void __launch_bounds__(kPlaneThreads) lin_plane_kernel(SwArgs p) {
    __shared__ __align__(16) float red[6 * 32];
    __shared__ float sh_F[2];
    __shared__ float sh_Sint, sh_Sfrac, sh_dS;

    const int b = blockIdx.x;
    if (p.only && p.only[b] == 0) return;  // fix-up launch: only problems a fast path flagged
    if (threadIdx.x == 0) atomicAdd(&g_plane_problems[0], 1ull);
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
    float* __restrict__ Fg = p.ws + (size_t)p.B * plane * lin_planes(MODE) + (size_t)b * frame_stride(L1m, L2m);
    float* __restrict__ out = p.out ? p.out + (size_t)b * plane : nullptr;

    zero_padding(out, L1m, L2m, L1, L2);
    const int W = L2m;  // row stride

    // ---------------- forward sweep ----------------
    FrameLse acc;
    acc.init();
    if (threadIdx.x == 0) {
        acc.add(0.f, 0.f, 0.f);  // alpha[0,0] = 0 (d alpha = 0)
        sh_F[0] = 0.f;           // F[2]
        sh_F[1] = 0.f;           // F[3] if diagonal 2 is empty
        Fg[0] = Fg[1] = 0.f;
    }
    __syncthreads();
    FrameWin fw{0.f, 0.f, 0.f};
    for (int k = 2; k <= L1 + L2; ++k) {
        fw.Fk2 = fw.Fk1;
        fw.Fk1 = fw.Fk;
        fw.Fk = sh_F[k & 1];
        const float d1 = fw.Fk - fw.Fk1, d2 = fw.Fk - fw.Fk2;
        const int ilo = max(1, k - L2), ihi = min(L1, k - 1);
        const int imid = (ilo + ihi) >> 1;
        if (threadIdx.x == 0) Fg[k] = fw.Fk;
        for (int i = ilo + threadIdx.x; i <= ihi; i += blockDim.x) {
            const int j = k - i;
            const size_t q = (size_t)(i - 1) * W + (j - 1);
            if (MODE == MODE_MARG) {
                // value + marginals keep alpha in score units, as the reference
                // does (src/sw/kernels_cpu.cpp:70-150): each exponent is a
                // difference of score-unit values, scaled by log2(e)/T only
                // after the largest term is subtracted
                const float sc = s[q];
                const bool up = i > 1, lf = j > 1, dg = up && lf;
                const float v0 = dg ? A[q - W - 1] + sc : kNeg;
                const float v1 = up ? A[q - W] + gapn : kNeg;
                const float v2 = lf ? A[q - 1] + gapn : kNeg;
                const float m = fmaxf(fmaxf(v0, v1), fmaxf(v2, sc));
                const float sum = (ex2f((v0 - m) * c) + ex2f((v1 - m) * c)) + (ex2f((v2 - m) * c) + ex2f((sc - m) * c));
                A[q] = m + lg2f(sum) * ic;
                continue;
            }
            const float x = s[q] * c;
            const bool up = i > 1, lf = j > 1, dg = up && lf;
            const float v0 = dg ? A[q - W - 1] + x - d2 : kNeg;
            const float v1 = up ? A[q - W] + g - d1 : kNeg;
            const float v2 = lf ? A[q - 1] + g - d1 : kNeg;
            const float v3 = x - fw.Fk;
            const Lse4 r = lse4(v0, v1, v2, v3);
            A[q] = r.a;
            if (i == imid) sh_F[(k + 1) & 1] = fw.Fk + rintf(r.a);
            float ya = 0.f;
            if (MODE != MODE_MARG) {
                const float inv = 1.f / r.sum;
                const float w0 = r.t0 * inv, w1 = r.t1 * inv, w2 = r.t2 * inv, w3 = r.t3 * inv;
                float tg;
                if (MODE == MODE_HVP) {
                    const float vv = V[q];
                    const float e0 = dg ? TG[q - W - 1] + vv : 0.f;
                    const float e1 = up ? TG[q - W] : 0.f;
                    const float e2 = lf ? TG[q - 1] : 0.f;
                    tg = w0 * e0 + w1 * e1 + w2 * e2 + w3 * vv;
                } else {
                    const float pg = (MODE == MODE_PGAP) ? 1.f : 0.f;
                    const float e0 = dg ? TG[q - W - 1] : 0.f;
                    const float e1 = (up ? TG[q - W] : 0.f) + pg;
                    const float e2 = (lf ? TG[q - 1] : 0.f) + pg;
                    tg = w0 * e0 + w1 * e1 + w2 * e2;
                    if (MODE == MODE_PT) {
                        // (alpha - E[v]) / T with E[v] over the four logits (framed, exact differences)
                        const float dv = w0 * (dg ? r.a - v0 : 0.f) + w1 * (up ? r.a - v1 : 0.f) +
                                         w2 * (lf ? r.a - v2 : 0.f) + w3 * (r.a - v3);
                        const float rt = dv * ic * iT;
                        RR[q] = rt;
                        tg += rt;
                    }
                }
                TG[q] = tg;
                ya = tg;
            }
            acc.add(r.a, fw.Fk, ya);
        }
        __syncthreads();
    }
    if (threadIdx.x == 0) {
        Fg[L1 + L2 + 1] = sh_F[(L1 + L2 + 1) & 1];
        Fg[L1 + L2 + 2] = Fg[L1 + L2 + 1];
    }
    if (MODE == MODE_MARG) {
        // S = M + T ln(exp(-M/T) + sum exp((alpha - M)/T)), M the largest alpha
        // (score units; the origin alpha[0,0] = 0 is the exp(-M/T) term)
        float mx = 0.f;
        for (int i = 1 + (threadIdx.x >> 5); i <= L1; i += blockDim.x >> 5)
            for (int j = 1 + (threadIdx.x & 31); j <= L2; j += 32) mx = fmaxf(mx, A[(size_t)(i - 1) * W + (j - 1)]);
        const float M = block_max(mx, red);
        double z = 0.0;
        for (int i = 1 + (threadIdx.x >> 5); i <= L1; i += blockDim.x >> 5)
            for (int j = 1 + (threadIdx.x & 31); j <= L2; j += 32)
                z += (double)ex2f((A[(size_t)(i - 1) * W + (j - 1)] - M) * c);
        const double zt = block_sum_d(z, reinterpret_cast<double*>(red));
        if (threadIdx.x == 0) {
            sh_Sint = M;  // S = Sint + Sfrac, score units
            sh_dS = 0.f;
            sh_Sfrac = lg2f((float)(zt + (double)ex2f(-M * c))) * ic;
            if (p.value) p.value[b] = sh_Sint + sh_Sfrac;
        }
        __syncthreads();
    }
    const FrameLse tot = block_frame_lse(acc, red);
    if (threadIdx.x == 0 && MODE != MODE_MARG) {
        const float l2 = tot.m + lg2f(tot.s);
        const float fl = floorf(l2);
        sh_Sint = tot.R + fl;
        sh_Sfrac = l2 - fl;
        float dS = 0.f;
        if (MODE == MODE_HVP || MODE == MODE_PGAP) dS = tot.y1 / tot.s;
        if (MODE == MODE_PT) dS = tot.y1 / tot.s + (lg2f(tot.s) - tot.y2 / tot.s) * ic * iT;
        sh_dS = dS;
        if (p.value) p.value[b] = (sh_Sint + sh_Sfrac) * ic;
    }
    __syncthreads();
    const float Sint = sh_Sint, Sfrac = sh_Sfrac;
    const float dS = sh_dS;

    // ---------------- reverse sweep (gather form) ----------------
    double gsum = 0.0, hsum = 0.0;
    float dsum = 0.f;
    for (int k = L1 + L2; k >= 2; --k) {
        const float F0 = Fg[k], Fm2 = Fg[k - 2], Fp1 = Fg[k + 1], Fp2 = Fg[k + 2];
        const int ilo = max(1, k - L2), ihi = min(L1, k - 1);
        for (int i = ilo + threadIdx.x; i <= ihi; i += blockDim.x) {
            const int j = k - i;
            const size_t q = (size_t)(i - 1) * W + (j - 1);
            const float a = A[q];
            const float sc = s[q];
            const float x = sc * c;
            const bool up = i > 1, lf = j > 1, dg = up && lf;
            const bool hasD = (i < L1) && (j < L2), hasU = i < L1, hasL = j < L2;
            if (MODE == MODE_MARG) {
                // score units (see the forward).  The incoming weights of this
                // cell are normalised by their own sum N, as the reference's
                // softmax does (src/sw/kernels_cpu.cpp:41-62, :200-260), so the
                // rounding of the stored alpha does not scale the flow through
                // the cell; Bt holds beta / N for the predecessors' gathers.
                const float lp = fminf(((a - Sint) - Sfrac) * c, 0.f);
                const float binit = ex2f(lp);
                float beta = binit;
                if (hasD) beta += Bt[q + W + 1] * ex2f(((a - A[q + W + 1]) + s[q + W + 1]) * c);
                if (hasU) beta += Bt[q + W] * ex2f(((a - A[q + W]) + gapn) * c);
                if (hasL) beta += Bt[q + 1] * ex2f(((a - A[q + 1]) + gapn) * c);
                const float ea = dg ? ((A[q - W - 1] - a) + sc) * c : kNeg;
                const float es = (sc - a) * c;
                const float eu = up ? ((A[q - W] - a) + gapn) * c : kNeg;
                const float el = lf ? ((A[q - 1] - a) + gapn) * c : kNeg;
                const float wa = dg ? ex2f(ea) : 0.f, wsk = ex2f(es);
                const float wu = up ? ex2f(eu) : 0.f, wl = lf ? ex2f(el) : 0.f;
                const float N = (wa + wsk) + (wu + wl);  // 1 up to rounding, >= 1/4
                const float bn = beta / N;
                Bt[q] = bn;
                if (out) out[q] = bn * (wa + wsk);
                gsum += (double)(bn * (wu + wl));
                // dS/dT = entropy of the path distribution: visit probability x
                // local choice entropy (of the normalised weights) + end-cell
                // entropy
                const float hloc = (dg ? -wa * ea : 0.f) + (up ? -wu * eu : 0.f) + (lf ? -wl * el : 0.f) - wsk * es;
                hsum += (double)bn * (double)hloc + (double)beta * (double)lg2f(N) - (double)binit * (double)lp;
                continue;
            }
            const float lp = fminf((a - Sfrac) + (F0 - Sint), 0.f);
            const float binit = ex2f(lp);
            float beta = binit;
            // successor weights: transitions (i,j) -> succ (exponents from framed differences)
            float wD = 0.f, wU = 0.f, wL = 0.f;
            if (hasD) { wD = ex2f(a - A[q + W + 1] + s[q + W + 1] * c + (F0 - Fp2)); beta += Bt[q + W + 1] * wD; }
            if (hasU) { wU = ex2f(a - A[q + W] + g + (F0 - Fp1)); beta += Bt[q + W] * wU; }
            if (hasL) { wL = ex2f(a - A[q + 1] + g + (F0 - Fp1)); beta += Bt[q + 1] * wL; }
            Bt[q] = beta;
            // own incoming weights, exponents ea = v - a
            const float ea = dg ? A[q - W - 1] + x + (Fm2 - F0) - a : kNeg;
            const float es = x - F0 - a;
            const float wa = dg ? ex2f(ea) : 0.f;
            const float wsk = ex2f(es);
            if (MODE == MODE_HVP) {
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
                if (PT) Wv -= binit * (((a - Sfrac) + (F0 - Sint)) * ic) * iT * iT;
                if (hasD) {
                    const size_t qs = q + W + 1;
                    const float rs = PT ? RR[qs] : 0.f;
                    float dw = wD * (u - (TG[qs] - rs)) * iT;
                    // E[v](succ) - logit(ij -> succ) = (alpha_s - T R_s) - (alpha + s_s)
                    if (PT) dw += wD * ((A[qs] - a + (Fp2 - F0)) * ic - T * rs - s[qs]) * iT * iT;
                    Wv += TB[qs] * wD + Bt[qs] * dw;
                }
                if (hasU) {
                    const size_t qs = q + W;
                    const float rs = PT ? RR[qs] : 0.f;
                    float dw = wU * (u + pg - (TG[qs] - rs)) * iT;
                    if (PT) dw += wU * ((A[qs] - a + (Fp1 - F0)) * ic - T * rs - gapn) * iT * iT;
                    Wv += TB[qs] * wU + Bt[qs] * dw;
                }
                if (hasL) {
                    const size_t qs = q + 1;
                    const float rs = PT ? RR[qs] : 0.f;
                    float dw = wL * (u + pg - (TG[qs] - rs)) * iT;
                    if (PT) dw += wL * ((A[qs] - a + (Fp1 - F0)) * ic - T * rs - gapn) * iT * iT;
                    Wv += TB[qs] * wL + Bt[qs] * dw;
                }
                TB[q] = Wv;
                const float r0 = PT ? RR[q] : 0.f;
                const float Edu = u - r0;
                const float dua = dg ? TG[q - W - 1] : 0.f;
                float dwa = wa * (dua - Edu) * iT;
                float dws = wsk * (0.f - Edu) * iT;
                if (PT) {
                    // E[v] - v_align = (alpha - T r0) - (alpha_diag + s);  E[v] - v_sky = alpha - T r0 - s
                    if (dg) dwa += wa * ((a - A[q - W - 1] + (F0 - Fm2)) * ic - T * r0 - sc) * iT * iT;
                    dws += wsk * ((a + F0) * ic - T * r0 - sc) * iT * iT;
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
        // the origin alpha[0,0] = 0 is a possible end state (empty alignment)
        if (threadIdx.x == 0) {
            const float lp0 = fminf((-Sint - Sfrac) * c, 0.f);  // score units
            hsum += (double)ex2f(lp0) * (double)(-lp0);
        }
        const double G = block_sum_d(gsum, reinterpret_cast<double*>(red));
        const double H = block_sum_d(hsum, reinterpret_cast<double*>(red));
        if (threadIdx.x == 0) {
            if (p.grad_gap) p.grad_gap[b] = (float)G;
            // dS/dT = (S - E[path score]) / T  (reference kernels_cpu.cpp:274-276)
            //       = entropy of the Gibbs path distribution (nats)
            if (p.grad_T) p.grad_T[b] = (float)(H * (double)kLn2);
        }
    }
}

// ==========================================================================
// AFFINE GAP
// ==========================================================================
// planes per problem: alpha M,I,D (0-2, framed), beta M,I,D (3-5), tangent fwd
// M,I,D (6-8), tangent bwd M,I,D (9-11), R M,I,D (12-14).
template <int MODE>
__global__ void __launch_bounds__(kPlaneThreads) aff_plane_kernel(SwArgs p) {
    __shared__ __align__(16) float red[6 * 32];
    __shared__ float sh_F[2];
    __shared__ float sh_Sint, sh_Sfrac, sh_dS;

    const int b = blockIdx.x;
    if (p.only && p.only[b] == 0) return;  // fix-up launch: only problems a fast path flagged
    if (threadIdx.x == 0) atomicAdd(&g_plane_problems[1], 1ull);
    const int L1m = p.L1, L2m = p.L2;
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
    float* __restrict__ Fg = p.ws + (size_t)p.B * plane * aff_planes(MODE) + (size_t)b * frame_stride(L1m, L2m);
    float* __restrict__ out = p.out ? p.out + (size_t)b * plane : nullptr;
    zero_padding(out, L1m, L2m, L1, L2);
    const int W = L2m;
    auto score = [&](size_t q) -> float { return sbf ? __bfloat162float(sbf[q]) : s[q]; };

    FrameLse acc;
    acc.init();
    if (threadIdx.x == 0) {
        acc.add(0.f, 0.f, 0.f);
        sh_F[0] = 0.f;
        sh_F[1] = 0.f;
        Fg[0] = Fg[1] = 0.f;
    }
    __syncthreads();
    const float pgo = (MODE == MODE_PGAP) ? 1.f : 0.f;   // param 0: gap_open
    const float pge = (MODE == MODE_PGE) ? 1.f : 0.f;    // param 1: gap_ext
    const bool PT = (MODE == MODE_PT);

    FrameWin fw{0.f, 0.f, 0.f};
    for (int k = 2; k <= L1 + L2; ++k) {
        fw.Fk2 = fw.Fk1;
        fw.Fk1 = fw.Fk;
        fw.Fk = sh_F[k & 1];
        const float d1 = fw.Fk - fw.Fk1, d2 = fw.Fk - fw.Fk2;
        const int ilo = max(1, k - L2), ihi = min(L1, k - 1);
        const int imid = (ilo + ihi) >> 1;
        if (threadIdx.x == 0) Fg[k] = fw.Fk;
        for (int i = ilo + threadIdx.x; i <= ihi; i += blockDim.x) {
            const int j = k - i;
            const size_t q = (size_t)(i - 1) * W + (j - 1);
            const float sc = score(q);
            const float x = sc * c;
            const bool up = i > 1, lf = j > 1, dg = up && lf;
            const float m0 = dg ? AM[q - W - 1] + x - d2 : kNeg;
            const float m1 = dg ? AI[q - W - 1] + x - d2 : kNeg;
            const float m2 = dg ? AD[q - W - 1] + x - d2 : kNeg;
            const float m3 = x - fw.Fk;
            const Lse4 rm = lse4(m0, m1, m2, m3);
            const float i0 = up ? AM[q - W] + go - d1 : kNeg;
            const float i1 = up ? AI[q - W] + ge - d1 : kNeg;
            const Lse2 ri = lse2(i0, i1);
            const float e0 = lf ? AM[q - 1] + go - d1 : kNeg;
            const float e1 = lf ? AD[q - 1] + ge - d1 : kNeg;
            const Lse2 rd = lse2(e0, e1);
            AM[q] = rm.a;
            AI[q] = ri.a;
            AD[q] = rd.a;
            if (i == imid) sh_F[(k + 1) & 1] = fw.Fk + rintf(rm.a);
            if (MODE == MODE_MARG) {
                acc.add(rm.a, fw.Fk);
                acc.add(ri.a, fw.Fk);
                acc.add(rd.a, fw.Fk);
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
                        const float dvm = wm0 * (dg ? rm.a - m0 : 0.f) + wm1 * (dg ? rm.a - m1 : 0.f) +
                                          wm2 * (dg ? rm.a - m2 : 0.f) + wm3 * (rm.a - m3);
                        const float rmv = dvm * ic * iT;
                        float riv = 0.f, rdv = 0.f;
                        if (ri.a > kNegThresh) riv = (wi0 * (ri.a - i0) + wi1 * (ri.a - i1)) * ic * iT;
                        if (rd.a > kNegThresh) rdv = (wd0 * (rd.a - e0) + wd1 * (rd.a - e1)) * ic * iT;
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
                acc.add(rm.a, fw.Fk, tm);
                acc.add(ri.a, fw.Fk, ti);
                acc.add(rd.a, fw.Fk, td);
            }
        }
        __syncthreads();
    }
    if (threadIdx.x == 0) {
        Fg[L1 + L2 + 1] = sh_F[(L1 + L2 + 1) & 1];
        Fg[L1 + L2 + 2] = Fg[L1 + L2 + 1];
    }
    const FrameLse tot = block_frame_lse(acc, red);
    if (threadIdx.x == 0) {
        const float l2 = tot.m + lg2f(tot.s);
        const float fl = floorf(l2);
        sh_Sint = tot.R + fl;
        sh_Sfrac = l2 - fl;
        float dS = 0.f;
        if (MODE == MODE_HVP || MODE == MODE_PGAP || MODE == MODE_PGE) dS = tot.y1 / tot.s;
        if (PT) dS = tot.y1 / tot.s + (lg2f(tot.s) - tot.y2 / tot.s) * ic * iT;
        sh_dS = dS;
        if (p.value) p.value[b] = (sh_Sint + sh_Sfrac) * ic;
    }
    __syncthreads();
    const float Sint = sh_Sint, Sfrac = sh_Sfrac, dS = sh_dS;

    double so = 0.0, se = 0.0, hsum = 0.0;
    float dsum = 0.f;
    for (int k = L1 + L2; k >= 2; --k) {
        const float F0 = Fg[k], Fm1 = Fg[k - 1], Fm2 = Fg[k - 2], Fp1 = Fg[k + 1], Fp2 = Fg[k + 2];
        const int ilo = max(1, k - L2), ihi = min(L1, k - 1);
        for (int i = ilo + threadIdx.x; i <= ihi; i += blockDim.x) {
            const int j = k - i;
            const size_t q = (size_t)(i - 1) * W + (j - 1);
            const float sc = score(q);
            const float x = sc * c;
            const bool up = i > 1, lf = j > 1, dg = up && lf;
            const bool hasD = (i < L1) && (j < L2), hasU = i < L1, hasL = j < L2;
            const float am = AM[q], ai = AI[q], ad = AD[q];
            const float lpm = fminf((am - Sfrac) + (F0 - Sint), 0.f);
            const float lpi = fminf((ai - Sfrac) + (F0 - Sint), 0.f);
            const float lpd = fminf((ad - Sfrac) + (F0 - Sint), 0.f);
            const float bim = ex2f(lpm), bii = ex2f(lpi), bid = ex2f(lpd);
            float bm = bim, bi = bii, bd = bid;
            if (MODE == MODE_MARG) {
                // Value + marginals, the fix-up of problems the linear-domain
                // kernels flag (low temperatures, extreme scores).  Every exponent
                // is formed with the two framed alphas cancelling first, and each
                // state's incoming weights are divided by their sum N, as the
                // reference's softmax normalises them (src/sw_affine/kernels_cpu.cpp:
                // 53-87, :199-346): the rounding of a large stored alpha then does
                // not scale the flow through the cell.  B* hold beta / N for the
                // predecessors' gathers; beta itself is the state's visit
                // probability (the marginal, for M).
                const size_t qD = q + W + 1, qU = q + W, qL = q + 1;
                if (hasD) {
                    const float xs = score(qD) * c, fd = F0 - Fp2, amD = AM[qD], bMD = BM[qD];
                    bm += bMD * ex2f(((am - amD) + fd) + xs);
                    bi += bMD * ex2f(((ai - amD) + fd) + xs);
                    bd += bMD * ex2f(((ad - amD) + fd) + xs);
                }
                if (hasU) {
                    const float f1 = F0 - Fp1, aiU = AI[qU], bIU = BI[qU];
                    bm += bIU * ex2f(((am - aiU) + f1) + go);
                    bi += bIU * ex2f(((ai - aiU) + f1) + ge);
                }
                if (hasL) {
                    const float f1 = F0 - Fp1, adL = AD[qL], bDL = BD[qL];
                    bm += bDL * ex2f(((am - adL) + f1) + go);
                    bd += bDL * ex2f(((ad - adL) + f1) + ge);
                }
                // own incoming weights (exponents e = v - a) and their sums
                const float es = (x - am) - F0;
                const float wsk = ex2f(es);
                float NM = wsk, hm = -wsk * es;
                if (dg) {
                    const float f2 = Fm2 - F0;
                    const float e0 = ((AM[q - W - 1] - am) + f2) + x;
                    const float e1 = ((AI[q - W - 1] - am) + f2) + x;
                    const float e2 = ((AD[q - W - 1] - am) + f2) + x;
                    const float w0 = ex2f(e0), w1 = ex2f(e1), w2 = ex2f(e2);
                    NM += (w0 + w1) + w2;
                    hm -= w0 * e0;
                    if (AI[q - W - 1] > kNegThresh) hm -= w1 * e1;
                    if (AD[q - W - 1] > kNegThresh) hm -= w2 * e2;
                }
                float NI = 0.f, hi = 0.f, woi = 0.f, wei = 0.f;
                if (up) {  // I(ij): opened from M above, extended from I above
                    const float f1 = Fm1 - F0;
                    const float e0 = ((AM[q - W] - ai) + f1) + go, e1 = ((AI[q - W] - ai) + f1) + ge;
                    woi = ex2f(e0);
                    wei = ex2f(e1);
                    NI = woi + wei;
                    hi = -woi * e0;
                    if (AI[q - W] > kNegThresh) hi -= wei * e1;
                }
                float ND = 0.f, hd = 0.f, wod = 0.f, wed = 0.f;
                if (lf) {  // D(ij): opened from M on the left, extended from D on the left
                    const float f1 = Fm1 - F0;
                    const float e0 = ((AM[q - 1] - ad) + f1) + go, e1 = ((AD[q - 1] - ad) + f1) + ge;
                    wod = ex2f(e0);
                    wed = ex2f(e1);
                    ND = wod + wed;
                    hd = -wod * e0;
                    if (AD[q - 1] > kNegThresh) hd -= wed * e1;
                }
                const float bmn = bm / NM;                      // NM >= 1/4
                const float bin = NI > 0.f ? bi / NI : 0.f;     // NI, ND >= 1/2 when reachable
                const float bdn = ND > 0.f ? bd / ND : 0.f;
                BM[q] = bmn;
                BI[q] = bin;
                BD[q] = bdn;
                if (out) out[q] = bm;
                so += (double)(bin * woi) + (double)(bdn * wod);
                se += (double)(bin * wei) + (double)(bdn * wed);
                // dS/dT: end-state terms + visit probability x local choice
                // entropy of the normalised weights (h / N + lg2 N)
                double hs = -(double)bim * (double)lpm;
                if (ai > kNegThresh) hs -= (double)bii * (double)lpi;
                if (ad > kNegThresh) hs -= (double)bid * (double)lpd;
                hs += (double)bmn * (double)hm + (double)bm * (double)lg2f(NM);
                if (NI > 0.f) hs += (double)bin * (double)hi + (double)bi * (double)lg2f(NI);
                if (ND > 0.f) hs += (double)bdn * (double)hd + (double)bd * (double)lg2f(ND);
                hsum += hs;
                continue;
            }
            // successor transition weights (framed exponents)
            float xs = 0.f, wMM = 0.f, wIM = 0.f, wDM = 0.f, wMI = 0.f, wII = 0.f, wMD = 0.f, wDD = 0.f;
            const size_t qD = q + W + 1, qU = q + W, qL = q + 1;
            if (hasD) {
                xs = score(qD) * c;
                const float base = xs - AM[qD] + (F0 - Fp2);
                wMM = ex2f(am + base);   // M(ij) -> M(D)
                wIM = ex2f(ai + base);   // I(ij) -> M(D)
                wDM = ex2f(ad + base);   // D(ij) -> M(D)
                const float bMD = BM[qD];
                bm += bMD * wMM;
                bi += bMD * wIM;
                bd += bMD * wDM;
            }
            if (hasU) {
                const float base = -AI[qU] + (F0 - Fp1);
                wMI = ex2f(am + go + base);   // M(ij) -> I(U)
                wII = ex2f(ai + ge + base);   // I(ij) -> I(U)
                const float bIU = BI[qU];
                bm += bIU * wMI;
                bi += bIU * wII;
            }
            if (hasL) {
                const float base = -AD[qL] + (F0 - Fp1);
                wMD = ex2f(am + go + base);   // M(ij) -> D(L)
                wDD = ex2f(ad + ge + base);   // D(ij) -> D(L)
                const float bDL = BD[qL];
                bm += bDL * wMD;
                bd += bDL * wDD;
            }
            BM[q] = bm;
            BI[q] = bi;
            BD[q] = bd;
            if (MODE == MODE_HVP) {
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
                    if (am > kNegThresh) Wm -= bim * (((am - Sfrac) + (F0 - Sint)) * ic) * iT * iT;
                    if (ai > kNegThresh) Wi -= bii * (((ai - Sfrac) + (F0 - Sint)) * ic) * iT * iT;
                    if (ad > kNegThresh) Wd -= bid * (((ad - Sfrac) + (F0 - Sint)) * ic) * iT * iT;
                }
                if (hasD) {
                    const float rs = PT ? RM[qD] : 0.f;
                    const float Edu = TM[qD] - rs;
                    // E[v](succ) - logit: (alpha_s - T R_s) - (alpha_state + s_s), framed differences
                    const float dEv = (AM[qD] + (Fp2 - F0)) * ic - T * rs - xs * ic;
                    const float xbD = XM[qD], bMD = BM[qD];
                    float dw;
                    dw = wMM * (um - Edu) * iT + (PT ? wMM * (dEv - am * ic) * iT * iT : 0.f);
                    Wm += xbD * wMM + bMD * dw;
                    dw = wIM * (ui - Edu) * iT + (PT ? wIM * (dEv - ai * ic) * iT * iT : 0.f);
                    Wi += xbD * wIM + bMD * dw;
                    dw = wDM * (ud - Edu) * iT + (PT ? wDM * (dEv - ad * ic) * iT * iT : 0.f);
                    Wd += xbD * wDM + bMD * dw;
                }
                if (hasU) {
                    const float rs = PT ? RI[qU] : 0.f;
                    const float Edu = TI[qU] - rs;
                    const float dEv = (AI[qU] + (Fp1 - F0)) * ic - T * rs;
                    const float xbU = XI[qU], bIU = BI[qU];
                    float dw;
                    dw = wMI * (um + pgo - Edu) * iT + (PT ? wMI * (dEv - (am * ic + gon)) * iT * iT : 0.f);
                    Wm += xbU * wMI + bIU * dw;
                    dw = wII * (ui + pge - Edu) * iT + (PT ? wII * (dEv - (ai * ic + gen)) * iT * iT : 0.f);
                    Wi += xbU * wII + bIU * dw;
                }
                if (hasL) {
                    const float rs = PT ? RD[qL] : 0.f;
                    const float Edu = TD[qL] - rs;
                    const float dEv = (AD[qL] + (Fp1 - F0)) * ic - T * rs;
                    const float xbL = XD[qL], bDL = BD[qL];
                    float dw;
                    dw = wMD * (um + pgo - Edu) * iT + (PT ? wMD * (dEv - (am * ic + gon)) * iT * iT : 0.f);
                    Wm += xbL * wMD + bDL * dw;
                    dw = wDD * (ud + pge - Edu) * iT + (PT ? wDD * (dEv - (ad * ic + gen)) * iT * iT : 0.f);
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
        if (threadIdx.x == 0) {  // origin M[0,0] = 0
            const float lp0 = fminf(-Sfrac - Sint, 0.f);
            hsum += (double)ex2f(lp0) * (double)(-lp0);
        }
        const double O = block_sum_d(so, reinterpret_cast<double*>(red));
        const double E = block_sum_d(se, reinterpret_cast<double*>(red));
        const double H = block_sum_d(hsum, reinterpret_cast<double*>(red));
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
