// sw_nw_affine.cu -- soft Needleman-Wunsch with affine gaps (three states: M
// match, I gap in the second sequence, D gap in the first): value, marginals,
// dS/d(gap_open), dS/d(gap_ext), dS/dT, the Hessian-vector product, the three
// parameter Jacobians, and their contraction with a weight plane
// (backward_full).
//
// Recurrences (src/nw_affine/kernels_cpu.cpp:101-185 restated, natural units):
//   M(0,0) = 0, I(i,0) = open + (i-1) ext, D(0,j) = open + (j-1) ext, every
//   other boundary state -inf;
//   M(i,j) = s_ij + LSE_T(M, I, D at (i-1, j-1)),
//   I(i,j) = LSE_T(M + open, I + ext, D + open at (i-1, j)),
//   D(i,j) = LSE_T(M + open, I + open, D + ext at (i, j-1)),
//   S = LSE_T(M, I, D at (L1, L2)).
// Each state's three options come from one predecessor cell, with normalised
// weights w.  The reverse is the flow of the path distribution over states:
// beta_X(c) = sum over the successor states Y at d of beta_Y(d) w_{Y<-X}(d),
// seeded at (L1, L2) with the final LSE's weights; the marginal of (i, j) is
// beta_M(i, j).  dS/dopen and dS/dext are the flows through opening and
// extending moves (plus the leading gaps of boundary states), and dS/dT is the
// entropy of the path distribution: each visited state's choice entropy
// weighted by its visit probability, plus the final choice's.  This equals
// the reference's (S - E[path score]) / T without its cancellation.
//
// Tangents (along V in the scores, or a parameter): the forward carries each
// state's d alpha = sum_k w_k (d alpha_k + the option's direct derivative)
// (+ V for M; + the choice entropy along T); the reverse carries d beta, with
// dw_k = w_k (u_k - sum_l w_l u_l) / T (+ w_k (E[v] - v_k) / T^2 along T), u
// the options' tangents, which all come from the one predecessor cell being
// updated, so a cell's reverse needs only its own forward tangents.  The
// output is d beta_M (src/nw_affine/kernels_cpu.cpp:362-1000).
//
// Engine: one CTA per problem sweeps the anti-diagonals, threads striding
// over a diagonal's cells, one barrier per diagonal; per-cell values live in
// diagonal-major planes ([k][i]) in the workspace.  The three alphas (and the
// forward tangents) are stored relative to an integer frame per diagonal, so
// options are formed from small values plus exact frame differences.  The
// reverse gathers from successors (no atomics: deterministic); per-problem
// sums are fp64 block reductions.
#include <math.h>
#include <stddef.h>
#include <stdint.h>

#include "../../include/d2p_b200.h"
#include "sw_common.cuh"
#include "sw_internal.h"

namespace d2pb {
namespace nwa {

constexpr int kThreads = 256;
constexpr float kNInf = -1.0e30f;   // absent state: exp((kNInf - m) / T) is 0, and 0 * kNInf is 0

// planes of one problem, each (L1m + L2m + 1) (L1m + 1) floats
enum Plane : int {
    kAM = 0, kAI, kAD,                 // alpha of M, I, D (minus the diagonal's frame)
    kWM1, kWM2, kWM3,                  // weights of M's options (from M, I, D)
    kWI1, kWI2, kWI3,                  //   of I's
    kWD1, kWD2, kWD3,                  //   of D's
    kBM, kBI, kBD,                     // beta
    kFM, kFI, kFD,                     // forward tangents (minus the diagonal's tangent frame)
    kRM, kRI, kRD,                     // reverse tangents
    kNumPlanes
};
__host__ __device__ inline size_t plane_floats(int L1m, int L2m) {
    return ((size_t)L1m + L2m + 1) * ((size_t)L1m + 1);
}
__host__ __device__ inline int planes_for(int mode) { return mode == MODE_MARG ? kBD + 1 : kNumPlanes; }
__host__ __device__ inline size_t per_problem_bytes(int L1m, int L2m, int mode) {
    const size_t b = (plane_floats(L1m, L2m) * planes_for(mode) + 2 * ((size_t)L1m + L2m + 1)) * sizeof(float);
    return (b + 255) & ~(size_t)255;
}

struct Ctx {
    float* p[kNumPlanes];
    float* O;     // alpha's frame of each diagonal (integer-valued)
    float* D;     // the forward tangents'
    int stride;
    __device__ float& at(int plane, int k, int i) const { return p[plane][(size_t)k * stride + i]; }
};

__device__ __forceinline__ double block_sum(double v, double* red) {
    for (int o = 16; o >= 1; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    __syncthreads();
    if (lane == 0) red[warp] = v;
    __syncthreads();
    double t = 0.0;
    if (threadIdx.x < 32) {
        t = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.0;
        for (int o = 16; o >= 1; o >>= 1) t += __shfl_xor_sync(0xffffffffu, t, o);
    }
    return t;   // valid in thread 0
}

// normalised weights of three options; returns the LSE (m + T ln sum), and
// through *h the choice's entropy -sum w ln w = ln(sum) + sum w (m - v) / T
__device__ __forceinline__ float lse3w(float v1, float v2, float v3, float T, float iT, float& w1, float& w2,
                                       float& w3, float* h) {
    const float m = fmaxf(v1, fmaxf(v2, v3));
    const float e1 = expf((v1 - m) * iT), e2 = expf((v2 - m) * iT), e3 = expf((v3 - m) * iT);
    const float sum = (e1 + e2) + e3;
    const float ls = logf(sum);
    const float is = 1.f / sum;
    w1 = e1 * is;
    w2 = e2 * is;
    w3 = e3 * is;
    if (h) *h = ls + iT * fmaf(w1, m - v1, fmaf(w2, m - v2, w3 * (m - v3)));
    return fmaf(T, ls, m);
}

// Rings: the last three diagonals of the three alphas (and forward tangents)
// during the forward, and of the three betas (and reverse tangents) during the
// reverse, sit in shared memory ([3][L1m + 1] floats each) when they fit, so
// the sweep reads its neighbours at shared-memory latency; the planes in the
// workspace still receive what the reverse reads back (the weights; for the
// tangent modes the alphas and the forward tangents).  When the rings do not
// fit, each ring is its quantity's plane.  The scores (and direction) of a
// diagonal, and in MODE_MARG the weights its reverse reads, are loaded one
// diagonal ahead, before the barrier.
constexpr int kPF = 2;                          // forward: cells per thread prefetched (diagonals of <= 512 cells)
constexpr int kPFR = 2;                         // reverse (18 weights a cell): diagonals of <= 512 cells
constexpr size_t kMaxRingBytes = 200 * 1024;    // dynamic shared memory cap of the rings
__host__ __device__ inline int rings_for(int mode) { return mode == MODE_MARG ? 6 : 12; }
__host__ __device__ inline size_t ring_bytes(int L1m, int mode) {
    return (size_t)rings_for(mode) * 3 * ((size_t)L1m + 1) * sizeof(float);
}
// ring ids: alphas 0..2, betas 3..5, forward tangents 6..8, reverse tangents 9..11
enum Ring : int { rAM = 0, rBM = 3, rFM = 6, rRM = 9 };

// the weights one cell's reverse reads (MODE_MARG): those its successors give
// its states (M at (i+1, j+1), I at (i+1, j), D at (i, j+1)) and its own
struct RevIn {
    float sm[3], si[3], sd[3];
    float om[3], oi[3], od[3];
};

// One CTA per problem.  MODE: MODE_MARG (value, marginals, the three
// parameter gradients), MODE_HVP (out = d marginals along p.tangent),
// MODE_PGAP / MODE_PGE / MODE_PT (out = dP/d(open, ext, T); with dot_with,
// dot_out[b] = sum dot_with * dP).
template <int MODE>
__global__ void __launch_bounds__(kThreads) nwa_kernel(SwArgs p) {
    extern __shared__ float ring_smem[];
    __shared__ double red[32];
    const int b = blockIdx.x;
    if (p.only && !p.only[b]) return;   // a fix-up launch: only the problems the wavefront kernel flagged
    const int L1m = p.L1, L2m = p.L2;
    const int L1 = p.lengths ? min(max(p.lengths[2 * b], 0), L1m) : L1m;
    const int L2 = p.lengths ? min(max(p.lengths[2 * b + 1], 0), L2m) : L2m;
    const float go = p.gap_dev ? __ldg(p.gap_dev) : p.gap;
    const float ge = p.gap2_dev ? __ldg(p.gap2_dev) : p.gap2;
    const float T = p.temp_dev ? __ldg(p.temp_dev) : p.temp;
    const float iT = 1.f / T;
    const size_t plane = (size_t)L1m * L2m;
    const float* __restrict__ S = p.scores + (size_t)b * plane;
    const float* __restrict__ V = MODE == MODE_HVP ? p.tangent + (size_t)b * plane : nullptr;
    const float* __restrict__ Gw = p.dot_with ? p.dot_with + (size_t)b * plane : nullptr;
    float* __restrict__ out = p.out ? p.out + (size_t)b * plane : nullptr;
    Ctx C;
    {
        float* base = reinterpret_cast<float*>(reinterpret_cast<char*>(p.ws) + (size_t)b * per_problem_bytes(L1m, L2m, MODE));
        const size_t pf = plane_floats(L1m, L2m);
        for (int q = 0; q < kNumPlanes; ++q) C.p[q] = q < planes_for(MODE) ? base + (size_t)q * pf : nullptr;
        C.O = base + pf * planes_for(MODE);
        C.D = C.O + (L1m + L2m + 1);
        C.stride = L1m + 1;
    }
    constexpr bool TAN = MODE != MODE_MARG;
    // the direct derivative of each option's gap term along the parameter
    constexpr float xI1 = MODE == MODE_PGAP ? 1.f : 0.f, xI2 = MODE == MODE_PGE ? 1.f : 0.f, xI3 = xI1;
    constexpr float xD1 = xI1, xD2 = xI1, xD3 = xI2;
    const int K = L1 + L2;
    const int tid = threadIdx.x;
    const bool smR = ring_bytes(L1m, MODE) <= kMaxRingBytes;
    const int RS = L1m + 1;
    // row of diagonal k of ring rg (its plane pl when the rings are the planes)
    auto row = [&](int rg, int pl, int k) -> float* {
        return smR ? ring_smem + (size_t)(3 * rg + k % 3) * RS : C.p[pl] + (size_t)k * C.stride;
    };

    if (out && (L1 < L1m || L2 < L2m)) {   // zeros outside the problem
        for (int i = 0; i < L1m; ++i)
            for (int j = (i < L1 ? L2 : 0) + (int)threadIdx.x; j < L2m; j += blockDim.x) out[(size_t)i * L2m + j] = 0.f;
    }

    // ------------------------------------------------------------- forward
    float pc[kPF], pv[kPF];   // scores (and direction) of this thread's first kPF cells of a diagonal
    auto fetch_fwd = [&](int k, float* c, float* v) {
        const int i0 = max(0, k - L2), i1 = min(L1, k);
#pragma unroll
        for (int r = 0; r < kPF; ++r) {
            const int i = i0 + tid + r * kThreads, j = k - i;
            const bool ok = i <= i1 && i >= 1 && j >= 1;
            const size_t si = ok ? (size_t)(i - 1) * L2m + (j - 1) : 0;
            c[r] = ok ? __ldg(S + si) : 0.f;
            if (MODE == MODE_HVP) v[r] = ok ? __ldg(V + si) : 0.f;
        }
    };
    fetch_fwd(0, pc, pv);
    float O1 = 0.f, O2 = 0.f, D1 = 0.f, D2 = 0.f;
    for (int k = 0; k <= K; ++k) {
        const int k1 = max(k - 1, 0), k2 = max(k - 2, 0);
        float* const aM0 = row(rAM, kAM, k);
        float* const aI0 = row(rAM + 1, kAI, k);
        float* const aD0 = row(rAM + 2, kAD, k);
        const float* const aM1 = row(rAM, kAM, k1);
        const float* const aI1 = row(rAM + 1, kAI, k1);
        const float* const aD1 = row(rAM + 2, kAD, k1);
        const float* const aM2 = row(rAM, kAM, k2);
        const float* const aI2 = row(rAM + 1, kAI, k2);
        const float* const aD2 = row(rAM + 2, kAD, k2);
        float* const fM0 = TAN ? row(rFM, kFM, k) : nullptr;
        float* const fI0 = TAN ? row(rFM + 1, kFI, k) : nullptr;
        float* const fD0 = TAN ? row(rFM + 2, kFD, k) : nullptr;
        const float* const fM1 = TAN ? row(rFM, kFM, k1) : nullptr;
        const float* const fI1 = TAN ? row(rFM + 1, kFI, k1) : nullptr;
        const float* const fD1 = TAN ? row(rFM + 2, kFD, k1) : nullptr;
        const float* const fM2 = TAN ? row(rFM, kFM, k2) : nullptr;
        const float* const fI2 = TAN ? row(rFM + 1, kFI, k2) : nullptr;
        const float* const fD2 = TAN ? row(rFM + 2, kFD, k2) : nullptr;
        float Ok = 0.f, Dk = 0.f;
        if (k >= 1) {   // from the previous diagonal's middle cell: its largest state
            const int im = (max(0, k - 1 - L2) + min(L1, k - 1)) >> 1;
            float x = aM1[im];
            int st = 0;
            if (aI1[im] > x) x = aI1[im], st = 1;
            if (aD1[im] > x) x = aD1[im], st = 2;
            Ok = O1 + rintf(x);
            if (TAN) Dk = D1 + rintf((st == 0 ? fM1 : st == 1 ? fI1 : fD1)[im]);
        }
        if (tid == 0) {
            C.O[k] = Ok;
            C.D[k] = Dk;
        }
        const float dO1 = O1 - Ok, dO2 = O2 - Ok, dD1 = D1 - Dk, dD2 = D2 - Dk;   // exact
        // the alphas (rings; the planes too where the tangent reverses read them)
        auto putA = [&](int i, float vM, float vI, float vD) {
            aM0[i] = vM;
            aI0[i] = vI;
            aD0[i] = vD;
            if (smR && TAN) {
                C.at(kAM, k, i) = vM;
                C.at(kAI, k, i) = vI;
                C.at(kAD, k, i) = vD;
            }
        };
        auto putF = [&](int i, float vM, float vI, float vD) {
            fM0[i] = vM;
            fI0[i] = vI;
            fD0[i] = vD;
            if (smR) {
                C.at(kFM, k, i) = vM;
                C.at(kFI, k, i) = vI;
                C.at(kFD, k, i) = vD;
            }
        };
        auto cell = [&](int i, float sc, float vv) {
            const int j = k - i;
            if (i == 0 || j == 0) {   // boundary states
                putA(i, k == 0 ? 0.f : kNInf, (j == 0 && i >= 1) ? fmaf((float)(i - 1), ge, go) - Ok : kNInf,
                     (i == 0 && j >= 1) ? fmaf((float)(j - 1), ge, go) - Ok : kNInf);
                if (TAN) {
                    const float lead = MODE == MODE_PGAP ? 1.f : MODE == MODE_PGE ? (float)(k - 1) : 0.f;
                    putF(i, -Dk, ((j == 0 && i >= 1) ? lead : 0.f) - Dk, ((i == 0 && j >= 1) ? lead : 0.f) - Dk);
                }
                return;
            }
            // M from (i-1, j-1)
            const float m1 = aM2[i - 1] + dO2, m2 = aI2[i - 1] + dO2, m3 = aD2[i - 1] + dO2;
            float wm1, wm2, wm3, hM;
            const float aM = sc + lse3w(m1, m2, m3, T, iT, wm1, wm2, wm3, MODE == MODE_PT ? &hM : nullptr);
            // I from (i-1, j)
            const float u1 = aM1[i - 1] + (go + dO1), u2 = aI1[i - 1] + (ge + dO1), u3 = aD1[i - 1] + (go + dO1);
            float wi1, wi2, wi3, hI;
            const float aI = lse3w(u1, u2, u3, T, iT, wi1, wi2, wi3, MODE == MODE_PT ? &hI : nullptr);
            // D from (i, j-1)
            const float l1 = aM1[i] + (go + dO1), l2 = aI1[i] + (go + dO1), l3 = aD1[i] + (ge + dO1);
            float wd1, wd2, wd3, hD;
            const float aD = lse3w(l1, l2, l3, T, iT, wd1, wd2, wd3, MODE == MODE_PT ? &hD : nullptr);
            putA(i, aM, aI, aD);
            C.at(kWM1, k, i) = wm1;
            C.at(kWM2, k, i) = wm2;
            C.at(kWM3, k, i) = wm3;
            C.at(kWI1, k, i) = wi1;
            C.at(kWI2, k, i) = wi2;
            C.at(kWI3, k, i) = wi3;
            C.at(kWD1, k, i) = wd1;
            C.at(kWD2, k, i) = wd2;
            C.at(kWD3, k, i) = wd3;
            if (TAN) {
                float fM = fmaf(wm1, fM2[i - 1] + dD2, fmaf(wm2, fI2[i - 1] + dD2, wm3 * (fD2[i - 1] + dD2)));
                float fI = fmaf(wi1, fM1[i - 1] + (xI1 + dD1),
                                fmaf(wi2, fI1[i - 1] + (xI2 + dD1), wi3 * (fD1[i - 1] + (xI3 + dD1))));
                float fD = fmaf(wd1, fM1[i] + (xD1 + dD1), fmaf(wd2, fI1[i] + (xD2 + dD1), wd3 * (fD1[i] + (xD3 + dD1))));
                if (MODE == MODE_HVP) fM += vv;
                if (MODE == MODE_PT) {   // + the choice's entropy (d LSE_T / dT at fixed options)
                    fM += hM;
                    fI += hI;
                    fD += hD;
                }
                putF(i, fM, fI, fD);
            }
        };
        const int i0 = max(0, k - L2), i1 = min(L1, k);
#pragma unroll
        for (int r = 0; r < kPF; ++r) {
            const int i = i0 + tid + r * kThreads;
            if (i <= i1) cell(i, pc[r], pv[r]);
        }
        for (int i = i0 + tid + kPF * kThreads; i <= i1; i += kThreads) {
            const int j = k - i;
            const bool ok = i >= 1 && j >= 1;
            const size_t si = ok ? (size_t)(i - 1) * L2m + (j - 1) : 0;
            cell(i, ok ? __ldg(S + si) : 0.f, MODE == MODE_HVP && ok ? __ldg(V + si) : 0.f);
        }
        if (k < K) {
            float nc[kPF], nv[kPF];
            fetch_fwd(k + 1, nc, nv);
            __syncthreads();
#pragma unroll
            for (int r = 0; r < kPF; ++r) {
                pc[r] = nc[r];
                pv[r] = nv[r];
            }
        } else {
            __syncthreads();
        }
        O2 = O1;
        O1 = Ok;
        D2 = D1;
        D1 = Dk;
    }

    // the final choice among the end cell's states (rings read before any reverse write)
    const float eM = row(rAM, kAM, K)[L1], eI = row(rAM + 1, kAI, K)[L1], eD = row(rAM + 2, kAD, K)[L1];
    float fw1, fw2, fw3, fh;
    const float aEnd = lse3w(eM, eI, eD, T, iT, fw1, fw2, fw3, &fh);
    float fr1 = 0.f, fr2 = 0.f, fr3 = 0.f;   // the final weights' tangents
    if (TAN) {
        const float t1 = row(rFM, kFM, K)[L1], t2 = row(rFM + 1, kFI, K)[L1], t3 = row(rFM + 2, kFD, K)[L1];
        const float E = fmaf(fw1, t1, fmaf(fw2, t2, fw3 * t3));
        fr1 = fw1 * (t1 - E) * iT;
        fr2 = fw2 * (t2 - E) * iT;
        fr3 = fw3 * (t3 - E) * iT;
        if (MODE == MODE_PT) {
            const float Ev = fmaf(fw1, eM, fmaf(fw2, eI, fw3 * eD));
            const float iT2 = iT * iT;
            fr1 = fmaf(fw1 * (Ev - eM), iT2, fr1);
            fr2 = fmaf(fw2 * (Ev - eI), iT2, fr2);
            fr3 = fmaf(fw3 * (Ev - eD), iT2, fr3);
        }
    }

    // ------------------------------------------------------------- reverse
    RevIn pre[kPFR];
    auto fetch_one = [&](int k, int i, RevIn& q) {
        const int j = k - i;
        const bool okM = i + 1 <= L1 && j + 1 <= L2, okI = i + 1 <= L1 && j >= 1, okD = j + 1 <= L2 && i >= 1;
        const bool own = i >= 1 && j >= 1;
#pragma unroll
        for (int s = 0; s < 3; ++s) {
            q.sm[s] = okM ? C.at(kWM1 + s, k + 2, i + 1) : 0.f;
            q.si[s] = okI ? C.at(kWI1 + s, k + 1, i + 1) : 0.f;
            q.sd[s] = okD ? C.at(kWD1 + s, k + 1, i) : 0.f;
            q.om[s] = own ? C.at(kWM1 + s, k, i) : 0.f;
            q.oi[s] = own ? C.at(kWI1 + s, k, i) : 0.f;
            q.od[s] = own ? C.at(kWD1 + s, k, i) : 0.f;
        }
    };
    auto fetch_rev = [&](int k, RevIn* q) {
        const int i0 = max(0, k - L2), i1 = min(L1, k);
#pragma unroll
        for (int r = 0; r < kPFR; ++r) {
            const int i = i0 + tid + r * kThreads;
            if (i <= i1) fetch_one(k, i, q[r]);
        }
    };
    if (MODE == MODE_MARG) fetch_rev(K, pre);
    double sopen = 0.0, sext = 0.0, sent = 0.0, sdot = 0.0;
    for (int k = K; k >= 0; --k) {
        const int k1 = min(k + 1, K), k2 = min(k + 2, K);
        float* const bM0 = row(rBM, kBM, k);
        float* const bI0 = row(rBM + 1, kBI, k);
        float* const bD0 = row(rBM + 2, kBD, k);
        const float* const bM2 = row(rBM, kBM, k2);     // M successors lie on diagonal k + 2
        const float* const bI1 = row(rBM + 1, kBI, k1);
        const float* const bD1 = row(rBM + 2, kBD, k1);
        const int i0 = max(0, k - L2), i1 = min(L1, k);
        if (MODE == MODE_MARG) {
            auto ent = [](const float* w) {   // a state's choice entropy -sum w ln w
                float h = 0.f;
#pragma unroll
                for (int q = 0; q < 3; ++q)
                    if (w[q] > 0.f) h = fmaf(-w[q], logf(w[q]), h);
                return h;
            };
            auto cell = [&](int i, const RevIn& q) {
                const int j = k - i;
                float bM = 0.f, bI = 0.f, bD = 0.f;
                if (k == K) {
                    bM = fw1;
                    bI = fw2;
                    bD = fw3;
                }
                if (i + 1 <= L1 && j + 1 <= L2) {
                    const float by = bM2[i + 1];
                    bM = fmaf(by, q.sm[0], bM);
                    bI = fmaf(by, q.sm[1], bI);
                    bD = fmaf(by, q.sm[2], bD);
                }
                if (i + 1 <= L1 && j >= 1) {
                    const float by = bI1[i + 1];
                    bM = fmaf(by, q.si[0], bM);
                    bI = fmaf(by, q.si[1], bI);
                    bD = fmaf(by, q.si[2], bD);
                }
                if (j + 1 <= L2 && i >= 1) {
                    const float by = bD1[i];
                    bM = fmaf(by, q.sd[0], bM);
                    bI = fmaf(by, q.sd[1], bI);
                    bD = fmaf(by, q.sd[2], bD);
                }
                bM0[i] = bM;
                bI0[i] = bI;
                bD0[i] = bD;
                if (i >= 1 && j >= 1) {
                    if (out) out[(size_t)(i - 1) * L2m + (j - 1)] = bM;
                    sopen += (double)bI * (double)(q.oi[0] + q.oi[2]) + (double)bD * (double)(q.od[0] + q.od[1]);
                    sext += (double)bI * (double)q.oi[1] + (double)bD * (double)q.od[2];
                    sent += (double)bM * (double)ent(q.om) + (double)bI * (double)ent(q.oi) +
                            (double)bD * (double)ent(q.od);
                } else if (k >= 1) {   // leading gaps of the boundary states
                    const float bb = i >= 1 ? bI : bD;
                    sopen += (double)bb;
                    sext += (double)bb * (double)(k - 1);
                }
            };
#pragma unroll
            for (int r = 0; r < kPFR; ++r) {
                const int i = i0 + tid + r * kThreads;
                if (i <= i1) cell(i, pre[r]);
            }
            for (int i = i0 + tid + kPFR * kThreads; i <= i1; i += kThreads) {
                RevIn q;
                fetch_one(k, i, q);
                cell(i, q);
            }
            if (k > 0) {
                RevIn nxt[kPFR];
                fetch_rev(k - 1, nxt);
                __syncthreads();
#pragma unroll
                for (int r = 0; r < kPFR; ++r) pre[r] = nxt[r];
            } else {
                __syncthreads();
            }
        } else {
            float* const rM0 = row(rRM, kRM, k);
            float* const rI0 = row(rRM + 1, kRI, k);
            float* const rD0 = row(rRM + 2, kRD, k);
            const float* const rM2 = row(rRM, kRM, k2);
            const float* const rI1 = row(rRM + 1, kRI, k1);
            const float* const rD1 = row(rRM + 2, kRD, k1);
            for (int i = i0 + tid; i <= i1; i += blockDim.x) {
                const int j = k - i;
                const bool interior = i >= 1 && j >= 1;
                float bM = 0.f, bI = 0.f, bD = 0.f, rM = 0.f, rI = 0.f, rD = 0.f;
                if (k == K) {
                    bM = fw1;
                    bI = fw2;
                    bD = fw3;
                    rM = fr1;
                    rI = fr2;
                    rD = fr3;
                }
                // this cell's states as options: their tangents (a shift common
                // to the three cancels in u - E) and, along T, their values
                const float t1 = C.at(kFM, k, i), t2 = C.at(kFI, k, i), t3 = C.at(kFD, k, i);
                float a1 = 0.f, a2 = 0.f, a3 = 0.f;
                if (MODE == MODE_PT) {
                    a1 = C.at(kAM, k, i);
                    a2 = C.at(kAI, k, i);
                    a3 = C.at(kAD, k, i);
                }
                // successor state Y at d (beta by, its tangent ry) takes this
                // cell's states with weights w1..w3; x1..x3: the options' direct
                // parameter derivatives, g1..g3 their gap terms
                auto take = [&](int kd, int id, float by, float ry, int pw, float x1, float x2, float x3, float g1,
                                float g2, float g3) {
                    const float w1 = C.at(pw, kd, id), w2 = C.at(pw + 1, kd, id), w3 = C.at(pw + 2, kd, id);
                    bM = fmaf(by, w1, bM);
                    bI = fmaf(by, w2, bI);
                    bD = fmaf(by, w3, bD);
                    const float u1 = t1 + x1, u2 = t2 + x2, u3 = t3 + x3;
                    const float E = fmaf(w1, u1, fmaf(w2, u2, w3 * u3));
                    float e1 = w1 * (u1 - E) * iT, e2 = w2 * (u2 - E) * iT, e3 = w3 * (u3 - E) * iT;
                    if (MODE == MODE_PT) {
                        const float v1 = a1 + g1, v2 = a2 + g2, v3 = a3 + g3;
                        const float Ev = fmaf(w1, v1, fmaf(w2, v2, w3 * v3));
                        const float iT2 = iT * iT;
                        e1 = fmaf(w1 * (Ev - v1), iT2, e1);
                        e2 = fmaf(w2 * (Ev - v2), iT2, e2);
                        e3 = fmaf(w3 * (Ev - v3), iT2, e3);
                    }
                    rM = fmaf(ry, w1, fmaf(by, e1, rM));
                    rI = fmaf(ry, w2, fmaf(by, e2, rI));
                    rD = fmaf(ry, w3, fmaf(by, e3, rD));
                };
                if (i + 1 <= L1 && j + 1 <= L2)
                    take(k + 2, i + 1, bM2[i + 1], rM2[i + 1], kWM1, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f);
                if (i + 1 <= L1 && j >= 1) take(k + 1, i + 1, bI1[i + 1], rI1[i + 1], kWI1, xI1, xI2, xI3, go, ge, go);
                if (j + 1 <= L2 && i >= 1) take(k + 1, i, bD1[i], rD1[i], kWD1, xD1, xD2, xD3, go, go, ge);
                bM0[i] = bM;
                bI0[i] = bI;
                bD0[i] = bD;
                rM0[i] = rM;
                rI0[i] = rI;
                rD0[i] = rD;
                if (interior) {
                    const size_t si = (size_t)(i - 1) * L2m + (j - 1);
                    if (out) out[si] = rM;
                    if (Gw) sdot += (double)Gw[si] * (double)rM;
                }
            }
            __syncthreads();
        }
    }

    if (MODE == MODE_MARG) {
        const double to = block_sum(sopen, red);
        const double te = block_sum(sext, red);
        const double th = block_sum(sent, red);
        if (tid == 0) {
            if (p.value) p.value[b] = (float)((double)aEnd + (double)C.O[K]);
            if (p.grad_gap) p.grad_gap[b] = (float)to;
            if (p.grad_gap2) p.grad_gap2[b] = (float)te;
            if (p.grad_T) p.grad_T[b] = (float)(th + (double)fh);
        }
    } else if (p.dot_out) {
        const double t = block_sum(sdot, red);
        if (tid == 0) p.dot_out[b] = (float)t;
    }
}

}  // namespace nwa

// ------------------------------------------------------------------ host side
size_t nwa_workspace_bytes(int op, int B, int L1, int L2) {
    const size_t fb = nwa::per_problem_bytes(L1, L2, op == D2P_OP_FORWARD_BACKWARD ? MODE_MARG : MODE_PT);
    size_t n = (fb * (size_t)(B > 0 ? B : 1) + 255) & ~(size_t)255;
    if (op == D2P_OP_FORWARD_BACKWARD) {   // the wavefront pass shares the area; + one flag per problem
        const size_t w = nwa_wave_area(B, L1, L2);
        if (w > n) n = w;
        n += ((size_t)(B > 0 ? B : 1) * sizeof(int) + 255) & ~(size_t)255;
    }
    if (op == D2P_OP_BACKWARD_FULL) n += ((size_t)3 * (B > 0 ? B : 1) * sizeof(float) + 255) & ~(size_t)255;
    return n;
}

int launch_nwa(const SwArgs& a, cudaStream_t st) {
    if (a.B == 0) return 0;
    static DeviceSetup setup;
    int dev = 0, sms = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return (int)e;
    int rc = device_setup(setup, dev, [] {
        const int cap = (int)nwa::kMaxRingBytes;
        const void* ks[] = {(const void*)nwa::nwa_kernel<MODE_MARG>, (const void*)nwa::nwa_kernel<MODE_HVP>,
                            (const void*)nwa::nwa_kernel<MODE_PGAP>, (const void*)nwa::nwa_kernel<MODE_PGE>,
                            (const void*)nwa::nwa_kernel<MODE_PT>};
        cudaError_t r = cudaSuccess;
        for (const void* k : ks)
            if (r == cudaSuccess) r = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, cap);
        return (int)r;
    }, &sms);
    if (rc) return rc;
    const size_t rb = nwa::ring_bytes(a.L1, a.mode);
    const size_t smem = rb <= nwa::kMaxRingBytes ? rb : 0;   // else the rings are the planes
    switch (a.mode) {
        case MODE_MARG: nwa::nwa_kernel<MODE_MARG><<<a.B, nwa::kThreads, smem, st>>>(a); break;
        case MODE_HVP: nwa::nwa_kernel<MODE_HVP><<<a.B, nwa::kThreads, smem, st>>>(a); break;
        case MODE_PGAP: nwa::nwa_kernel<MODE_PGAP><<<a.B, nwa::kThreads, smem, st>>>(a); break;
        case MODE_PGE: nwa::nwa_kernel<MODE_PGE><<<a.B, nwa::kThreads, smem, st>>>(a); break;
        case MODE_PT: nwa::nwa_kernel<MODE_PT><<<a.B, nwa::kThreads, smem, st>>>(a); break;
        default: return kErrInvalid;
    }
    return (int)cudaGetLastError();
}

}  // namespace d2pb

using namespace d2pb;

// ---------------------------------------------------------------- C ABI
extern "C" {

// the reference's affine table limit: 3 (L1 + 1) (L2 + 1) <= INT_MAX
static bool nwa_dims_ok(int B, int L1, int L2) {
    if (B < 0 || L1 < 0 || L2 < 0) return false;
    return 3LL * (long long)(L1 + 1) * (long long)(L2 + 1) <= 2147483647LL;
}

static SwArgs nwa_args(const float* scores, const int* lengths, int B, int L1, int L2, float go, float ge, float T,
                       void* ws) {
    SwArgs a{};
    a.scores = scores;
    a.lengths = lengths;
    a.B = B;
    a.L1 = L1;
    a.L2 = L2;
    a.gap = go;
    a.gap2 = ge;
    a.temp = T;
    a.ws = (float*)ws;
    return a;
}

int d2p_nw_affine_forward_backward(const float* scores, const int* lengths, int B, int L1, int L2,
                                   float gap_open, float gap_ext, float temperature, const float* gap_open_dev,
                                   const float* gap_ext_dev, const float* temperature_dev, float* value,
                                   float* marginals, float* grad_gap_open, float* grad_gap_ext,
                                   float* grad_temperature, void* workspace, size_t workspace_bytes, void* stream) {
    if (!nwa_dims_ok(B, L1, L2)) return D2P_ERR_TOO_LARGE;
    if (B == 0) return D2P_OK;
    if (!scores || !value || !marginals) return D2P_ERR_INVALID_ARGUMENT;
    if (!workspace || workspace_bytes < nwa_workspace_bytes(D2P_OP_FORWARD_BACKWARD, B, L1, L2))
        return D2P_ERR_WORKSPACE_TOO_SMALL;
    SwArgs a = nwa_args(scores, lengths, B, L1, L2, gap_open, gap_ext, temperature, workspace);
    a.gap_dev = gap_open_dev;
    a.gap2_dev = gap_ext_dev;
    a.temp_dev = temperature_dev;
    a.mode = MODE_MARG;
    a.value = value;
    a.out = marginals;
    a.grad_gap = grad_gap_open;
    a.grad_gap2 = grad_gap_ext;
    a.grad_T = grad_temperature;
    cudaStream_t st = (cudaStream_t)stream;
    // the wavefront pass; the engine recomputes the problems it flags
    const size_t eng = (nwa::per_problem_bytes(L1, L2, MODE_MARG) * (size_t)B + 255) & ~(size_t)255;
    const size_t wav = nwa_wave_area(B, L1, L2);
    int* flags = (int*)((char*)workspace + (eng > wav ? eng : wav));
    int rc = (int)cudaMemsetAsync(flags, 0, (size_t)B * sizeof(int), st);
    if (rc) return rc;
    SwArgs w = a;
    w.redo = flags;
    rc = launch_nwa_wave(w, st);
    if (rc == 0) a.only = flags;
    else if (rc != -1) return rc;
    return launch_nwa(a, st);
}

int d2p_nw_affine_hvp(const float* scores, const float* tangent, const int* lengths, int B, int L1, int L2,
                      float gap_open, float gap_ext, float temperature, float* hvp, void* workspace,
                      size_t workspace_bytes, void* stream) {
    if (!nwa_dims_ok(B, L1, L2)) return D2P_ERR_TOO_LARGE;
    if (B == 0) return D2P_OK;
    if (!scores || !tangent || !hvp) return D2P_ERR_INVALID_ARGUMENT;
    if (!workspace || workspace_bytes < nwa_workspace_bytes(D2P_OP_HVP, B, L1, L2)) return D2P_ERR_WORKSPACE_TOO_SMALL;
    SwArgs a = nwa_args(scores, lengths, B, L1, L2, gap_open, gap_ext, temperature, workspace);
    a.mode = MODE_HVP;
    a.tangent = tangent;
    a.out = hvp;
    return launch_nwa(a, (cudaStream_t)stream);
}

int d2p_nw_affine_param_jacobian(const float* scores, const int* lengths, int B, int L1, int L2, int param_type,
                                 float gap_open, float gap_ext, float temperature, float* jacobian, void* workspace,
                                 size_t workspace_bytes, void* stream) {
    if (!nwa_dims_ok(B, L1, L2)) return D2P_ERR_TOO_LARGE;
    if (param_type < 0 || param_type > 2) return D2P_ERR_INVALID_ARGUMENT;
    if (B == 0) return D2P_OK;
    if (!scores || !jacobian) return D2P_ERR_INVALID_ARGUMENT;
    if (!workspace || workspace_bytes < nwa_workspace_bytes(D2P_OP_PARAM_JACOBIAN, B, L1, L2))
        return D2P_ERR_WORKSPACE_TOO_SMALL;
    SwArgs a = nwa_args(scores, lengths, B, L1, L2, gap_open, gap_ext, temperature, workspace);
    a.mode = param_type == 0 ? MODE_PGAP : param_type == 1 ? MODE_PGE : MODE_PT;
    a.out = jacobian;
    return launch_nwa(a, (cudaStream_t)stream);
}

int d2p_nw_affine_backward_full(const float* scores, const float* grad_marginals, const int* lengths, int B, int L1,
                                int L2, float gap_open, float gap_ext, float temperature, float* grad_scores,
                                float* grad_gap_open, float* grad_gap_ext, float* grad_temperature,
                                void* workspace, size_t workspace_bytes, void* stream) {
    if (!nwa_dims_ok(B, L1, L2)) return D2P_ERR_TOO_LARGE;
    if (!grad_scores || !grad_gap_open || !grad_gap_ext || !grad_temperature) return D2P_ERR_INVALID_ARGUMENT;
    cudaStream_t st = (cudaStream_t)stream;
    if (B == 0) {
        float* outs[3] = {grad_gap_open, grad_gap_ext, grad_temperature};
        for (float* o : outs) {
            const cudaError_t e = cudaMemsetAsync(o, 0, sizeof(float), st);
            if (e != cudaSuccess) return (int)e;
        }
        return D2P_OK;
    }
    if (!scores || !grad_marginals) return D2P_ERR_INVALID_ARGUMENT;
    if (!workspace || workspace_bytes < nwa_workspace_bytes(D2P_OP_BACKWARD_FULL, B, L1, L2))
        return D2P_ERR_WORKSPACE_TOO_SMALL;
    // grad_scores = H . grad_marginals (the Hessian of S is symmetric); the
    // parameter parts = sum grad_marginals * dP/dtheta
    const size_t area = nwa::per_problem_bytes(L1, L2, MODE_PT) * (size_t)B;
    float* partials = (float*)((char*)workspace + ((area + 255) & ~(size_t)255));
    SwArgs a = nwa_args(scores, lengths, B, L1, L2, gap_open, gap_ext, temperature, workspace);
    a.mode = MODE_HVP;
    a.tangent = grad_marginals;
    a.out = grad_scores;
    int rc = launch_nwa(a, st);
    if (rc) return rc;
    a.tangent = nullptr;
    a.out = nullptr;
    a.dot_with = grad_marginals;
    const int modes[3] = {MODE_PGAP, MODE_PGE, MODE_PT};
    float* outs[3] = {grad_gap_open, grad_gap_ext, grad_temperature};
    for (int q = 0; q < 3; ++q) {
        a.mode = modes[q];
        a.dot_out = partials + (size_t)q * B;
        rc = launch_nwa(a, st);
        if (rc) return rc;
        rc = launch_sum_batches(partials + (size_t)q * B, 1, B, outs[q], 0, st);
        if (rc) return rc;
    }
    return D2P_OK;
}

}  // extern "C"
