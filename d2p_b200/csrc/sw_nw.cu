// sw_nw.cu -- soft Needleman-Wunsch (global alignment, linear gap): value,
// marginals, dS/dgap and dS/dT, the Hessian-vector product, the parameter
// Jacobians dP/dgap and dP/dT, and their contraction with a weight plane
// (backward_full).
//
// Recurrences (src/nw/kernels_cpu.cpp:79-642 restated, natural units):
//   alpha[0,0] = 0, alpha[i,0] = i gap, alpha[0,j] = j gap,
//   alpha[i,j] = T log sum_k exp(v_k / T),  v = (alpha[i-1,j-1] + s_ij,
//                alpha[i-1,j] + gap, alpha[i,j-1] + gap),
//   S = alpha[L1, L2];  w_k = exp((v_k - alpha[i,j]) / T) normalised by their sum.
// The reverse is the flow of the path distribution: beta[L1,L2] = 1 and
// beta[c] = sum over the successors d of c of beta[d] w_{c->d}(d); the marginal
// of cell (i,j) is beta[i,j] w_diag(i,j).  dS/dgap = E[gaps] = the flow
// through gap moves (beta (w_up + w_left) per cell, plus k gaps for a path
// that reaches the boundary cell (i, 0) or (0, j), k = i + j), and dS/dT =
// (S - E[path score]) / T is the entropy of the path distribution: the sum of
// each cell's choice entropy -sum w ln w weighted by beta (equal to the
// reference's (S - sum s mu - gap dS/dgap) / T, src/nw/kernels_cpu.cpp:161-262,
// without its cancellation).
//
// Tangents along a direction (V in the scores, or gap, or T): the forward
// carries d alpha = sum_k w_k dv_k (+ (alpha - E[v]) / T along T), the
// reverse d beta[c] = sum_d (d beta[d] w_{c->d}(d) + beta[d] dw_{c->d}(d)),
// dw_k = w_k (dv_k - d alpha) / T (+ w_k (E[v] - v_k) / T^2 along T), and the
// marginal's tangent d beta w_diag + beta dw_diag (src/nw/kernels_cpu.cpp:278-642).
//
// Value + marginals without parameter gradients run on the column-sweep strip
// kernel (sw_strip.cu, its NW form) for problems of at most 512 rows; this
// engine takes the rest and recomputes whatever the strip kernel flags.
//
// Engine.  One CTA per problem sweeps the anti-diagonals (k = i + j), the
// threads striding over the cells of a diagonal, with one barrier per
// diagonal.  Per-cell values live in diagonal-major planes in the workspace
// ([k][i]: one diagonal is contiguous, so its loads and stores coalesce):
// alpha and the three normalised weights from the forward, beta from the
// reverse, and for a tangent its forward and reverse values.  alpha and the
// forward tangent are stored relative to an integer frame per diagonal.  The reverse is a
// gather over the successors (no atomics: deterministic).  A general engine:
// any size, every mode; per-problem sums are block reductions in fp64.
#include <math.h>
#include <stddef.h>
#include <stdint.h>

#include "../../include/d2p_b200.h"
#include "sw_common.cuh"
#include "sw_internal.h"

namespace d2pb {
namespace nw {

constexpr int kThreads = 256;

// planes of one problem, each (L1m + L2m + 1) (L1m + 1) floats, then the
// frames of the diagonals (alpha's and the forward tangent's), L1m + L2m + 1
// floats each
enum Plane : int { kA = 0, kWd, kWu, kWl, kB, kT1, kT2, kT3, kNumPlanes };
__host__ __device__ inline size_t plane_floats(int L1m, int L2m) {
    return ((size_t)L1m + L2m + 1) * ((size_t)L1m + 1);
}
__host__ __device__ inline int planes_for(int mode) {
    // MARG: alpha, weights, beta, each cell's choice entropy; HVP / PGAP:
    // alpha, weights, beta, the forward tangent and the reverse tangent; PT:
    // + E[v] as well
    return mode == MODE_MARG ? 6 : (mode == MODE_PT ? 8 : 7);
}
__host__ __device__ inline size_t per_problem_bytes(int L1m, int L2m, int mode) {
    const size_t b = (plane_floats(L1m, L2m) * planes_for(mode) + 2 * ((size_t)L1m + L2m + 1)) * sizeof(float);
    return (b + 255) & ~(size_t)255;
}

struct Ctx {
    float* p[kNumPlanes];
    float* O;     // alpha's frame of each diagonal (integer-valued): alpha = A + O[k]
    float* D;     // the forward tangent's: dalpha = F + D[k]
    int stride;   // L1m + 1
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

// Rings: the last three diagonals of alpha (and the forward tangent) during
// the forward, and of beta (and the reverse tangent) during the reverse, sit
// in shared memory ([3][L1m + 1] floats each) when they fit, so the sweep reads
// its neighbours at shared-memory latency; the planes still receive what the
// reverse reads back (weights and entropies; the forward tangent; alpha and
// E[v] for MODE_PT).  When the rings do not fit, each ring is its quantity's
// plane.  The scores (and direction) of a diagonal are loaded one diagonal
// ahead, before the barrier.
constexpr int kPF = 2;                          // cells per thread prefetched (diagonals of <= 512 cells)
constexpr size_t kMaxRingBytes = 200 * 1024;    // dynamic shared memory cap of the rings
__host__ __device__ inline int rings_for(int mode) { return mode == MODE_MARG ? 2 : 4; }
__host__ __device__ inline size_t ring_bytes(int L1m, int mode) {
    return (size_t)rings_for(mode) * 3 * ((size_t)L1m + 1) * sizeof(float);
}

// One CTA per problem.  MODE: MODE_MARG (value, marginals, dS/dgap, dS/dT),
// MODE_HVP (out = d marginals along p.tangent), MODE_PGAP / MODE_PT (out =
// dP/dtheta; with dot_with, dot_out[b] = sum dot_with * dP/dtheta).
//
// Frames.  alpha grows along the diagonals (about k gap on diagonal k), so it
// is stored as A = alpha - O[k], with O[k] an integer-valued float taken from
// the previous diagonal's middle cell: every option v - alpha is then formed
// from small stored values plus an exact difference of frames, instead of as
// a difference of two large rounded numbers.  The forward tangent (which grows
// like the expected number of gaps, or the path's sum of V) keeps a frame D[k]
// the same way.
template <int MODE>
__global__ void __launch_bounds__(kThreads) nw_kernel(SwArgs p) {
    extern __shared__ float ring_smem[];
    __shared__ double red[32];
    const int b = blockIdx.x;
    if (p.only && !p.only[b]) return;   // a fix-up launch: only the problems the strip kernel flagged
    const int L1m = p.L1, L2m = p.L2;
    const int L1 = p.lengths ? min(max(p.lengths[2 * b], 0), L1m) : L1m;
    const int L2 = p.lengths ? min(max(p.lengths[2 * b + 1], 0), L2m) : L2m;
    const float gap = p.gap_dev ? __ldg(p.gap_dev) : p.gap;
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
    const bool TAN = MODE != MODE_MARG;
    // the forward tangent (dalpha, or U) and the reverse tangent (dbeta, or W)
    const int kF = kT1, kR = kT2, kEv = kT3;
    const int K = L1 + L2;   // the end cell's diagonal
    const int tid = threadIdx.x;
    const bool smR = ring_bytes(L1m, MODE) <= kMaxRingBytes;
    const int RS = L1m + 1;
    // row of diagonal k of ring rg (alpha 0, beta 1, forward tangent 2,
    // reverse tangent 3), or of its plane pl when the rings are the planes
    auto row = [&](int rg, int pl, int k) -> float* {
        return smR ? ring_smem + (size_t)(3 * rg + k % 3) * RS : C.p[pl] + (size_t)k * C.stride;
    };

    // padding of the output: zeros outside the problem
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
    float O1 = 0.f, O2 = 0.f, D1 = 0.f, D2 = 0.f;   // frames of diagonals k-1, k-2
    for (int k = 0; k <= K; ++k) {
        float* const a0 = row(0, kA, k);
        const float* const a1 = row(0, kA, max(k - 1, 0));
        const float* const a2 = row(0, kA, max(k - 2, 0));
        float* const f0 = TAN ? row(2, kF, k) : nullptr;
        const float* const f1 = TAN ? row(2, kF, max(k - 1, 0)) : nullptr;
        const float* const f2 = TAN ? row(2, kF, max(k - 2, 0)) : nullptr;
        float Ok = 0.f, Dk = 0.f;
        if (k >= 2) {   // from the previous diagonal's middle cell (the same value in every thread)
            const int im = (max(0, k - 1 - L2) + min(L1, k - 1)) >> 1;
            Ok = O1 + rintf(a1[im]);
            if (TAN) Dk = D1 + rintf(f1[im]);
        }
        if (tid == 0) {
            C.O[k] = Ok;
            C.D[k] = Dk;
        }
        const float dO1 = O1 - Ok, dO2 = O2 - Ok, dD1 = D1 - Dk, dD2 = D2 - Dk;   // exact
        auto putA = [&](int i, float v) {
            a0[i] = v;
            if (smR && MODE == MODE_PT) C.at(kA, k, i) = v;
        };
        auto putF = [&](int i, float v) {
            f0[i] = v;
            if (smR) C.at(kF, k, i) = v;
        };
        auto cell = [&](int i, float sc, float vv) {
            const int j = k - i;
            if (i == 0 || j == 0) {   // boundary: alpha = k gap; the gap tangent is k
                putA(i, fmaf((float)k, gap, -Ok));
                if (TAN) putF(i, (MODE == MODE_PGAP ? (float)k : 0.f) - Dk);
                return;
            }
            const float vd = a2[i - 1] + (sc + dO2);
            const float vu = a1[i - 1] + (gap + dO1);
            const float vl = a1[i] + (gap + dO1);
            const float m = fmaxf(vd, fmaxf(vu, vl));
            const float ed = expf((vd - m) * iT), eu = expf((vu - m) * iT), el = expf((vl - m) * iT);
            const float sum = (ed + eu) + el;
            const float a = fmaf(T, logf(sum), m);
            const float is = 1.f / sum;
            const float wd = ed * is, wu = eu * is, wl = el * is;
            putA(i, a);
            C.at(kWd, k, i) = wd;
            C.at(kWu, k, i) = wu;
            C.at(kWl, k, i) = wl;
            if (MODE == MODE_MARG) {
                // the entropy of the cell's choice, -sum w ln w = ln(sum) +
                // sum w (m - v) / T: a sum of non-negative terms
                C.at(kT1, k, i) = logf(sum) + iT * fmaf(wd, m - vd, fmaf(wu, m - vu, wl * (m - vl)));
            }
            if (TAN) {
                // tangents of the three options, in this diagonal's frame
                float td = f2[i - 1] + dD2, tu = f1[i - 1] + dD1, tl = f1[i] + dD1;
                if (MODE == MODE_HVP) td += vv;
                if (MODE == MODE_PGAP) {
                    tu += 1.f;
                    tl += 1.f;
                }
                float f = fmaf(wd, td, fmaf(wu, tu, wl * tl));
                if (MODE == MODE_PT) {
                    const float ev = fmaf(wd, vd, fmaf(wu, vu, wl * vl));
                    C.at(kEv, k, i) = ev;
                    f = fmaf(a - ev, iT, f);
                }
                putF(i, f);
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
    const float aEnd = row(0, kA, K)[L1];   // read before any reverse write (separate rings)

    // ------------------------------------------------------------- reverse
    double sgap = 0.0, sent = 0.0, sdot = 0.0;
    for (int k = K; k >= 0; --k) {
        const float Ok = C.O[k], Dk = C.D[k];
        const float Ok1 = k + 1 <= K ? C.O[k + 1] : 0.f, Ok2 = k + 2 <= K ? C.O[k + 2] : 0.f;
        const float Dk1 = k + 1 <= K ? C.D[k + 1] : 0.f, Dk2 = k + 2 <= K ? C.D[k + 2] : 0.f;
        const float Om2 = k >= 2 ? C.O[k - 2] : 0.f, Dm2 = k >= 2 ? C.D[k - 2] : 0.f;
        float* const b0 = row(1, kB, k);
        const float* const b1 = row(1, kB, min(k + 1, K));
        const float* const b2 = row(1, kB, min(k + 2, K));
        float* const r0 = TAN ? row(3, kR, k) : nullptr;
        const float* const r1 = TAN ? row(3, kR, min(k + 1, K)) : nullptr;
        const float* const r2 = TAN ? row(3, kR, min(k + 2, K)) : nullptr;
        const int i0 = max(0, k - L2), i1 = min(L1, k);
        for (int i = i0 + tid; i <= i1; i += blockDim.x) {
            const int j = k - i;
            const bool interior = i >= 1 && j >= 1;
            float be = 0.f, tb = 0.f;
            const float fc = TAN ? C.at(kF, k, i) : 0.f;
            const float ac = MODE == MODE_PT ? C.at(kA, k, i) : 0.f;
            if (k == K) {
                be = 1.f;   // the end cell (L1, L2); its tangent is 0
            } else {
                // successors: (i+1, j+1) by its diagonal option, (i+1, j) by
                // its up option (if j >= 1), (i, j+1) by its left option (if i >= 1)
                auto take = [&](int kd, int id, int opt, int si_d, float dO, float dD) {
                    // dO, dD: this cell's frames minus the successor's (exact)
                    const float bd = (kd == k + 1 ? b1 : b2)[id];
                    const float w = C.at(opt, kd, id);
                    be = fmaf(bd, w, be);
                    if (TAN) {
                        // dw of the option c -> d at d: w (dv - d alpha_d) / T (+ the T term)
                        float dv = fc + dD;
                        if (MODE == MODE_HVP && opt == kWd) dv += V[si_d];
                        if (MODE == MODE_PGAP && opt != kWd) dv += 1.f;
                        const float fd = C.at(kF, kd, id);
                        float eu = fd;
                        if (MODE == MODE_PT) eu = fd - (C.at(kA, kd, id) - C.at(kEv, kd, id)) * iT;
                        float dw = w * (dv - eu) * iT;
                        if (MODE == MODE_PT) {
                            const float v = ac + ((opt == kWd ? S[si_d] : gap) + dO);
                            dw = fmaf(w * (C.at(kEv, kd, id) - v), iT * iT, dw);
                        }
                        tb = fmaf((kd == k + 1 ? r1 : r2)[id], w, fmaf(bd, dw, tb));
                    }
                };
                if (i + 1 <= L1 && j + 1 <= L2) take(k + 2, i + 1, kWd, i * L2m + j, Ok - Ok2, Dk - Dk2);
                if (i + 1 <= L1 && j >= 1) take(k + 1, i + 1, kWu, 0, Ok - Ok1, Dk - Dk1);
                if (j + 1 <= L2 && i >= 1) take(k + 1, i, kWl, 0, Ok - Ok1, Dk - Dk1);
            }
            b0[i] = be;
            if (TAN) r0[i] = tb;
            if (MODE == MODE_MARG && !interior) sgap += (double)be * (double)k;   // a path ending at (i, 0) or (0, j) takes k more gaps
            if (interior) {
                const size_t si = (size_t)(i - 1) * L2m + (j - 1);
                const float wd = C.at(kWd, k, i);
                if (MODE == MODE_MARG) {
                    const float mu = be * wd;
                    if (out) out[si] = mu;
                    sgap += (double)be * (double)(C.at(kWu, k, i) + C.at(kWl, k, i));
                    sent += (double)be * (double)C.at(kT1, k, i);
                } else {
                    // the tangent of this cell's diagonal weight
                    float dv = C.at(kF, k - 2, i - 1) + (Dm2 - Dk);
                    if (MODE == MODE_HVP) dv += V[si];
                    float eu = fc;
                    if (MODE == MODE_PT) eu = fc - (ac - C.at(kEv, k, i)) * iT;
                    float dwd = wd * (dv - eu) * iT;
                    if (MODE == MODE_PT) {
                        const float vd = C.at(kA, k - 2, i - 1) + (S[si] + (Om2 - Ok));
                        dwd = fmaf(wd * (C.at(kEv, k, i) - vd), iT * iT, dwd);
                    }
                    const float dmu = fmaf(tb, wd, be * dwd);
                    if (out) out[si] = dmu;
                    if (Gw) sdot += (double)Gw[si] * (double)dmu;
                }
            }
        }
        __syncthreads();
    }

    if (MODE == MODE_MARG) {
        // dS/dgap = E[gaps]: the flows through gap moves; dS/dT = (S - E[path
        // score]) / T, the entropy of the path distribution: the cells' choice
        // entropies weighted by their visit probabilities (both sums of
        // non-negative terms, free of the cancellation in S - sum s mu - gap
        // dS/dgap)
        const double tgap = block_sum(sgap, red);
        const double tent = block_sum(sent, red);
        if (threadIdx.x == 0) {
            const double Sv = (double)aEnd + (double)C.O[K];
            if (p.value) p.value[b] = (float)Sv;
            if (p.grad_gap) p.grad_gap[b] = (float)tgap;
            if (p.grad_T) p.grad_T[b] = (float)tent;
        }
    } else if (p.dot_out) {
        const double t = block_sum(sdot, red);
        if (threadIdx.x == 0) p.dot_out[b] = (float)t;
    }
}

}  // namespace nw

// ------------------------------------------------------------------ host side
static size_t a256(size_t x) { return (x + 255) & ~(size_t)255; }

// value + marginals: the engine's planes or the strip kernel's workspace,
// whichever is larger, then the strip kernel's flags and CTA order (B ints each)
static size_t nw_fb_area(int B, int L1, int L2) {
    size_t n = a256(nw::per_problem_bytes(L1, L2, MODE_MARG) * (size_t)(B > 0 ? B : 1));
    const size_t sf = lin_strip_workspace_bytes(B, L1, L2);
    return n > sf ? n : a256(sf);
}

// the area the engine and the wavefront tangent passes share
static size_t nw_tan_area(int B, int L1, int L2) {
    const size_t nb = (size_t)(B > 0 ? B : 1);
    const size_t e = a256(nw::per_problem_bytes(L1, L2, MODE_PT) * nb), w = nw_wave_tan_area(B, L1, L2);
    return e > w ? e : w;
}

// tangent ops: [shared area][partials (backward_full)][a flag per problem]
size_t nw_workspace_bytes(int op, int B, int L1, int L2) {
    const size_t nb = (size_t)(B > 0 ? B : 1);
    if (op == D2P_OP_FORWARD_BACKWARD) return nw_fb_area(B, L1, L2) + 2 * a256(nb * sizeof(int));
    size_t n = nw_tan_area(B, L1, L2);
    if (op == D2P_OP_BACKWARD_FULL) n += a256((size_t)2 * nb * sizeof(float));
    return n + a256(nb * sizeof(int));
}

// one tangent sweep: the wavefront form, then the engine for the problems it
// flags (all of them when the wavefront form does not take the shape)
static int nw_tan_sweep(SwArgs a, int* flags, cudaStream_t st) {
    int rc = (int)cudaMemsetAsync(flags, 0, (size_t)a.B * sizeof(int), st);
    if (rc) return rc;
    SwArgs w = a;
    w.redo = flags;
    rc = launch_nw_wave_tan(w, st);
    if (rc == 0) a.only = flags;
    else if (rc != -1) return rc;
    return launch_nw(a, st);
}

int launch_nw(const SwArgs& a, cudaStream_t st) {
    if (a.B == 0) return 0;
    static DeviceSetup setup;
    int dev = 0, sms = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return (int)e;
    int rc = device_setup(setup, dev, [] {
        const int cap = (int)nw::kMaxRingBytes;
        const void* ks[] = {(const void*)nw::nw_kernel<MODE_MARG>, (const void*)nw::nw_kernel<MODE_HVP>,
                            (const void*)nw::nw_kernel<MODE_PGAP>, (const void*)nw::nw_kernel<MODE_PT>};
        cudaError_t r = cudaSuccess;
        for (const void* k : ks)
            if (r == cudaSuccess) r = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, cap);
        return (int)r;
    }, &sms);
    if (rc) return rc;
    const size_t rb = nw::ring_bytes(a.L1, a.mode);
    const size_t smem = rb <= nw::kMaxRingBytes ? rb : 0;   // else the rings are the planes
    switch (a.mode) {
        case MODE_MARG: nw::nw_kernel<MODE_MARG><<<a.B, nw::kThreads, smem, st>>>(a); break;
        case MODE_HVP: nw::nw_kernel<MODE_HVP><<<a.B, nw::kThreads, smem, st>>>(a); break;
        case MODE_PGAP: nw::nw_kernel<MODE_PGAP><<<a.B, nw::kThreads, smem, st>>>(a); break;
        case MODE_PT: nw::nw_kernel<MODE_PT><<<a.B, nw::kThreads, smem, st>>>(a); break;
        default: return kErrInvalid;
    }
    return (int)cudaGetLastError();
}

}  // namespace d2pb

using namespace d2pb;

// ---------------------------------------------------------------- C ABI
extern "C" {

static bool nw_dims_ok(int B, int L1, int L2) {
    if (B < 0 || L1 < 0 || L2 < 0) return false;
    return (long long)(L1 + 1) * (long long)(L2 + 1) <= 2147483647LL;
}

static SwArgs nw_args(const float* scores, const int* lengths, int B, int L1, int L2, float gap, float T,
                      void* ws) {
    SwArgs a{};
    a.scores = scores;
    a.lengths = lengths;
    a.B = B;
    a.L1 = L1;
    a.L2 = L2;
    a.gap = gap;
    a.temp = T;
    a.ws = (float*)ws;
    return a;
}

int d2p_nw_forward_backward(const float* scores, const int* lengths, int B, int L1, int L2, float gap,
                            float temperature, const float* gap_dev, const float* temperature_dev, float* value,
                            float* marginals, float* grad_gap, float* grad_temperature, void* workspace,
                            size_t workspace_bytes, void* stream) {
    if (!nw_dims_ok(B, L1, L2)) return D2P_ERR_TOO_LARGE;
    if (B == 0) return D2P_OK;
    if (!scores || !value || !marginals) return D2P_ERR_INVALID_ARGUMENT;
    if (!workspace || workspace_bytes < nw_workspace_bytes(D2P_OP_FORWARD_BACKWARD, B, L1, L2))
        return D2P_ERR_WORKSPACE_TOO_SMALL;
    SwArgs a = nw_args(scores, lengths, B, L1, L2, gap, temperature, workspace);
    a.gap_dev = gap_dev;
    a.temp_dev = temperature_dev;
    a.mode = MODE_MARG;
    a.value = value;
    a.out = marginals;
    a.grad_gap = grad_gap;
    a.grad_T = grad_temperature;
    cudaStream_t st = (cudaStream_t)stream;
    if (!grad_gap && !grad_temperature) {
        // value + marginals: the column-sweep strip kernel (problems of at most
        // 512 rows); the engine recomputes only the problems it flags
        const size_t area = nw_fb_area(B, L1, L2);
        int* flags = (int*)((char*)workspace + area);
        int* order = (int*)((char*)flags + a256((size_t)B * sizeof(int)));
        a.redo = flags;
        if (lengths) {
            const int ro = launch_lin_order(lengths, B, L1, L2, order, st);
            if (ro == D2P_OK) a.order = order;
            else if (ro != -1) return ro;
        }
        const int rc = launch_lin_strip(a, area, st, true);
        a.order = nullptr;
        a.redo = nullptr;
        if (rc == D2P_OK) {
            a.only = flags;
            return launch_nw(a, st);
        }
        if (rc != -1) return rc;
    }
    return launch_nw(a, st);
}

int d2p_nw_hvp(const float* scores, const float* tangent, const int* lengths, int B, int L1, int L2, float gap,
               float temperature, float* hvp, void* workspace, size_t workspace_bytes, void* stream) {
    if (!nw_dims_ok(B, L1, L2)) return D2P_ERR_TOO_LARGE;
    if (B == 0) return D2P_OK;
    if (!scores || !tangent || !hvp) return D2P_ERR_INVALID_ARGUMENT;
    if (!workspace || workspace_bytes < nw_workspace_bytes(D2P_OP_HVP, B, L1, L2)) return D2P_ERR_WORKSPACE_TOO_SMALL;
    SwArgs a = nw_args(scores, lengths, B, L1, L2, gap, temperature, workspace);
    a.mode = MODE_HVP;
    a.tangent = tangent;
    a.out = hvp;
    int* flags = (int*)((char*)workspace + nw_tan_area(B, L1, L2));
    return nw_tan_sweep(a, flags, (cudaStream_t)stream);
}

int d2p_nw_param_jacobian(const float* scores, const int* lengths, int B, int L1, int L2, int param_type,
                          float gap, float temperature, float* jacobian, void* workspace,
                          size_t workspace_bytes, void* stream) {
    if (!nw_dims_ok(B, L1, L2)) return D2P_ERR_TOO_LARGE;
    if (param_type != 0 && param_type != 1) return D2P_ERR_INVALID_ARGUMENT;
    if (B == 0) return D2P_OK;
    if (!scores || !jacobian) return D2P_ERR_INVALID_ARGUMENT;
    if (!workspace || workspace_bytes < nw_workspace_bytes(D2P_OP_PARAM_JACOBIAN, B, L1, L2))
        return D2P_ERR_WORKSPACE_TOO_SMALL;
    SwArgs a = nw_args(scores, lengths, B, L1, L2, gap, temperature, workspace);
    a.mode = param_type == 0 ? MODE_PGAP : MODE_PT;
    a.out = jacobian;
    int* flags = (int*)((char*)workspace + nw_tan_area(B, L1, L2));
    return nw_tan_sweep(a, flags, (cudaStream_t)stream);
}

int d2p_nw_backward_full(const float* scores, const float* grad_marginals, const int* lengths, int B, int L1,
                         int L2, float gap, float temperature, float* grad_scores, float* grad_gap,
                         float* grad_temperature, void* workspace, size_t workspace_bytes, void* stream) {
    if (!nw_dims_ok(B, L1, L2)) return D2P_ERR_TOO_LARGE;
    if (!grad_scores || !grad_gap || !grad_temperature) return D2P_ERR_INVALID_ARGUMENT;
    cudaStream_t st = (cudaStream_t)stream;
    if (B == 0) {
        cudaError_t e1 = cudaMemsetAsync(grad_gap, 0, sizeof(float), st);
        cudaError_t e2 = cudaMemsetAsync(grad_temperature, 0, sizeof(float), st);
        return (int)(e1 != cudaSuccess ? e1 : e2);
    }
    if (!scores || !grad_marginals) return D2P_ERR_INVALID_ARGUMENT;
    if (!workspace || workspace_bytes < nw_workspace_bytes(D2P_OP_BACKWARD_FULL, B, L1, L2))
        return D2P_ERR_WORKSPACE_TOO_SMALL;
    // grad_scores = H . grad_marginals (the Hessian of S is symmetric);
    // grad_gap / grad_T = sum grad_marginals * dP/dgap, dP/dT
    const size_t area = nw_tan_area(B, L1, L2);
    float* partials = (float*)((char*)workspace + area);
    int* flags = (int*)((char*)workspace + area + a256((size_t)2 * B * sizeof(float)));
    SwArgs a = nw_args(scores, lengths, B, L1, L2, gap, temperature, workspace);
    a.mode = MODE_HVP;
    a.tangent = grad_marginals;
    a.out = grad_scores;
    int rc = nw_tan_sweep(a, flags, st);
    if (rc) return rc;
    a.tangent = nullptr;
    a.out = nullptr;
    a.dot_with = grad_marginals;
    const int modes[2] = {MODE_PGAP, MODE_PT};
    float* outs[2] = {grad_gap, grad_temperature};
    for (int q = 0; q < 2; ++q) {
        a.mode = modes[q];
        a.dot_out = partials + (size_t)q * B;
        rc = nw_tan_sweep(a, flags, st);
        if (rc) return rc;
        rc = launch_sum_batches(partials + (size_t)q * B, 1, B, outs[q], 0, st);
        if (rc) return rc;
    }
    return D2P_OK;
}

}  // extern "C"
