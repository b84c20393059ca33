// sw_dtw.cu -- soft dynamic time warping with an optional Sakoe-Chiba band:
// value, alignment marginals, dS/dT, the Hessian-vector product, the
// temperature Jacobian dP/dT, and its contraction with a weight plane
// (backward_full).
//
// Recurrence (src/dtw/kernels_cpu.cpp:58-128 restated, natural units):
//   alpha[0,0] = 0, every other cell +inf until reached;
//   alpha[i,j] = c_ij + softmin_T(alpha[i-1,j-1], alpha[i-1,j], alpha[i,j-1])
//   for cells inside the band (|j - i L2 / L1| <= bandwidth, in the
//   reference's float arithmetic; bandwidth < 0: no band); S = alpha[L1, L2]
//   (+inf, the sentinel 1e30, when one sequence is empty).
// softmin_T(v) = m - T ln sum exp((m - v_k) / T), m = min v, with normalised
// weights w_k.  The reverse is the flow of the path distribution: beta[L1,L2] =
// 1 and beta[c] = sum over the successors d of c of beta[d] w_c(d); the
// marginal of (i, j) is beta[i, j] itself (every visited cell pays its cost).
// dS/dT = -(the entropy of the path distribution): minus each visited cell's
// choice entropy -sum w ln w weighted by beta, a sum of non-negative terms
// (equal to the reference's sum beta (softmin - E[alpha]) / T).
//
// Tangents: the forward carries d alpha = V + sum w d alpha_k (along V) or
// -entropy + sum w u_k (along T); the reverse carries d beta with
// dw_c(d) = w_c(d) (E_d - t_c) / T, E_d = sum_k w_k(d) t_k (+ w_c(d) (a_c -
// E[a](d)) / T^2 along T); the output is d beta
// (src/dtw/kernels_cpu.cpp:236-534).
//
// Engine: one CTA per problem sweeps the anti-diagonals, threads striding
// over a diagonal's cells, one barrier per diagonal; per-cell values live in
// diagonal-major planes ([k][i]) in the workspace.  alpha and the forward
// tangent are stored relative to an integer frame per diagonal (taken from
// the diagonal's cell nearest the band's centre line), so options are formed
// from small values plus exact frame differences.  Gather-form reverse, no
// atomics; fp64 block sums.
#include <math.h>
#include <stddef.h>
#include <stdint.h>

#include "../../include/d2p_b200.h"
#include "sw_common.cuh"
#include "sw_internal.h"

namespace d2pb {
namespace dtw {

constexpr int kThreads = 256;
constexpr float kPInf = 1.0e30f;   // unreached cell, as the reference's sentinel
constexpr float kFin = 0.5e30f;    // values below this are reached

enum Plane : int { kA = 0, kWd, kWu, kWl, kB, kH, kF, kR, kNumPlanes };
__host__ __device__ inline size_t plane_floats(int L1m, int L2m) {
    return ((size_t)L1m + L2m + 1) * ((size_t)L1m + 1);
}
// MARG: alpha, weights, beta, entropy; tangents: + forward and reverse tangent
__host__ __device__ inline int planes_for(int mode) { return mode == MODE_MARG ? kH + 1 : kNumPlanes; }
__host__ __device__ inline size_t per_problem_bytes(int L1m, int L2m, int mode) {
    const size_t b = (plane_floats(L1m, L2m) * planes_for(mode) + 2 * ((size_t)L1m + L2m + 1)) * sizeof(float);
    return (b + 255) & ~(size_t)255;
}

struct Ctx {
    float* p[kNumPlanes];
    float* O;
    float* D;
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

// the reference's band test (src/dtw/kernels_cpu.cpp:23-29), float arithmetic
__device__ __forceinline__ bool in_band(int i, int j, int L1, int L2, int bw) {
    if (bw < 0 || L1 == 0 || L2 == 0) return true;
    const float e = (float)((long long)i * L2) / (float)L1;
    return fabsf((float)j - e) <= (float)bw;
}

// Rings: the last three diagonals of alpha (and the forward tangent) during
// the forward, and of beta (and the reverse tangent) during the reverse, sit
// in shared memory ([3][L1m + 1] floats each) when they fit, so the sweep reads
// its neighbours at shared-memory latency; the planes in the workspace still
// receive what the reverse reads back (weights, entropies; for the tangent
// modes alpha and the forward tangent).  When the rings do not fit, each ring is its
// quantity's plane.  The global loads of a diagonal (costs, direction, the
// successors' weights) are issued one diagonal ahead, before the barrier.
constexpr int kPF = 2;                          // cells per thread prefetched (diagonals of <= 512 cells)
constexpr size_t kMaxRingBytes = 200 * 1024;    // dynamic shared memory cap of the rings
__host__ __device__ inline int rings_for(int mode) { return mode == MODE_MARG ? 2 : 4; }
__host__ __device__ inline size_t ring_bytes(int L1m, int mode) {
    return (size_t)rings_for(mode) * 3 * ((size_t)L1m + 1) * sizeof(float);
}

// One CTA per problem.  MODE: MODE_MARG (value, marginals, dS/dT), MODE_HVP
// (out = d marginals along p.tangent), MODE_PT (out = dP/dT; with dot_with,
// dot_out[b] = sum dot_with * dP/dT).  p.gap2 carries nothing; the band is
// p.parts (an int, < 0 for none).
template <int MODE>
__global__ void __launch_bounds__(kThreads) dtw_kernel(SwArgs p) {
    extern __shared__ float ring_smem[];
    __shared__ double red[32];
    const int b = blockIdx.x;
    if (p.only && !p.only[b]) return;   // a fix-up launch: only the problems the wavefront kernel flagged
    const int L1m = p.L1, L2m = p.L2;
    const int L1 = p.lengths ? min(max(p.lengths[2 * b], 0), L1m) : L1m;
    const int L2 = p.lengths ? min(max(p.lengths[2 * b + 1], 0), L2m) : L2m;
    const int bw = p.parts;
    const float T = p.temp_dev ? __ldg(p.temp_dev) : p.temp;
    const float iT = 1.f / T;
    const size_t plane = (size_t)L1m * L2m;
    const float* __restrict__ Cst = p.scores + (size_t)b * plane;
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
    const int K = L1 + L2;
    const int tid = threadIdx.x;
    // rings in shared memory (the launch gives them their bytes) or in the planes
    const bool smR = ring_bytes(L1m, MODE) <= kMaxRingBytes;
    const int S = L1m + 1;
    float* const rgA = ring_smem;
    float* const rgB = ring_smem + 3 * S;
    float* const rgF = ring_smem + 6 * S;   // TAN only
    float* const rgR = ring_smem + 9 * S;   // TAN only
    auto row = [&](float* rg, int pl, int k) -> float* {
        return smR ? rg + (k % 3) * S : C.p[pl] + (size_t)k * C.stride;
    };

    if (out && (L1 < L1m || L2 < L2m)) {   // zeros outside the problem
        for (int i = 0; i < L1m; ++i)
            for (int j = (i < L1 ? L2 : 0) + (int)threadIdx.x; j < L2m; j += blockDim.x) out[(size_t)i * L2m + j] = 0.f;
    }

    // ------------------------------------------------------------- forward
    // costs (and direction) of this thread's first kPF cells of diagonal k
    float pc[kPF], pv[kPF];
    auto fetch_fwd = [&](int k, float* c, float* v) {
        const int i0 = max(0, k - L2), i1 = min(L1, k);
#pragma unroll
        for (int r = 0; r < kPF; ++r) {
            const int i = i0 + tid + r * kThreads, j = k - i;
            const bool ok = i <= i1 && i >= 1 && j >= 1;
            const size_t si = ok ? (size_t)(i - 1) * L2m + (j - 1) : 0;
            c[r] = ok ? __ldg(Cst + si) : 0.f;
            if (MODE == MODE_HVP) v[r] = ok ? __ldg(V + si) : 0.f;
        }
    };
    fetch_fwd(0, pc, pv);
    float O1 = 0.f, O2 = 0.f, D1 = 0.f, D2 = 0.f;
    for (int k = 0; k <= K; ++k) {
        float* const a0 = row(rgA, kA, k);
        const float* const a1 = row(rgA, kA, max(k - 1, 0));
        const float* const a2 = row(rgA, kA, max(k - 2, 0));
        float* const f0 = TAN ? row(rgF, kF, k) : nullptr;
        const float* const f1 = TAN ? row(rgF, kF, max(k - 1, 0)) : nullptr;
        const float* const f2 = TAN ? row(rgF, kF, max(k - 2, 0)) : nullptr;
        float Ok = O1, Dk = D1;
        if (k >= 2) {   // the previous diagonal's cell nearest the band's centre line
            const int lo = max(0, k - 1 - L2), hi = min(L1, k - 1);
            int im = K > 0 ? (int)(((long long)(k - 1) * L1 + K / 2) / K) : 0;
            im = min(max(im, lo), hi);
            const float a = a1[im];
            if (a < kFin) {
                Ok = O1 + rintf(a);
                if (TAN) Dk = D1 + rintf(f1[im]);
            }
        }
        if (tid == 0) {
            C.O[k] = Ok;
            C.D[k] = Dk;
        }
        const float dO1 = O1 - Ok, dO2 = O2 - Ok, dD1 = D1 - Dk, dD2 = D2 - Dk;   // exact
        const int i0 = max(0, k - L2), i1 = min(L1, k);
        auto cell = [&](int i, float cst, float vv) {
            const int j = k - i;
            float a = kPInf, wd = 0.f, wu = 0.f, wl = 0.f, h = 0.f, f = 0.f;
            if (k == 0) {
                a = 0.f;
            } else if (i >= 1 && j >= 1 && in_band(i, j, L1, L2, bw)) {
                const float vd = a2[i - 1] + dO2, vu = a1[i - 1] + dO1, vl = a1[i] + dO1;
                const float m = fminf(vd, fminf(vu, vl));
                if (m < kFin) {
                    const float ed = expf((m - vd) * iT), eu = expf((m - vu) * iT), el = expf((m - vl) * iT);
                    const float sum = (ed + eu) + el;
                    const float ls = logf(sum);
                    const float is = 1.f / sum;
                    wd = ed * is;
                    wu = eu * is;
                    wl = el * is;
                    a = cst + fmaf(-T, ls, m);
                    // the choice's entropy -sum w ln w = ln(sum) + sum w (v - m) / T
                    h = ls + iT * fmaf(wd, vd - m, fmaf(wu, vu - m, wl * (vl - m)));
                    if (TAN) {
                        f = fmaf(wd, f2[i - 1] + dD2, fmaf(wu, f1[i - 1] + dD1, wl * (f1[i] + dD1)));
                        if (MODE == MODE_HVP) f += vv;
                        if (MODE == MODE_PT) f -= h;
                    }
                }
            }
            const float as = a < kFin ? a : kPInf;
            a0[i] = as;
            if (smR && TAN) C.at(kA, k, i) = as;   // the tangent reverses read alpha back
            C.at(kWd, k, i) = wd;
            C.at(kWu, k, i) = wu;
            C.at(kWl, k, i) = wl;
            C.at(kH, k, i) = h;
            if (TAN) {
                f0[i] = f;
                if (smR) C.at(kF, k, i) = f;
            }
        };
#pragma unroll
        for (int r = 0; r < kPF; ++r) {
            const int i = i0 + tid + r * kThreads;
            if (i <= i1) cell(i, pc[r], pv[r]);
        }
        for (int i = i0 + tid + kPF * kThreads; i <= i1; i += kThreads) {
            const int j = k - i;
            const bool ok = i >= 1 && j >= 1;
            const size_t si = ok ? (size_t)(i - 1) * L2m + (j - 1) : 0;
            cell(i, ok ? __ldg(Cst + si) : 0.f, MODE == MODE_HVP && ok ? __ldg(V + si) : 0.f);
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
    const float aE = row(rgA, kA, K)[L1];   // read before any reverse write (separate rings)

    // ------------------------------------------------------------- reverse
    // this thread's first kPF cells of diagonal k: entropy and the three
    // weights its successors give it (MODE_MARG)
    float ph[kPF], pd[kPF], pu[kPF], pl[kPF];
    auto fetch_rev = [&](int k, float* h, float* wd, float* wu, float* wl) {
        const int i0 = max(0, k - L2), i1 = min(L1, k);
#pragma unroll
        for (int r = 0; r < kPF; ++r) {
            const int i = i0 + tid + r * kThreads, j = k - i;
            const bool ok = i <= i1;
            h[r] = ok && i >= 1 && j >= 1 ? C.at(kH, k, i) : 0.f;
            wd[r] = ok && i + 1 <= L1 && j + 1 <= L2 ? C.at(kWd, k + 2, i + 1) : 0.f;
            wu[r] = ok && i + 1 <= L1 && j >= 1 ? C.at(kWu, k + 1, i + 1) : 0.f;
            wl[r] = ok && j + 1 <= L2 && i >= 1 ? C.at(kWl, k + 1, i) : 0.f;
        }
    };
    if (MODE == MODE_MARG) fetch_rev(K, ph, pd, pu, pl);
    double sent = 0.0, sdot = 0.0;
    for (int k = K; k >= 0; --k) {
        const float Ok = C.O[k], Dk = C.D[k];
        const float Ok1 = k + 1 <= K ? C.O[k + 1] : 0.f, Ok2 = k + 2 <= K ? C.O[k + 2] : 0.f;
        const float Dk1 = k + 1 <= K ? C.D[k + 1] : 0.f, Dk2 = k + 2 <= K ? C.D[k + 2] : 0.f;
        float* const b0 = row(rgB, kB, k);
        const float* const b1 = row(rgB, kB, min(k + 1, K));
        const float* const b2 = row(rgB, kB, min(k + 2, K));
        float* const r0 = TAN ? row(rgR, kR, k) : nullptr;
        const float* const r1 = TAN ? row(rgR, kR, min(k + 1, K)) : nullptr;
        const float* const r2 = TAN ? row(rgR, kR, min(k + 2, K)) : nullptr;
        const int i0 = max(0, k - L2), i1 = min(L1, k);
        if (MODE == MODE_MARG) {
            // An unreached cell gets weight 0 from each successor, so its flow
            // is 0 without a test; the end cell keeps its 1, as in the reference.
            auto cell = [&](int i, float h, float wd, float wu, float wl) {
                const int j = k - i;
                float be = k == K ? 1.f : 0.f;
                if (i + 1 <= L1 && j + 1 <= L2) be = fmaf(b2[i + 1], wd, be);
                if (i + 1 <= L1 && j >= 1) be = fmaf(b1[i + 1], wu, be);
                if (j + 1 <= L2 && i >= 1) be = fmaf(b1[i], wl, be);
                b0[i] = be;
                if (i >= 1 && j >= 1) {
                    if (out) out[(size_t)(i - 1) * L2m + (j - 1)] = be;
                    sent += (double)be * (double)h;
                }
            };
#pragma unroll
            for (int r = 0; r < kPF; ++r) {
                const int i = i0 + tid + r * kThreads;
                if (i <= i1) cell(i, ph[r], pd[r], pu[r], pl[r]);
            }
            for (int i = i0 + tid + kPF * kThreads; i <= i1; i += kThreads) {
                const int j = k - i;
                cell(i, i >= 1 && j >= 1 ? C.at(kH, k, i) : 0.f,
                     i + 1 <= L1 && j + 1 <= L2 ? C.at(kWd, k + 2, i + 1) : 0.f,
                     i + 1 <= L1 && j >= 1 ? C.at(kWu, k + 1, i + 1) : 0.f,
                     j + 1 <= L2 && i >= 1 ? C.at(kWl, k + 1, i) : 0.f);
            }
            if (k > 0) {
                float nh[kPF], nd[kPF], nu[kPF], nl[kPF];
                fetch_rev(k - 1, nh, nd, nu, nl);
                __syncthreads();
#pragma unroll
                for (int r = 0; r < kPF; ++r) {
                    ph[r] = nh[r];
                    pd[r] = nd[r];
                    pu[r] = nu[r];
                    pl[r] = nl[r];
                }
            } else {
                __syncthreads();
            }
        } else {
        for (int i = i0 + tid; i <= i1; i += blockDim.x) {
            const int j = k - i;
            float be = k == K ? 1.f : 0.f, tb = 0.f;
            const float tc = C.at(kF, k, i);
            const float ac = C.at(kA, k, i);
            // successor d of this cell by its option with weight plane pw;
            // dO, dD: the successor's frames minus this cell's (exact)
            auto take = [&](int kd, int id, int pw, float dO, float dD) {
                const float bd = (kd == k + 1 ? b1 : b2)[id];
                const float w = C.at(pw, kd, id);
                be = fmaf(bd, w, be);
                const size_t sd = (size_t)(id - 1) * L2m + (kd - id - 1);
                // E_d - t_c: the successor's options' mean tangent minus this cell's
                float g = C.at(kF, kd, id) - tc + dD;
                if (MODE == MODE_HVP) g -= V[sd];
                float dw;
                if (MODE == MODE_PT) {
                    const float hd = C.at(kH, kd, id);
                    // a_c - E[a](d) = a_c - (alpha_d - c_d) - T h_d
                    const float da = (ac - C.at(kA, kd, id)) + (Cst[sd] - dO) - T * hd;
                    dw = w * fmaf(g + hd, iT, da * iT * iT);
                } else {
                    dw = w * g * iT;
                }
                tb = fmaf((kd == k + 1 ? r1 : r2)[id], w, fmaf(bd, dw, tb));
            };
            // an unreached cell takes no flow (its successors give it weight 0);
            // the end cell keeps its 1 even when unreached, as in the reference
            if (ac < kFin) {
                if (i + 1 <= L1 && j + 1 <= L2) take(k + 2, i + 1, kWd, Ok2 - Ok, Dk2 - Dk);
                if (i + 1 <= L1 && j >= 1) take(k + 1, i + 1, kWu, Ok1 - Ok, Dk1 - Dk);
                if (j + 1 <= L2 && i >= 1) take(k + 1, i, kWl, Ok1 - Ok, Dk1 - Dk);
            }
            b0[i] = be;
            r0[i] = tb;
            if (i >= 1 && j >= 1) {
                const size_t si = (size_t)(i - 1) * L2m + (j - 1);
                if (out) out[si] = tb;
                if (Gw) sdot += (double)Gw[si] * (double)tb;
            }
        }
        __syncthreads();
        }
    }

    if (MODE == MODE_MARG) {
        const double th = block_sum(sent, red);
        if (tid == 0) {
            if (p.value) p.value[b] = aE < kFin ? (float)((double)aE + (double)C.O[K]) : kPInf;
            if (p.grad_T) p.grad_T[b] = (float)(-th);
        }
    } else if (p.dot_out) {
        const double t = block_sum(sdot, red);
        if (tid == 0) p.dot_out[b] = (float)t;
    }
}

}  // namespace dtw

// ------------------------------------------------------------------ host side
// the area the engine and the wavefront passes of one operator share
static size_t dtw_area(int op, int B, int L1, int L2) {
    const size_t fb = dtw::per_problem_bytes(L1, L2, op == D2P_OP_FORWARD_BACKWARD ? MODE_MARG : MODE_PT);
    size_t n = (fb * (size_t)(B > 0 ? B : 1) + 255) & ~(size_t)255;
    size_t w = 0;
    if (op == D2P_OP_FORWARD_BACKWARD) w = dtw_wave_area(B, L1, L2);
    if (op != D2P_OP_FORWARD_BACKWARD) w = dtw_wave_tan_area(B, L1, L2);
    return w > n ? w : n;
}
static size_t dtw_vec_bytes(int B) { return ((size_t)(B > 0 ? B : 1) * 4 + 255) & ~(size_t)255; }

// [shared area][partials (backward_full)][a flag per problem (wavefront passes)]
size_t dtw_workspace_bytes(int op, int B, int L1, int L2) {
    size_t n = dtw_area(op, B, L1, L2);
    if (op == D2P_OP_BACKWARD_FULL) n += dtw_vec_bytes(B);
    return n + dtw_vec_bytes(B);
}

static int launch_dtw(const SwArgs& a, cudaStream_t st) {
    if (a.B == 0) return 0;
    static DeviceSetup setup;
    int dev = 0, sms = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return (int)e;
    int rc = device_setup(setup, dev, [] {
        const int cap = (int)dtw::kMaxRingBytes;
        cudaError_t r = cudaFuncSetAttribute(dtw::dtw_kernel<MODE_MARG>, cudaFuncAttributeMaxDynamicSharedMemorySize, cap);
        if (r == cudaSuccess)
            r = cudaFuncSetAttribute(dtw::dtw_kernel<MODE_HVP>, cudaFuncAttributeMaxDynamicSharedMemorySize, cap);
        if (r == cudaSuccess)
            r = cudaFuncSetAttribute(dtw::dtw_kernel<MODE_PT>, cudaFuncAttributeMaxDynamicSharedMemorySize, cap);
        return (int)r;
    }, &sms);
    if (rc) return rc;
    const size_t rb = dtw::ring_bytes(a.L1, a.mode);
    const size_t smem = rb <= dtw::kMaxRingBytes ? rb : 0;   // else the rings are the planes
    switch (a.mode) {
        case MODE_MARG: dtw::dtw_kernel<MODE_MARG><<<a.B, dtw::kThreads, smem, st>>>(a); break;
        case MODE_HVP: dtw::dtw_kernel<MODE_HVP><<<a.B, dtw::kThreads, smem, st>>>(a); break;
        case MODE_PT: dtw::dtw_kernel<MODE_PT><<<a.B, dtw::kThreads, smem, st>>>(a); break;
        default: return kErrInvalid;
    }
    return (int)cudaGetLastError();
}

}  // namespace d2pb

using namespace d2pb;

// ---------------------------------------------------------------- C ABI
extern "C" {

static bool dtw_dims_ok(int B, int L1, int L2) {
    if (B < 0 || L1 < 0 || L2 < 0) return false;
    return (long long)(L1 + 1) * (long long)(L2 + 1) <= 2147483647LL;
}

static SwArgs dtw_args(const float* costs, const int* lengths, int B, int L1, int L2, float T, int bandwidth,
                       void* ws) {
    SwArgs a{};
    a.scores = costs;
    a.lengths = lengths;
    a.B = B;
    a.L1 = L1;
    a.L2 = L2;
    a.temp = T;
    a.parts = bandwidth < 0 ? -1 : bandwidth;
    a.ws = (float*)ws;
    return a;
}

int d2p_dtw_forward_backward(const float* costs, const int* lengths, int B, int L1, int L2, float temperature,
                             const float* temperature_dev, int bandwidth, float* value, float* marginals,
                             float* grad_temperature, void* workspace, size_t workspace_bytes, void* stream) {
    if (!dtw_dims_ok(B, L1, L2)) return D2P_ERR_TOO_LARGE;
    if (B == 0) return D2P_OK;
    if (!costs || !value || !marginals) return D2P_ERR_INVALID_ARGUMENT;
    if (!workspace || workspace_bytes < dtw_workspace_bytes(D2P_OP_FORWARD_BACKWARD, B, L1, L2))
        return D2P_ERR_WORKSPACE_TOO_SMALL;
    SwArgs a = dtw_args(costs, lengths, B, L1, L2, temperature, bandwidth, workspace);
    a.temp_dev = temperature_dev;
    a.mode = MODE_MARG;
    a.value = value;
    a.out = marginals;
    a.grad_T = grad_temperature;
    cudaStream_t st = (cudaStream_t)stream;
    // the wavefront pass; the engine recomputes the problems it flags
    int* flags = (int*)((char*)workspace + dtw_area(D2P_OP_FORWARD_BACKWARD, B, L1, L2));
    int rc = (int)cudaMemsetAsync(flags, 0, (size_t)B * sizeof(int), st);
    if (rc) return rc;
    SwArgs w = a;
    w.redo = flags;
    rc = launch_dtw_wave(w, st);
    if (rc == 0) a.only = flags;
    else if (rc != -1) return rc;
    return launch_dtw(a, st);
}

int d2p_dtw_hvp(const float* costs, const float* tangent, const int* lengths, int B, int L1, int L2,
                float temperature, int bandwidth, float* hvp, void* workspace, size_t workspace_bytes,
                void* stream) {
    if (!dtw_dims_ok(B, L1, L2)) return D2P_ERR_TOO_LARGE;
    if (B == 0) return D2P_OK;
    if (!costs || !tangent || !hvp) return D2P_ERR_INVALID_ARGUMENT;
    if (!workspace || workspace_bytes < dtw_workspace_bytes(D2P_OP_HVP, B, L1, L2)) return D2P_ERR_WORKSPACE_TOO_SMALL;
    SwArgs a = dtw_args(costs, lengths, B, L1, L2, temperature, bandwidth, workspace);
    a.mode = MODE_HVP;
    a.tangent = tangent;
    a.out = hvp;
    cudaStream_t st = (cudaStream_t)stream;
    // the wavefront pass; the engine recomputes the problems it flags
    int* flags = (int*)((char*)workspace + dtw_area(D2P_OP_HVP, B, L1, L2));
    int rc = (int)cudaMemsetAsync(flags, 0, (size_t)B * sizeof(int), st);
    if (rc) return rc;
    SwArgs w = a;
    w.redo = flags;
    rc = launch_dtw_wave_tan(w, st);
    if (rc == 0) a.only = flags;
    else if (rc != -1) return rc;
    return launch_dtw(a, st);
}

int d2p_dtw_param_jacobian(const float* costs, const int* lengths, int B, int L1, int L2, float temperature,
                           int bandwidth, float* jacobian, void* workspace, size_t workspace_bytes, void* stream) {
    if (!dtw_dims_ok(B, L1, L2)) return D2P_ERR_TOO_LARGE;
    if (B == 0) return D2P_OK;
    if (!costs || !jacobian) return D2P_ERR_INVALID_ARGUMENT;
    if (!workspace || workspace_bytes < dtw_workspace_bytes(D2P_OP_PARAM_JACOBIAN, B, L1, L2))
        return D2P_ERR_WORKSPACE_TOO_SMALL;
    SwArgs a = dtw_args(costs, lengths, B, L1, L2, temperature, bandwidth, workspace);
    a.mode = MODE_PT;
    a.out = jacobian;
    cudaStream_t st = (cudaStream_t)stream;
    // the wavefront pass; the engine recomputes the problems it flags
    int* flags = (int*)((char*)workspace + dtw_area(D2P_OP_PARAM_JACOBIAN, B, L1, L2));
    int rc = (int)cudaMemsetAsync(flags, 0, (size_t)B * sizeof(int), st);
    if (rc) return rc;
    SwArgs w = a;
    w.redo = flags;
    rc = launch_dtw_wave_tan(w, st);
    if (rc == 0) a.only = flags;
    else if (rc != -1) return rc;
    return launch_dtw(a, st);
}

int d2p_dtw_backward_full(const float* costs, const float* grad_marginals, const int* lengths, int B, int L1, int L2,
                          float temperature, int bandwidth, float* grad_costs, float* grad_temperature,
                          void* workspace, size_t workspace_bytes, void* stream) {
    if (!dtw_dims_ok(B, L1, L2)) return D2P_ERR_TOO_LARGE;
    if (!grad_costs || !grad_temperature) return D2P_ERR_INVALID_ARGUMENT;
    cudaStream_t st = (cudaStream_t)stream;
    if (B == 0) return (int)cudaMemsetAsync(grad_temperature, 0, sizeof(float), st);
    if (!costs || !grad_marginals) return D2P_ERR_INVALID_ARGUMENT;
    if (!workspace || workspace_bytes < dtw_workspace_bytes(D2P_OP_BACKWARD_FULL, B, L1, L2))
        return D2P_ERR_WORKSPACE_TOO_SMALL;
    // grad_costs = H . grad_marginals (the Hessian of S is symmetric); grad_T
    // = sum grad_marginals * dP/dT: two wavefront sweeps, the engine for the
    // problems they flag
    const size_t area = dtw_area(D2P_OP_BACKWARD_FULL, B, L1, L2);
    float* partials = (float*)((char*)workspace + area);
    int* flags = (int*)((char*)workspace + area + dtw_vec_bytes(B));
    SwArgs a = dtw_args(costs, lengths, B, L1, L2, temperature, bandwidth, workspace);
    a.mode = MODE_HVP;
    a.tangent = grad_marginals;
    a.out = grad_costs;
    int rc = (int)cudaMemsetAsync(flags, 0, (size_t)B * sizeof(int), st);
    if (rc) return rc;
    SwArgs w = a;
    w.redo = flags;
    rc = launch_dtw_wave_tan(w, st);
    if (rc == 0) a.only = flags;
    else if (rc != -1) return rc;
    rc = launch_dtw(a, st);
    if (rc) return rc;
    a.tangent = nullptr;
    a.out = nullptr;
    a.dot_with = grad_marginals;
    a.mode = MODE_PT;
    a.dot_out = partials;
    w = a;
    w.only = nullptr;
    w.redo = flags;
    rc = launch_dtw_wave_tan(w, st);
    if (rc == 0) a.only = flags;
    else if (rc != -1) return rc;
    else a.only = nullptr;
    rc = launch_dtw(a, st);
    if (rc) return rc;
    return launch_sum_batches(partials, 1, B, grad_temperature, 0, st);
}

}  // extern "C"
