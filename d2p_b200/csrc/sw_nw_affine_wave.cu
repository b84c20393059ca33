// sw_nw_affine_wave.cu -- soft Needleman-Wunsch with affine gaps: value,
// marginals, dS/d(gap_open), dS/d(gap_ext) and dS/dT in row-block wavefront
// form, the value pass behind soft_nw_affine when no tangent is wanted (same
// recurrence and outputs as nwa_kernel<MODE_MARG> in sw_nw_affine.cu,
// src/nw_affine/kernels_cpu.cpp:101-360 restated).
//
// Sweep (as in sw_dtw_wave.cu).  One CTA per problem, kW warps; warp w takes
// row-blocks w, w + kW, ... (lane l = row 32 rb + l + 1) and sweeps steps t;
// at step t lane l works on column j = t - l + 1, carrying the three states
// M, I, D of its cell:
//   M(i,j) = s_ij + LSE_T(M, I, D at (i-1, j-1)),
//   I(i,j) = LSE_T(M + open, I + ext, D + open at (i-1, j)),
//   D(i,j) = LSE_T(M + open, I + open, D + ext at (i, j-1)).
// Up (three shuffles) and diagonal (the up of the step before) come from lane
// l-1, left from the lane's own registers; lane 0 reads the row above from an
// L2-resident boundary row (three states and their frame per column) that
// the warp above writes with lane 31, behind a release / acquire progress
// word.  Row 0 and column 0 (M(0,0) = 0, I(i,0) = open + (i-1) ext, D(0,j) =
// open + (j-1) ext, every other boundary state absent) are formed where they
// are read.
//
// Reverse (gather form, bottom row-block first, steps t = L2 + 30 .. -1).  A
// state's beta is the end cell's final weight (at (L1, L2)) plus the flows of
// the successor states that take it: D(i, j+1) (the lane's own previous step,
// kept in registers), I(i+1, j) and M(i+1, j+1) (lane l+1's up flows of the
// previous step plus its diagonal flows of the step before, three shuffles).
// The extra step t = -1 brings every lane to its column-0 cell, whose I state
// takes the leading gap: dS/dopen += beta_I, dS/dext += beta_I (i - 1); row
// 0's D states take their flows from row-block 0's lane 0 in the same way.
// Per cell: marginal = beta_M; dS/dopen and dS/dext sum the flows through
// opening and extending options; dS/dT sums each state's choice entropy
// weighted by its beta, plus the final choice's.
//
// Numerics: an integer frame per step of a row-block, advanced by rint of the
// largest state at the anchor lane (lane 16, or the nearest live one);
// boundary rows carry their frame.  The reverse multiplies probabilities
// only.
//
// Memory.  The forward writes per cell three float4 (w_M1..3 with h_M, w_I..
// with h_I, w_D.. with h_D) in the layout [row-block][step][lane] and reads
// the scores through a per-warp ring [32][64] filled by 4-byte cp.async; the
// reverse reads the float4s back 2 steps ahead and stages the marginals in
// the ring.  HBM per cell: score 4 B, 48 B written and read, marginal 4 B.
//
// A problem whose wait gave up, or with an empty sequence, is flagged in
// p.redo; the caller recomputes flagged problems with nwa_kernel.
#include <math.h>
#include <stddef.h>
#include <stdint.h>

#include "../../include/d2p_b200.h"
#include "sw_common.cuh"
#include "sw_internal.h"
#include "sw_ring.cuh"

namespace d2pb {
namespace nwaw {

using ring::cp_async4_zfill;
using ring::kAll;

constexpr int kW = 8;                 // warps per CTA
constexpr int kThreads = 32 * kW;
constexpr int kCW = 16;               // columns per stage / ring chunk
constexpr int kRW = 64;               // ring width (columns)
constexpr int kPD = 2;                // reverse: steps of weights loaded ahead
constexpr int kMaxL1 = 8192;          // rows per problem (256 row-blocks)
constexpr int kMaxL2 = 1000000;       // columns (stage counts fit the progress word's 16 bits)
constexpr float kNInf = -1.0e30f;     // absent state
constexpr float kLow = -0.5e30f;      // values above this are present

struct WarpSmem {
    float ring[32 * kRW];             // forward: scores; reverse: marginals before their store
    float4 bin[kCW];                  // forward: the stage's row above (M, I, D - frame, frame)
    float4 bbin[kCW];                 // reverse: the stage's flows from the row below (M, I, D)
};
struct CtaSmem {
    WarpSmem w[kW];
    int progF[kW], progR[kW];         // (row-block key << 16) | stages done, per warp
    int err;
    double red[3][kW];
    double val;                       // S
    float fw[3], fh;                  // the final choice's weights and entropy
};

__host__ __device__ inline int nrb_of(int L1m) { return (L1m + 31) / 32; }
__host__ __device__ inline int steps_of(int L2m) { return (L2m + 31 + kCW - 1) / kCW * kCW; }
__host__ __device__ inline size_t slots_of(int L1m, int L2m) { return (size_t)nrb_of(L1m) * steps_of(L2m) * 32; }
__host__ __device__ inline size_t row_elems(int L2m) { return (size_t)L2m + kCW + 1; }
__host__ __device__ inline size_t per_problem_bytes(int L1m, int L2m) {
    const size_t nr = (size_t)nrb_of(L1m) * row_elems(L2m);
    return ring::align_up(3 * slots_of(L1m, L2m) * sizeof(float4), 256) + 2 * ring::align_up(nr * sizeof(float4), 256);
}

// normalised weights of three options; returns the LSE (m + T ln sum), and
// through h the choice's entropy -sum w ln w = ln(sum) + sum w (m - v) / T
__device__ __forceinline__ float lse3(float v1, float v2, float v3, float T, float iT, float& w1, float& w2,
                                      float& w3, float& h) {
    const float m = fmaxf(v1, fmaxf(v2, v3));
    const float e1 = expf((v1 - m) * iT), e2 = expf((v2 - m) * iT), e3 = expf((v3 - m) * iT);
    const float sum = (e1 + e2) + e3;
    const float ls = logf(sum);
    const float is = 1.f / sum;
    w1 = e1 * is;
    w2 = e2 * is;
    w3 = e3 * is;
    h = ls + iT * fmaf(w1, m - v1, fmaf(w2, m - v2, w3 * (m - v3)));
    return fmaf(T, ls, m);
}

__device__ __forceinline__ float rel(float v, float shift) { return v > kLow ? v + shift : kNInf; }

__global__ void __launch_bounds__(kThreads, 2) nwa_wave_kernel(SwArgs p) {
    extern __shared__ __align__(16) unsigned char smem_raw[];
    CtaSmem& sm = *reinterpret_cast<CtaSmem*>(smem_raw);
    const int b = blockIdx.x;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int L1m = p.L1, L2m = p.L2;
    const int L1 = p.lengths ? min(max(p.lengths[2 * b], 0), L1m) : L1m;
    const int L2 = p.lengths ? min(max(p.lengths[2 * b + 1], 0), L2m) : L2m;
    if (L1 == 0 || L2 == 0) {   // the engine writes the boundary-only value and the zeros
        if (tid == 0) p.redo[b] = 1;
        return;
    }
    const float go = p.gap_dev ? __ldg(p.gap_dev) : p.gap;
    const float ge = p.gap2_dev ? __ldg(p.gap2_dev) : p.gap2;
    const float T = p.temp_dev ? __ldg(p.temp_dev) : p.temp;
    const float iT = 1.f / T;
    const size_t plane = (size_t)L1m * L2m;
    const float* __restrict__ Sc = p.scores + (size_t)b * plane;
    float* __restrict__ out = p.out + (size_t)b * plane;
    const int TP = steps_of(L2m);
    char* base = reinterpret_cast<char*>(p.ws) + (size_t)b * per_problem_bytes(L1m, L2m);
    const size_t ns = slots_of(L1m, L2m);
    float4* const PM = reinterpret_cast<float4*>(base);   // (w_M1, w_M2, w_M3, h_M) per cell
    float4* const PI = PM + ns;                            // (w_I1, w_I2, w_I3, h_I)
    float4* const PD = PI + ns;                            // (w_D1, w_D2, w_D3, h_D)
    const size_t nrb_bytes = ring::align_up((size_t)nrb_of(L1m) * row_elems(L2m) * sizeof(float4), 256);
    float4* const bnd = reinterpret_cast<float4*>(base + ring::align_up(3 * ns * sizeof(float4), 256));
    float4* const bbr = reinterpret_cast<float4*>(reinterpret_cast<char*>(bnd) + nrb_bytes);
    const int nRB = nrb_of(L1);
    const int nstF = (L2 + 31 + kCW - 1) / kCW;   // forward stages: t = 0 .. L2 + 30
    const int nstR = (L2 + 32 + kCW - 1) / kCW;   // reverse stages: t = L2 + 30 .. -1
    WarpSmem& ws = sm.w[warp];

    if (tid < kW) {
        sm.progF[tid] = -1;
        sm.progR[tid] = -1;
    }
    if (tid == 0) {
        sm.err = 0;
        sm.val = 0.0;
        sm.fw[0] = sm.fw[1] = sm.fw[2] = sm.fh = 0.f;
    }
    if (L1 < L1m || L2 < L2m) {   // zeros outside the problem
        for (int i = 0; i < L1m; ++i)
            for (int j = (i < L1 ? L2 : 0) + tid; j < L2m; j += kThreads) out[(size_t)i * L2m + j] = 0.f;
    }
    __syncthreads();

    // ------------------------------------------------------------- forward
    for (int rb = warp; rb < nRB; rb += kW) {
        const int i = 32 * rb + lane + 1;
        const bool rowok = i <= L1;
        const size_t poff = (size_t)rb * TP * 32 + lane;
        const int hiRow = min(31, L1 - 1 - 32 * rb);
        auto load_chunk = [&](int c) {
            const int col = c * kCW + (lane & 15);
            const bool cin = col < L2;
#pragma unroll 4
            for (int q = 0; q < 16; ++q) {
                const int r = (lane >> 4) + 2 * q;
                const bool ok = cin && 32 * rb + r < L1;
                const float* g = ok ? Sc + (size_t)(32 * rb + r) * L2m + col : Sc;
                cp_async4_zfill(&ws.ring[r * kRW + (col & (kRW - 1))], g, ok ? 4 : 0);
            }
            ring::cp_async_commit();
        };
        load_chunk(0);
        float pM = kNInf, pI = kNInf, pD = kNInf;      // own outputs of the previous step (rel O)
        float uM = kNInf, uI = kNInf, uD = kNInf;      // the up received the step before (rel O - dprev)
        float dprev = 0.f, O = 0.f;
        int lstar = 0;
        const int prodKey = (rb - 1) << 16;
        const float4* bin_g = bnd + (size_t)(rb > 0 ? rb - 1 : 0) * row_elems(L2m);
        float4* bout = bnd + (size_t)rb * row_elems(L2m);
        for (int c = 0; c < nstF; ++c) {
            ring::cp_async_wait0();
            __syncwarp();
            load_chunk(c + 1);
            if (rb > 0) {
                ring::wait_flag(&sm.progF[(rb - 1) % kW], prodKey | min(c + 3, nstF), &sm.err);
                if (lane < kCW) {
                    const int jj = c * kCW + lane + 1;
                    ws.bin[lane] = jj <= L2 ? __ldcg(bin_g + jj) : make_float4(kNInf, kNInf, kNInf, 0.f);
                }
                __syncwarp();
            }
#pragma unroll 2
            for (int q = 0; q < kCW; ++q) {
                const int t = c * kCW + q;
                const float an = __shfl_sync(kAll, fmaxf(pM, fmaxf(pI, pD)), lstar);
                const float d = an > kLow ? rintf(an) : 0.f;
                const int j = t - lane + 1;
                // up: (i-1, j)
                float vM = __shfl_up_sync(kAll, pM, 1), vI = __shfl_up_sync(kAll, pI, 1),
                      vD = __shfl_up_sync(kAll, pD, 1);
                if (lane == 0) {
                    if (rb == 0) {   // row 0
                        vM = kNInf;
                        vI = kNInf;
                        vD = fmaf((float)(j - 1), ge, go) - O;
                    } else {
                        const float4 bv = ws.bin[q];
                        const float sh = bv.w - O;
                        vM = rel(bv.x, sh);
                        vI = rel(bv.y, sh);
                        vD = rel(bv.z, sh);
                    }
                }
                // diag: (i-1, j-1); left: (i, j-1)
                float gM = rel(uM, -dprev), gI = rel(uI, -dprev), gD = rel(uD, -dprev);
                float lM = pM, lI = pI, lD = pD;
                if (j == 1) {   // column 0
                    gM = i == 1 ? -O : kNInf;
                    gI = i >= 2 ? fmaf((float)(i - 2), ge, go) - O : kNInf;
                    gD = kNInf;
                    lM = kNInf;
                    lI = fmaf((float)(i - 1), ge, go) - O;
                    lD = kNInf;
                }
                const bool live = rowok && j >= 1 && j <= L2;
                float oM = kNInf, oI = kNInf, oD = kNInf;
                float4 qM = make_float4(0.f, 0.f, 0.f, 0.f), qI = qM, qD = qM;
                if (live) {
                    const float sc = ws.ring[lane * kRW + ((t - lane) & (kRW - 1))];
                    const float aM = sc + lse3(gM, gI, gD, T, iT, qM.x, qM.y, qM.z, qM.w);
                    const float aI = lse3(vM + go, vI + ge, vD + go, T, iT, qI.x, qI.y, qI.z, qI.w);
                    const float aD = lse3(lM + go, lI + go, lD + ge, T, iT, qD.x, qD.y, qD.z, qD.w);
                    oM = aM > kLow ? aM - d : kNInf;
                    oI = aI > kLow ? aI - d : kNInf;
                    oD = aD > kLow ? aD - d : kNInf;
                    if (i == L1 && j == L2) {   // the final choice among the end cell's states
                        float w1, w2, w3, h;
                        const float fin = lse3(aM, aI, aD, T, iT, w1, w2, w3, h);
                        sm.val = (double)fin + (double)O;
                        sm.fw[0] = w1;
                        sm.fw[1] = w2;
                        sm.fw[2] = w3;
                        sm.fh = h;
                    }
                }
                const size_t pi = poff + (size_t)t * 32;
                PM[pi] = qM;
                PI[pi] = qI;
                PD[pi] = qD;
                if (lane == 31 && live) bout[j] = make_float4(oM, oI, oD, O + d);
                uM = vM;
                uI = vI;
                uD = vD;
                dprev = d;
                pM = oM;
                pI = oI;
                pD = oD;
                O += d;
                const int lo = max(0, t - L2 + 1), hi = min(t, hiRow);
                lstar = lo <= hi ? min(max(16, lo), hi) : 0;
            }
            if (lane == 31) ring::st_release(&sm.progF[warp], (rb << 16) | (c + 1));
        }
        ring::cp_async_wait0();
        __syncwarp();
    }
    __syncthreads();

    // ------------------------------------------------------------- reverse
    const float fw1 = sm.fw[0], fw2 = sm.fw[1], fw3 = sm.fw[2];
    double sopen = 0.0, sext = 0.0, sent = 0.0;
    for (int n = warp; n < nRB; n += kW) {
        const int rb = nRB - 1 - n;
        const int i = 32 * rb + lane + 1;
        const bool rowok = i <= L1;
        const size_t poff = (size_t)rb * TP * 32 + lane;
        const int T0 = L2 + 30;
        float4 bM4[kPD], bI4[kPD], bD4[kPD];
#pragma unroll
        for (int s = 0; s < kPD; ++s) {
            const size_t pi = poff + (size_t)max(T0 - s, 0) * 32;
            bM4[s] = PM[pi];
            bI4[s] = PI[pi];
            bD4[s] = PD[pi];
        }
        float lM = 0.f, lI = 0.f, lD = 0.f;      // flows from the right successor D(i, j+1)
        float dM = 0.f, dI = 0.f, dD = 0.f;      // diagonal flows of the previous cell, M(i, j+1) -> (i-1, j)
        float XM = 0.f, XI = 0.f, XD = 0.f;      // this step's message to lane l-1
        const bool below = rb + 1 < nRB;
        const int prodKey = (n - 1) << 16;
        const float4* bb_in = bbr + (size_t)rb * row_elems(L2m);
        float4* bb_out = bbr + (size_t)(rb > 0 ? rb - 1 : 0) * row_elems(L2m);
        for (int c = 0; c < nstR; ++c) {
            if (below) {
                ring::wait_flag(&sm.progR[(n - 1) % kW], prodKey | min(c + 3, nstR), &sm.err);
                if (lane < kCW) {
                    const int jj = L2 - (c * kCW + lane);
                    ws.bbin[lane] = jj >= 0 ? __ldcg(bb_in + jj) : make_float4(0.f, 0.f, 0.f, 0.f);
                }
            }
            __syncwarp();
#pragma unroll
            for (int q = 0; q < kCW; ++q) {
                const int s = c * kCW + q;
                const int t = T0 - s;
                if (t < -1) break;
                const float4 wm = bM4[q % kPD], wi = bI4[q % kPD], wd = bD4[q % kPD];
                {
                    const size_t pi = poff + (size_t)max(t - kPD, 0) * 32;
                    bM4[q % kPD] = PM[pi];
                    bI4[q % kPD] = PI[pi];
                    bD4[q % kPD] = PD[pi];
                }
                float xM = __shfl_down_sync(kAll, XM, 1), xI = __shfl_down_sync(kAll, XI, 1),
                      xD = __shfl_down_sync(kAll, XD, 1);
                if (lane == 31) {
                    const float4 bv = below ? ws.bbin[q] : make_float4(0.f, 0.f, 0.f, 0.f);
                    xM = bv.x;
                    xI = bv.y;
                    xD = bv.z;
                }
                const int j = t - lane + 1;
                const bool live = rowok && j >= 1 && j <= L2;
                const bool edge = rowok && j == 0;   // the column-0 cell (i, 0)
                const bool end = i == L1 && j == L2;
                if (live) {
                    const float bM = ((end ? fw1 : 0.f) + lM) + xM;
                    const float bI = ((end ? fw2 : 0.f) + lI) + xI;
                    const float bD = ((end ? fw3 : 0.f) + lD) + xD;
                    ws.ring[lane * kRW + ((t - lane) & (kRW - 1))] = bM;
                    sopen += (double)bI * (double)(wi.x + wi.z) + (double)bD * (double)(wd.x + wd.y);
                    sext += (double)bI * (double)wi.y + (double)bD * (double)wd.z;
                    sent += (double)bM * (double)wm.w + (double)bI * (double)wi.w + (double)bD * (double)wd.w;
                    lM = bD * wd.x;
                    lI = bD * wd.y;
                    lD = bD * wd.z;
                    XM = fmaf(bI, wi.x, dM);
                    XI = fmaf(bI, wi.y, dI);
                    XD = fmaf(bI, wi.z, dD);
                    dM = bM * wm.x;
                    dI = bM * wm.y;
                    dD = bM * wm.z;
                } else {
                    if (edge) {   // the leading gap of I(i, 0): one opening, i - 1 extensions
                        const double bb = (double)(lI + xI);
                        sopen += bb;
                        sext += bb * (double)(i - 1);
                    }
                    lM = lI = lD = 0.f;
                    XM = dM;
                    XI = dI;
                    XD = dD;
                    dM = dI = dD = 0.f;
                }
                if (lane == 0 && (live || edge)) {
                    if (rb > 0) {
                        bb_out[j] = make_float4(XM, XI, XD, 0.f);
                    } else if (j >= 1) {   // row 0: the leading gap of D(0, j)
                        sopen += (double)XD;
                        sext += (double)XD * (double)(j - 1);
                    }
                }
                if (t >= 0 && (t & (kCW - 1)) == 0) {   // chunk t / 16 is complete
                    __syncwarp();
                    const int col = t + (lane & 15);
                    if (col < L2) {
#pragma unroll 4
                        for (int r2 = 0; r2 < 16; ++r2) {
                            const int r = (lane >> 4) + 2 * r2;
                            if (32 * rb + r < L1) out[(size_t)(32 * rb + r) * L2m + col] = ws.ring[r * kRW + (col & (kRW - 1))];
                        }
                    }
                    __syncwarp();
                }
            }
            if (lane == 0) ring::st_release(&sm.progR[warp], (n << 16) | (c + 1));
        }
    }

    for (int o = 16; o >= 1; o >>= 1) {
        sopen += __shfl_xor_sync(kAll, sopen, o);
        sext += __shfl_xor_sync(kAll, sext, o);
        sent += __shfl_xor_sync(kAll, sent, o);
    }
    if (lane == 0) {
        sm.red[0][warp] = sopen;
        sm.red[1][warp] = sext;
        sm.red[2][warp] = sent;
    }
    __syncthreads();
    if (tid == 0) {
        double to = 0.0, te = 0.0, th = 0.0;
        for (int w = 0; w < kW; ++w) {
            to += sm.red[0][w];
            te += sm.red[1][w];
            th += sm.red[2][w];
        }
        p.value[b] = (float)sm.val;
        if (p.grad_gap) p.grad_gap[b] = (float)to;
        if (p.grad_gap2) p.grad_gap2[b] = (float)te;
        if (p.grad_T) p.grad_T[b] = (float)(th + (double)sm.fh);
        if (sm.err) p.redo[b] = 1;
    }
}

}  // namespace nwaw

size_t nwa_wave_area(int B, int L1, int L2) {
    return ring::align_up(nwaw::per_problem_bytes(L1, L2) * (size_t)(B > 0 ? B : 1), 256);
}

// Value, marginals and the three parameter gradients of every problem
// (a.mode == MODE_MARG, a.redo a zeroed flag per problem).  Returns -1 when
// the shape is not covered (nothing launched).
int launch_nwa_wave(const SwArgs& a, cudaStream_t st) {
    if (a.mode != MODE_MARG || !a.redo || !a.out || !a.value || a.L1 > nwaw::kMaxL1 || a.L2 > nwaw::kMaxL2 ||
        a.L1 < 1 || a.L2 < 1)
        return -1;
    if (a.B == 0) return 0;
    static DeviceSetup setup;
    int dev = 0, sms = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return (int)e;
    const size_t smem = sizeof(nwaw::CtaSmem);
    int rc = device_setup(setup, dev, [smem] {
        return (int)cudaFuncSetAttribute(nwaw::nwa_wave_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    }, &sms);
    if (rc) return rc;
    nwaw::nwa_wave_kernel<<<a.B, nwaw::kThreads, smem, st>>>(a);
    return (int)cudaGetLastError();
}

}  // namespace d2pb
