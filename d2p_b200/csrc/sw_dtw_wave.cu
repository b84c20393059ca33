// sw_dtw_wave.cu -- soft DTW value + marginals + dS/dT in row-block wavefront
// form: the value pass behind soft_dtw / soft_dtw_float when the temperature
// needs no Jacobian (same recurrence and outputs as dtw_kernel<MODE_MARG> in
// sw_dtw.cu, src/dtw/kernels_cpu.cpp:58-234 restated).
//
// Layout of the sweep.  One CTA per problem, kW warps.  Warp w takes the
// row-blocks w, w + kW, ... (32 rows each, lane l = row 32 rb + l + 1) and
// sweeps each one in steps t = 0 .. L2 + 30; at step t lane l works on column
// j = t - l + 1, so the 32 lanes of a warp sit on one anti-diagonal.
//   forward: up = lane l-1's output of the previous step (a shuffle), left =
//     the lane's own previous output, diag = the up it received the step
//     before; lane 0 takes row 32 rb (the row-block above) from an L2-resident
//     boundary row that the warp above writes with lane 31, 16 columns at a
//     time behind a release / acquire progress word (bounded waits).
//   reverse (gather form, row-blocks bottom to top, steps t = L2 + 30 .. 0):
//     beta_c = [c = end] + beta_right w_l(right) + beta_down w_u(down) +
//     beta_diag w_d(diag).  Each cell hands its left neighbour beta w_l in a
//     register and its upper neighbour beta w_u plus the diagonal flow it
//     computed one step earlier, in one shuffle; lane 0 hands row-block
//     rb - 1 the same sum through an L2-resident row.
// The marginal of a cell is its beta; dS/dT = -sum beta h, h the cell's choice
// entropy (a sum of non-negative terms).
//
// Numerics.  Each warp keeps an integer frame O_t per step of a row-block (all
// its lanes share the anti-diagonal): outputs are stored as alpha - O_t, the
// next frame adds rint of the previous step's output at an anchor lane (the
// lane nearest the band's centre line, else lane 16), and every option is a
// small stored value plus an exact integer frame difference.  Boundary rows
// carry (value - frame, frame).  The options' weights are normalised as in
// the reference's softmin; the reverse multiplies probabilities only (no
// frames).
//
// Memory.  The forward writes, per cell, the three weights and the entropy as
// one float4 in the layout [row-block][step][lane] (each warp store is four
// whole 128-byte lines), and reads the costs through a per-warp ring [32
// rows][64 columns] filled 16 columns at a time by 4-byte cp.async (any
// width); lane l at step t reads ring column (t - l) mod 64, a different bank
// in every lane.  The reverse
// reads the weights back in the same layout, 4 steps ahead, and stages the
// marginals in the same ring, storing each 16-column chunk once all its rows
// are done.  HBM per cell: cost 4 B, weights and entropy written and read
// 32 B, marginal 4 B.
//
// A problem whose wait gave up, or with an empty sequence, is flagged in
// p.redo; the caller recomputes flagged problems with dtw_kernel.
#include <math.h>
#include <stddef.h>
#include <stdint.h>

#include "../../include/d2p_b200.h"
#include "sw_common.cuh"
#include "sw_internal.h"
#include "sw_ring.cuh"

namespace d2pb {
namespace dtww {

using ring::cp_async4_zfill;
using ring::kAll;

constexpr int kW = 8;                 // warps per CTA
constexpr int kThreads = 32 * kW;
constexpr int kCW = 16;               // columns per stage / ring chunk
constexpr int kRW = 64;               // ring width (columns)
constexpr int kPD = 4;                // reverse: steps of weights loaded ahead
constexpr int kMaxL1 = 8192;          // rows per problem (256 row-blocks)
constexpr int kMaxL2 = 1000000;       // columns (stage counts fit the progress word's 16 bits)
constexpr float kPInf = 1.0e30f;      // unreached cell, as the reference's sentinel
constexpr float kFin = 0.5e30f;       // values below this are reached

struct WarpSmem {
    float ring[32 * kRW];             // forward: costs; reverse: marginals before their store
    float2 bin[kCW];                  // forward: the stage's row above (value - frame, frame)
    float bbin[kCW];                  // reverse: the stage's flows from the row below
};
struct CtaSmem {
    WarpSmem w[kW];
    int progF[kW], progR[kW];         // (row-block key << 16) | stages done, per warp
    int err;
    double red[kW];
    double val;                       // alpha at the end cell
};

__host__ __device__ inline int nrb_of(int L1m) { return (L1m + 31) / 32; }
__host__ __device__ inline int steps_of(int L2m) { return (L2m + 31 + kCW - 1) / kCW * kCW; }
__host__ __device__ inline size_t plane_floats(int L1m, int L2m) {
    return (size_t)nrb_of(L1m) * steps_of(L2m) * 32;
}
__host__ __device__ inline size_t row_elems(int L2m) { return (size_t)L2m + kCW + 1; }
__host__ __device__ inline size_t per_problem_bytes(int L1m, int L2m) {
    const size_t nr = (size_t)nrb_of(L1m) * row_elems(L2m);
    return ring::align_up(4 * plane_floats(L1m, L2m) * sizeof(float), 256) + ring::align_up(nr * sizeof(float2), 256) +
           ring::align_up(nr * sizeof(float), 256);
}

__global__ void __launch_bounds__(kThreads, 2) dtw_wave_kernel(SwArgs p) {
    extern __shared__ __align__(16) unsigned char smem_raw[];
    CtaSmem& sm = *reinterpret_cast<CtaSmem*>(smem_raw);
    const int b = blockIdx.x;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int L1m = p.L1, L2m = p.L2;
    const int L1 = p.lengths ? min(max(p.lengths[2 * b], 0), L1m) : L1m;
    const int L2 = p.lengths ? min(max(p.lengths[2 * b + 1], 0), L2m) : L2m;
    if (L1 == 0 || L2 == 0) {   // the engine writes the sentinel value and the zeros
        if (tid == 0) p.redo[b] = 1;
        return;
    }
    const int bw = p.parts;
    const float T = p.temp_dev ? __ldg(p.temp_dev) : p.temp;
    const float iT = 1.f / T;
    const size_t plane = (size_t)L1m * L2m;
    const float* __restrict__ Cst = p.scores + (size_t)b * plane;
    float* __restrict__ out = p.out + (size_t)b * plane;
    const int TP = steps_of(L2m);
    char* base = reinterpret_cast<char*>(p.ws) + (size_t)b * per_problem_bytes(L1m, L2m);
    const size_t pfl = plane_floats(L1m, L2m);
    float4* const Wp = reinterpret_cast<float4*>(base);   // (w_d, w_u, w_l, h) per cell
    float2* const bnd = reinterpret_cast<float2*>(base + ring::align_up(4 * pfl * sizeof(float), 256));
    float* const bbr = reinterpret_cast<float*>(reinterpret_cast<char*>(bnd) +
                                                ring::align_up((size_t)nrb_of(L1m) * row_elems(L2m) * sizeof(float2), 256));
    const int nRB = nrb_of(L1);
    const int nst = (L2 + 31 + kCW - 1) / kCW;   // stages of a row-block's sweep
    WarpSmem& ws = sm.w[warp];

    if (tid < kW) {
        sm.progF[tid] = -1;
        sm.progR[tid] = -1;
    }
    if (tid == 0) {
        sm.err = 0;
        sm.val = kPInf;
    }
    if (L1 < L1m || L2 < L2m) {   // zeros outside the problem
        for (int i = 0; i < L1m; ++i)
            for (int j = (i < L1 ? L2 : 0) + tid; j < L2m; j += kThreads) out[(size_t)i * L2m + j] = 0.f;
    }
    __syncthreads();

    const float ratio = (float)L1 / (float)(L1 + L2);   // anchor: the band's centre row of an anti-diagonal

    // ------------------------------------------------------------- forward
    for (int rb = warp; rb < nRB; rb += kW) {
        const int i = 32 * rb + lane + 1;
        const bool rowok = i <= L1;
        const float ei = (float)((long long)i * L2) / (float)L1;   // the band's centre column of this row
        const size_t poff = (size_t)rb * TP * 32 + lane;
        // chunk c of the cost rows: columns [16c, 16c + 16), lane = column
        // (lane & 15) of rows (lane >> 4) + 2q
        auto load_chunk = [&](int c) {
            const int col = c * kCW + (lane & 15);
            const bool cin = col < L2;
#pragma unroll 4
            for (int q = 0; q < 16; ++q) {
                const int r = (lane >> 4) + 2 * q;
                const bool ok = cin && 32 * rb + r < L1;
                const float* g = ok ? Cst + (size_t)(32 * rb + r) * L2m + col : Cst;
                cp_async4_zfill(&ws.ring[r * kRW + (col & (kRW - 1))], g, ok ? 4 : 0);
            }
            ring::cp_async_commit();
        };
        load_chunk(0);
        float prev = kPInf;                                   // own output of the previous step (rel O)
        float upPrev = (rb == 0 && lane == 0) ? 0.f : kPInf;  // the up received the step before (alpha[0][0] = 0)
        float dprev = 0.f;                                    // the previous step's frame increment
        float O = 0.f;                                        // frame of the previous step's outputs
        int lstar = 0;
        const int prodKey = (rb - 1) << 16;
        const float2* bin_g = bnd + (size_t)(rb > 0 ? rb - 1 : 0) * row_elems(L2m);
        float2* bout = bnd + (size_t)rb * row_elems(L2m);
        for (int c = 0; c < nst; ++c) {
            ring::cp_async_wait0();
            __syncwarp();
            load_chunk(c + 1);
            if (rb > 0) {
                ring::wait_flag(&sm.progF[(rb - 1) % kW], prodKey | min(c + 3, nst), &sm.err);
                if (lane < kCW) {
                    const int jj = c * kCW + lane + 1;
                    ws.bin[lane] = jj <= L2 ? __ldcg(bin_g + jj) : make_float2(kPInf, 0.f);
                }
                __syncwarp();
            }
#pragma unroll 4
            for (int q = 0; q < kCW; ++q) {
                const int t = c * kCW + q;
                // this step's frame: the previous outputs at the anchor lane
                const float an = __shfl_sync(kAll, prev, lstar);
                const float d = an < kFin ? rintf(an) : 0.f;
                float up = __shfl_up_sync(kAll, prev, 1);
                if (lane == 0) {
                    if (rb == 0) {
                        up = kPInf;
                    } else {
                        const float2 bv = ws.bin[q];
                        up = bv.x < kFin ? bv.x + (bv.y - O) : kPInf;
                    }
                }
                const float dg = upPrev < kFin ? upPrev - dprev : kPInf;
                const float lf = prev;
                const int j = t - lane + 1;
                const bool live = rowok && j >= 1 && j <= L2;
                const bool act = live && (bw < 0 || fabsf((float)j - ei) <= (float)bw);
                float a = kPInf, wd = 0.f, wu = 0.f, wl = 0.f, h = 0.f;
                if (act) {
                    const float m = fminf(dg, fminf(up, lf));
                    if (m < kFin) {
                        const float cst = ws.ring[lane * kRW + ((t - lane) & (kRW - 1))];
                        const float ed = expf((m - dg) * iT), eu = expf((m - up) * iT), el = expf((m - lf) * iT);
                        const float sum = (ed + eu) + el;
                        const float ls = logf(sum);
                        const float is = 1.f / sum;
                        wd = ed * is;
                        wu = eu * is;
                        wl = el * is;
                        a = cst + fmaf(-T, ls, m);
                        h = ls + iT * fmaf(wd, dg - m, fmaf(wu, up - m, wl * (lf - m)));
                    }
                }
                const float o = a < kFin ? a - d : kPInf;   // relative to this step's frame O + d
                Wp[poff + (size_t)t * 32] = make_float4(wd, wu, wl, h);
                if (lane == 31 && live) bout[j] = make_float2(o, O + d);
                if (i == L1 && j == L2) sm.val = a < kFin ? (double)o + (double)(O + d) : (double)kPInf;
                upPrev = up;
                dprev = d;
                prev = o;
                O += d;
                // anchor lane of this step's outputs (for the next step's frame)
                const int lo = max(0, t - L2 + 1), hi = min(min(t, 31), L1 - 1 - 32 * rb);
                int lc = 16;
                if (bw >= 0) lc = (int)rintf((float)(32 * rb + t + 2) * ratio) - (32 * rb + 1);
                lstar = lo <= hi ? min(max(lc, lo), hi) : 0;
            }
            if (lane == 31) ring::st_release(&sm.progF[warp], (rb << 16) | (c + 1));
        }
        ring::cp_async_wait0();
        __syncwarp();
    }
    __syncthreads();

    // ------------------------------------------------------------- reverse
    double sent = 0.0;
    for (int n = warp; n < nRB; n += kW) {
        const int rb = nRB - 1 - n;   // key n: bottom row-block first
        const int i = 32 * rb + lane + 1;
        const bool rowok = i <= L1;
        const size_t poff = (size_t)rb * TP * 32 + lane;
        const int T0 = L2 + 30;       // the first step (t runs down to 0)
        float4 buf[kPD];
#pragma unroll
        for (int s = 0; s < kPD; ++s) buf[s] = Wp[poff + (size_t)max(T0 - s, 0) * 32];
        float pleft = 0.f, pdiag = 0.f, X = 0.f;
        const bool below = rb + 1 < nRB;
        const int prodKey = (n - 1) << 16;
        const float* bb_in = bbr + (size_t)rb * row_elems(L2m);          // flows into row 32 rb + 32
        float* bb_out = bbr + (size_t)(rb > 0 ? rb - 1 : 0) * row_elems(L2m);
        for (int c = 0; c < nst; ++c) {
            if (below) {
                ring::wait_flag(&sm.progR[(n - 1) % kW], prodKey | min(c + 3, nst), &sm.err);
                if (lane < kCW) {
                    const int jj = L2 - (c * kCW + lane);
                    ws.bbin[lane] = jj >= 1 ? __ldcg(bb_in + jj) : 0.f;
                }
            }
            __syncwarp();
#pragma unroll
            for (int q = 0; q < kCW; ++q) {
                const int s = c * kCW + q;
                const int t = T0 - s;
                if (t < 0) break;
                const float4 wv = buf[q % kPD];
                const float wd = wv.x, wu = wv.y, wl = wv.z, h = wv.w;
                buf[q % kPD] = Wp[poff + (size_t)max(t - kPD, 0) * 32];
                float xin = __shfl_down_sync(kAll, X, 1);
                if (lane == 31) xin = below ? ws.bbin[q] : 0.f;
                const int j = t - lane + 1;
                const bool live = rowok && j >= 1 && j <= L2;
                const float seed = (i == L1 && j == L2) ? 1.f : 0.f;
                const float beta = live ? (seed + pleft) + xin : 0.f;
                pleft = beta * wl;
                X = fmaf(beta, wu, pdiag);
                pdiag = beta * wd;
                if (live) ws.ring[lane * kRW + ((t - lane) & (kRW - 1))] = beta;
                sent += (double)beta * (double)h;
                if (lane == 0 && rb > 0 && live) bb_out[j] = X;
                if ((t & (kCW - 1)) == 0) {   // chunk t / 16 (columns t .. t + 15) is complete
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

    // dS/dT = -sum beta h over the problem
    for (int o = 16; o >= 1; o >>= 1) sent += __shfl_xor_sync(kAll, sent, o);
    if (lane == 0) sm.red[warp] = sent;
    __syncthreads();
    if (tid == 0) {
        double th = 0.0;
        for (int w = 0; w < kW; ++w) th += sm.red[w];
        const double v = sm.val;
        p.value[b] = v < (double)kFin ? (float)v : kPInf;
        if (p.grad_T) p.grad_T[b] = (float)(-th);
        if (sm.err) p.redo[b] = 1;
    }
}


// ============================================================================
// The Hessian-vector product H V = d(marginals)/d(costs) . V in the same form.
// The forward carries each cell's tangent along V, f = sum_k w_k f_k + V_c
// (framed per step like alpha, frame D_t), and stores (w_d, w_u, w_l, f) and
// V per cell.  The reverse carries beta and its tangent r: a cell d hands each
// predecessor k the flow b_d w_k and r_d w_k + b_d w_k (f_d - V_d - f_k + D_d -
// D_k) / T, the difference of tangents formed per successor as in the
// reference (src/dtw/kernels_cpu.cpp:236-420 restated as flows): it reads its
// predecessors' forward tangents itself (its own prefetched slot for the left
// one, lane l-1's by shuffle for the upper two, the row-block above's for lane
// 0); the predecessor's r is the sum of what it receives.
// ============================================================================
__host__ __device__ inline size_t hvp_problem_bytes(int L1m, int L2m) {
    const size_t nr = (size_t)nrb_of(L1m) * row_elems(L2m);
    const size_t sl = plane_floats(L1m, L2m);   // slots [rb][t][lane]
    return 2 * ring::align_up(sl * sizeof(float4), 256) + 2 * ring::align_up(nr * sizeof(float4), 256) +
           2 * ring::align_up((size_t)nrb_of(L1m) * steps_of(L2m) * 4, 256);
}

// MODE_HVP: out = H p.tangent.  MODE_PT: out = dP/dT (if p.out), and with
// p.dot_with, dot_out[b] = sum dot_with * dP/dT.
template <int MODE>
__global__ void __launch_bounds__(kThreads, 2) dtw_wave_tan_kernel(SwArgs p) {
    extern __shared__ __align__(16) unsigned char smem_raw[];
    CtaSmem& sm = *reinterpret_cast<CtaSmem*>(smem_raw);
    const int b = blockIdx.x;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int L1m = p.L1, L2m = p.L2;
    const int L1 = p.lengths ? min(max(p.lengths[2 * b], 0), L1m) : L1m;
    const int L2 = p.lengths ? min(max(p.lengths[2 * b + 1], 0), L2m) : L2m;
    if (L1 == 0 || L2 == 0) {
        if (tid == 0) p.redo[b] = 1;
        return;
    }
    const int bw = p.parts;
    const float T = p.temp_dev ? __ldg(p.temp_dev) : p.temp;
    const float iT = 1.f / T;
    const size_t plane = (size_t)L1m * L2m;
    const float* __restrict__ Cst = p.scores + (size_t)b * plane;
    const float* __restrict__ Vin = MODE == MODE_HVP ? p.tangent + (size_t)b * plane : nullptr;
    float* __restrict__ out = p.out ? p.out + (size_t)b * plane : nullptr;
    const float* __restrict__ Gw = p.dot_with ? p.dot_with + (size_t)b * plane : nullptr;
    const int TP = steps_of(L2m);
    char* base = reinterpret_cast<char*>(p.ws) + (size_t)b * hvp_problem_bytes(L1m, L2m);
    const size_t sl = plane_floats(L1m, L2m);
    float4* const Wp = reinterpret_cast<float4*>(base);   // (w_d, w_u, w_l, f)
    // HVP: (V, -, -, -); PT: (alpha - O, h, alpha - O - cost, -), alpha 0 where unreached
    float4* const Xp = Wp + ring::align_up(sl * sizeof(float4), 256) / sizeof(float4);
    const size_t nr = (size_t)nrb_of(L1m) * row_elems(L2m);
    float4* const bnd = Xp + ring::align_up(sl * sizeof(float4), 256) / sizeof(float4);
    float4* const bbr = bnd + ring::align_up(nr * sizeof(float4), 256) / sizeof(float4);
    float* const Dst = reinterpret_cast<float*>(bbr + ring::align_up(nr * sizeof(float4), 256) / sizeof(float4));
    float* const Ost = Dst + ring::align_up((size_t)nrb_of(L1m) * TP * 4, 256) / 4;   // alpha's frames
    const int nRB = nrb_of(L1);
    const int nst = (L2 + 31 + kCW - 1) / kCW;
    WarpSmem& ws = sm.w[warp];
    __shared__ float4 binF[kW][kCW];   // forward: the row above (alpha - O, O, f - D, D)
    __shared__ float4 bbinR[kW][kCW];  // reverse: flows from the row below (flow, q, p, -)

    if (tid < kW) {
        sm.progF[tid] = -1;
        sm.progR[tid] = -1;
    }
    if (tid == 0) sm.err = 0;
    if (out && (L1 < L1m || L2 < L2m)) {   // zeros outside the problem (no plane: only the dot is wanted)
        for (int i = 0; i < L1m; ++i)
            for (int j = (i < L1 ? L2 : 0) + tid; j < L2m; j += kThreads) out[(size_t)i * L2m + j] = 0.f;
    }
    __syncthreads();
    const float ratio = (float)L1 / (float)(L1 + L2);

    // ------------------------------------------------------------- forward
    for (int rb = warp; rb < nRB; rb += kW) {
        const int i = 32 * rb + lane + 1;
        const bool rowok = i <= L1;
        const float ei = (float)((long long)i * L2) / (float)L1;
        const size_t poff = (size_t)rb * TP * 32 + lane;
        const float* vrow = MODE == MODE_HVP ? Vin + (size_t)(rowok ? i - 1 : 0) * L2m : nullptr;
        // V of this lane's column, two steps ahead (steps t and t + 1 in flight)
        auto vload = [&](int jj) {
            return MODE == MODE_HVP && rowok && jj >= 1 && jj <= L2 ? __ldg(vrow + (jj - 1)) : 0.f;
        };
        float vcur = vload(1 - lane), vnext = vload(2 - lane);
        auto load_chunk = [&](int c) {
            const int col = c * kCW + (lane & 15);
            const bool cin = col < L2;
#pragma unroll 4
            for (int q = 0; q < 16; ++q) {
                const int r = (lane >> 4) + 2 * q;
                const bool ok = cin && 32 * rb + r < L1;
                const float* g = ok ? Cst + (size_t)(32 * rb + r) * L2m + col : Cst;
                cp_async4_zfill(&ws.ring[r * kRW + (col & (kRW - 1))], g, ok ? 4 : 0);
            }
            ring::cp_async_commit();
        };
        load_chunk(0);
        float prev = kPInf, upPrev = (rb == 0 && lane == 0) ? 0.f : kPInf, dprev = 0.f, O = 0.f;
        float prevF = 0.f, upPrevF = 0.f, ddprev = 0.f, Dfr = 0.f;
        int lstar = 0;
        const int prodKey = (rb - 1) << 16;
        const float4* bin_g = bnd + (size_t)(rb > 0 ? rb - 1 : 0) * row_elems(L2m);
        float4* bout = bnd + (size_t)rb * row_elems(L2m);
        for (int c = 0; c < nst; ++c) {
            ring::cp_async_wait0();
            __syncwarp();
            load_chunk(c + 1);
            if (rb > 0) {
                ring::wait_flag(&sm.progF[(rb - 1) % kW], prodKey | min(c + 3, nst), &sm.err);
                if (lane < kCW) {
                    const int jj = c * kCW + lane + 1;
                    binF[warp][lane] = jj <= L2 ? __ldcg(bin_g + jj) : make_float4(kPInf, 0.f, 0.f, 0.f);
                }
                __syncwarp();
            }
#pragma unroll 2
            for (int q = 0; q < kCW; ++q) {
                const int t = c * kCW + q;
                const float an = __shfl_sync(kAll, prev, lstar), anF = __shfl_sync(kAll, prevF, lstar);
                const float d = an < kFin ? rintf(an) : 0.f;
                const float dd = an < kFin ? rintf(anF) : 0.f;
                float up = __shfl_up_sync(kAll, prev, 1), upF = __shfl_up_sync(kAll, prevF, 1);
                if (lane == 0) {
                    if (rb == 0) {
                        up = kPInf;
                        upF = 0.f;
                    } else {
                        const float4 bv = binF[warp][q];
                        up = bv.x < kFin ? bv.x + (bv.y - O) : kPInf;
                        upF = bv.x < kFin ? bv.z + (bv.w - Dfr) : 0.f;
                    }
                }
                const float dg = upPrev < kFin ? upPrev - dprev : kPInf;
                const float dgF = upPrevF - ddprev;
                const float lf = prev, lfF = prevF;
                const int j = t - lane + 1;
                const bool live = rowok && j >= 1 && j <= L2;
                const bool act = live && (bw < 0 || fabsf((float)j - ei) <= (float)bw);
                const float vv = live ? vcur : 0.f;
                vcur = vnext;
                vnext = vload(j + 2);
                float a = kPInf, wd = 0.f, wu = 0.f, wl = 0.f, f = 0.f, h = 0.f, cst = 0.f;
                if (act) {
                    const float m = fminf(dg, fminf(up, lf));
                    if (m < kFin) {
                        cst = ws.ring[lane * kRW + ((t - lane) & (kRW - 1))];
                        const float ed = expf((m - dg) * iT), eu = expf((m - up) * iT), el = expf((m - lf) * iT);
                        const float sum = (ed + eu) + el;
                        const float ls = logf(sum);
                        const float is = 1.f / sum;
                        wd = ed * is;
                        wu = eu * is;
                        wl = el * is;
                        a = cst + fmaf(-T, ls, m);
                        f = fmaf(wd, dgF, fmaf(wu, upF, wl * lfF));
                        if (MODE == MODE_HVP) {
                            f += vv;
                        } else {   // along T: minus the choice's entropy
                            h = ls + iT * fmaf(wd, dg - m, fmaf(wu, up - m, wl * (lf - m)));
                            f -= h;
                        }
                    }
                }
                const bool reached = a < kFin;
                const float o = reached ? a - d : kPInf;
                const float oF = reached ? f - dd : 0.f;
                const size_t pi = poff + (size_t)t * 32;
                Wp[pi] = make_float4(wd, wu, wl, oF);
                if (MODE == MODE_HVP) Xp[pi] = make_float4(vv, 0.f, 0.f, 0.f);
                else Xp[pi] = reached ? make_float4(o, h, o - cst, 0.f) : make_float4(0.f, 0.f, 0.f, 0.f);
                if (lane == 31 && live) bout[j] = make_float4(o, O + d, oF, Dfr + dd);
                if (lane == 0) {
                    Dst[(size_t)rb * TP + t] = Dfr + dd;
                    Ost[(size_t)rb * TP + t] = O + d;
                }
                upPrev = up;
                upPrevF = upF;
                dprev = d;
                ddprev = dd;
                prev = o;
                prevF = oF;
                O += d;
                Dfr += dd;
                const int lo = max(0, t - L2 + 1), hi = min(min(t, 31), L1 - 1 - 32 * rb);
                int lc = 16;
                if (bw >= 0) lc = (int)rintf((float)(32 * rb + t + 2) * ratio) - (32 * rb + 1);
                lstar = lo <= hi ? min(max(lc, lo), hi) : 0;
            }
            if (lane == 31) ring::st_release(&sm.progF[warp], (rb << 16) | (c + 1));
        }
        ring::cp_async_wait0();
        __syncwarp();
    }
    __syncthreads();

    // ------------------------------------------------------------- reverse
    constexpr bool XPT = MODE == MODE_PT;
    constexpr int kPT = 4;   // steps loaded ahead (a divisor of kCW: slot q % kPT is step s % kPT)
    double sdot = 0.0;
    for (int n = warp; n < nRB; n += kW) {
        const int rb = nRB - 1 - n;
        const int i = 32 * rb + lane + 1;
        const bool rowok = i <= L1;
        const size_t poff = (size_t)rb * TP * 32 + lane;
        const size_t rup = (size_t)(rb > 0 ? rb - 1 : 0);
        const float* Drb = Dst + (size_t)rb * TP;
        const float* Dup = Dst + rup * TP;
        const float* Orb = Ost + (size_t)rb * TP;
        const float* Oup = Ost + rup * TP;
        const float4* Wup = Wp + rup * TP * 32 + 31;   // the row above: lane 31
        const float4* Xup = Xp + rup * TP * 32 + 31;
        const int T0 = L2 + 30;
        float4 wbuf[kPT], xbuf[kPT];
#pragma unroll
        for (int s = 0; s < kPT; ++s) {
            const size_t pi = poff + (size_t)max(T0 - s, 0) * 32;
            wbuf[s] = Wp[pi];
            xbuf[s] = Xp[pi];
        }
        float upf[kPT], upa[kPT];   // the row above's lane-31 tangent (and alpha) at steps T0 + 30 - s
#pragma unroll
        for (int s = 0; s < kPT; ++s) {
            const size_t ss = (size_t)min(T0 + 30 - s, TP - 1) * 32;
            upf[s] = Wup[ss].w;
            upa[s] = XPT ? Xup[ss].x : 0.f;
        }
        float fuaC = Wup[(size_t)min(T0 + 31, TP - 1) * 32].w;
        float auaC = XPT ? Xup[(size_t)min(T0 + 31, TP - 1) * 32].x : 0.f;
        float Lf = 0.f, Lq = 0.f;   // from the right successor (own previous step)
        float Df = 0.f, Dq = 0.f;   // the diagonal message of the previous step
        float Xf = 0.f, Xq = 0.f;   // this step's message to lane l-1
        const bool below = rb + 1 < nRB;
        const int prodKey = (n - 1) << 16;
        const float4* bb_in = bbr + (size_t)rb * row_elems(L2m);
        float4* bb_out = bbr + rup * row_elems(L2m);
        for (int c = 0; c < nst; ++c) {
            if (below) {
                ring::wait_flag(&sm.progR[(n - 1) % kW], prodKey | min(c + 3, nst), &sm.err);
                if (lane < kCW) {
                    const int jj = L2 - (c * kCW + lane);
                    bbinR[warp][lane] = jj >= 1 ? __ldcg(bb_in + jj) : make_float4(0.f, 0.f, 0.f, 0.f);
                }
            }
            __syncwarp();
#pragma unroll
            for (int q = 0; q < kCW; ++q) {
                const int s = c * kCW + q;
                const int t = T0 - s;
                if (t < 0) break;
                const float4 wv = wbuf[q % kPT];
                const float4 xv = xbuf[q % kPT];
                // the predecessors' forward tangents (and along T their alphas), in
                // their frames: left = this lane's step t-1; up / diagonal = lane
                // l-1's steps t-1 / t-2 (in flight there), for lane 0 the row-block
                // above's last row at its steps t+31 / t+30
                const float fl = wbuf[(q + 1) % kPT].w;
                float fu = __shfl_up_sync(kAll, fl, 1);
                float fd = __shfl_up_sync(kAll, wbuf[(q + 2) % kPT].w, 1);
                const int su = min(t + 31, TP - 1), sd = min(t + 30, TP - 1);
                // the row above's lane 31 at steps t + 31 / t + 30, loaded kPT steps ahead
                const float fda = upf[q % kPT], fua = fuaC;
                const float ada = upa[q % kPT], aua = auaC;
                fuaC = fda;
                auaC = ada;
                {
                    const size_t ss = (size_t)max(min(t - kPT + 30, TP - 1), 0) * 32;
                    upf[q % kPT] = Wup[ss].w;
                    if (XPT) upa[q % kPT] = Xup[ss].x;
                }
                float al = 0.f, au = 0.f, ad = 0.f;
                if (MODE == MODE_PT) {
                    al = xbuf[(q + 1) % kPT].x;
                    au = __shfl_up_sync(kAll, al, 1);
                    ad = __shfl_up_sync(kAll, xbuf[(q + 2) % kPT].x, 1);
                }
                {
                    const size_t pi = poff + (size_t)max(t - kPT, 0) * 32;
                    wbuf[q % kPT] = Wp[pi];
                    xbuf[q % kPT] = Xp[pi];
                }
                float xf = __shfl_down_sync(kAll, Xf, 1), xq = __shfl_down_sync(kAll, Xq, 1);
                if (lane == 31) {
                    const float4 bv = below ? bbinR[warp][q] : make_float4(0.f, 0.f, 0.f, 0.f);
                    xf = bv.x;
                    xq = bv.y;
                }
                const int j = t - lane + 1;
                const bool live = rowok && j >= 1 && j <= L2;
                const float seed = (i == L1 && j == L2) ? 1.f : 0.f;
                float beta = 0.f, r = 0.f;
                if (live) {
                    beta = (seed + Lf) + xf;
                    r = Lq + xq;
                }
                const float Dt = __ldg(Drb + t);
                const float Dl = __ldg(Drb + max(t - 1, 0));
                const float Dd = __ldg(Drb + max(t - 2, 0));
                const float Dua = __ldg(Dup + su), Dda = __ldg(Dup + sd);
                float Ot = 0.f, Ol = 0.f, Od = 0.f, Oua = 0.f, Oda = 0.f;
                if (MODE == MODE_PT) {
                    Ot = __ldg(Orb + t);
                    Ol = __ldg(Orb + max(t - 1, 0));
                    Od = __ldg(Orb + max(t - 2, 0));
                    Oua = __ldg(Oup + su);
                    Oda = __ldg(Oup + sd);
                }
                const bool top = lane == 0 && rb > 0;
                float Du = Dl, Ddg = Dd, Ou = Ol, Odg = Od;
                if (top) {
                    fu = fua;
                    fd = fda;
                    au = aua;
                    ad = ada;
                    Du = Dua;
                    Ddg = Dda;
                    Ou = Oua;
                    Odg = Oda;
                }
                // to predecessor k with weight w: r w + b dw, with
                //   HVP: dw = w (f - V - f_k + D - D_k) / T
                //   PT:  dw = w ((f - f_k + D - D_k + h) / T + (a_k - s + O_k - O - T h) / T^2)
                auto msg = [&](float w, float fk, float Dk, float ak, float Ok) {
                    float dw;
                    if (MODE == MODE_HVP) {
                        dw = w * (((wv.w - xv.x) - fk) + (Dt - Dk)) * iT;
                    } else {
                        const float g = (wv.w - fk) + (Dt - Dk);
                        const float da = (ak - xv.z) + (Ok - Ot) - T * xv.y;
                        dw = w * fmaf(g + xv.y, iT, da * iT * iT);
                    }
                    return fmaf(r, w, beta * dw);
                };
                Lf = beta * wv.z;
                Lq = msg(wv.z, fl, Dl, al, Ol);
                Xf = fmaf(beta, wv.y, Df);
                Xq = msg(wv.y, fu, Du, au, Ou) + Dq;
                Df = beta * wv.x;
                Dq = msg(wv.x, fd, Ddg, ad, Odg);
                if (live) ws.ring[lane * kRW + ((t - lane) & (kRW - 1))] = r;
                if (lane == 0 && rb > 0 && live) bb_out[j] = make_float4(Xf, Xq, 0.f, 0.f);
                if ((t & (kCW - 1)) == 0) {
                    __syncwarp();
                    const int col = t + (lane & 15);
                    if (col < L2) {
#pragma unroll 4
                        for (int r2 = 0; r2 < 16; ++r2) {
                            const int rr = (lane >> 4) + 2 * r2;
                            if (32 * rb + rr < L1) {
                                const float hv = ws.ring[rr * kRW + (col & (kRW - 1))];
                                const size_t gi = (size_t)(32 * rb + rr) * L2m + col;
                                if (out) out[gi] = hv;
                                if (Gw) sdot += (double)__ldg(Gw + gi) * (double)hv;
                            }
                        }
                    }
                    __syncwarp();
                }
            }
            if (lane == 0) ring::st_release(&sm.progR[warp], (n << 16) | (c + 1));
        }
    }
    for (int o = 16; o >= 1; o >>= 1) sdot += __shfl_xor_sync(kAll, sdot, o);
    if (lane == 0) sm.red[warp] = sdot;
    __syncthreads();
    if (tid == 0) {
        if (p.dot_out) {
            double th = 0.0;
            for (int w = 0; w < kW; ++w) th += sm.red[w];
            p.dot_out[b] = (float)th;
        }
        if (sm.err) p.redo[b] = 1;
    }
}

}  // namespace dtww

size_t dtw_wave_area(int B, int L1, int L2) {
    return ring::align_up(dtww::per_problem_bytes(L1, L2) * (size_t)(B > 0 ? B : 1), 256);
}

size_t dtw_wave_tan_area(int B, int L1, int L2) {
    return ring::align_up(dtww::hvp_problem_bytes(L1, L2) * (size_t)(B > 0 ? B : 1), 256);
}

// a.mode MODE_HVP: H V of every problem (a.tangent = V, a.out = H V);
// MODE_PT: dP/dT (a.out, optional) and dot_out[b] = sum dot_with * dP/dT (with
// a.dot_with).  a.redo a zeroed flag per problem.  Returns -1 when the shape is
// not covered (nothing launched).
int launch_dtw_wave_tan(const SwArgs& a, cudaStream_t st) {
    if (!a.redo || a.L1 > dtww::kMaxL1 || a.L2 > dtww::kMaxL2 || a.L1 < 1 || a.L2 < 1) return -1;
    if (a.mode == MODE_HVP && (!a.out || !a.tangent)) return -1;
    if (a.mode == MODE_PT && !a.out && !(a.dot_with && a.dot_out)) return -1;
    if (a.mode != MODE_HVP && a.mode != MODE_PT) return -1;
    if (a.B == 0) return 0;
    static DeviceSetup setup;
    int dev = 0, sms = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return (int)e;
    const size_t smem = sizeof(dtww::CtaSmem);
    int rc = device_setup(setup, dev, [smem] {
        cudaError_t r = cudaFuncSetAttribute(dtww::dtw_wave_tan_kernel<MODE_HVP>,
                                             cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (r == cudaSuccess)
            r = cudaFuncSetAttribute(dtww::dtw_wave_tan_kernel<MODE_PT>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     (int)smem);
        return (int)r;
    }, &sms);
    if (rc) return rc;
    if (a.mode == MODE_HVP) dtww::dtw_wave_tan_kernel<MODE_HVP><<<a.B, dtww::kThreads, smem, st>>>(a);
    else dtww::dtw_wave_tan_kernel<MODE_PT><<<a.B, dtww::kThreads, smem, st>>>(a);
    return (int)cudaGetLastError();
}

// Value + marginals + dS/dT of every problem (a.mode == MODE_MARG, a.redo set
// to a zeroed flag per problem).  Returns -1 when the shape is not covered
// (nothing launched).
int launch_dtw_wave(const SwArgs& a, cudaStream_t st) {
    if (a.mode != MODE_MARG || !a.redo || !a.out || !a.value || a.L1 > dtww::kMaxL1 || a.L2 > dtww::kMaxL2 ||
        a.L1 < 1 || a.L2 < 1)
        return -1;
    if (a.B == 0) return 0;
    static DeviceSetup setup;
    int dev = 0, sms = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return (int)e;
    const size_t smem = sizeof(dtww::CtaSmem);
    int rc = device_setup(setup, dev, [smem] {
        return (int)cudaFuncSetAttribute(dtww::dtw_wave_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    }, &sms);
    if (rc) return rc;
    dtww::dtw_wave_kernel<<<a.B, dtww::kThreads, smem, st>>>(a);
    return (int)cudaGetLastError();
}

}  // namespace d2pb
