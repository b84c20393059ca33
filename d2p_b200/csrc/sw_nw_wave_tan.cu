// sw_nw_wave_tan.cu -- soft Needleman-Wunsch (linear gap) tangent operators in
// row-block wavefront form: the Hessian-vector product (MODE_HVP), dP/dgap
// (MODE_PGAP) and dP/dT (MODE_PT), each optionally contracted with a weight
// plane (backward_full); the same recurrences and outputs as nw_kernel's
// tangent modes in sw_nw.cu (src/nw/kernels_cpu.cpp restated).
//
// Sweep as in sw_dtw_wave.cu: one CTA of kW warps per problem, warp w takes
// row-blocks w, w + kW, ..., lane l = row 32 rb + l + 1, step t on column j = t
// - l + 1; up and diagonal by shuffles, left in registers, the row above
// through an L2-resident boundary row behind release / acquire progress words
// (bounded waits); integer frames per step for alpha (O) and its tangent (D),
// taken at the lane nearest the main diagonal.
//
// Forward (max-LSE):  alpha = LSE_T(alpha_diag + s, alpha_up + gap, alpha_left
// + gap) with boundary alpha(i,0) = i gap, alpha(0,j) = j gap formed where
// read; the tangent f = w_d t_d + w_u t_u + w_l t_l with t_d = f_diag (+ V),
// t_u,l = f_up,left (+ 1 along gap), and along T + (alpha - E[v]) / T.  Per
// cell it stores (w_d, w_u, w_l, f) and (HVP: V; PT: alpha, E[v], s).
//
// Reverse (gather form, flows): a cell d hands each predecessor k the flow
// b_d w_k and q_k = r_d w_k + b_d dw_k, dw_k = w_k (dv_k - eu_d) / T with dv_k
// = f_k + D_k - D_d (+ V_d for the diagonal option, + 1 for a gap option along
// gap) and eu_d = f_d (along T: - (alpha_d - E[v]_d) / T, and dw_k += w_k
// (E[v]_d - v_k) / T^2, v_k = alpha_k + (s_d or gap) + O_k - O_d); the
// predecessors' tangents and alphas come from the lane's own prefetched slot
// (left), lane l-1's by shuffle (up, diagonal) or the row-block above (lane
// 0), boundary predecessors in absolute terms.  A cell's r is the sum of what
// it receives; its marginal's tangent r w_d + b dw_d is exactly the message it
// hands its diagonal predecessor.
//
// A problem whose wait gave up, or with an empty sequence, is flagged in
// p.redo; the caller recomputes flagged problems with nw_kernel.
#include <math.h>
#include <stddef.h>
#include <stdint.h>

#include "../../include/d2p_b200.h"
#include "sw_common.cuh"
#include "sw_internal.h"
#include "sw_ring.cuh"

namespace d2pb {
namespace nwt {

using ring::cp_async4_zfill;
using ring::kAll;

constexpr int kW = 8;
constexpr int kThreads = 32 * kW;
constexpr int kCW = 16;
constexpr int kRW = 64;
constexpr int kPT = 4;                // reverse: steps loaded ahead (a divisor of kCW)
constexpr int kMaxL1 = 8192;
constexpr int kMaxL2 = 1000000;
constexpr float kNInf = -1.0e30f;     // no value (lanes outside the problem)
constexpr float kLow = -0.5e30f;

struct WarpSmem {
    float ring[32 * kRW];             // forward: scores; reverse: outputs before their store
};
struct CtaSmem {
    WarpSmem w[kW];
    float4 binF[kW][kCW];             // forward: the row above (alpha - O, O, f - D, D)
    float4 bbinR[kW][kCW];            // reverse: flows from the row below (flow, q, -, -)
    int progF[kW], progR[kW];
    int err;
    double red[kW];
};

__host__ __device__ inline int nrb_of(int L1m) { return (L1m + 31) / 32; }
__host__ __device__ inline int steps_of(int L2m) { return (L2m + 31 + kCW - 1) / kCW * kCW; }
__host__ __device__ inline size_t slots_of(int L1m, int L2m) { return (size_t)nrb_of(L1m) * steps_of(L2m) * 32; }
__host__ __device__ inline size_t row_elems(int L2m) { return (size_t)L2m + kCW + 1; }
__host__ __device__ inline size_t per_problem_bytes(int L1m, int L2m) {
    const size_t sl = slots_of(L1m, L2m), nr = (size_t)nrb_of(L1m) * row_elems(L2m);
    return 2 * ring::align_up(sl * sizeof(float4), 256) + 2 * ring::align_up(nr * sizeof(float4), 256) +
           2 * ring::align_up((size_t)nrb_of(L1m) * steps_of(L2m) * 4, 256);
}

template <int MODE>
__global__ void __launch_bounds__(kThreads, 2) nw_wave_tan_kernel(SwArgs p) {
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
    constexpr bool PG = MODE == MODE_PGAP, PT = MODE == MODE_PT, HV = MODE == MODE_HVP;
    const float gap = p.gap_dev ? __ldg(p.gap_dev) : p.gap;
    const float T = p.temp_dev ? __ldg(p.temp_dev) : p.temp;
    const float iT = 1.f / T;
    const size_t plane = (size_t)L1m * L2m;
    const float* __restrict__ Sc = p.scores + (size_t)b * plane;
    const float* __restrict__ Vin = HV ? p.tangent + (size_t)b * plane : nullptr;
    float* __restrict__ out = p.out ? p.out + (size_t)b * plane : nullptr;
    const float* __restrict__ Gw = p.dot_with ? p.dot_with + (size_t)b * plane : nullptr;
    const int TP = steps_of(L2m);
    char* base = reinterpret_cast<char*>(p.ws) + (size_t)b * per_problem_bytes(L1m, L2m);
    const size_t sl = slots_of(L1m, L2m), nr = (size_t)nrb_of(L1m) * row_elems(L2m);
    float4* const Wp = reinterpret_cast<float4*>(base);   // (w_d, w_u, w_l, f)
    float4* const Xp = Wp + ring::align_up(sl * sizeof(float4), 256) / sizeof(float4);   // HVP: V; PT: (alpha, E[v], s)
    float4* const bnd = Xp + ring::align_up(sl * sizeof(float4), 256) / sizeof(float4);
    float4* const bbr = bnd + ring::align_up(nr * sizeof(float4), 256) / sizeof(float4);
    float* const Dst = reinterpret_cast<float*>(bbr + ring::align_up(nr * sizeof(float4), 256) / sizeof(float4));
    float* const Ost = Dst + ring::align_up((size_t)nrb_of(L1m) * TP * 4, 256) / 4;
    const int nRB = nrb_of(L1);
    const int nst = (L2 + 31 + kCW - 1) / kCW;
    WarpSmem& ws = sm.w[warp];

    if (tid < kW) {
        sm.progF[tid] = -1;
        sm.progR[tid] = -1;
    }
    if (tid == 0) sm.err = 0;
    if (out && (L1 < L1m || L2 < L2m)) {   // zeros outside the problem
        for (int i = 0; i < L1m; ++i)
            for (int j = (i < L1 ? L2 : 0) + tid; j < L2m; j += kThreads) out[(size_t)i * L2m + j] = 0.f;
    }
    __syncthreads();
    const float ratio = (float)L1 / (float)(L1 + L2);   // the main diagonal's row on an anti-diagonal

    // ------------------------------------------------------------- forward
    for (int rb = warp; rb < nRB; rb += kW) {
        const int i = 32 * rb + lane + 1;
        const bool rowok = i <= L1;
        const size_t poff = (size_t)rb * TP * 32 + lane;
        const float* vrow = HV ? Vin + (size_t)(rowok ? i - 1 : 0) * L2m : nullptr;
        // V of this lane's column, two steps ahead (steps t and t + 1 in flight)
        auto vload = [&](int jj) { return HV && rowok && jj >= 1 && jj <= L2 ? __ldg(vrow + (jj - 1)) : 0.f; };
        float vcur = vload(1 - lane), vnext = vload(2 - lane);
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
        float prev = kNInf, prevF = 0.f;        // own outputs of the previous step (rel O, D)
        float upPrev = kNInf, upPrevF = 0.f;    // the up received the step before
        float dprev = 0.f, ddprev = 0.f, O = 0.f, Dfr = 0.f;
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
                    sm.binF[warp][lane] = jj <= L2 ? __ldcg(bin_g + jj) : make_float4(kNInf, 0.f, 0.f, 0.f);
                }
                __syncwarp();
            }
#pragma unroll 2
            for (int q = 0; q < kCW; ++q) {
                const int t = c * kCW + q;
                const float an = __shfl_sync(kAll, prev, lstar), anF = __shfl_sync(kAll, prevF, lstar);
                const float d = an > kLow ? rintf(an) : 0.f;
                const float dd = an > kLow ? rintf(anF) : 0.f;
                const int j = t - lane + 1;
                // up: (i-1, j)
                float up = __shfl_up_sync(kAll, prev, 1), upF = __shfl_up_sync(kAll, prevF, 1);
                if (lane == 0) {
                    if (rb == 0) {   // row 0: j gap (the gap tangent j)
                        up = fmaf((float)j, gap, -O);
                        upF = (PG ? (float)j : 0.f) - Dfr;
                    } else {
                        const float4 bv = sm.binF[warp][q];
                        up = bv.x + (bv.y - O);
                        upF = bv.z + (bv.w - Dfr);
                    }
                }
                // diag: (i-1, j-1), the up of the step before; left: (i, j-1)
                float dg = upPrev - dprev, dgF = upPrevF - ddprev;
                float lf = prev, lfF = prevF;
                if (j == 1) {   // column 0: i gap
                    dg = fmaf((float)(i - 1), gap, -O);
                    dgF = (PG ? (float)(i - 1) : 0.f) - Dfr;
                    lf = fmaf((float)i, gap, -O);
                    lfF = (PG ? (float)i : 0.f) - Dfr;
                }
                const bool live = rowok && j >= 1 && j <= L2;
                float o = kNInf, oF = 0.f;
                float4 wq = make_float4(0.f, 0.f, 0.f, 0.f), xq = wq;
                if (live) {
                    const float sc = ws.ring[lane * kRW + ((t - lane) & (kRW - 1))];
                    const float vv = vcur;
                    const float vd = dg + sc, vu = up + gap, vl = lf + gap;
                    const float m = fmaxf(vd, fmaxf(vu, vl));
                    const float ed = expf((vd - m) * iT), eu = expf((vu - m) * iT), el = expf((vl - m) * iT);
                    const float sum = (ed + eu) + el;
                    const float a = fmaf(T, logf(sum), m);
                    const float is = 1.f / sum;
                    const float wd = ed * is, wu = eu * is, wl = el * is;
                    float td = dgF, tu = upF, tl = lfF;
                    if (HV) td += vv;
                    if (PG) {
                        tu += 1.f;
                        tl += 1.f;
                    }
                    float f = fmaf(wd, td, fmaf(wu, tu, wl * tl));
                    float ev = 0.f;
                    if (PT) {
                        ev = fmaf(wd, vd, fmaf(wu, vu, wl * vl));
                        f = fmaf(a - ev, iT, f);
                    }
                    o = a - d;
                    oF = f - dd;
                    wq = make_float4(wd, wu, wl, oF);
                    if (HV) xq.x = vv;
                    if (PT) xq = make_float4(o, ev - d, sc, 0.f);
                }
                vcur = vnext;
                vnext = vload(j + 2);
                const size_t pi = poff + (size_t)t * 32;
                Wp[pi] = wq;
                if (!PG) Xp[pi] = xq;
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
                // anchor: the lane nearest the main diagonal (where the alignment mass is)
                const int lo = max(0, t - L2 + 1), hi = min(t, hiRow);
                const int lc = (int)rintf((float)(32 * rb + t + 2) * ratio) - (32 * rb + 1);
                lstar = lo <= hi ? min(max(lc, lo), hi) : 0;
            }
            if (lane == 31) ring::st_release(&sm.progF[warp], (rb << 16) | (c + 1));
        }
        ring::cp_async_wait0();
        __syncwarp();
    }
    __syncthreads();

    // ------------------------------------------------------------- reverse
    constexpr bool XPT = PT;
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
        const float4* Wup = Wp + rup * TP * 32 + 31;
        const float4* Xup = Xp + rup * TP * 32 + 31;
        const int T0 = L2 + 30;
        float4 wbuf[kPT], xbuf[kPT];
#pragma unroll
        for (int s = 0; s < kPT; ++s) {
            const size_t pi = poff + (size_t)max(T0 - s, 0) * 32;
            wbuf[s] = Wp[pi];
            xbuf[s] = PG ? make_float4(0.f, 0.f, 0.f, 0.f) : Xp[pi];
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
        float Lf = 0.f, Lq = 0.f, Df = 0.f, Dq = 0.f, Xf = 0.f, Xq = 0.f;
        const bool below = rb + 1 < nRB;
        const int prodKey = (n - 1) << 16;
        const float4* bb_in = bbr + (size_t)rb * row_elems(L2m);
        float4* bb_out = bbr + rup * row_elems(L2m);
        for (int c = 0; c < nst; ++c) {
            if (below) {
                ring::wait_flag(&sm.progR[(n - 1) % kW], prodKey | min(c + 3, nst), &sm.err);
                if (lane < kCW) {
                    const int jj = L2 - (c * kCW + lane);
                    sm.bbinR[warp][lane] = jj >= 1 ? __ldcg(bb_in + jj) : make_float4(0.f, 0.f, 0.f, 0.f);
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
                const float fl0 = wbuf[(q + 1) % kPT].w;
                float fu = __shfl_up_sync(kAll, fl0, 1);
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
                if (PT) {
                    al = xbuf[(q + 1) % kPT].x;
                    au = __shfl_up_sync(kAll, al, 1);
                    ad = __shfl_up_sync(kAll, xbuf[(q + 2) % kPT].x, 1);
                }
                {
                    const size_t pi = poff + (size_t)max(t - kPT, 0) * 32;
                    wbuf[q % kPT] = Wp[pi];
                    if (!PG) xbuf[q % kPT] = Xp[pi];
                }
                float xf = __shfl_down_sync(kAll, Xf, 1), xq2 = __shfl_down_sync(kAll, Xq, 1);
                if (lane == 31) {
                    const float4 bv = below ? sm.bbinR[warp][q] : make_float4(0.f, 0.f, 0.f, 0.f);
                    xf = bv.x;
                    xq2 = bv.y;
                }
                const int j = t - lane + 1;
                const bool live = rowok && j >= 1 && j <= L2;
                const float seed = (i == L1 && j == L2) ? 1.f : 0.f;
                float beta = 0.f, r = 0.f;
                if (live) {
                    beta = (seed + Lf) + xf;
                    r = Lq + xq2;
                }
                // predecessors' frames: left t-1, up t-1 / diag t-2 (lane 0: the row above's t+31 / t+30);
                // boundary predecessors (column 0, row 0) in absolute terms with frame 0
                const float Dt = __ldg(Drb + t);
                float Dl = __ldg(Drb + max(t - 1, 0)), Dd = __ldg(Drb + max(t - 2, 0));
                const float Dua = __ldg(Dup + su), Dda = __ldg(Dup + sd);
                float Ot = 0.f, Ol = 0.f, Od = 0.f, Oua = 0.f, Oda = 0.f;
                if (PT) {
                    Ot = __ldg(Orb + t);
                    Ol = __ldg(Orb + max(t - 1, 0));
                    Od = __ldg(Orb + max(t - 2, 0));
                    Oua = __ldg(Oup + su);
                    Oda = __ldg(Oup + sd);
                }
                float fl = fl0, Du = Dl, Ddg = Dd, Ou = Ol, Odg = Od;
                if (lane == 0 && rb > 0) {
                    fu = fua;
                    fd = fda;
                    au = aua;
                    ad = ada;
                    Du = Dua;
                    Ddg = Dda;
                    Ou = Oua;
                    Odg = Oda;
                }
                if (lane == 0 && rb == 0) {   // row 0: up (0, j), diagonal (0, j-1)
                    fu = PG ? (float)j : 0.f;
                    fd = PG ? (float)(j - 1) : 0.f;
                    au = (float)j * gap;
                    ad = (float)(j - 1) * gap;
                    Du = Ddg = Ou = Odg = 0.f;
                }
                if (j == 1) {   // column 0: left (i, 0), diagonal (i-1, 0)
                    fl = PG ? (float)i : 0.f;
                    fd = PG ? (float)(i - 1) : 0.f;
                    al = (float)i * gap;
                    ad = (float)(i - 1) * gap;
                    Dl = Ddg = Ol = Odg = 0.f;
                }
                // message to predecessor k with weight w: r w + b dw
                float eu = wv.w;
                if (PT) eu -= (xv.x - xv.y) * iT;
                auto msg = [&](float w, float fk, float Dk, float ak, float Ok, bool diag) {
                    float dv = fk + (Dk - Dt);
                    if (HV && diag) dv += xv.x;
                    if (PG && !diag) dv += 1.f;
                    float dw = w * (dv - eu) * iT;
                    if (PT) {
                        const float v = ak + ((diag ? xv.z : gap) + (Ok - Ot));
                        dw = fmaf(w * (xv.y - v), iT * iT, dw);
                    }
                    return fmaf(r, w, beta * dw);
                };
                Lf = beta * wv.z;
                Lq = msg(wv.z, fl, Dl, al, Ol, false);
                Xf = fmaf(beta, wv.y, Df);
                Xq = msg(wv.y, fu, Du, au, Ou, false) + Dq;
                Df = beta * wv.x;
                Dq = msg(wv.x, fd, Ddg, ad, Odg, true);
                // the marginal's tangent r w_d + b dw_d: the diagonal message
                if (live) ws.ring[lane * kRW + ((t - lane) & (kRW - 1))] = Dq;
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

}  // namespace nwt

size_t nw_wave_tan_area(int B, int L1, int L2) {
    return ring::align_up(nwt::per_problem_bytes(L1, L2) * (size_t)(B > 0 ? B : 1), 256);
}

// a.mode MODE_HVP (a.tangent, a.out), MODE_PGAP or MODE_PT (a.out, and / or
// dot_out[b] = sum dot_with * dP with a.dot_with); a.redo a zeroed flag per
// problem.  Returns -1 when the shape is not covered (nothing launched).
int launch_nw_wave_tan(const SwArgs& a, cudaStream_t st) {
    if (!a.redo || a.L1 > nwt::kMaxL1 || a.L2 > nwt::kMaxL2 || a.L1 < 1 || a.L2 < 1) return -1;
    if (a.mode == MODE_HVP && (!a.out || !a.tangent)) return -1;
    if ((a.mode == MODE_PGAP || a.mode == MODE_PT) && !a.out && !(a.dot_with && a.dot_out)) return -1;
    if (a.mode != MODE_HVP && a.mode != MODE_PGAP && a.mode != MODE_PT) return -1;
    if (a.B == 0) return 0;
    static DeviceSetup setup;
    int dev = 0, sms = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return (int)e;
    const size_t smem = sizeof(nwt::CtaSmem);
    int rc = device_setup(setup, dev, [smem] {
        const void* ks[] = {(const void*)nwt::nw_wave_tan_kernel<MODE_HVP>, (const void*)nwt::nw_wave_tan_kernel<MODE_PGAP>,
                            (const void*)nwt::nw_wave_tan_kernel<MODE_PT>};
        cudaError_t r = cudaSuccess;
        for (const void* k : ks)
            if (r == cudaSuccess) r = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        return (int)r;
    }, &sms);
    if (rc) return rc;
    switch (a.mode) {
        case MODE_HVP: nwt::nw_wave_tan_kernel<MODE_HVP><<<a.B, nwt::kThreads, smem, st>>>(a); break;
        case MODE_PGAP: nwt::nw_wave_tan_kernel<MODE_PGAP><<<a.B, nwt::kThreads, smem, st>>>(a); break;
        default: nwt::nw_wave_tan_kernel<MODE_PT><<<a.B, nwt::kThreads, smem, st>>>(a); break;
    }
    return (int)cudaGetLastError();
}

}  // namespace d2pb
