// sw_affine_fast.cu -- linear-domain fast path for affine-gap soft
// Smith-Waterman value + marginals.
//
// The reference's three-state log-sum-exp recurrence
// (src/sw_affine/kernels_cpu.cpp:94-197) in the linear domain, with
// P = 2^(s c), Go = 2^(gap_open c), Ge = 2^(gap_ext c), c = log2(e)/T:
//   M_ij = P_ij (T_{i-1,j-1} + 1)            T = M + I + D
//   I_ij = Go M_{i-1,j} + Ge I_{i-1,j}       (gap in the second sequence)
//   D_ij = Go M_{i,j-1} + Ge D_{i,j-1}       (gap in the first sequence)
//   Z_total = 1 + sum_ij T_ij
// and its reverse (src/sw_affine/kernels_cpu.cpp:199-346) as outside sums:
//   BM_ij = 1 + P_{i+1,j+1} BM_{i+1,j+1} + Go BI_{i+1,j} + Go BD_{i,j+1}
//   BI_ij = 1 + P_{i+1,j+1} BM_{i+1,j+1} + Ge BI_{i+1,j}
//   BD_ij = 1 + P_{i+1,j+1} BM_{i+1,j+1} + Ge BD_{i,j+1}
//   marginal_ij = BM_ij M_ij / Z_total
// (cells outside the problem are 0; the diagonal inputs of row 1 and column
// 1 are 0, the reference's `dg` condition).
//
// Organisation, frames, stages, boundary rows and fix-up contract are those
// of the linear kernel (sw_linear.cu), with two values per neighbour:
//   forward:  lane l-1 sends (u, T) of its cell (i-1, j): u = Go M + Ge I is
//             I_ij, and T becomes the diagonal input of (i, j+1);
//   reverse:  lane l+1 sends (BI, X) of its cell (i+1, j): BI is the Y input
//             of (i, j) and X = P BM of its previous cell (i+1, j+1).
// The forward stores M per cell (all the reverse needs of it): marginal =
// BM M 2^(Q + E - S).  One frame per lane covers all three states.
#include <cuda_bf16.h>
#include <stddef.h>
#include <stdint.h>

#include "sw_common.cuh"
#include "sw_internal.h"
#include "sw_lindomain.cuh"
#include "sw_ring.cuh"

namespace d2pb {
namespace aff {
using namespace ring;
using namespace ld;

constexpr int kMaxRB = 512;              // row-blocks per problem (L1 <= 16384)
constexpr int kNW = 6;                   // warps per CTA, two CTAs per SM
constexpr int kNWWide = 12;              // warps per CTA when the batch leaves SMs idle (one CTA per SM)

struct WarpSmem {
    float ringS[32 * kRW];    // scores [rows][64]; reverse: marginals written in place
    float zr[2][16 * 32];     // reverse: the forward's M of 16 anti-diagonals, two slots
    float er[16 * 32];        // reverse: forward frames, 16 group slots
    // staging of the neighbouring row-block's boundary values: two per step
    // (forward u, T of the row above's last lane; reverse BI, X of the
    // row-block below's lane 0) and its frames, by its group
    float sa[kHR];
    float sb[kHR];
    float sf[kHR / 4];
    // which neighbour stage each of the 8 stage slots holds when the
    // neighbour pushed it there itself: (ordinal << 16) | stage
    int tag[kHR / 16];
};
static_assert(sizeof(WarpSmem) % 16 == 0, "per-warp shared blocks must stay 16-byte aligned");
static_assert(offsetof(WarpSmem, sb) == offsetof(WarpSmem, sa) + 4 * kHR &&
                  offsetof(WarpSmem, sf) == offsetof(WarpSmem, sa) + 8 * kHR,
              "sa, sb, sf are contiguous");

struct Layout {  // per-problem workspace
    float* mpl;      // [nRB][ZT][32]   M of forward step t (frame E) at row t
    float* efr;      // [nRB][GT][32]   frame of each lane for each group of 4 forward steps
    float* hva;      // [nRB][ZT]       boundary values of each row-block by its step: u / BI
    float* hvb;      // [nRB][ZT]                                                    T / X
    float* hfr;      // [nRB][GT]       and their frames, by its group
};
__host__ __device__ inline size_t per_problem_bytes(int L1m, int L2m) {
    const size_t nrb = (size_t)(L1m + 31) / 32;
    return align_up(nrb * zt_rows(L2m) * 32 * 4, 256) + align_up(nrb * gt_rows(L2m) * 32 * 4, 256) +
           2 * align_up(nrb * hz_stride(L2m) * 4, 256) + align_up(nrb * hf_stride(L2m) * 4, 256);
}
__device__ inline Layout carve(float* ws, int b, int L1m, int L2m) {
    const size_t nrb = (size_t)(L1m + 31) / 32;
    char* base = (char*)ws + (size_t)b * per_problem_bytes(L1m, L2m);
    Layout L;
    L.mpl = (float*)base;
    base += align_up(nrb * zt_rows(L2m) * 32 * 4, 256);
    L.efr = (float*)base;
    base += align_up(nrb * gt_rows(L2m) * 32 * 4, 256);
    L.hva = (float*)base;
    base += align_up(nrb * hz_stride(L2m) * 4, 256);
    L.hvb = (float*)base;
    base += align_up(nrb * hz_stride(L2m) * 4, 256);
    L.hfr = (float*)base;
    return L;
}

// One group of the boundary lane's (bnd) two values and its frame: into the
// staging ring of the consumer row-block's warp while it keeps up (push, pp;
// ring at shared address pv: sa, sb, sf), else to the row-block's boundary
// rows in global memory, from where the consumer copies it (the linear
// kernel's handoff, sw_linear.cu).
template <class Ctx>
__device__ __forceinline__ void handoff(const Ctx& C, int g, float4 a, float4 b, float fr, bool bnd, bool pp) {
    stg_pair_pred(C.oa + 4 * g, C.ob + 4 * g, C.of + g, a, b, fr, bnd && !pp);
    const unsigned sa = C.pv + 16u * (unsigned)(g & (kHR / 4 - 1));
    sts_group_pred_s(sa, C.pv + 8u * kHR + 4u * (unsigned)(g & (kHR / 4 - 1)), a, fr, pp);
    sts_group_pred_s(sa + 4u * kHR, C.pv + 8u * kHR + 4u * (unsigned)(g & (kHR / 4 - 1)), b, fr, pp);
}

// ==========================================================================
// forward
// ==========================================================================
struct FwdF {
    float d0, d1;       // 2^(E_{l-1} - E) for the inputs of the first / other steps (lane 0: 0)
    float Ged0, Ged1;   // Ge d0, Ge d1
    float fs;           // 2^-E
    float ua[4];        // lane 0: I from the row above for each step, frame E (other lanes: 0)
    float ta[4];        // lane 0: T of the row above's cell (i-1, j) for each step (the next diagonal)
};

struct FwdVars {
    bool push;          // lane 31, this stage: its values go to the consumer's staging ring
    float Mp, Dp, Td;   // own M, D of the previous step; diagonal T of this step (own frame)
    float ur, Tr;       // lane l-1's u and T of the previous step (its frame)
    float Tl;           // own T of the previous step (frame anchor)
    float E, Esent;
    FwdF f;
    float nE, nfJ;
    FwdF nf;
    float gsum;
    double acc;         // partition of this lane's cells so far: sum T 2^-ab
    float ab;           // base (log2) of acc, raised with the frames
    int ebmin, ebmax;
    float emax;         // largest E - ab of a group
};

struct FwdCtx {
    const float* ring;
    const float* au;    // lane 0: the row above's u, T staged by its step, frames by group; zeros otherwise
    const float* at;
    const float* af;
    float* oa;          // this row-block's boundary rows (global) for the row-block below: u, T
    float* ob;
    float* of;
    unsigned pv;        // shared address of the staging ring of the warp computing the row-block below
    float* mrow;        // mpl row 0 of this row-block, this lane
    float* erow;
    float c, Go, Ge;
    float notl0;
    int lane, nv, L2;
    bool l0, l31;
};

__device__ __forceinline__ FwdF fwd_factors(const FwdCtx& C, float E, float eup0, float eup1) {
    FwdF f;
    f.d0 = p2(eup0 - E) * C.notl0;
    f.d1 = p2(eup1 - E) * C.notl0;
    f.Ged0 = C.Ge * f.d0;
    f.Ged1 = C.Ge * f.d1;
    f.fs = p2(-E);
#pragma unroll
    for (int q = 0; q < 4; ++q) f.ua[q] = f.ta[q] = 0.f;
    return f;
}

// next group's frame and factors (see fwd_lookahead in sw_linear.cu); lane 0
// takes the frames of the row above's last lane, whose step 4g + 31 (group
// g + 7) feeds lane 0's step 4g and steps 4g + 32 .. 4g + 34 (group g + 8) the rest
__device__ __forceinline__ void fwd_lookahead(const FwdCtx& C, FwdVars& V, int g) {
    const int eb = efield(V.Tl);
    V.ebmin = min(V.ebmin, eb);
    V.ebmax = max(V.ebmax, eb);
    const float ea0 = C.af[(g + 7) & (kHR / 4 - 1)], ea1 = C.af[(g + 8) & (kHR / 4 - 1)];
    const float w = p2(ea0 - ea1);
    V.nE = C.l0 ? ea1 : V.E + efield_j(eb);
    V.nfJ = C.l0 ? w : __int_as_float(0x7f000000 - eb);
    const float p2J = C.l0 ? inv_p2(w) : __int_as_float(eb);
    const float p2Jup = __shfl_up_sync(kAll, p2J, 1);
    V.nf.d0 = V.f.d1 * V.nfJ;
    V.nf.d1 = V.nf.d0 * p2Jup;
    V.nf.Ged0 = C.Ge * V.nf.d0;
    V.nf.Ged1 = C.Ge * V.nf.d1;
    V.nf.fs = p2(-V.nE);
    const int s0 = (4 * g + 31) & (kHR - 1), s1 = (4 * g + 32) & (kHR - 1);
    const float4 u = *reinterpret_cast<const float4*>(C.au + s1);
    const float4 t = *reinterpret_cast<const float4*>(C.at + s1);
    V.nf.ua[0] = C.au[s0] * w;
    V.nf.ua[1] = u.x;
    V.nf.ua[2] = u.y;
    V.nf.ua[3] = u.z;
    V.nf.ta[0] = C.at[s0] * w;
    V.nf.ta[1] = t.x;
    V.nf.ta[2] = t.y;
    V.nf.ta[3] = t.z;
}

__device__ __forceinline__ void fwd_apply(FwdVars& V) {
    const float dE = V.E - V.ab;
    V.acc = fma((double)V.gsum, p2d(dE), V.acc);
    V.emax = fmaxf(V.emax, dE);
    V.gsum = 0.f;
    V.Mp *= V.nfJ;
    V.Dp *= V.nfJ;
    V.Td *= V.nfJ;
    V.E = V.nE;
    V.f = V.nf;
}

struct FwdOut {
    float M, D, T, u, Tdn;
};
// one cell, step i of its group
__device__ __forceinline__ FwdOut fwd_cell(const FwdCtx& C, const FwdVars& V, int i, float sc) {
    FwdOut o;
    const float P = ex2f(sc * C.c);
    const float d = i == 0 ? V.f.d0 : V.f.d1;
    o.M = P * (V.Td + V.f.fs);
    const float I = fmaf(V.ur, d, V.f.ua[i]);
    o.D = fmaf(C.Ge, V.Dp, C.Go * V.Mp);
    o.T = o.M + I + o.D;
    o.u = fmaf(i == 0 ? V.f.Ged0 : V.f.Ged1, V.ur, fmaf(C.Go, o.M, C.Ge * V.f.ua[i]));
    o.Tdn = fmaf(V.Tr, d, V.f.ta[i]);
    return o;
}

template <bool MASK>
__device__ __forceinline__ void fwd_stage_full(const FwdCtx& C, FwdVars& V, int k, int thr) {
    const int c0 = (kCW * k - C.lane) & (kRW - 1);
    const float* const pA = C.ring + c0;
    const float* const pB = pA - kRW;
    float scv[kCW];
#pragma unroll
    for (int u = 0; u < kCW; ++u) scv[u] = ((u < kRW - c0) ? pA : pB)[u];
    float* const pm = C.mrow + (size_t)(kCW * k) * 32;
    float* const pe = C.erow + (size_t)(kCW * k / 4) * 32;
    float uq[4], tq[4];
#pragma unroll
    for (int u = 0; u < kCW; ++u) {
        const int i = u & 3;
        if (i == 0) fwd_apply(V);
        if (i == 3) {
            if (u == kCW - 1) cp_async_wait1();  // the last look-ahead's boundary values (copied at stage start)
            fwd_lookahead(C, V, 4 * k + (u >> 2) + 1);
        }
        FwdOut o = fwd_cell(C, V, i, scv[u]);
        if (MASK) {
            const bool act = u < thr;
            o.T = act ? o.T : 0.f;
            o.u = act ? o.u : 0.f;
        }
        V.gsum += o.T;
        pm[(size_t)u * 32] = o.M;
        uq[i] = o.u;
        tq[i] = o.T;
        if (i == 3) {
            const int g = 4 * k + (u >> 2);
            pe[(u >> 2) * 32] = V.E;
            handoff(C, g, make_float4(uq[0], uq[1], uq[2], uq[3]), make_float4(tq[0], tq[1], tq[2], tq[3]), V.E, C.l31, V.push);
        }
        V.Mp = o.M;
        V.Dp = o.D;
        V.Td = o.Tdn;
        V.Tl = o.T;
        V.ur = __shfl_up_sync(kAll, o.u, 1);
        V.Tr = __shfl_up_sync(kAll, o.T, 1);
    }
}

__device__ __forceinline__ void fwd_stage_start(const FwdCtx& C, FwdVars& V, int k) {
    const bool live = C.lane < C.nv;
    float uq[4], tq[4];
#pragma unroll 1
    for (int q = 0; q < 4; ++q) {
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const int t = kCW * k + 4 * q + i;
            const int j0 = t - C.lane;
            const bool act = live & (j0 >= 0) & (j0 < C.L2);
            if (i == 0) fwd_apply(V);
            const float eup_now = __shfl_up_sync(kAll, V.E, 1);
            if (live && j0 == 0 && !C.l0) {
                V.E = V.Esent;
                V.f = fwd_factors(C, V.E, V.Esent, i == 0 ? eup_now : V.Esent);
            }
            if (i == 3) {
                if (q == 3) cp_async_wait1();
                fwd_lookahead(C, V, 4 * k + q + 1);
            }
            FwdOut o = fwd_cell(C, V, i, C.ring[j0 & (kRW - 1)]);
            o.M = act ? o.M : 0.f;
            o.D = act ? o.D : 0.f;
            o.T = act ? o.T : 0.f;
            o.u = act ? o.u : 0.f;
            V.gsum += o.T;
            C.mrow[(size_t)t * 32] = o.M;
            uq[i] = o.u;
            tq[i] = o.T;
            if (i == 3) {
                const int g = t >> 2;
                C.erow[(size_t)g * 32] = V.E;
                handoff(C, g, make_float4(uq[0], uq[1], uq[2], uq[3]), make_float4(tq[0], tq[1], tq[2], tq[3]), V.E, C.l31, V.push);
            }
            V.Mp = o.M;
            V.Dp = o.D;
            V.Td = act ? o.Tdn : 0.f;
            V.Tl = o.T;
            V.ur = __shfl_up_sync(kAll, o.u, 1);
            V.Tr = __shfl_up_sync(kAll, o.T, 1);
            V.Esent = __shfl_up_sync(kAll, V.E, 1);
        }
    }
}

// ==========================================================================
// reverse
// ==========================================================================
struct RevF {
    float d0, d1;       // 2^(Q_{l+1} - Q) for the messages of the first / other steps (bottom lane: 0)
    float Ged0, Ged1, God0, God1;
    float fsq;          // 2^-Q
    float xa[4], ya[4]; // bottom lane: X and BI from the row-block below, frame Q (other lanes: 0)
    float kE;           // 2^(Q + E - S)
};

struct RevVars {
    bool push;          // lane 0, this stage: its messages go to the consumer's staging ring
    float BDp, PBp;     // own BD and P BM of column j+1
    float Yr, Xr;       // lane l+1's BI and X of the previous step (its frame)
    float BMl;          // own BM of the previous step (frame anchor)
    float Q, Qsent;
    RevF f;
    float nQ, nfJ;
    RevF nf;
    int ebmin, ebmax;
};

struct RevCtx {
    float* ring;
    const float* zr;
    const float* er;
    const float* by;    // bottom lane: the row-block below's BI, X staged by its step (frames by
    const float* bx;    //   group); zeros otherwise
    const float* bf;
    float* oa;          // this row-block's boundary rows (global) for the row-block above: BI, X
    float* ob;
    float* of;
    unsigned pv;        // shared address of the staging ring of the warp computing the row-block above
    float c, Go, Ge, cS;
    float notBot;
    float Sint;
    int lane, nv, L2, P;
    bool l0, bot;
};

__device__ __forceinline__ void rev_kfactors(const RevCtx& C, RevF& f, float Q, int h) {
    const int gA = C.P / 4 + 7 - h;
    f.kE = p2(Q + C.er[(gA & 15) * 32 + C.lane] - C.Sint) * C.cS;
}

__device__ __forceinline__ RevF rev_factors(const RevCtx& C, float Q, float qdn0, float qdn1, int h) {
    RevF f;
    f.d0 = p2(qdn0 - Q) * C.notBot;
    f.d1 = p2(qdn1 - Q) * C.notBot;
    f.Ged0 = C.Ge * f.d0;
    f.Ged1 = C.Ge * f.d1;
    f.God0 = C.Go * f.d0;
    f.God1 = C.Go * f.d1;
    f.fsq = p2(-Q);
#pragma unroll
    for (int q = 0; q < 4; ++q) f.xa[q] = f.ya[q] = 0.f;
    rev_kfactors(C, f, Q, h);
    return f;
}

// the bottom lane follows the frames of the row-block below's lane 0, whose
// step tau + 31 (same column) feeds step tau here: entry 4h + 31 (its group
// h + 7) for the group's first step, 4h + 32 .. 4h + 34 (group h + 8) the rest
__device__ __forceinline__ void rev_lookahead(const RevCtx& C, RevVars& V, int h) {
    const int eb = efield(V.BMl);
    V.ebmin = min(V.ebmin, eb);
    V.ebmax = max(V.ebmax, eb);
    const float qb0 = C.bf[(h + 7) & (kHR / 4 - 1)], qb1 = C.bf[(h + 8) & (kHR / 4 - 1)];
    const float w = p2(qb0 - qb1);
    V.nQ = C.bot ? qb1 : V.Q + efield_j(eb);
    V.nfJ = C.bot ? w : __int_as_float(0x7f000000 - eb);
    const float p2J = C.bot ? inv_p2(w) : __int_as_float(eb);
    const float p2Jdn = __shfl_down_sync(kAll, p2J, 1);
    V.nf.d0 = V.f.d1 * V.nfJ;
    V.nf.d1 = V.nf.d0 * p2Jdn;
    V.nf.Ged0 = C.Ge * V.nf.d0;
    V.nf.Ged1 = C.Ge * V.nf.d1;
    V.nf.God0 = C.Go * V.nf.d0;
    V.nf.God1 = C.Go * V.nf.d1;
    V.nf.fsq = p2(-V.nQ);
    const int s0 = (4 * h + 31) & (kHR - 1), s1 = (4 * h + 32) & (kHR - 1);
    const float4 y = *reinterpret_cast<const float4*>(C.by + s1);
    const float4 x = *reinterpret_cast<const float4*>(C.bx + s1);
    V.nf.ya[0] = C.by[s0] * w;
    V.nf.ya[1] = y.x;
    V.nf.ya[2] = y.y;
    V.nf.ya[3] = y.z;
    V.nf.xa[0] = C.bx[s0] * w;
    V.nf.xa[1] = x.x;
    V.nf.xa[2] = x.y;
    V.nf.xa[3] = x.z;
    rev_kfactors(C, V.nf, V.nQ, h);
}

__device__ __forceinline__ void rev_apply(RevVars& V) {
    V.BDp *= V.nfJ;
    V.PBp *= V.nfJ;
    V.Q = V.nQ;
    V.f = V.nf;
}

struct RevOut {
    float BM, BI, BD, PB, mu;
};
__device__ __forceinline__ RevOut rev_cell(const RevCtx& C, const RevVars& V, int i, float sc, float m) {
    RevOut o;
    const float P = ex2f(sc * C.c);
    const float c1 = V.f.fsq + fmaf(V.Xr, i == 0 ? V.f.d0 : V.f.d1, V.f.xa[i]);
    o.BD = fmaf(C.Ge, V.BDp, c1);
    o.BI = fmaf(i == 0 ? V.f.Ged0 : V.f.Ged1, V.Yr, fmaf(C.Ge, V.f.ya[i], c1));
    o.BM = fmaf(i == 0 ? V.f.God0 : V.f.God1, V.Yr, fmaf(C.Go, V.f.ya[i], fmaf(C.Go, V.BDp, c1)));
    o.PB = P * o.BM;
    o.mu = o.BM * (m * V.f.kE);
    return o;
}

template <bool MASK>
__device__ __forceinline__ void rev_stage_full(const RevCtx& C, RevVars& V, int k, int thr) {
    const int m16 = C.P + 16 - kCW * k;
    const float* const zb = C.zr + ((m16 >> 4) & 1) * (16 * 32) + C.lane;
    const int cb = (C.P + 31 - kCW * k - C.lane) & (kRW - 1);
    float* const qA = C.ring + cb;
    float* const qB = qA + kRW;
    float scv[kCW];
#pragma unroll
    for (int u = 0; u < kCW; ++u) scv[u] = (((u <= cb) ? qA : qB) - u)[0];
    float yq[4], xq[4];
#pragma unroll
    for (int u = 0; u < kCW; ++u) {
        const int i = u & 3;
        if (i == 0) rev_apply(V);
        if (i == 3) {
            if (u == kCW - 1) cp_async_wait1();
            rev_lookahead(C, V, 4 * k + (u >> 2) + 1);
        }
        RevOut o = rev_cell(C, V, i, scv[u], zb[(15 - u) * 32]);
        (((u <= cb) ? qA : qB) - u)[0] = o.mu;
        if (MASK) {
            const bool act = u < thr;
            o.BM = act ? o.BM : 0.f;
            o.BI = act ? o.BI : 0.f;
            o.BD = act ? o.BD : 0.f;
            o.PB = act ? o.PB : 0.f;
        }
        const float xs = V.PBp;  // X for the row above's next cell: P BM of this lane's previous cell
        yq[i] = o.BI;
        xq[i] = xs;
        if (i == 3) {
            const int h = 4 * k + (u >> 2);
            handoff(C, h, make_float4(yq[0], yq[1], yq[2], yq[3]), make_float4(xq[0], xq[1], xq[2], xq[3]), V.Q, C.l0, V.push);
        }
        V.Yr = __shfl_down_sync(kAll, o.BI, 1);
        V.Xr = __shfl_down_sync(kAll, xs, 1);
        V.BDp = o.BD;
        V.PBp = o.PB;
        V.BMl = o.BM;
    }
}

__device__ __forceinline__ void rev_stage_part(const RevCtx& C, RevVars& V, int k) {
    const int m16 = C.P + 16 - kCW * k;
    const float* const zb = C.zr + ((m16 >> 4) & 1) * (16 * 32) + C.lane;
    const bool live = C.lane < C.nv;
    float yq[4], xq[4];
#pragma unroll 1
    for (int q = 0; q < 4; ++q) {
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const int u = 4 * q + i;
            const int tf = m16 + 15 - u;
            const int j0 = tf - C.lane;
            const bool act = live & (j0 >= 0) & (j0 < C.L2);
            if (i == 0) rev_apply(V);
            const float qdn_now = __shfl_down_sync(kAll, V.Q, 1);
            if (live && j0 == C.L2 - 1 && !C.bot) {
                V.Q = 0.f;
                V.f = rev_factors(C, 0.f, V.Qsent, i == 0 ? qdn_now : V.Qsent, 4 * k + q);
            }
            if (i == 3) {
                if (q == 3) cp_async_wait1();
                rev_lookahead(C, V, 4 * k + q + 1);
            }
            const int ci = j0 & (kRW - 1);
            RevOut o = rev_cell(C, V, i, C.ring[ci], zb[(15 - u) * 32]);
            if (act) C.ring[ci] = o.mu;
            o.BM = act ? o.BM : 0.f;
            o.BI = act ? o.BI : 0.f;
            o.BD = act ? o.BD : 0.f;
            o.PB = act ? o.PB : 0.f;
            const float xs = V.PBp;
            yq[i] = o.BI;
            xq[i] = xs;
            if (i == 3) {
                const int h = 4 * k + q;
                handoff(C, h, make_float4(yq[0], yq[1], yq[2], yq[3]), make_float4(xq[0], xq[1], xq[2], xq[3]), V.Q, C.l0, V.push);
            }
            V.Yr = __shfl_down_sync(kAll, o.BI, 1);
            V.Xr = __shfl_down_sync(kAll, xs, 1);
            V.BDp = o.BD;
            V.PBp = o.PB;
            V.BMl = o.BM;
            V.Qsent = __shfl_down_sync(kAll, V.Q, 1);
        }
    }
}

// ==========================================================================
// kernel
// ==========================================================================
// SPLIT: the launch is cooperative and spreads each problem over p.parts CTAs
// (sw_linear.cu's scheme): row-block r goes to warp r mod NW of part
// (r / NW) mod parts, the handoff from a part's last warp to the next part's
// warp 0 takes the global route, and the progress words, the forward ->
// reverse barrier and the partition partials sit in the problem's p.sync words.
template <int NW, int MINB, bool SPLIT>
__global__ void __launch_bounds__(NW * 32, MINB) aff_fast_kernel(SwArgs p) {
    extern __shared__ __align__(16) unsigned char smem_raw[];
    WarpSmem& W = reinterpret_cast<WarpSmem*>(smem_raw)[threadIdx.x >> 5];
    __shared__ int progF[NW], progR[NW];
    __shared__ __align__(16) float red[4 * 32];
    __shared__ int sh_Sint, sh_err, sh_bad;
    __shared__ float sh_Sfrac;
    __shared__ __align__(16) float zv[kHR];   // staging of a missing neighbour: zeros
    __shared__ float zf[kHR / 4];

    const int K = SPLIT ? p.parts : 1;
    const int part = SPLIT ? (int)(blockIdx.x % K) : 0;
    const int bi = SPLIT ? (int)(blockIdx.x / K) : (int)blockIdx.x;
    const int b = p.order ? p.order[bi] : bi;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int gw = part * NW + warp, NWt = K * NW;  // this warp among the problem's warps
    // cross-CTA links: warp 0's producer and warp NW-1's consumer sit in the
    // neighbouring parts; their progress words are global
    int* const gsync = SPLIT ? p.sync + (size_t)b * (kSyncBytes / 4) : nullptr;
    const bool xin = SPLIT && K > 1 && warp == 0;
    const bool xout = SPLIT && K > 1 && warp == NW - 1;
    const int pin = (part + K - 1) % K;
    const int L1m = p.L1, L2m = p.L2;
    const int L1 = p.lengths ? min(max(p.lengths[2 * b], 0), L1m) : L1m;
    const int L2 = p.lengths ? min(max(p.lengths[2 * b + 1], 0), L2m) : L2m;
    const float go = p.gap_dev ? __ldg(p.gap_dev) : p.gap;
    const float ge = p.gap2_dev ? __ldg(p.gap2_dev) : p.gap2;
    const float T = p.temp_dev ? __ldg(p.temp_dev) : p.temp;
    const float c = kLog2e / T;
    const float Go = ex2f(go * c), Ge = ex2f(ge * c);
    const size_t plane = (size_t)L1m * L2m;
    const float* __restrict__ S = p.scores + (size_t)b * plane;
    float* __restrict__ out = p.out ? p.out + (size_t)b * plane : nullptr;
    const Layout LY = carve(p.ws, b, L1m, L2m);
    const int nRB = (L1 + 31) / 32;
    const int nch = (L2 + kCW - 1) / kCW;
    const size_t zst = (size_t)zt_rows(L2m) * 32;
    const size_t est = (size_t)gt_rows(L2m) * 32;

    if (out && (L1 < L1m || L2 < L2m)) {
        for (int i = gw; i < L1m; i += NWt) {
            float* row = out + (size_t)i * L2m;
            for (int j = (i < L1 ? L2 : 0) + lane; j < L2m; j += 32) row[j] = 0.f;
        }
    }
    if (L1 == 0 || L2 == 0) {
        if (threadIdx.x == 0 && part == 0) {
            if (p.value) p.value[b] = 0.f;
            if (p.redo) p.redo[b] = 0;
        }
        return;
    }
    if (threadIdx.x < NW) {
        progF[threadIdx.x] = -1;
        progR[threadIdx.x] = -1;
    }
    if (threadIdx.x < kHR) zv[threadIdx.x] = 0.f;
    if (threadIdx.x < kHR / 4) zf[threadIdx.x] = 0.f;
    if (lane < kHR / 16) W.tag[lane] = -1;
    if (threadIdx.x == 0) {
        sh_err = 0;
        sh_bad = 0;
    }
    __syncthreads();
    // the warps of the neighbouring row-blocks: wprev produces this warp's
    // inputs, wnext consumes its outputs
    const int wprev = (warp + NW - 1) % NW, wnext = (warp + 1) % NW;
    WarpSmem& Wn = reinterpret_cast<WarpSmem*>(smem_raw)[wnext];
    const size_t hzst = (size_t)hz_stride(L2m), hfst = (size_t)hf_stride(L2m);

    // Boundary values of the neighbouring row-block, staged by the one lane
    // that reads them, on the linear kernel's schedule (sw_linear.cu): the
    // prologue copies the neighbour's stages 1 and 2 (from step 28 and group 4
    // on); stage k, once the neighbour has finished its stage k+3, copies that
    // stage as a copy group of its own, which the stage's last look-ahead waits
    // for.  Stages the neighbour pushed into the ring itself (tag) are not copied.
    auto copy_stage = [&](int ordinal, int x, const float* ga, const float* gb, const float* gf) {
        if (W.tag[x & (kHR / 16 - 1)] == ((ordinal << 16) | x)) return;  // pushed
        const int s0 = x == 1 ? 28 : kCW * x, ns = x == 1 ? 1 : 4, g0 = 4 * x;
        for (int i = 0; i < ns; ++i) {
            cp_async16(W.sa + ((s0 + 4 * i) & (kHR - 1)), ga + s0 + 4 * i, 16);
            cp_async16(W.sb + ((s0 + 4 * i) & (kHR - 1)), gb + s0 + 4 * i, 16);
        }
        cp_async16(W.sf + (g0 & (kHR / 4 - 1)), gf + g0, 16);
    };
    auto wait_prog = [&](const int* prog, int need) {
        if (xin)
            wait_flag_gpu(prog, need, &sh_err);
        else
            wait_flag(prog, need, &sh_err);
    };
    auto stage_first = [&](const int* prog, int ordinal, const float* ga, const float* gb, const float* gf,
                           bool reader) {
        wait_prog(prog, (ordinal << 16) + 3);
        if (reader) {
            copy_stage(ordinal, 1, ga, gb, gf);
            copy_stage(ordinal, 2, ga, gb, gf);
        }
    };
    auto stage_next = [&](const int* prog, int ordinal, int k, const float* ga, const float* gb, const float* gf,
                          bool reader) {
        wait_prog(prog, (ordinal << 16) + min(k + 4, kStageMask));
        if (reader) copy_stage(ordinal, k + 3, ga, gb, gf);
    };
    // past its last stage a row-block's neighbour reads up to 48 steps and 12
    // groups further: zeros, in the final frame (one lane writes them)
    auto write_tail = [&](float* oa, float* ob, float* of, int n, float fr) {
#pragma unroll 4
        for (int i = 0; i < 12; ++i) {
            *reinterpret_cast<float4*>(oa + kCW * n + 4 * i) = make_float4(0.f, 0.f, 0.f, 0.f);
            *reinterpret_cast<float4*>(ob + kCW * n + 4 * i) = make_float4(0.f, 0.f, 0.f, 0.f);
        }
#pragma unroll
        for (int i = 0; i < 3; ++i) *reinterpret_cast<float4*>(of + 4 * n + 4 * i) = make_float4(fr, fr, fr, fr);
    };

    // ============================== forward ==============================
    FwdVars V;
    V.acc = 0.0;
    V.ab = 0.f;
    V.gsum = 0.f;
    V.E = 0.f;
    V.ebmin = V.ebmax = 0x3f800000;
    V.emax = 0.f;
    const int* const prodF = xin ? gsync + pin : &progF[wprev];
    const int* const prodR = xin ? gsync + kMaxParts + pin : &progR[wprev];
    for (int r = gw; r < nRB; r += NWt) {
        const int nv = min(32, L1 - 32 * r);
        const int nst = (L2 + nv - 1 + kCW - 1) / kCW;
        const float* srow = S + (size_t)(32 * r) * L2m;
        const bool hasB = r > 0;
        FwdCtx C;
        C.ring = W.ringS + lane * kRW;
        const bool fromAbove = hasB && lane == 0;
        C.au = fromAbove ? W.sa : zv;
        C.at = fromAbove ? W.sb : zv;
        C.af = fromAbove ? W.sf : zf;
        C.oa = LY.hva + (size_t)r * hzst;
        C.ob = LY.hvb + (size_t)r * hzst;
        C.of = LY.hfr + (size_t)r * hfst;
        C.pv = (unsigned)__cvta_generic_to_shared(Wn.sa);
        C.mrow = LY.mpl + (size_t)r * zst + lane;
        C.erow = LY.efr + (size_t)r * est + lane;
        C.c = c;
        C.Go = Go;
        C.Ge = Ge;
        C.notl0 = lane == 0 ? 0.f : 1.f;
        C.lane = lane;
        C.nv = nv;
        C.L2 = L2;
        C.l0 = lane == 0;
        C.l31 = lane == 31;
        const Tile tS = make_tile(srow, L2m, W.ringS, nv, lane);

        const size_t rA = (size_t)(r - 1);
        const float *const gaA = LY.hva + rA * hzst, *const gbA = LY.hvb + rA * hzst, *const gfA = LY.hfr + rA * hfst;
        const bool hasD = r + 1 < nRB;
        __syncwarp();
        if (lane == 31) st_release(&progF[warp], r << 16);  // started: the row above may push to this warp
        if (0 < nch) tile_load<4>(tS, 0, L2);
        if (hasB) stage_first(prodF, r - 1, gaA, gbA, gfA, lane == 0);
        cp_async_commit();
        V.Mp = V.Dp = V.Td = V.ur = V.Tr = V.Tl = 0.f;
        V.f.d1 = 0.f;
        for (int k = 0; k < nst; ++k) {
            __syncwarp();
            if (hasB) stage_next(prodF, r - 1, k, gaA, gbA, gfA, lane == 0);
            cp_async_commit();
            if (k + 1 < nch) tile_load<4>(tS, k + 1, L2);
            cp_async_commit();
            cp_async_wait2();  // everything but this stage's two groups
            __syncwarp();
            // push while the row-block below is on its warp and has done at least
            // k - 8 stages (the linear kernel's rule, sw_linear.cu)
            V.push = false;
            if (lane == 31 && hasD && !xout) {
                const int cw = ld_acquire(&progF[wnext]);
                V.push = (cw >> 16) == r + 1 && (cw & kStageMask) + 8 >= k;
            }
            if (k == 0) {
                if (lane == 0) V.E = C.af[7];
                V.Esent = __shfl_up_sync(kAll, V.E, 1);
                fwd_lookahead(C, V, 0);
            }
            if (kCW * k < 31)
                fwd_stage_start(C, V, k);
            else if (nv == 32 && kCW * k + kCW - 1 <= L2 - 1)
                fwd_stage_full<false>(C, V, k, 0);
            else
                fwd_stage_full<true>(C, V, k, lane < nv ? L2 + lane - kCW * k : -1);
            acc_rebase(V.acc, V.ab, V.E);
            if (V.push) Wn.tag[k & (kHR / 16 - 1)] = (r << 16) | k;
            __syncwarp();
            if (lane == 31) {
                st_release(&progF[warp], (r << 16) | min(k + 1, kStageMask - 1));
                if (xout) st_release_gpu(gsync + part, (r << 16) | min(k + 1, kStageMask - 1));
            }
        }
        V.acc = fma((double)V.gsum, p2d(V.E - V.ab), V.acc);
        V.emax = fmaxf(V.emax, V.E - V.ab);
        V.gsum = 0.f;
        if (lane == 31) write_tail(C.oa, C.ob, C.of, nst, V.E);
        cp_async_wait0();
        __syncwarp();
        if (lane == 31) {
            st_release(&progF[warp], (r << 16) | kStageMask);
            if (xout) st_release_gpu(gsync + part, (r << 16) | kStageMask);
        }
    }

    if (lane < kHR / 16) W.tag[lane] = -1;  // forward pushes are no reverse pushes
    // ---- S = log2(1 + sum of every lane's partition), kept as integer + fraction
    {
        // every lane's acc brought to the largest base; M[0,0] = 0 adds 2^-abmax
        const float abl = block_max(V.ab, red);
        const double totl = block_sum_d(V.acc * p2d(V.ab - abl), reinterpret_cast<double*>(red));
        if (threadIdx.x == 0) {
            float abmax = abl;
            double tot = totl;
            if (SPLIT && K > 1) {  // every part's partial, after every part's forward
                double* const gp = reinterpret_cast<double*>(gsync + 64);
                gp[kSyncPartDoubles * part] = (double)abl;
                gp[kSyncPartDoubles * part + 1] = totl;
                atom_add_release_gpu(gsync + 2 * kMaxParts, 1);
                int it = 0;
                while (ld_acquire_gpu(gsync + 2 * kMaxParts) < K) {
                    if (++it > kSpinLimit) {
                        sh_err = 1;
                        break;
                    }
                    __nanosleep(64);
                }
                abmax = -3.0e38f;
                for (int k = 0; k < K; ++k) abmax = fmaxf(abmax, (float)gp[kSyncPartDoubles * k]);
                tot = 0.0;
                for (int k = 0; k < K; ++k)
                    tot = fma(gp[kSyncPartDoubles * k + 1], p2d((float)gp[kSyncPartDoubles * k] - abmax), tot);
            }
            tot += p2d(-abmax);
            const int hi = __double2hiint(tot);
            const int ef = (hi >> 20) & 0x7ff;
            const int e = ef - 1023 + (int)abmax;
            const bool fin = ef != 0x7ff && ef != 0;
            const double m = __hiloint2double((hi & 0x800fffff) | 0x3ff00000, __double2loint(tot));
            sh_Sint = e;
            sh_Sfrac = lg2_rr((float)m);
            if (!fin) sh_bad = 1;
            if (p.value && part == 0) p.value[b] = ((float)sh_Sint + sh_Sfrac) / c;
        }
        __syncthreads();
    }

    // the forward's range checks, folded into one word before the reverse
    const int fwd_out = ((V.ebmin < ((127 - kJMax) << 23) || V.ebmax > ((127 + kJMax) << 23)) ? 1 : 0) |
                        (V.emax > 1000.f ? 8 : 0);

    // ============================== reverse ==============================
    const int P = kCW * ((L2 - 1 + kCW - 1) / kCW);
    const int nstR = P / kCW + 2;
    RevVars RV;
    RV.ebmin = RV.ebmax = 0x3f800000;
    for (int q = gw; q < nRB; q += NWt) {
        const int r = nRB - 1 - q;
        const int nv = min(32, L1 - 32 * r);
        const float* srow = S + (size_t)(32 * r) * L2m;
        const bool hasBelow = r + 1 < nRB, hasAbove = r > 0;
        const float* const mblk = LY.mpl + (size_t)r * zst;
        const float* const eblk = LY.efr + (size_t)r * est;
        RevCtx C;
        C.ring = W.ringS + lane * kRW;
        C.zr = &W.zr[0][0];
        C.er = W.er;
        const bool fromBelow = hasBelow && lane == nv - 1;
        C.by = fromBelow ? W.sa : zv;
        C.bx = fromBelow ? W.sb : zv;
        C.bf = fromBelow ? W.sf : zf;
        C.oa = LY.hva + (size_t)r * hzst;
        C.ob = LY.hvb + (size_t)r * hzst;
        C.of = LY.hfr + (size_t)r * hfst;
        C.pv = (unsigned)__cvta_generic_to_shared(Wn.sa);
        C.c = c;
        C.Go = Go;
        C.Ge = Ge;
        C.cS = ex2f(-sh_Sfrac);
        C.notBot = lane == nv - 1 ? 0.f : 1.f;
        C.bot = lane == nv - 1;
        C.Sint = (float)sh_Sint;
        C.lane = lane;
        C.nv = nv;
        C.L2 = L2;
        C.P = P;
        C.l0 = lane == 0;
        const Tile tS = make_tile(srow, L2m, W.ringS, nv, lane);
        const Tile tM = make_tile(out ? out + (size_t)(32 * r) * L2m : srow, L2m, W.ringS, nv, lane);

        auto batch = [&](int kb) {
            const int M = P / kCW + 1 - kb;
            float* const zd = &W.zr[M & 1][0];
            const float* const zs = mblk + (size_t)(16 * M) * 32;
#pragma unroll
            for (int it = 0; it < 4; ++it) cp_async16(zd + 4 * (lane + 32 * it), zs + 4 * (lane + 32 * it), 16);
            const int gl = 4 * M - 1;
#pragma unroll
            for (int it = 0; it < 2; ++it) {
                const int cc = lane + 32 * it, g = gl + (cc >> 3), c4 = cc & 7;
                if (cc < 40 && g >= 0) cp_async16(W.er + (g & 15) * 32 + 4 * c4, eblk + (size_t)g * 32 + 4 * c4, 16);
            }
        };
        const size_t rB = (size_t)(r + 1);
        const float *const gaB = LY.hva + rB * hzst, *const gbB = LY.hvb + rB * hzst, *const gfB = LY.hfr + rB * hfst;

        __syncwarp();
        if (lane == 0) st_release(&progR[warp], q << 16);  // started: the row-block below may push to this warp
        {
            const int M0 = P / kCW + 1;
            for (int ch = M0; ch >= M0 - 2; --ch)
                if (ch >= 0 && ch < nch) tile_load<4>(tS, ch, L2);
        }
        batch(0);
        if (hasBelow) stage_first(prodR, q - 1, gaB, gbB, gfB, lane == nv - 1);
        cp_async_commit();

        RV.BDp = RV.PBp = RV.Yr = RV.Xr = RV.BMl = 0.f;
        RV.Q = 0.f;
        RV.Qsent = 0.f;
        RV.f.d1 = 0.f;
        for (int k = 0; k < nstR; ++k) {
            const int M = P / kCW + 1 - k;
            __syncwarp();
            if (hasBelow) stage_next(prodR, q - 1, k, gaB, gbB, gfB, lane == nv - 1);
            cp_async_commit();
            if (out && M + 1 < nch && M + 1 >= 0) tile_store(tM, M + 1, L2);
            if (M - 3 >= 0 && M - 3 < nch) tile_load<4>(tS, M - 3, L2);
            if (k + 1 < nstR) batch(k + 1);
            cp_async_commit();
            cp_async_wait2();
            __syncwarp();
            RV.push = false;
            if (lane == 0 && hasAbove && !xout) {
                const int cw = ld_acquire(&progR[wnext]);
                RV.push = (cw >> 16) == q + 1 && (cw & kStageMask) + 8 >= k;
            }
            if (k == 0) rev_lookahead(C, RV, 0);
            if (kCW * k <= P + 32 - L2)
                rev_stage_part(C, RV, k);
            else if (nv == 32 && kCW * k + kCW - 1 <= P - 1)
                rev_stage_full<false>(C, RV, k, 0);
            else
                rev_stage_full<true>(C, RV, k, lane < nv ? 16 * M + 16 - lane : -1);
            if (RV.push) Wn.tag[k & (kHR / 16 - 1)] = (q << 16) | k;
            __syncwarp();
            if (lane == 0) {
                st_release(&progR[warp], (q << 16) | min(k + 1, kStageMask - 1));
                if (xout) st_release_gpu(gsync + kMaxParts + part, (q << 16) | min(k + 1, kStageMask - 1));
            }
        }
        if (lane == 0) write_tail(C.oa, C.ob, C.of, nstR, RV.Q);
        __syncwarp();
        if (out && nch > 0) tile_store(tM, 0, L2);
        cp_async_wait0();
        __syncwarp();
        if (lane == 0) {
            st_release(&progR[warp], (q << 16) | kStageMask);
            if (xout) st_release_gpu(gsync + kMaxParts + part, (q << 16) | kStageMask);
        }
    }

    const bool outside = (fwd_out & 1) || RV.ebmin < ((127 - kJMax) << 23) || RV.ebmax > ((127 + kJMax) << 23);
    const int o_win = __syncthreads_or(outside ? 1 : 0);
    const int o_acc = __syncthreads_or(fwd_out & 8);
    // nonzero = recompute; the bits say why (1 frame step, 2 wait gave up,
    // 4 partition not finite, 8 partition base)
    const int redo = (o_win ? 1 : 0) | (sh_err ? 2 : 0) | (sh_bad ? 4 : 0) | (o_acc ? 8 : 0);
    if (threadIdx.x == 0 && p.redo) {
        if (SPLIT)
            atomicOr(p.redo + b, redo);  // zeroed by the launcher
        else
            p.redo[b] = redo;
    }
}

// bf16 scores are widened into the workspace once per call
__global__ void bf16_to_f32_kernel(const __nv_bfloat16* __restrict__ in, float* __restrict__ out, size_t n) {
    const size_t i0 = ((size_t)blockIdx.x * blockDim.x + threadIdx.x) * 8;
    const size_t stride = (size_t)gridDim.x * blockDim.x * 8;
    for (size_t i = i0; i < n; i += stride) {
        if (i + 8 <= n) {
            const uint4 v = *reinterpret_cast<const uint4*>(in + i);
            const unsigned w[4] = {v.x, v.y, v.z, v.w};
            float4 a, bb;
            a.x = __uint_as_float(w[0] << 16);
            a.y = __uint_as_float(w[0] & 0xffff0000u);
            a.z = __uint_as_float(w[1] << 16);
            a.w = __uint_as_float(w[1] & 0xffff0000u);
            bb.x = __uint_as_float(w[2] << 16);
            bb.y = __uint_as_float(w[2] & 0xffff0000u);
            bb.z = __uint_as_float(w[3] << 16);
            bb.w = __uint_as_float(w[3] & 0xffff0000u);
            *reinterpret_cast<float4*>(out + i) = a;
            *reinterpret_cast<float4*>(out + i + 4) = bb;
        } else {
            for (size_t k = i; k < n; ++k) out[k] = __bfloat162float(in[k]);
        }
    }
}

}  // namespace aff

// ------------------------------------------------------------------ host side
int launch_bf16_widen(const __nv_bfloat16* in, float* out, size_t n, cudaStream_t st) {
    if (n == 0) return 0;
    if ((((uintptr_t)in) & 15) != 0 || (((uintptr_t)out) & 15) != 0) return -1;
    aff::bf16_to_f32_kernel<<<1184, 256, 0, st>>>(in, out, n);
    return (int)cudaGetLastError();
}

size_t aff_fast_workspace_bytes(int B, int L1, int L2, bool bf16) {
    if (L1 > 32 * aff::kMaxRB || L2 % 4 != 0) return 0;
    size_t b = aff::per_problem_bytes(L1, L2) * (size_t)B;
    if (bf16) b += ring::align_up((size_t)B * L1 * L2 * sizeof(float), 256);  // widened scores
    return b;
}

int launch_aff_fast(const SwArgs& a0, size_t ws_bytes, cudaStream_t st) {
    SwArgs a = a0;
    if (a.mode != MODE_MARG || !a.redo || a.grad_gap || a.grad_gap2 || a.grad_T) return -1;
    if (engine_forced_plane()) return -1;
    if (a.L2 % 4 != 0 || a.L1 > 32 * aff::kMaxRB || a.L1 == 0 || a.L2 == 0) return -1;
    const bool bf16 = a.scores_bf16 != nullptr;
    if ((((uintptr_t)a.ws) & 255) != 0 || !a.ws) return -1;
    if (a.out && (((uintptr_t)a.out) & 15) != 0) return -1;
    if (ws_bytes < aff_fast_workspace_bytes(a.B, a.L1, a.L2, bf16)) return -1;
    if (bf16) {
        if ((((uintptr_t)a.scores_bf16) & 15) != 0) return -1;
        float* wide = (float*)((char*)a.ws + aff::per_problem_bytes(a.L1, a.L2) * (size_t)a.B);
        const size_t n = (size_t)a.B * a.L1 * a.L2;
        aff::bf16_to_f32_kernel<<<1184, 256, 0, st>>>(a.scores_bf16, wide, n);
        cudaError_t e = cudaGetLastError();
        if (e != cudaSuccess) return (int)e;
        a.scores = wide;
        a.scores_bf16 = nullptr;
    } else if (!a.scores || (((uintptr_t)a.scores) & 15) != 0) {
        return -1;
    }
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return (int)e;
    static DeviceSetup setup;
    const size_t s6 = sizeof(aff::WarpSmem) * aff::kNW, s12 = sizeof(aff::WarpSmem) * aff::kNWWide;
    int nsm = 0;
    const int se = device_setup(setup, dev, [s6, s12] {
        const void* ks[3] = {(const void*)aff::aff_fast_kernel<aff::kNW, 2, false>,
                             (const void*)aff::aff_fast_kernel<aff::kNWWide, 1, false>,
                             (const void*)aff::aff_fast_kernel<aff::kNWWide, 1, true>};
        cudaError_t r = cudaSuccess;
        for (int i = 0; i < 3 && r == cudaSuccess; ++i) {
            r = cudaFuncSetAttribute(ks[i], cudaFuncAttributeMaxDynamicSharedMemorySize, (int)(i == 0 ? s6 : s12));
            if (r == cudaSuccess)
                r = cudaFuncSetAttribute(ks[i], cudaFuncAttributePreferredSharedMemoryCarveout,
                                         (int)cudaSharedmemCarveoutMaxShared);
        }
        return (int)r;
    }, &nsm);
    if (se != 0) return se;
    // A batch that leaves most SMs idle spreads each problem over several CTAs
    // of 12 warps (cooperative launch: every part resident at once); at most
    // one problem per SM runs 12 warps per problem when that pays (see
    // launch_lin_fast).
    const int K = a.sync ? lin_parts_nw(a.B, a.L1, a.L2, nsm, aff::kNWWide) : 1;
    if (K > 1) {
        SwArgs s = a;
        s.parts = K;
        e = cudaMemsetAsync(s.sync, 0, kSyncBytes * (size_t)a.B, st);
        if (e == cudaSuccess) e = cudaMemsetAsync(s.redo, 0, sizeof(int) * (size_t)a.B, st);
        if (e != cudaSuccess) return (int)e;
        void* args[1] = {&s};
        e = cudaLaunchCooperativeKernel((const void*)aff::aff_fast_kernel<aff::kNWWide, 1, true>, dim3(a.B * K),
                                        dim3(aff::kNWWide * 32), args, s12, st);
        if (e == cudaSuccess) return 0;
        cudaGetLastError();  // a cooperative launch that does not fit: one CTA per problem instead
    }
    if (a.B <= nsm && lin_wide_pays(a.L1, a.L2)) {
        aff::aff_fast_kernel<aff::kNWWide, 1, false><<<a.B, aff::kNWWide * 32, s12, st>>>(a);
    } else {
        aff::aff_fast_kernel<aff::kNW, 2, false><<<a.B, aff::kNW * 32, s6, st>>>(a);
    }
    return (int)cudaGetLastError();
}

}  // namespace d2pb
