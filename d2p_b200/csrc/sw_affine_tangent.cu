// sw_affine_tangent.cu -- linear-domain tangent sweeps for affine-gap soft
// Smith-Waterman: the directional derivative of the marginals along a
// direction V in the scores (HVP, src/sw_affine/kernels_cpu.cpp:352-620), along
// gap_open, gap_ext or T (the parameter Jacobians, :630-921), and contracted
// with a weight plane (the parameter half of backward_full,
// src/sw_affine/torch_cuda.cpp).
//
// The value recurrences are sw_affine_fast.cu's (P = 2^(s c), Go = 2^(go c),
// Ge = 2^(ge c), c = log2(e)/T):
//   M = P (T_diag + 1)        I = Go M_up + Ge I_up      D = Go M_left + Ge D_left
//   T = M + I + D
//   BM = c1 + Go (BI_down + BD_right)   BI = c1 + Ge BI_down   BD = c1 + Ge BD_right
//   c1 = 1 + P' BM' (the diagonal successor's),   mu = BM M / Z_total.
// With dP = P vp (vp = V/T along V; -s/T^2 along T), dGo = Go go_ (go_ = 1/T
// along gap_open, -go/T^2 along T) and dGe = Ge ge_ likewise, each tangent is
// the same recurrence with source terms:
//   dM = M vp + P dT_diag
//   dI = Go (dM_up + go_ M_up) + Ge (dI_up + ge_ I_up)      (the u a lane sends down)
//   dD = Go (dM_left + go_ M_left) + Ge (dD_left + ge_ D_left)
//   dc1 = P' (vp' BM' + dBM')
//   dBI = dc1 + Ge (dBI_down + ge_ BI_down), dBD likewise to the right,
//   dBM = dc1 + Go (dBI_down + go_ BI_down + dBD_right + go_ BD_right)
//   dmu = (dBM M + BM dM) / Z_total - mu dZ_total / Z_total.
// A tangent shares its value's frame; frames, stages, the row-block pipeline,
// the handoff routes (four values per step cross a row-block boundary: u, T
// and their tangents forward, BI, X and theirs in the reverse), the split of
// large problems over several CTAs and the fix-up contract are those of
// sw_tangent.cu.
//
// PG (value + marginals + dS/dgap_open, dS/dgap_ext, dS/dT, for gap parameters
// that need gradients), one sweep pair: the forward carries the tangent along
// gap_open, so dS/dgo = T dZ/Z, the expected number of gap openings.  Every
// visit of an I or D state is entered by exactly one opening or one extension,
// so the expected number of extensions, dS/dge, is the sum of the I and D
// visit probabilities (BI I + BD D) / Z_total minus dS/dgo; the forward keeps
// I and D per cell for it.  The reverse also writes the marginals and sums
// score x marginal, and dS/dT follows from Euler's identity for the degree-1
// homogeneous S(s, go, ge, T): S = sum s mu + go dS/dgo + ge dS/dge + T dS/dT.
//
// BF (backward_full): the HVP along the weight plane g gives grad_scores = H g
// (the Hessian of S is symmetric); the parameter parts are the tangents along
// g of dS/dgo, dS/dge and dS/dT.  A gap is opened from an M cell with weight
// Go (BI_down + BD_right) = BM - c1, so
//   dS/dgo = E[openings] = sum M (BM - c1) / Z_total,
// a sum over cells of values the HVP sweeps hold, and so is its tangent (dM,
// dBM, dc1).  The sweep pair also sums s H g; d(dS/dT)[g] = -(sum s H g + go
// d(dS/dgo)[g] + ge d(dS/dge)[g]) / T by Euler's identity, with d(dS/dge)[g]
// read from dot_out[B + b], which the caller's dot sweep along gap_ext wrote
// before this launch.  (dS/dge as gap cells minus openings, the gap cells from
// the position sums of path ends and starts, needs no second sweep pair but
// cancels: its fp32 error reached 3.7x the reference's.)
#include <stddef.h>
#include <stdint.h>

#include "sw_common.cuh"
#include "sw_internal.h"
#include "sw_lindomain.cuh"
#include "sw_ring.cuh"

namespace d2pb {
namespace atan_ {
using namespace ring;
using namespace ld;

constexpr int kMaxRB = 512;
constexpr int kNW = 6;

struct WarpSmem {
    float ringS[32 * kRW];    // scores; reverse: dmu written in place
    float ringV[32 * kRW];    // the direction (HVP) or the dot-mode weights
    float zr[2][16 * 32];     // reverse: the forward's M of 16 anti-diagonals, two slots
    float dzr[2][16 * 32];    //          and its dM (PG: the forward's I)
    float xr[2][16 * 32];     //          PG: the forward's D
    float er[16 * 32];        // reverse: forward frames
    // staging of the neighbouring row-block's boundary values by its step
    // (forward: u, T, du, dT; reverse: BI, X, dBI, dX) and frames by group
    float s0[kHR];
    float s1[kHR];
    float s2[kHR];
    float s3[kHR];
    float sf[kHR / 4];
    int tag[kHR / 16];
};
static_assert(sizeof(WarpSmem) % 16 == 0, "per-warp shared blocks must stay 16-byte aligned");
static_assert(offsetof(WarpSmem, s1) == offsetof(WarpSmem, s0) + 4 * kHR &&
                  offsetof(WarpSmem, s2) == offsetof(WarpSmem, s0) + 8 * kHR &&
                  offsetof(WarpSmem, s3) == offsetof(WarpSmem, s0) + 12 * kHR &&
                  offsetof(WarpSmem, sf) == offsetof(WarpSmem, s0) + 16 * kHR,
              "staging rows are contiguous");

struct Layout {
    float* mpl;   // [nRB][ZT][32] M of forward step t at row t
    float* dmpl;  // [nRB][ZT][32] dM
    float* efr;   // [nRB][GT][32] frames
    float* h[4];  // [nRB][HZ]     boundary rows (the four values above)
    float* hfr;   // [nRB][HF]     their frames
    float* xpl;   // [nRB][ZT][32] PG: D of forward step t (dmpl then holds I)
};
__host__ __device__ inline size_t per_problem_bytes(int L1m, int L2m, bool pg = false) {
    const size_t nrb = (size_t)(L1m + 31) / 32;
    return (pg ? 3 : 2) * align_up(nrb * zt_rows(L2m) * 32 * 4, 256) + align_up(nrb * gt_rows(L2m) * 32 * 4, 256) +
           4 * align_up(nrb * hz_stride(L2m) * 4, 256) + align_up(nrb * hf_stride(L2m) * 4, 256);
}
__device__ inline Layout carve(float* ws, int b, int L1m, int L2m, bool pg) {
    const size_t nrb = (size_t)(L1m + 31) / 32;
    char* base = (char*)ws + (size_t)b * per_problem_bytes(L1m, L2m, pg);
    Layout L;
    L.mpl = (float*)base;
    base += align_up(nrb * zt_rows(L2m) * 32 * 4, 256);
    L.dmpl = (float*)base;
    base += align_up(nrb * zt_rows(L2m) * 32 * 4, 256);
    L.efr = (float*)base;
    base += align_up(nrb * gt_rows(L2m) * 32 * 4, 256);
    for (int i = 0; i < 4; ++i) {
        L.h[i] = (float*)base;
        base += align_up(nrb * hz_stride(L2m) * 4, 256);
    }
    L.hfr = (float*)base;
    base += align_up(nrb * hf_stride(L2m) * 4, 256);
    L.xpl = pg ? (float*)base : nullptr;
    return L;
}

struct Dir {
    float vs, ss, go, ge;  // dP = P (vs V + ss s), dGo = Go go, dGe = Ge ge
};

// the boundary lane's four values of a group and its frame (sw_tangent.cu's
// handoff with four rows)
template <class Ctx>
__device__ __forceinline__ void handoff4(const Ctx& C, int g, float4 a, float4 b, float4 da, float4 db, float fr,
                                         bool bnd, bool pp) {
    const bool pg = bnd && !pp;
    stg_pair_pred(C.oh[0] + 4 * g, C.oh[1] + 4 * g, C.of + g, a, b, fr, pg);
    stg_pair_pred(C.oh[2] + 4 * g, C.oh[3] + 4 * g, C.of + g, da, db, fr, pg);
    const unsigned sv = C.pv + 16u * (unsigned)(g & (kHR / 4 - 1));
    const unsigned sf = C.pv + 16u * kHR + 4u * (unsigned)(g & (kHR / 4 - 1));
    sts_group_pred_s(sv, sf, a, fr, pp);
    sts_group_pred_s(sv + 4u * kHR, sf, b, fr, pp);
    sts_group_pred_s(sv + 8u * kHR, sf, da, fr, pp);
    sts_group_pred_s(sv + 12u * kHR, sf, db, fr, pp);
}

// ==========================================================================
// forward
// ==========================================================================
struct FwdF {
    float d0, d1;
    float Ged0, Ged1;
    float fs;
    float ua[4], ta[4], dua[4], dta[4];  // lane 0: the row above's u, T and tangents, frame E
};

struct FwdVars {
    bool push;
    float Mp, Dp, Td;       // own M, D of the previous step; diagonal T of this step
    float ur, Tr;           // lane l-1's u and T of the previous step (its frame)
    float dMp, dDp, dTd, dur, dTr;
    float Tl;               // own T of the previous step (frame anchor)
    float E, Esent;
    FwdF f;
    float nE, nfJ;
    FwdF nf;
    float gsum, dgsum;
    double acc, dacc;
    float ab;
    int ebmin, ebmax;
    float emax;
};

struct FwdCtx {
    const float* ring;
    const float* vring;
    const float* as;     // lane 0: staging rows u, T, du, dT (as + i kHR) of the row above; zeros otherwise
    const float* af;
    float* oh[4];
    float* of;
    unsigned pv;
    float* mrow;
    float* dmrow;
    float* xrow;         // PG: xpl row 0 of this row-block, this lane
    float* erow;
    float c, Go, Ge;
    Dir dir;
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
    for (int q = 0; q < 4; ++q) f.ua[q] = f.ta[q] = f.dua[q] = f.dta[q] = 0.f;
    return f;
}

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
    float* const tgt[4] = {V.nf.ua, V.nf.ta, V.nf.dua, V.nf.dta};
#pragma unroll
    for (int r = 0; r < 4; ++r) {
        const float* row = C.as + r * kHR;
        const float4 x = *reinterpret_cast<const float4*>(row + s1);
        tgt[r][0] = row[s0] * w;
        tgt[r][1] = x.x;
        tgt[r][2] = x.y;
        tgt[r][3] = x.z;
    }
}

__device__ __forceinline__ void fwd_apply(FwdVars& V) {
    const float dE = V.E - V.ab;
    const double sc = p2d(dE);
    V.acc = fma((double)V.gsum, sc, V.acc);
    V.dacc = fma((double)V.dgsum, sc, V.dacc);
    V.emax = fmaxf(V.emax, dE);
    V.gsum = V.dgsum = 0.f;
    V.Mp *= V.nfJ;
    V.Dp *= V.nfJ;
    V.Td *= V.nfJ;
    V.dMp *= V.nfJ;
    V.dDp *= V.nfJ;
    V.dTd *= V.nfJ;
    V.E = V.nE;
    V.f = V.nf;
}

__device__ __forceinline__ void acc_rebase2(FwdVars& V) {
    if (V.E - V.ab > 700.f) {
        const double sc = p2d(V.ab - V.E);
        V.acc *= sc;
        V.dacc *= sc;
        V.ab = V.E;
    }
}

struct FwdOut {
    float M, D, T, u, Tdn, I;
    float dM, dD, dT, du, dTdn;
};
__device__ __forceinline__ FwdOut fwd_cell(const FwdCtx& C, const FwdVars& V, int i, float sc, float vv) {
    FwdOut o;
    const float P = ex2f(sc * C.c);
    const float vp = fmaf(C.dir.vs, vv, C.dir.ss * sc);
    const float d = i == 0 ? V.f.d0 : V.f.d1;
    o.M = P * (V.Td + V.f.fs);
    const float I = fmaf(V.ur, d, V.f.ua[i]);
    o.I = I;
    o.D = fmaf(C.Ge, V.Dp, C.Go * V.Mp);
    o.T = o.M + I + o.D;
    o.u = fmaf(i == 0 ? V.f.Ged0 : V.f.Ged1, V.ur, fmaf(C.Go, o.M, C.Ge * V.f.ua[i]));
    o.Tdn = fmaf(V.Tr, d, V.f.ta[i]);
    o.dM = fmaf(o.M, vp, P * V.dTd);
    const float dI = fmaf(V.dur, d, V.f.dua[i]);
    o.dD = fmaf(C.Go, fmaf(C.dir.go, V.Mp, V.dMp), C.Ge * fmaf(C.dir.ge, V.Dp, V.dDp));
    o.dT = o.dM + dI + o.dD;
    o.du = fmaf(C.Go, fmaf(C.dir.go, o.M, o.dM), C.Ge * fmaf(C.dir.ge, I, dI));
    o.dTdn = fmaf(V.dTr, d, V.f.dta[i]);
    return o;
}

__device__ __forceinline__ void fwd_commit(FwdVars& V, const FwdOut& o) {
    V.Mp = o.M;
    V.Dp = o.D;
    V.Td = o.Tdn;
    V.Tl = o.T;
    V.dMp = o.dM;
    V.dDp = o.dD;
    V.dTd = o.dTdn;
    V.ur = __shfl_up_sync(kAll, o.u, 1);
    V.Tr = __shfl_up_sync(kAll, o.T, 1);
    V.dur = __shfl_up_sync(kAll, o.du, 1);
    V.dTr = __shfl_up_sync(kAll, o.dT, 1);
}

template <bool MASK, bool HV, bool PG>
__device__ __forceinline__ void fwd_stage_full(const FwdCtx& C, FwdVars& V, int k, int thr) {
    const int c0 = (kCW * k - C.lane) & (kRW - 1);
    float scv[kCW], vvv[kCW];
#pragma unroll
    for (int u = 0; u < kCW; ++u) {
        const int col = (u < kRW - c0) ? c0 + u : c0 + u - kRW;
        scv[u] = C.ring[col];
        vvv[u] = HV ? C.vring[col] : 0.f;
    }
    float* const pm = C.mrow + (size_t)(kCW * k) * 32;
    float* const pdm = C.dmrow + (size_t)(kCW * k) * 32;
    float* const px = PG ? C.xrow + (size_t)(kCW * k) * 32 : nullptr;
    float* const pe = C.erow + (size_t)(kCW * k / 4) * 32;
    float uq[4], tq[4], duq[4], dtq[4];
#pragma unroll
    for (int u = 0; u < kCW; ++u) {
        const int i = u & 3;
        if (i == 0) fwd_apply(V);
        if (i == 3) {
            if (u == kCW - 1) cp_async_wait1();
            fwd_lookahead(C, V, 4 * k + (u >> 2) + 1);
        }
        FwdOut o = fwd_cell(C, V, i, scv[u], vvv[u]);
        if (MASK) {
            const bool act = u < thr;
            o.T = act ? o.T : 0.f;
            o.u = act ? o.u : 0.f;
            o.dT = act ? o.dT : 0.f;
            o.du = act ? o.du : 0.f;
        }
        V.gsum += o.T;
        V.dgsum += o.dT;
        pm[(size_t)u * 32] = o.M;
        if (PG) {  // the reverse needs no dM: the I and D visit sums take I and D
            pdm[(size_t)u * 32] = o.I;
            px[(size_t)u * 32] = o.D;
        } else {
            pdm[(size_t)u * 32] = o.dM;
        }
        uq[i] = o.u;
        tq[i] = o.T;
        duq[i] = o.du;
        dtq[i] = o.dT;
        if (i == 3) {
            pe[(u >> 2) * 32] = V.E;
            handoff4(C, 4 * k + (u >> 2), make_float4(uq[0], uq[1], uq[2], uq[3]),
                     make_float4(tq[0], tq[1], tq[2], tq[3]), make_float4(duq[0], duq[1], duq[2], duq[3]),
                     make_float4(dtq[0], dtq[1], dtq[2], dtq[3]), V.E, C.l31, V.push);
        }
        fwd_commit(V, o);
    }
}

template <bool HV, bool PG>
__device__ __forceinline__ void fwd_stage_start(const FwdCtx& C, FwdVars& V, int k) {
    const bool live = C.lane < C.nv;
    float uq[4], tq[4], duq[4], dtq[4];
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
            const int col = j0 & (kRW - 1);
            FwdOut o = fwd_cell(C, V, i, C.ring[col], HV ? C.vring[col] : 0.f);
            o.M = act ? o.M : 0.f;
            o.D = act ? o.D : 0.f;
            o.T = act ? o.T : 0.f;
            o.u = act ? o.u : 0.f;
            o.dM = act ? o.dM : 0.f;
            o.dD = act ? o.dD : 0.f;
            o.dT = act ? o.dT : 0.f;
            o.du = act ? o.du : 0.f;
            V.gsum += o.T;
            V.dgsum += o.dT;
            C.mrow[(size_t)t * 32] = o.M;
            if (PG) {
                C.dmrow[(size_t)t * 32] = act ? o.I : 0.f;
                C.xrow[(size_t)t * 32] = o.D;
            } else {
                C.dmrow[(size_t)t * 32] = o.dM;
            }
            uq[i] = o.u;
            tq[i] = o.T;
            duq[i] = o.du;
            dtq[i] = o.dT;
            if (i == 3) {
                C.erow[(size_t)(t >> 2) * 32] = V.E;
                handoff4(C, 4 * k + q, make_float4(uq[0], uq[1], uq[2], uq[3]),
                         make_float4(tq[0], tq[1], tq[2], tq[3]), make_float4(duq[0], duq[1], duq[2], duq[3]),
                         make_float4(dtq[0], dtq[1], dtq[2], dtq[3]), V.E, C.l31, V.push);
            }
            if (!act) {
                o.Tdn = 0.f;
                o.dTdn = 0.f;
            }
            fwd_commit(V, o);
            V.Esent = __shfl_up_sync(kAll, V.E, 1);
        }
    }
}

// ==========================================================================
// reverse
// ==========================================================================
struct RevF {
    float d0, d1;
    float Ged0, Ged1, God0, God1;
    float fsq;
    float xa[4], ya[4], dxa[4], dya[4];  // bottom lane: X, BI and tangents from the row-block below, frame Q
    float kE;
};

struct RevVars {
    bool push;
    float BDp, PBp;         // own BD and P BM of column j+1
    float Yr, Xr;           // lane l+1's BI and X of the previous step (its frame)
    float dBDp, dPBp, dYr, dXr;
    float BMl;
    float Q, Qsent;
    RevF f;
    float nQ, nfJ;
    RevF nf;
    int ebmin, ebmax;
    float chk;
    float sdot;
    double dot;
    float sgap;             // PG: this stage's sum of the I and D visit probabilities
    double dot2;
    float sx1;              // BF: this stage's sum of the openings' tangent
    double dot3;
};

struct RevCtx {
    float* ring;
    const float* vring;
    const float* zr;
    const float* dzr;
    const float* xr;       // PG: WarpSmem::xr
    const float* er;
    const float* bs;     // bottom lane: staging rows BI, X, dBI, dX (bs + i kHR) of the row-block below
    const float* bf;
    float* oh[4];
    float* of;
    unsigned pv;
    float c, Go, Ge, cS;
    Dir dir;
    float dSr;
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
    for (int q = 0; q < 4; ++q) f.xa[q] = f.ya[q] = f.dxa[q] = f.dya[q] = 0.f;
    rev_kfactors(C, f, Q, h);
    return f;
}

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
    float* const tgt[4] = {V.nf.ya, V.nf.xa, V.nf.dya, V.nf.dxa};
#pragma unroll
    for (int r = 0; r < 4; ++r) {
        const float* row = C.bs + r * kHR;
        const float4 x = *reinterpret_cast<const float4*>(row + s1);
        tgt[r][0] = row[s0] * w;
        tgt[r][1] = x.x;
        tgt[r][2] = x.y;
        tgt[r][3] = x.z;
    }
    rev_kfactors(C, V.nf, V.nQ, h);
}

__device__ __forceinline__ void rev_apply(RevVars& V) {
    V.BDp *= V.nfJ;
    V.PBp *= V.nfJ;
    V.dBDp *= V.nfJ;
    V.dPBp *= V.nfJ;
    V.Q = V.nQ;
    V.f = V.nf;
}

struct RevOut {
    float BM, BI, BD, PB, dBI, dBD, dPB, dmu, gv;
    float x1;               // BF: the cell's share of d(dS/dgo)[g]
};
// m / dm: the forward's M and dM of this cell.  PG: the marginal itself (in
// dmu) and the cell's I and D visit probabilities (in gv; dm is then the
// forward's I, x its D), no tangent of the reverse.
template <bool PG, bool BF>
__device__ __forceinline__ RevOut rev_cell(const RevCtx& C, const RevVars& V, int i, float sc, float vv, float m,
                                           float dm, float x) {
    RevOut o;
    const float P = ex2f(sc * C.c);
    const float vp = fmaf(C.dir.vs, vv, C.dir.ss * sc);
    const float d = i == 0 ? V.f.d0 : V.f.d1;
    const float c1 = V.f.fsq + fmaf(V.Xr, d, V.f.xa[i]);
    o.BD = fmaf(C.Ge, V.BDp, c1);
    o.BI = fmaf(i == 0 ? V.f.Ged0 : V.f.Ged1, V.Yr, fmaf(C.Ge, V.f.ya[i], c1));
    o.BM = fmaf(i == 0 ? V.f.God0 : V.f.God1, V.Yr, fmaf(C.Go, V.f.ya[i], fmaf(C.Go, V.BDp, c1)));
    o.PB = P * o.BM;
    o.x1 = 0.f;
    if (PG) {
        o.dBI = o.dBD = o.dPB = 0.f;
        o.dmu = o.BM * (m * V.f.kE);
        o.gv = fmaf(o.BI, dm, o.BD * x) * V.f.kE;
        return o;
    }
    o.gv = 0.f;
    const float BIdn = fmaf(V.Yr, d, V.f.ya[i]);
    const float dBIdn = fmaf(V.dYr, d, V.f.dya[i]);
    const float dc1 = fmaf(V.dXr, d, V.f.dxa[i]);
    o.dBD = fmaf(C.Ge, fmaf(C.dir.ge, V.BDp, V.dBDp), dc1);
    o.dBI = fmaf(C.Ge, fmaf(C.dir.ge, BIdn, dBIdn), dc1);
    const float dBM = fmaf(C.Go, fmaf(C.dir.go, BIdn + V.BDp, dBIdn + V.dBDp), dc1);
    o.dPB = P * fmaf(vp, o.BM, dBM);
    const float mu = o.BM * (m * V.f.kE);
    o.dmu = fmaf(fmaf(dBM, m, o.BM * dm), V.f.kE, -mu * C.dSr);
    if (BF) {   // openings from this M cell, M (BM - c1) / Z, and their tangent
        const float op = o.BM - c1;
        const float mk = m * V.f.kE;
        o.x1 = fmaf(fmaf(dm, op, m * (dBM - dc1)), V.f.kE, -(mk * op) * C.dSr);
    }
    return o;
}

// BF: the cell's shares of sum s dmu and of the openings' tangent
__device__ __forceinline__ void bf_emit(RevVars& V, const RevOut& o, float sc, bool act) {
    if (!act) return;
    V.sdot = fmaf(sc, o.dmu, V.sdot);
    V.sx1 += o.x1;
}

// DOT: sum gm * dmu; PG: write the marginal and sum score * marginal (gm is
// the score); otherwise write dmu
template <bool DOT, bool PG>
__device__ __forceinline__ void rev_emit(RevVars& V, float* slot, float gm, float dmu, bool act, float gv) {
    if (act) V.chk = fmaf(dmu, 0.f, V.chk);
    if (DOT || PG) {
        if (act) V.sdot = fmaf(gm, dmu, V.sdot);
    }
    if (PG) {
        if (act) {
            V.chk = fmaf(gv, 0.f, V.chk);
            V.sgap += gv;
        }
    }
    if (!DOT) {
        if (act) *slot = dmu;
    }
}

// the cell's outputs into the lane's state: messages (BI, X = P BM of the
// previous cell) and their tangents go to lane l-1
__device__ __forceinline__ void rev_commit(RevVars& V, const RevOut& o, bool act, float& yq, float& xq, float& dyq,
                                           float& dxq) {
    const float BI = act ? o.BI : 0.f, dBI = act ? o.dBI : 0.f;
    const float xs = V.PBp, dxs = V.dPBp;
    yq = BI;
    xq = xs;
    dyq = dBI;
    dxq = dxs;
    V.Yr = __shfl_down_sync(kAll, BI, 1);
    V.Xr = __shfl_down_sync(kAll, xs, 1);
    V.dYr = __shfl_down_sync(kAll, dBI, 1);
    V.dXr = __shfl_down_sync(kAll, dxs, 1);
    V.BDp = act ? o.BD : 0.f;
    V.PBp = act ? o.PB : 0.f;
    V.dBDp = act ? o.dBD : 0.f;
    V.dPBp = act ? o.dPB : 0.f;
    V.BMl = act ? o.BM : 0.f;
}

template <bool MASK, bool HV, bool DOT, bool PG, bool BF>
__device__ __forceinline__ void rev_stage_full(const RevCtx& C, RevVars& V, int k, int thr) {
    const int m16 = C.P + 16 - kCW * k;
    const int slot = ((m16 >> 4) & 1) * (16 * 32) + C.lane;
    const float* const zb = C.zr + slot;
    const float* const dzb = C.dzr + slot;
    const float* const xb = C.xr + slot;
    const int cb = (C.P + 31 - kCW * k - C.lane) & (kRW - 1);
    float scv[kCW], vvv[kCW];
#pragma unroll
    for (int u = 0; u < kCW; ++u) {
        const int col = (u <= cb) ? cb - u : cb - u + kRW;
        scv[u] = C.ring[col];
        vvv[u] = HV ? C.vring[col] : 0.f;
    }
    float yq[4], xq[4], dyq[4], dxq[4];
#pragma unroll
    for (int u = 0; u < kCW; ++u) {
        const int i = u & 3;
        if (i == 0) rev_apply(V);
        if (i == 3) {
            if (u == kCW - 1) cp_async_wait1();
            rev_lookahead(C, V, 4 * k + (u >> 2) + 1);
        }
        const RevOut o = rev_cell<PG, BF>(C, V, i, scv[u], DOT ? 0.f : vvv[u], zb[(15 - u) * 32],
                                          dzb[(15 - u) * 32], PG ? xb[(15 - u) * 32] : 0.f);
        const bool act = !MASK || u < thr;
        const int col = (u <= cb) ? cb - u : cb - u + kRW;
        rev_emit<DOT, PG>(V, C.ring + col, PG ? scv[u] : vvv[u], o.dmu, act, o.gv);
        if (BF) bf_emit(V, o, scv[u], act);
        rev_commit(V, o, act, yq[i], xq[i], dyq[i], dxq[i]);
        if (i == 3)
            handoff4(C, 4 * k + (u >> 2), make_float4(yq[0], yq[1], yq[2], yq[3]),
                     make_float4(xq[0], xq[1], xq[2], xq[3]), make_float4(dyq[0], dyq[1], dyq[2], dyq[3]),
                     make_float4(dxq[0], dxq[1], dxq[2], dxq[3]), V.Q, C.l0, V.push);
    }
}

template <bool HV, bool DOT, bool PG, bool BF>
__device__ __forceinline__ void rev_stage_part(const RevCtx& C, RevVars& V, int k) {
    const int m16 = C.P + 16 - kCW * k;
    const int slot = ((m16 >> 4) & 1) * (16 * 32) + C.lane;
    const float* const zb = C.zr + slot;
    const float* const dzb = C.dzr + slot;
    const float* const xb = C.xr + slot;
    const bool live = C.lane < C.nv;
    float yq[4], xq[4], dyq[4], dxq[4];
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
            const float vv = HV ? C.vring[ci] : 0.f;
            const float sc = C.ring[ci];
            const RevOut o = rev_cell<PG, BF>(C, V, i, sc, DOT ? 0.f : vv, zb[(15 - u) * 32], dzb[(15 - u) * 32],
                                              PG ? xb[(15 - u) * 32] : 0.f);
            rev_emit<DOT, PG>(V, C.ring + ci, PG ? sc : vv, o.dmu, act, o.gv);
            if (BF) bf_emit(V, o, sc, act);
            rev_commit(V, o, act, yq[i], xq[i], dyq[i], dxq[i]);
            if (i == 3)
                handoff4(C, 4 * k + q, make_float4(yq[0], yq[1], yq[2], yq[3]),
                         make_float4(xq[0], xq[1], xq[2], xq[3]), make_float4(dyq[0], dyq[1], dyq[2], dyq[3]),
                         make_float4(dxq[0], dxq[1], dxq[2], dxq[3]), V.Q, C.l0, V.push);
            V.Qsent = __shfl_down_sync(kAll, V.Q, 1);
        }
    }
}

// ==========================================================================
// kernel (sw_tangent.cu's lin_tan_kernel with the affine cell)
// ==========================================================================
template <bool HV, bool DOT, bool SPLIT, bool PG, bool BF>
__global__ void __launch_bounds__(kNW * 32, 1) aff_tan_kernel(SwArgs p) {
    extern __shared__ __align__(16) unsigned char smem_raw[];
    WarpSmem& W = reinterpret_cast<WarpSmem*>(smem_raw)[threadIdx.x >> 5];
    __shared__ int progF[kNW], progR[kNW];
    __shared__ __align__(16) double red[2 * 32];
    __shared__ int sh_Sint, sh_err, sh_bad;
    __shared__ float sh_Sfrac, sh_dSr;
    __shared__ __align__(16) float zv[4 * kHR];   // staging of a missing neighbour: zeros
    __shared__ float zf[kHR / 4];

    const int K = SPLIT ? p.parts : 1;
    const int part = SPLIT ? (int)(blockIdx.x % K) : 0;
    const int b = SPLIT ? (int)(blockIdx.x / K) : (int)blockIdx.x;
    if (p.only && p.only[b] == 0) return;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int gw = part * kNW + warp, NWt = K * kNW;
    int* const gsync = SPLIT ? p.sync + (size_t)b * (kSyncBytes / 4) : nullptr;
    double* const gpart = SPLIT ? reinterpret_cast<double*>(gsync + 64) : nullptr;
    const bool xin = SPLIT && K > 1 && warp == 0;
    const bool xout = SPLIT && K > 1 && warp == kNW - 1;
    const int pin = (part + K - 1) % K;
    const int L1m = p.L1, L2m = p.L2;
    const int L1 = p.lengths ? min(max(p.lengths[2 * b], 0), L1m) : L1m;
    const int L2 = p.lengths ? min(max(p.lengths[2 * b + 1], 0), L2m) : L2m;
    const float go = p.gap_dev ? __ldg(p.gap_dev) : p.gap;
    const float ge = p.gap2_dev ? __ldg(p.gap2_dev) : p.gap2;
    const float T = p.temp_dev ? __ldg(p.temp_dev) : p.temp;
    const float c = kLog2e / T;
    const float Go = ex2f(go * c), Ge = ex2f(ge * c);
    Dir dir;
    const float iT = 1.f / T, iT2 = 1.f / (T * T);
    dir.vs = p.mode == MODE_HVP ? iT : 0.f;
    dir.ss = p.mode == MODE_PT ? -iT2 : 0.f;
    dir.go = PG ? iT : (p.mode == MODE_PGAP ? iT : (p.mode == MODE_PT ? -go * iT2 : 0.f));
    dir.ge = PG ? 0.f : (p.mode == MODE_PGE ? iT : (p.mode == MODE_PT ? -ge * iT2 : 0.f));
    const size_t plane = (size_t)L1m * L2m;
    const float* __restrict__ S = p.scores + (size_t)b * plane;
    const float* __restrict__ Vp = HV ? (DOT ? p.dot_with : p.tangent) + (size_t)b * plane : nullptr;
    float* __restrict__ out = (!DOT && p.out) ? p.out + (size_t)b * plane : nullptr;
    const Layout LY = carve(p.ws, b, L1m, L2m, PG);
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
            if (DOT && p.dot_out) p.dot_out[b] = 0.f;
            if (BF && p.dot_out) p.dot_out[b] = p.dot_out[2 * p.B + b] = 0.f;
            if (PG) {  // S = log(1) = 0, and so its derivatives
                if (p.value) p.value[b] = 0.f;
                if (p.grad_gap) p.grad_gap[b] = 0.f;
                if (p.grad_gap2) p.grad_gap2[b] = 0.f;
                if (p.grad_T) p.grad_T[b] = 0.f;
            }
            if (p.redo && !PG) p.redo[b] = 0;  // PG: zeroed by the launcher
        }
        return;
    }
    if (threadIdx.x < kNW) {
        progF[threadIdx.x] = -1;
        progR[threadIdx.x] = -1;
    }
    for (int i = threadIdx.x; i < 4 * kHR; i += blockDim.x) zv[i] = 0.f;
    if (threadIdx.x < kHR / 4) zf[threadIdx.x] = 0.f;
    if (lane < kHR / 16) W.tag[lane] = -1;
    if (threadIdx.x == 0) {
        sh_err = 0;
        sh_bad = 0;
    }
    __syncthreads();
    const int wprev = (warp + kNW - 1) % kNW, wnext = (warp + 1) % kNW;
    WarpSmem& Wn = reinterpret_cast<WarpSmem*>(smem_raw)[wnext];
    const size_t hzst = (size_t)hz_stride(L2m), hfst = (size_t)hf_stride(L2m);

    auto copy_stage = [&](int ordinal, int x, int rb) {
        if (W.tag[x & (kHR / 16 - 1)] == ((ordinal << 16) | x)) return;
        const int s0 = x == 1 ? 28 : kCW * x, ns = x == 1 ? 1 : 4, g0 = 4 * x;
        float* const rows[4] = {W.s0, W.s1, W.s2, W.s3};
#pragma unroll
        for (int h = 0; h < 4; ++h) {
            const float* const src = LY.h[h] + (size_t)rb * hzst;
            for (int i = 0; i < ns; ++i) cp_async16(rows[h] + ((s0 + 4 * i) & (kHR - 1)), src + s0 + 4 * i, 16);
        }
        cp_async16(W.sf + (g0 & (kHR / 4 - 1)), LY.hfr + (size_t)rb * hfst + g0, 16);
    };
    auto wait_prog = [&](const int* prog, int need) {
        if (xin)
            wait_flag_gpu(prog, need, &sh_err);
        else
            wait_flag(prog, need, &sh_err);
    };
    auto stage_first = [&](const int* prog, int ordinal, int rb, bool reader) {
        wait_prog(prog, (ordinal << 16) + 3);
        if (reader) {
            copy_stage(ordinal, 1, rb);
            copy_stage(ordinal, 2, rb);
        }
    };
    auto stage_need = [&](const int* prog, int ordinal, int k, int rb, bool reader) {
        wait_prog(prog, (ordinal << 16) + min(k + 4, kStageMask));
        if (reader) copy_stage(ordinal, k + 3, rb);
    };
    auto write_tail = [&](int rb, int n, float fr) {
#pragma unroll
        for (int h = 0; h < 4; ++h) {
            float* const o = LY.h[h] + (size_t)rb * hzst + kCW * n;
#pragma unroll 4
            for (int i = 0; i < 12; ++i) *reinterpret_cast<float4*>(o + 4 * i) = make_float4(0.f, 0.f, 0.f, 0.f);
        }
        float* const of = LY.hfr + (size_t)rb * hfst + 4 * n;
#pragma unroll
        for (int i = 0; i < 3; ++i) *reinterpret_cast<float4*>(of + 4 * i) = make_float4(fr, fr, fr, fr);
    };

    // ============================== forward ==============================
    FwdVars V;
    V.acc = V.dacc = 0.0;
    V.ab = 0.f;
    V.gsum = V.dgsum = 0.f;
    V.E = 0.f;
    V.ebmin = V.ebmax = 0x3f800000;
    V.emax = 0.f;
    const int* const prodF = xin ? gsync + pin : &progF[wprev];
    const int* const prodR = xin ? gsync + kMaxParts + pin : &progR[wprev];
    for (int r = gw; r < nRB; r += NWt) {
        const int nv = min(32, L1 - 32 * r);
        const int nst = (L2 + nv - 1 + kCW - 1) / kCW;
        const bool hasB = r > 0, hasD = r + 1 < nRB;
        FwdCtx C;
        C.ring = W.ringS + lane * kRW;
        C.vring = W.ringV + lane * kRW;
        C.as = (hasB && lane == 0) ? W.s0 : zv;
        C.af = (hasB && lane == 0) ? W.sf : zf;
#pragma unroll
        for (int h = 0; h < 4; ++h) C.oh[h] = LY.h[h] + (size_t)r * hzst;
        C.of = LY.hfr + (size_t)r * hfst;
        C.pv = (unsigned)__cvta_generic_to_shared(Wn.s0);
        C.mrow = LY.mpl + (size_t)r * zst + lane;
        C.dmrow = LY.dmpl + (size_t)r * zst + lane;
        C.xrow = PG ? LY.xpl + (size_t)r * zst + lane : nullptr;
        C.erow = LY.efr + (size_t)r * est + lane;
        C.c = c;
        C.Go = Go;
        C.Ge = Ge;
        C.dir = dir;
        C.notl0 = lane == 0 ? 0.f : 1.f;
        C.lane = lane;
        C.nv = nv;
        C.L2 = L2;
        C.l0 = lane == 0;
        C.l31 = lane == 31;
        const Tile tS = make_tile(S + (size_t)(32 * r) * L2m, L2m, W.ringS, nv, lane);
        const Tile tV = make_tile(HV && !DOT ? Vp + (size_t)(32 * r) * L2m : S, L2m, W.ringV, nv, lane);

        __syncwarp();
        if (lane == 31) st_release(&progF[warp], r << 16);
        if (0 < nch) {
            tile_load<4>(tS, 0, L2);
            if (HV && !DOT) tile_load<4>(tV, 0, L2);
        }
        if (hasB) stage_first(prodF, r - 1, r - 1, lane == 0);
        cp_async_commit();
        V.Mp = V.Dp = V.Td = V.ur = V.Tr = V.Tl = 0.f;
        V.dMp = V.dDp = V.dTd = V.dur = V.dTr = 0.f;
        V.f.d1 = 0.f;
        for (int k = 0; k < nst; ++k) {
            __syncwarp();
            if (hasB) stage_need(prodF, r - 1, k, r - 1, lane == 0);
            cp_async_commit();
            if (k + 1 < nch) {
                tile_load<4>(tS, k + 1, L2);
                if (HV && !DOT) tile_load<4>(tV, k + 1, L2);
            }
            cp_async_commit();
            cp_async_wait2();
            __syncwarp();
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
                fwd_stage_start<HV && !DOT, PG>(C, V, k);
            else if (nv == 32 && kCW * k + kCW - 1 <= L2 - 1)
                fwd_stage_full<false, HV && !DOT, PG>(C, V, k, 0);
            else
                fwd_stage_full<true, HV && !DOT, PG>(C, V, k, lane < nv ? L2 + lane - kCW * k : -1);
            acc_rebase2(V);
            if (V.push) Wn.tag[k & (kHR / 16 - 1)] = (r << 16) | k;
            __syncwarp();
            if (lane == 31) {
                st_release(&progF[warp], (r << 16) | min(k + 1, kStageMask - 1));
                if (xout) st_release_gpu(gsync + part, (r << 16) | min(k + 1, kStageMask - 1));
            }
        }
        {
            const double sc = p2d(V.E - V.ab);
            V.acc = fma((double)V.gsum, sc, V.acc);
            V.dacc = fma((double)V.dgsum, sc, V.dacc);
        }
        V.emax = fmaxf(V.emax, V.E - V.ab);
        V.gsum = V.dgsum = 0.f;
        if (lane == 31) write_tail(r, nst, V.E);
        cp_async_wait0();
        __syncwarp();
        if (lane == 31) {
            st_release(&progF[warp], (r << 16) | kStageMask);
            if (xout) st_release_gpu(gsync + part, (r << 16) | kStageMask);
        }
    }
    const int fwd_out = ((V.ebmin < ((127 - kJMax) << 23) || V.ebmax > ((127 + kJMax) << 23)) ? 1 : 0) |
                        (V.emax > 1000.f ? 8 : 0);
    if (lane < kHR / 16) W.tag[lane] = -1;

    {
        float* redf = reinterpret_cast<float*>(red);
        const float abl = block_max(V.ab, redf);
        const double scl = p2d(V.ab - abl);
        const double totl = block_sum_d(V.acc * scl, red);
        const double dtotl = block_sum_d(V.dacc * scl, red);
        if (threadIdx.x == 0) {
            float abmax = abl;
            double tot = totl, dtot = dtotl;
            if (SPLIT && K > 1) {
                double* const g = gpart + kSyncPartDoubles * part;
                g[0] = (double)abl;
                g[1] = totl;
                g[2] = dtotl;
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
                for (int k = 0; k < K; ++k) abmax = fmaxf(abmax, (float)gpart[kSyncPartDoubles * k]);
                tot = dtot = 0.0;
                for (int k = 0; k < K; ++k) {
                    const double sk = p2d((float)gpart[kSyncPartDoubles * k] - abmax);
                    tot = fma(gpart[kSyncPartDoubles * k + 1], sk, tot);
                    dtot = fma(gpart[kSyncPartDoubles * k + 2], sk, dtot);
                }
            }
            tot += p2d(-abmax);  // M[0,0] = 0
            const int hi = __double2hiint(tot);
            const int ef = (hi >> 20) & 0x7ff;
            const bool fin = ef != 0x7ff && ef != 0;
            const double m = __hiloint2double((hi & 0x800fffff) | 0x3ff00000, __double2loint(tot));
            sh_Sint = ef - 1023 + (int)abmax;
            sh_Sfrac = lg2_rr((float)m);
            const double q = dtot / tot;
            sh_dSr = (float)q;
            if (!fin || !(fabs(q) < 1e30)) sh_bad = 1;
            if (PG && part == 0) {
                if (p.value) p.value[b] = ((float)sh_Sint + sh_Sfrac) / c;
                if (p.grad_gap) p.grad_gap[b] = (float)(q * (double)T);
            }
        }
        __syncthreads();
    }

    // ============================== reverse ==============================
    const int P = kCW * ((L2 - 1 + kCW - 1) / kCW);
    const int nstR = P / kCW + 2;
    RevVars RV;
    RV.ebmin = RV.ebmax = 0x3f800000;
    RV.chk = 0.f;
    RV.dot = 0.0;
    RV.dot2 = 0.0;
    RV.dot3 = 0.0;
    for (int q = gw; q < nRB; q += NWt) {
        const int r = nRB - 1 - q;
        const int nv = min(32, L1 - 32 * r);
        const bool hasBelow = r + 1 < nRB, hasAbove = r > 0;
        const float* const mblk = LY.mpl + (size_t)r * zst;
        const float* const dmblk = LY.dmpl + (size_t)r * zst;
        const float* const xblk = PG ? LY.xpl + (size_t)r * zst : nullptr;
        const float* const eblk = LY.efr + (size_t)r * est;
        RevCtx C;
        C.ring = W.ringS + lane * kRW;
        C.vring = W.ringV + lane * kRW;
        C.zr = &W.zr[0][0];
        C.dzr = &W.dzr[0][0];
        C.xr = &W.xr[0][0];
        C.er = W.er;
        C.bs = (hasBelow && lane == nv - 1) ? W.s0 : zv;
        C.bf = (hasBelow && lane == nv - 1) ? W.sf : zf;
#pragma unroll
        for (int h = 0; h < 4; ++h) C.oh[h] = LY.h[h] + (size_t)r * hzst;
        C.of = LY.hfr + (size_t)r * hfst;
        C.pv = (unsigned)__cvta_generic_to_shared(Wn.s0);
        C.c = c;
        C.Go = Go;
        C.Ge = Ge;
        C.cS = ex2f(-sh_Sfrac);
        C.dir = dir;
        C.dSr = sh_dSr;
        C.notBot = lane == nv - 1 ? 0.f : 1.f;
        C.bot = lane == nv - 1;
        C.Sint = (float)sh_Sint;
        C.lane = lane;
        C.nv = nv;
        C.L2 = L2;
        C.P = P;
        C.l0 = lane == 0;
        const float* const srow = S + (size_t)(32 * r) * L2m;
        const Tile tS = make_tile(srow, L2m, W.ringS, nv, lane);
        const Tile tV = make_tile(HV ? Vp + (size_t)(32 * r) * L2m : srow, L2m, W.ringV, nv, lane);
        const Tile tM = make_tile(out ? out + (size_t)(32 * r) * L2m : srow, L2m, W.ringS, nv, lane);

        auto batch = [&](int kb) {
            const int M = P / kCW + 1 - kb;
            const size_t o16 = (size_t)(16 * M) * 32;
#pragma unroll
            for (int it = 0; it < 4; ++it) {
                const int e = 4 * (lane + 32 * it);
                cp_async16(&W.zr[M & 1][0] + e, mblk + o16 + e, 16);
                cp_async16(&W.dzr[M & 1][0] + e, dmblk + o16 + e, 16);  // PG: I
                if (PG) cp_async16(&W.xr[M & 1][0] + e, xblk + o16 + e, 16);
            }
            const int gl = 4 * M - 1;
#pragma unroll
            for (int it = 0; it < 2; ++it) {
                const int cc = lane + 32 * it, g = gl + (cc >> 3), c4 = cc & 7;
                if (cc < 40 && g >= 0) cp_async16(W.er + (g & 15) * 32 + 4 * c4, eblk + (size_t)g * 32 + 4 * c4, 16);
            }
        };
        auto loads = [&](int ch) {
            if (ch >= 0 && ch < nch) {
                tile_load<4>(tS, ch, L2);
                if (HV) tile_load<4>(tV, ch, L2);
            }
        };

        __syncwarp();
        if (lane == 0) st_release(&progR[warp], q << 16);
        {
            const int M0 = P / kCW + 1;
            for (int ch = M0; ch >= M0 - 2; --ch) loads(ch);
        }
        batch(0);
        if (hasBelow) stage_first(prodR, q - 1, r + 1, lane == nv - 1);
        cp_async_commit();

        RV.BDp = RV.PBp = RV.Yr = RV.Xr = RV.BMl = 0.f;
        RV.dBDp = RV.dPBp = RV.dYr = RV.dXr = 0.f;
        RV.Q = 0.f;
        RV.Qsent = 0.f;
        RV.f.d1 = 0.f;
        for (int k = 0; k < nstR; ++k) {
            const int M = P / kCW + 1 - k;
            __syncwarp();
            if (hasBelow) stage_need(prodR, q - 1, k, r + 1, lane == nv - 1);
            cp_async_commit();
            if (out && M + 1 < nch && M + 1 >= 0) tile_store(tM, M + 1, L2);
            loads(M - 3);
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
            RV.sdot = 0.f;
            RV.sgap = 0.f;
            RV.sx1 = 0.f;
            if (kCW * k <= P + 32 - L2)
                rev_stage_part<HV, DOT, PG, BF>(C, RV, k);
            else if (nv == 32 && kCW * k + kCW - 1 <= P - 1)
                rev_stage_full<false, HV, DOT, PG, BF>(C, RV, k, 0);
            else
                rev_stage_full<true, HV, DOT, PG, BF>(C, RV, k, lane < nv ? 16 * M + 16 - lane : -1);
            if (DOT || PG || BF) RV.dot += (double)RV.sdot;
            if (PG) RV.dot2 += (double)RV.sgap;
            if (BF) RV.dot3 += (double)RV.sx1;
            if (RV.push) Wn.tag[k & (kHR / 16 - 1)] = (q << 16) | k;
            __syncwarp();
            if (lane == 0) {
                st_release(&progR[warp], (q << 16) | min(k + 1, kStageMask - 1));
                if (xout) st_release_gpu(gsync + kMaxParts + part, (q << 16) | min(k + 1, kStageMask - 1));
            }
        }
        if (lane == 0) write_tail(r, nstR, RV.Q);
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
    const int o_tan = __syncthreads_or(RV.chk != 0.f ? 1 : 0);
    const int redo = (o_win ? 1 : 0) | (sh_err ? 2 : 0) | (sh_bad ? 4 : 0) | (o_acc ? 8 : 0) | (o_tan ? 16 : 0);
    if (DOT || PG || BF) {
        const double tot = block_sum_d(RV.dot, red);
        const double tot2 = PG ? block_sum_d(RV.dot2, red) : 0.0;
        const double tot3 = BF ? block_sum_d(RV.dot3, red) : 0.0;
        if (threadIdx.x == 0) {
            // DOT: the weighted sum.  PG: dS/dge = (I and D visits) - dS/dgo,
            // dS/dT = (S - sum s mu - go dS/dgo - ge dS/dge) / T.  BF: the
            // tangents along g of dS/dgo (all3) and, by Euler, of dS/dT from
            // sum s dmu (all) and the caller's d(dS/dge)[g] in dot_out[B + b]
            auto finish = [&](double all, double visits, double all3) {
                if (BF && p.dot_out) {
                    const double gge = (double)p.dot_out[p.B + b];
                    p.dot_out[b] = (float)all3;
                    p.dot_out[2 * p.B + b] = (float)(-(all + (double)go * all3 + (double)ge * gge) / (double)T);
                }
                if (DOT && p.dot_out) p.dot_out[b] = (float)all;
                if (PG) {
                    const double S = ((double)sh_Sint + (double)sh_Sfrac) / (double)c;
                    const double eo = (double)sh_dSr * (double)T;
                    const double ee = visits - eo;
                    if (p.grad_gap2) p.grad_gap2[b] = (float)ee;
                    if (p.grad_T) p.grad_T[b] = (float)((S - all - (double)go * eo - (double)ge * ee) / (double)T);
                }
            };
            if (SPLIT && K > 1) {
                gpart[kSyncPartDoubles * part + 3] = tot;
                if (PG) gpart[kSyncPartDoubles * part + 4] = tot2;
                if (BF) gpart[kSyncPartDoubles * part + 4] = tot3;   // (slot 4: PG's, unused by BF)
                if (atom_add_release_gpu(gsync + 2 * kMaxParts + 1, 1) == K - 1) {
                    (void)ld_acquire_gpu(gsync + 2 * kMaxParts + 1);
                    double all = 0.0, all2 = 0.0, all3 = 0.0;
                    for (int k = 0; k < K; ++k) {
                        all += gpart[kSyncPartDoubles * k + 3];
                        if (PG) all2 += gpart[kSyncPartDoubles * k + 4];
                        if (BF) all3 += gpart[kSyncPartDoubles * k + 4];
                    }
                    finish(all, all2, all3);
                }
            } else {
                finish(tot, tot2, tot3);
            }
        }
    }
    if (threadIdx.x == 0 && p.redo) {
        if (SPLIT || PG)
            atomicOr(p.redo + b, redo);
        else
            p.redo[b] = redo;
    }
}

}  // namespace atan_

// ------------------------------------------------------------------ host side
size_t aff_tan_workspace_bytes(int B, int L1, int L2, bool pg) {
    if (L1 > 32 * atan_::kMaxRB || L2 % 4 != 0) return 0;
    return atan_::per_problem_bytes(L1, L2, pg) * (size_t)B;
}

int launch_aff_tan(const SwArgs& a, size_t ws_bytes, cudaStream_t st) {
    // PG: value + marginals + parameter gradients (one sweep pair, see the kernel)
    const bool pg = a.mode == MODE_MARG && (a.grad_gap || a.grad_gap2 || a.grad_T);
    if (a.mode != MODE_HVP && a.mode != MODE_PGAP && a.mode != MODE_PGE && a.mode != MODE_PT && !pg) return -1;
    if (!a.redo || engine_forced_plane()) return -1;
    if (a.L2 % 4 != 0 || a.L1 > 32 * atan_::kMaxRB || a.L1 == 0 || a.L2 == 0) return -1;
    const bool dot = a.dot_with != nullptr;
    const bool hv = a.mode == MODE_HVP || dot;
    // BF: backward_full's sweep pair -- the HVP along a.tangent into a.out,
    // and per problem d(dS/dgo) and d(dS/dT) along it into a.dot_out[b] and
    // [2 B + b], from d(dS/dge) in a.dot_out[B + b] (written before)
    const bool bf = a.mode == MODE_HVP && !dot && a.dot_out != nullptr;
    if (a.mode == MODE_HVP && (dot || !a.tangent)) return -1;
    if (dot && !a.dot_out) return -1;
    if (!dot && !a.out && !pg) return -1;
    if (pg && (dot || a.tangent)) return -1;
    auto al16 = [](const void* q) { return (((uintptr_t)q) & 15) == 0; };
    if (!a.scores || !al16(a.scores) || (a.out && !al16(a.out)) || !a.ws) return -1;
    if ((a.tangent && !al16(a.tangent)) || (dot && !al16(a.dot_with))) return -1;
    if ((((uintptr_t)a.ws) & 255) != 0) return -1;
    if (ws_bytes < atan_::per_problem_bytes(a.L1, a.L2, pg) * (size_t)a.B) return -1;
    const size_t smem = sizeof(atan_::WarpSmem) * atan_::kNW;
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return (int)e;
    static DeviceSetup setup;
    int nsm = 0;
    const int se = device_setup(setup, dev, [smem] {
        const void* ks[10] = {(const void*)atan_::aff_tan_kernel<true, false, false, false, false>,
                              (const void*)atan_::aff_tan_kernel<false, false, false, false, false>,
                              (const void*)atan_::aff_tan_kernel<true, true, false, false, false>,
                              (const void*)atan_::aff_tan_kernel<true, false, true, false, false>,
                              (const void*)atan_::aff_tan_kernel<false, false, true, false, false>,
                              (const void*)atan_::aff_tan_kernel<true, true, true, false, false>,
                              (const void*)atan_::aff_tan_kernel<false, false, false, true, false>,
                              (const void*)atan_::aff_tan_kernel<false, false, true, true, false>,
                              (const void*)atan_::aff_tan_kernel<true, false, false, false, true>,
                              (const void*)atan_::aff_tan_kernel<true, false, true, false, true>};
        for (const void* k : ks) {
            cudaError_t r = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
            if (r == cudaSuccess)
                r = cudaFuncSetAttribute(k, cudaFuncAttributePreferredSharedMemoryCarveout,
                                         (int)cudaSharedmemCarveoutMaxShared);
            if (r != cudaSuccess) return (int)r;
        }
        return 0;
    }, &nsm);
    if (se != 0) return se;
    const int K = a.sync ? lin_parts_nw(a.B, a.L1, a.L2, nsm, atan_::kNW) : 1;
    // one sweep pair; a spread launch zeroes the flags itself unless told not
    // to (PG zeroes them before the launch: its kernels OR their bits in)
    auto sweep = [&](const SwArgs& x, bool zero_redo) -> cudaError_t {
        cudaError_t err;
        if (K > 1) {
            SwArgs s = x;
            s.parts = K;
            err = cudaMemsetAsync(s.sync, 0, kSyncBytes * (size_t)s.B, st);
            if (err == cudaSuccess && zero_redo) err = cudaMemsetAsync(s.redo, 0, sizeof(int) * (size_t)s.B, st);
            if (err != cudaSuccess) return err;
            void* args[1] = {&s};
            const void* k = pg    ? (const void*)atan_::aff_tan_kernel<false, false, true, true, false>
                            : bf  ? (const void*)atan_::aff_tan_kernel<true, false, true, false, true>
                            : dot ? (const void*)atan_::aff_tan_kernel<true, true, true, false, false>
                            : hv  ? (const void*)atan_::aff_tan_kernel<true, false, true, false, false>
                                  : (const void*)atan_::aff_tan_kernel<false, false, true, false, false>;
            err = cudaLaunchCooperativeKernel(k, dim3(s.B * K), dim3(atan_::kNW * 32), args, smem, st);
            if (err == cudaSuccess) return err;
            cudaGetLastError();  // does not fit: one CTA per problem instead
        }
        if (pg)
            atan_::aff_tan_kernel<false, false, false, true, false><<<x.B, atan_::kNW * 32, smem, st>>>(x);
        else if (bf)
            atan_::aff_tan_kernel<true, false, false, false, true><<<x.B, atan_::kNW * 32, smem, st>>>(x);
        else if (dot)
            atan_::aff_tan_kernel<true, true, false, false, false><<<x.B, atan_::kNW * 32, smem, st>>>(x);
        else if (hv)
            atan_::aff_tan_kernel<true, false, false, false, false><<<x.B, atan_::kNW * 32, smem, st>>>(x);
        else
            atan_::aff_tan_kernel<false, false, false, false, false><<<x.B, atan_::kNW * 32, smem, st>>>(x);
        return cudaGetLastError();
    };
    if (!pg) return (int)sweep(a, true);
    // PG: one sweep pair; its flags are ORed in (zeroed here)
    e = cudaMemsetAsync(a.redo, 0, sizeof(int) * (size_t)a.B, st);
    if (e != cudaSuccess) return (int)e;
    return (int)sweep(a, false);
}

}  // namespace d2pb
