// sw_tangent.cu -- linear-domain tangent sweeps for linear-gap soft
// Smith-Waterman: the directional derivative of the marginals,
//   dmu = d/de mu(s + e V, gap + e dgap, T + e dT),
// which is the Hessian-vector product (src/sw/kernels_cpu.cpp:288-485,
// direction V in the scores), the parameter Jacobians dP/dgap and dP/dT
// (src/sw/kernels_cpu.cpp:500-710), and, contracted with a weight plane, the
// parameter half of the marginals' vector-Jacobian product (backward_full,
// src/sw/torch_cuda.cpp:666-771).
//
// In the linear domain of sw_linear.cu (Z = 2^a, P = 2^(s c), G = 2^(gap c),
// c = log2(e)/T) every quantity is a product of P's and G's, so the tangent
// of each recurrence is the same recurrence with a source term.  With
// dP = P vp (vp = V/T for a direction V; -s/T^2 for T) and dG = G gam
// (gam = 1/T for gap; -gap/T^2 for T):
//   w = P (Z_diag + 1)                 dw = w vp + P dZ_diag
//   Z = w + G (Z_up + Z_left)          dZ = dw + G (dZ_up + dZ_left) + gam (Z - w)
//   B = 1 + P' B' + G (B_down + B_right)     (P' B' the diagonal successor's)
//   dB = d(P' B') + G (dB_down + dB_right) + gam G (B_down + B_right),
//   d(P B) = P (vp B + dB)
//   mu = B w / Z_total                 dmu = (dB w + B dw) / Z_total - mu dZ_total / Z_total
// A tangent shares its value's power-of-two frame, so the frames, stages,
// row-block pipeline and handoff routes are sw_linear.cu's, with a second
// value (the tangent) wherever a value crosses lanes or row-blocks.  The
// forward stores w and dw per cell; the reverse writes dmu, or, in the dot
// mode, sums weight * dmu per problem.  A problem whose frames leave the
// window, whose partition is not finite, or whose tangent overflowed, is
// flagged, and the caller recomputes it with the plane engine (sw_plane.cu).
//
// BF (backward_full in one sweep pair): the HVP along the weight plane g gives
// grad_scores = H g (the Hessian of S is symmetric).  The parameter parts are
// sum g dP/dgap = d(dS/dgap)[g] and sum g dP/dT = d(dS/dT)[g].  dS/dgap is
// the sum over cells of the gap flow B gz / Z_total, with gz = G (Z_up +
// Z_left) the gap part of Z, so its tangent along g is a per-cell sum in the
// reverse, from gz and dgz kept by the forward.  Differentiating Euler's
// identity S = sum s mu + gap dS/dgap + T dS/dT along g gives
// d(dS/dT)[g] = -(sum s H g + gap d(dS/dgap)[g]) / T.
#include <stddef.h>
#include <stdint.h>

#include "sw_common.cuh"
#include "sw_internal.h"
#include "sw_lindomain.cuh"
#include "sw_ring.cuh"

namespace d2pb {
namespace ltan {
using namespace ring;
using namespace ld;

constexpr int kMaxRB = 512;  // row-blocks per problem (L1 <= 16384)
constexpr int kNW = 6;       // warps per CTA, one CTA per SM

struct WarpSmem {
    float ringS[32 * kRW];    // scores [rows][64]; reverse: dmu written in place
    float ringV[32 * kRW];    // the direction V (HVP) or the weights of the dot mode, likewise
    float zr[2][16 * 32];     // reverse: the forward's w of 16 anti-diagonals, two slots
    float dzr[2][16 * 32];    //          and its dw
    float gzr[2][16 * 32];    //          BF: the gap part of Z
    float dgzr[2][16 * 32];   //          and its tangent
    float er[16 * 32];        // reverse: forward frames, 16 group slots
    // staging of the neighbouring row-block's boundary values and tangents by
    // its step, and their frames by its group; tags as in sw_linear.cu
    float sv[kHR];
    float sdv[kHR];
    float sf[kHR / 4];
    int tag[kHR / 16];
};
static_assert(sizeof(WarpSmem) % 16 == 0, "per-warp shared blocks must stay 16-byte aligned");
static_assert(offsetof(WarpSmem, sdv) == offsetof(WarpSmem, sv) + 4 * kHR &&
                  offsetof(WarpSmem, sf) == offsetof(WarpSmem, sv) + 8 * kHR,
              "sv, sdv, sf are contiguous");

struct Layout {  // per-problem workspace
    float* zpl;   // [nRB][ZT][32]   w of forward step t (frame E) at row t
    float* dzpl;  // [nRB][ZT][32]   dw likewise
    float* efr;   // [nRB][GT][32]   frame of each lane for each group of 4 forward steps
    float* hz;    // [nRB][HZ]       boundary values of each row-block, by its step
    float* hdz;   // [nRB][HZ]       and their tangents
    float* hfr;   // [nRB][HF]       and their frames, by its group
    float* gzpl;  // [nRB][ZT][32]   BF: gap part of Z (frame E)
    float* dgzpl; // [nRB][ZT][32]   BF: its tangent
};
__host__ __device__ inline size_t per_problem_bytes(int L1m, int L2m, bool bf = false) {
    const size_t nrb = (size_t)(L1m + 31) / 32;
    return (bf ? 4 : 2) * align_up(nrb * zt_rows(L2m) * 32 * 4, 256) + align_up(nrb * gt_rows(L2m) * 32 * 4, 256) +
           2 * align_up(nrb * hz_stride(L2m) * 4, 256) + align_up(nrb * hf_stride(L2m) * 4, 256);
}
__device__ inline Layout carve(float* ws, int b, int L1m, int L2m, bool bf) {
    const size_t nrb = (size_t)(L1m + 31) / 32;
    char* base = (char*)ws + (size_t)b * per_problem_bytes(L1m, L2m, bf);
    Layout L;
    L.zpl = (float*)base;
    base += align_up(nrb * zt_rows(L2m) * 32 * 4, 256);
    L.dzpl = (float*)base;
    base += align_up(nrb * zt_rows(L2m) * 32 * 4, 256);
    L.efr = (float*)base;
    base += align_up(nrb * gt_rows(L2m) * 32 * 4, 256);
    L.hz = (float*)base;
    base += align_up(nrb * hz_stride(L2m) * 4, 256);
    L.hdz = (float*)base;
    base += align_up(nrb * hz_stride(L2m) * 4, 256);
    L.hfr = (float*)base;
    base += align_up(nrb * hf_stride(L2m) * 4, 256);
    L.gzpl = bf ? (float*)base : nullptr;
    base += align_up(nrb * zt_rows(L2m) * 32 * 4, 256);
    L.dgzpl = bf ? (float*)base : nullptr;
    return L;
}

// the direction of the sweep: dP = P (vs V + ss s), dG = G gam
struct Dir {
    float vs, ss, gam;
};

// One group of the boundary lane's (bnd) values, tangents and frame: into the
// consumer warp's staging ring while it keeps up (pp), else to the row-block's
// boundary rows in global memory (sw_linear.cu's handoff, with two values).
template <class Ctx>
__device__ __forceinline__ void handoff(const Ctx& C, int g, float4 v, float4 dv, float fr, bool bnd, bool pp) {
    stg_pair_pred(C.ov + 4 * g, C.odv + 4 * g, C.of + g, v, dv, fr, bnd && !pp);
    const unsigned sv = C.pv + 16u * (unsigned)(g & (kHR / 4 - 1));
    const unsigned sf = C.pv + 8u * kHR + 4u * (unsigned)(g & (kHR / 4 - 1));
    sts_group_pred_s(sv, sf, v, fr, pp);
    sts_group_pred_s(sv + 4u * kHR, sf, dv, fr, pp);
}

// ==========================================================================
// forward sweep of one row-block
// ==========================================================================
struct FwdF {
    float d0, d1;       // 2^(E_{l-1} - E) for the up input of the first / other steps (lane 0: 0)
    float Gd0, Gd1;
    float fs;           // 2^-E
    float za[4], dza[4];  // lane 0: the row above's value and tangent for each step, frame E
};

struct FwdVars {
    bool push;
    float zl, zd, zsh;      // own z of the previous step; diagonal input; lane l-1's last z
    float dzl, dzd, dzsh;   // their tangents
    float E, Esent;
    FwdF f;
    float nE, nfJ;
    FwdF nf;
    float gsum, dgsum;      // this group's sums of z and dz (frame E)
    double acc, dacc;       // partition and its tangent so far: sum Z 2^-ab, sum dZ 2^-ab
    float ab;
    int ebmin, ebmax;
    float emax;
};

struct FwdCtx {
    const float* ring;   // this lane's score ring row
    const float* vring;  // this lane's V ring row (HVP)
    const float* av;     // lane 0: staged values, tangents (av + kHR) and frames of the row above
    const float* af;
    float* ov;           // this row-block's boundary rows (global)
    float* odv;
    float* of;
    unsigned pv;         // shared address of the consumer warp's staging ring
    float* zrow;         // zpl row 0 of this row-block, this lane
    float* dzrow;        // dzpl likewise
    float* gzrow;        // BF: gzpl, dgzpl likewise
    float* dgzrow;
    float* erow;
    float c, G;
    Dir dir;
    float notl0;
    int lane, nv, L2;
    bool l0, l31;
};

__device__ __forceinline__ FwdF fwd_factors(const FwdCtx& C, float E, float eup0, float eup1) {
    FwdF f;
    f.d0 = p2(eup0 - E) * C.notl0;
    f.d1 = p2(eup1 - E) * C.notl0;
    f.Gd0 = C.G * f.d0;
    f.Gd1 = C.G * f.d1;
    f.fs = p2(-E);
#pragma unroll
    for (int q = 0; q < 4; ++q) f.za[q] = f.dza[q] = 0.f;
    return f;
}

// the next group's frame and factors (sw_linear.cu's fwd_lookahead), with the
// row above's tangents converted like its values
__device__ __forceinline__ void fwd_lookahead(const FwdCtx& C, FwdVars& V, int g) {
    const int eb = efield(V.zl);
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
    V.nf.Gd0 = C.G * V.nf.d0;
    V.nf.Gd1 = C.G * V.nf.d1;
    V.nf.fs = p2(-V.nE);
    const int s0 = (4 * g + 31) & (kHR - 1), s1 = (4 * g + 32) & (kHR - 1);
    const float4 a = *reinterpret_cast<const float4*>(C.av + s1);
    const float4 da = *reinterpret_cast<const float4*>(C.av + kHR + s1);
    V.nf.za[0] = C.av[s0] * w;
    V.nf.za[1] = a.x;
    V.nf.za[2] = a.y;
    V.nf.za[3] = a.z;
    V.nf.dza[0] = C.av[kHR + s0] * w;
    V.nf.dza[1] = da.x;
    V.nf.dza[2] = da.y;
    V.nf.dza[3] = da.z;
}

__device__ __forceinline__ void fwd_apply(FwdVars& V) {
    const float dE = V.E - V.ab;
    const double sc = p2d(dE);
    V.acc = fma((double)V.gsum, sc, V.acc);
    V.dacc = fma((double)V.dgsum, sc, V.dacc);
    V.emax = fmaxf(V.emax, dE);
    V.gsum = V.dgsum = 0.f;
    V.zl *= V.nfJ;
    V.zd *= V.nfJ;
    V.dzl *= V.nfJ;
    V.dzd *= V.nfJ;
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
    float z, dz, zuin, dzuin, w, dw, gz, dgz;
};
// one cell, step i of its group (vv: the lane's V at this cell, HVP only).
// BF: also the gap part of Z and its tangent (gam = 0 along a score direction).
template <bool BF>
__device__ __forceinline__ FwdOut fwd_cell(const FwdCtx& C, const FwdVars& V, int i, float sc, float vv) {
    FwdOut o;
    const float P = ex2f(sc * C.c);
    const float vp = fmaf(C.dir.vs, vv, C.dir.ss * sc);
    const float d = i == 0 ? V.f.d0 : V.f.d1, Gd = i == 0 ? V.f.Gd0 : V.f.Gd1;
    o.w = P * (V.zd + V.f.fs);
    o.dw = fmaf(o.w, vp, P * V.dzd);
    const float zin = V.zl + V.f.za[i], dzin = V.dzl + V.f.dza[i];
    const float rest = fmaf(C.G, zin, o.w);
    o.z = fmaf(Gd, V.zsh, rest);
    const float drest = fmaf(C.G, dzin, o.dw);
    o.dz = fmaf(C.dir.gam, o.z - o.w, fmaf(Gd, V.dzsh, drest));
    o.gz = BF ? fmaf(Gd, V.zsh, C.G * zin) : 0.f;
    o.dgz = BF ? fmaf(Gd, V.dzsh, C.G * dzin) : 0.f;
    o.zuin = fmaf(V.zsh, d, V.f.za[i]);
    o.dzuin = fmaf(V.dzsh, d, V.f.dza[i]);
    return o;
}

template <bool MASK, bool HV, bool BF>
__device__ __forceinline__ void fwd_stage_full(const FwdCtx& C, FwdVars& V, int k, int thr) {
    const int c0 = (kCW * k - C.lane) & (kRW - 1);
    float scv[kCW], vvv[kCW];
#pragma unroll
    for (int u = 0; u < kCW; ++u) {
        const int col = (u < kRW - c0) ? c0 + u : c0 + u - kRW;
        scv[u] = C.ring[col];
        vvv[u] = HV ? C.vring[col] : 0.f;
    }
    float* const pz = C.zrow + (size_t)(kCW * k) * 32;
    float* const pdz = C.dzrow + (size_t)(kCW * k) * 32;
    float* const pgz = BF ? C.gzrow + (size_t)(kCW * k) * 32 : nullptr;
    float* const pdgz = BF ? C.dgzrow + (size_t)(kCW * k) * 32 : nullptr;
    float* const pe = C.erow + (size_t)(kCW * k / 4) * 32;
    float zq[4], dzq[4];
#pragma unroll
    for (int u = 0; u < kCW; ++u) {
        const int i = u & 3;
        if (i == 0) fwd_apply(V);
        if (i == 3) {
            if (u == kCW - 1) cp_async_wait1();
            fwd_lookahead(C, V, 4 * k + (u >> 2) + 1);
        }
        FwdOut o = fwd_cell<BF>(C, V, i, scv[u], vvv[u]);
        if (MASK) {
            const bool act = u < thr;
            o.z = act ? o.z : 0.f;
            o.dz = act ? o.dz : 0.f;
        }
        V.gsum += o.z;
        V.dgsum += o.dz;
        pz[(size_t)u * 32] = o.w;
        pdz[(size_t)u * 32] = o.dw;
        if (BF) {
            pgz[(size_t)u * 32] = o.gz;
            pdgz[(size_t)u * 32] = o.dgz;
        }
        zq[i] = o.z;
        dzq[i] = o.dz;
        if (i == 3) {
            pe[(u >> 2) * 32] = V.E;
            handoff(C, 4 * k + (u >> 2), make_float4(zq[0], zq[1], zq[2], zq[3]),
                    make_float4(dzq[0], dzq[1], dzq[2], dzq[3]), V.E, C.l31, V.push);
        }
        V.zd = o.zuin;
        V.dzd = o.dzuin;
        V.zl = o.z;
        V.dzl = o.dz;
        V.zsh = __shfl_up_sync(kAll, o.z, 1);
        V.dzsh = __shfl_up_sync(kAll, o.dz, 1);
    }
}

template <bool HV, bool BF>
__device__ __forceinline__ void fwd_stage_start(const FwdCtx& C, FwdVars& V, int k) {
    const bool live = C.lane < C.nv;
    float zq[4], dzq[4];
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
            FwdOut o = fwd_cell<BF>(C, V, i, C.ring[col], HV ? C.vring[col] : 0.f);
            o.z = act ? o.z : 0.f;
            o.dz = act ? o.dz : 0.f;
            V.gsum += o.z;
            V.dgsum += o.dz;
            C.zrow[(size_t)t * 32] = o.w;
            C.dzrow[(size_t)t * 32] = o.dw;
            if (BF) {
                C.gzrow[(size_t)t * 32] = o.gz;
                C.dgzrow[(size_t)t * 32] = o.dgz;
            }
            zq[i] = o.z;
            dzq[i] = o.dz;
            if (i == 3) {
                C.erow[(size_t)(t >> 2) * 32] = V.E;
                handoff(C, 4 * k + q, make_float4(zq[0], zq[1], zq[2], zq[3]),
                        make_float4(dzq[0], dzq[1], dzq[2], dzq[3]), V.E, C.l31, V.push);
            }
            V.zd = act ? o.zuin : 0.f;
            V.dzd = act ? o.dzuin : 0.f;
            V.zl = o.z;
            V.dzl = o.dz;
            V.zsh = __shfl_up_sync(kAll, o.z, 1);
            V.dzsh = __shfl_up_sync(kAll, o.dz, 1);
            V.Esent = __shfl_up_sync(kAll, V.E, 1);
        }
    }
}

// ==========================================================================
// reverse sweep of one row-block
// ==========================================================================
struct RevF {
    float d0, d1;        // 2^(Q_{l+1} - Q) for the message of the first / other steps (bottom lane: 0)
    float Gd0, Gd1;
    float fb[4];         // 2^-Q, plus for the bottom lane the message from below (frame Q)
    float dfb[4];        // bottom lane: the tangent of that message
    float kE;            // 2^(Q + E - S)
};

struct RevVars {
    bool push;
    float br, pbp, rsh;     // own b and P b of column j+1; message from lane l+1
    float dbr, dpbp, drsh;  // their tangents
    float Q, Qsent;
    RevF f;
    float nQ, nfJ;
    RevF nf;
    int ebmin, ebmax;
    float chk;              // fma(dmu, 0, chk) over the lane's cells: not 0 if a tangent overflowed
    float sdot;             // dot mode: this stage's sum of weight * dmu (BF: score * dmu)
    double dot;
    float sgap;             // BF: this stage's sum of the gap flows' tangents
    double dot2;
};

struct RevCtx {
    float* ring;
    const float* vring;
    const float* zr;      // WarpSmem::zr, dzr
    const float* dzr;
    const float* gzr;     // BF: WarpSmem::gzr, dgzr
    const float* dgzr;
    const float* er;
    const float* bv;      // bottom lane: staged messages, tangents (bv + kHR), frames of the row-block below
    const float* bf;
    float* ov;
    float* odv;
    float* of;
    unsigned pv;
    float c, G, cS;
    Dir dir;
    float dSr;            // dZ_total / Z_total
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
    f.Gd0 = C.G * f.d0;
    f.Gd1 = C.G * f.d1;
    f.fb[0] = f.fb[1] = f.fb[2] = f.fb[3] = p2(-Q);
    f.dfb[0] = f.dfb[1] = f.dfb[2] = f.dfb[3] = 0.f;
    rev_kfactors(C, f, Q, h);
    return f;
}

// the next group's frame and factors (sw_linear.cu's rev_lookahead), with the
// row-block below's tangents converted like its messages
__device__ __forceinline__ void rev_lookahead(const RevCtx& C, RevVars& V, int h) {
    const int eb = efield(V.br);
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
    V.nf.Gd0 = C.G * V.nf.d0;
    V.nf.Gd1 = C.G * V.nf.d1;
    const float fsq = p2(-V.nQ);
    const int s0 = (4 * h + 31) & (kHR - 1), s1 = (4 * h + 32) & (kHR - 1);
    const float4 e = *reinterpret_cast<const float4*>(C.bv + s1);
    const float4 de = *reinterpret_cast<const float4*>(C.bv + kHR + s1);
    V.nf.fb[0] = fmaf(C.bv[s0], w, fsq);
    V.nf.fb[1] = fsq + e.x;
    V.nf.fb[2] = fsq + e.y;
    V.nf.fb[3] = fsq + e.z;
    V.nf.dfb[0] = C.bv[kHR + s0] * w;
    V.nf.dfb[1] = de.x;
    V.nf.dfb[2] = de.y;
    V.nf.dfb[3] = de.z;
    rev_kfactors(C, V.nf, V.nQ, h);
}

__device__ __forceinline__ void rev_apply(RevVars& V) {
    V.br *= V.nfJ;
    V.pbp *= V.nfJ;
    V.dbr *= V.nfJ;
    V.dpbp *= V.nfJ;
    V.Q = V.nQ;
    V.f = V.nf;
}

struct RevOut {
    float b, pb, msg, db, dpb, dmsg, dmu, dgf;
};
// one cell, step i of its group: vv the lane's V here (HVP), w / dw the
// forward's diagonal term and its tangent.  PG: the marginal itself (in dmu),
// no tangent of the reverse.
// BF: gz / dgz the forward's gap part of Z and its tangent; dgf the tangent of
// the cell's gap flow B gz / Z_total
template <bool PG, bool BF>
__device__ __forceinline__ RevOut rev_cell(const RevCtx& C, const RevVars& V, int i, float sc, float vv, float w,
                                           float dw, float gz, float dgz) {
    RevOut o;
    const float P = ex2f(sc * C.c);
    const float vp = fmaf(C.dir.vs, vv, C.dir.ss * sc);
    const float d = i == 0 ? V.f.d0 : V.f.d1, Gd = i == 0 ? V.f.Gd0 : V.f.Gd1;
    const float rest = fmaf(C.G, V.br, V.f.fb[i]);
    o.b = fmaf(d, V.rsh, rest);
    o.msg = fmaf(Gd, V.rsh, fmaf(C.G, rest, V.pbp));
    o.pb = P * o.b;
    o.dgf = 0.f;
    if (PG) {
        o.db = o.dmsg = o.dpb = 0.f;
        o.dmu = o.b * (w * V.f.kE);
        return o;
    }
    const float drest = fmaf(C.G, fmaf(C.dir.gam, V.br, V.dbr), V.f.dfb[i]);
    o.db = fmaf(d, V.drsh, drest);
    o.dmsg = fmaf(C.G, fmaf(C.dir.gam, o.b, o.db), V.dpbp);
    o.dpb = P * fmaf(vp, o.b, o.db);
    const float mu = o.b * (w * V.f.kE);
    o.dmu = fmaf(fmaf(o.db, w, o.b * dw), V.f.kE, -mu * C.dSr);
    if (BF) {
        const float gf = o.b * (gz * V.f.kE);
        o.dgf = fmaf(fmaf(o.db, gz, o.b * dgz), V.f.kE, -gf * C.dSr);
    }
    return o;
}

// DOT: sum gm * dmu; PG: write the marginal and sum score * marginal (gm is
// the score); otherwise write dmu
template <bool DOT, bool PG, bool BF>
__device__ __forceinline__ void rev_emit(const RevCtx& C, RevVars& V, float* slot, float gm, float dmu, bool act,
                                         float sc, float dgf) {
    if (act) V.chk = fmaf(dmu, 0.f, V.chk);
    if (DOT || PG) {
        if (act) V.sdot = fmaf(gm, dmu, V.sdot);  // a cell outside the problem may hold inf: no 0 * inf
    }
    if (BF) {
        if (act) {
            V.chk = fmaf(dgf, 0.f, V.chk);
            V.sdot = fmaf(sc, dmu, V.sdot);
            V.sgap += dgf;
        }
    }
    if (!DOT) {
        if (act) *slot = dmu;
    }
}

template <bool MASK, bool HV, bool DOT, bool PG, bool BF>
__device__ __forceinline__ void rev_stage_full(const RevCtx& C, RevVars& V, int k, int thr) {
    const int m16 = C.P + 16 - kCW * k;
    const int slot = ((m16 >> 4) & 1) * (16 * 32) + C.lane;
    const float* const zb = C.zr + slot;
    const float* const dzb = C.dzr + slot;
    const float* const gzb = BF ? C.gzr + slot : nullptr;
    const float* const dgzb = BF ? C.dgzr + slot : nullptr;
    const int cb = (C.P + 31 - kCW * k - C.lane) & (kRW - 1);
    float scv[kCW], vvv[kCW];
#pragma unroll
    for (int u = 0; u < kCW; ++u) {
        const int col = (u <= cb) ? cb - u : cb - u + kRW;
        scv[u] = C.ring[col];
        vvv[u] = HV ? C.vring[col] : 0.f;
    }
    float mq[4], dmq[4];
#pragma unroll
    for (int u = 0; u < kCW; ++u) {
        const int i = u & 3;
        if (i == 0) rev_apply(V);
        if (i == 3) {
            if (u == kCW - 1) cp_async_wait1();
            rev_lookahead(C, V, 4 * k + (u >> 2) + 1);
        }
        const RevOut o = rev_cell<PG, BF>(C, V, i, scv[u], DOT ? 0.f : vvv[u], zb[(15 - u) * 32],
                                          PG ? 0.f : dzb[(15 - u) * 32], BF ? gzb[(15 - u) * 32] : 0.f,
                                          BF ? dgzb[(15 - u) * 32] : 0.f);
        const bool act = !MASK || u < thr;
        const int col = (u <= cb) ? cb - u : cb - u + kRW;
        rev_emit<DOT, PG, BF>(C, V, C.ring + col, PG ? scv[u] : vvv[u], o.dmu, act, scv[u], o.dgf);
        const float msg = act ? o.msg : 0.f, dmsg = act ? o.dmsg : 0.f;
        mq[i] = msg;
        dmq[i] = dmsg;
        if (i == 3)
            handoff(C, 4 * k + (u >> 2), make_float4(mq[0], mq[1], mq[2], mq[3]),
                    make_float4(dmq[0], dmq[1], dmq[2], dmq[3]), V.Q, C.l0, V.push);
        V.rsh = __shfl_down_sync(kAll, msg, 1);
        V.drsh = __shfl_down_sync(kAll, dmsg, 1);
        V.br = act ? o.b : 0.f;
        V.pbp = act ? o.pb : 0.f;
        V.dbr = act ? o.db : 0.f;
        V.dpbp = act ? o.dpb : 0.f;
    }
}

template <bool HV, bool DOT, bool PG, bool BF>
__device__ __forceinline__ void rev_stage_part(const RevCtx& C, RevVars& V, int k) {
    const int m16 = C.P + 16 - kCW * k;
    const int slot = ((m16 >> 4) & 1) * (16 * 32) + C.lane;
    const float* const zb = C.zr + slot;
    const float* const dzb = C.dzr + slot;
    const float* const gzb = BF ? C.gzr + slot : nullptr;
    const float* const dgzb = BF ? C.dgzr + slot : nullptr;
    const bool live = C.lane < C.nv;
    float mq[4], dmq[4];
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
            const float vv = HV ? C.vring[ci] : 0.f, sc = C.ring[ci];
            const RevOut o = rev_cell<PG, BF>(C, V, i, sc, DOT ? 0.f : vv, zb[(15 - u) * 32],
                                              PG ? 0.f : dzb[(15 - u) * 32], BF ? gzb[(15 - u) * 32] : 0.f,
                                              BF ? dgzb[(15 - u) * 32] : 0.f);
            rev_emit<DOT, PG, BF>(C, V, C.ring + ci, PG ? sc : vv, o.dmu, act, sc, o.dgf);
            const float msg = act ? o.msg : 0.f, dmsg = act ? o.dmsg : 0.f;
            mq[i] = msg;
            dmq[i] = dmsg;
            if (i == 3)
                handoff(C, 4 * k + q, make_float4(mq[0], mq[1], mq[2], mq[3]),
                        make_float4(dmq[0], dmq[1], dmq[2], dmq[3]), V.Q, C.l0, V.push);
            V.rsh = __shfl_down_sync(kAll, msg, 1);
            V.drsh = __shfl_down_sync(kAll, dmsg, 1);
            V.br = act ? o.b : 0.f;
            V.pbp = act ? o.pb : 0.f;
            V.dbr = act ? o.db : 0.f;
            V.dpbp = act ? o.dpb : 0.f;
            V.Qsent = __shfl_down_sync(kAll, V.Q, 1);
        }
    }
}

// ==========================================================================
// kernel: the row-block pipeline of sw_linear.cu's lin_fast_kernel, with the
// tangent carried beside each value.  HV: the V ring is loaded (HVP: the
// direction; DOT: the weights); DOT: sum weight * dmu per problem into
// dot_out instead of writing dmu to out.
// ==========================================================================
// SPLIT: a cooperative launch spreads each problem over p.parts CTAs, as in
// sw_linear.cu's lin_fast_kernel (the partition's tangent and the dot-mode
// sums are combined across the parts in part order).
// PG: value + marginals + dS/dgap + dS/dT (soft_sw_with_grads): the forward
// carries the tangent along gap (dS/dgap = T dZ/Z), the reverse writes the
// marginals and sums score x marginal, and dS/dT follows from Euler's identity
// for the degree-1 homogeneous S(s, gap, T): S = sum s mu + gap dS/dgap + T dS/dT.
template <bool HV, bool DOT, bool SPLIT, bool PG, bool BF>
__global__ void __launch_bounds__(kNW * 32, 1) lin_tan_kernel(SwArgs p) {
    extern __shared__ __align__(16) unsigned char smem_raw[];
    WarpSmem& W = reinterpret_cast<WarpSmem*>(smem_raw)[threadIdx.x >> 5];
    __shared__ int progF[kNW], progR[kNW];
    __shared__ __align__(16) double red[2 * 32];
    __shared__ int sh_Sint, sh_err, sh_bad;
    __shared__ float sh_Sfrac, sh_dSr;
    __shared__ __align__(16) float zv[2 * kHR];   // staging of a missing neighbour: zeros
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
    const float gapn = p.gap_dev ? __ldg(p.gap_dev) : p.gap;
    const float T = p.temp_dev ? __ldg(p.temp_dev) : p.temp;
    const float c = kLog2e / T;
    const float G = ex2f(gapn * c);
    Dir dir;  // dP = P (vs V + ss s), dG = G gam
    dir.vs = p.mode == MODE_HVP ? 1.f / T : 0.f;
    dir.ss = p.mode == MODE_PT ? -1.f / (T * T) : 0.f;
    dir.gam = (PG || p.mode == MODE_PGAP) ? 1.f / T : (p.mode == MODE_PT ? -gapn / (T * T) : 0.f);
    const size_t plane = (size_t)L1m * L2m;
    const float* __restrict__ S = p.scores + (size_t)b * plane;
    const float* __restrict__ Vp = HV ? (DOT ? p.dot_with : p.tangent) + (size_t)b * plane : nullptr;
    float* __restrict__ out = (!DOT && p.out) ? p.out + (size_t)b * plane : nullptr;
    const Layout LY = carve(p.ws, b, L1m, L2m, BF);
    const int nRB = (L1 + 31) / 32;
    const int nch = (L2 + kCW - 1) / kCW;
    const size_t zst = (size_t)zt_rows(L2m) * 32;
    const size_t est = (size_t)gt_rows(L2m) * 32;

    if (out && (L1 < L1m || L2 < L2m)) {  // zero the padded part of the output
        for (int i = gw; i < L1m; i += NWt) {
            float* row = out + (size_t)i * L2m;
            for (int j = (i < L1 ? L2 : 0) + lane; j < L2m; j += 32) row[j] = 0.f;
        }
    }
    if (L1 == 0 || L2 == 0) {  // no cells: the output is all zeros
        if (threadIdx.x == 0 && part == 0) {
            if (DOT && p.dot_out) p.dot_out[b] = 0.f;
            if (BF && p.dot_out) p.dot_out[b] = p.dot_out[p.B + b] = 0.f;
            if (PG) {  // S = log(1) = 0, and so its derivatives
                if (p.value) p.value[b] = 0.f;
                if (p.grad_gap) p.grad_gap[b] = 0.f;
                if (p.grad_T) p.grad_T[b] = 0.f;
            }
            if (p.redo) p.redo[b] = 0;
        }
        return;
    }
    if (threadIdx.x < kNW) {
        progF[threadIdx.x] = -1;
        progR[threadIdx.x] = -1;
    }
    for (int i = threadIdx.x; i < 2 * kHR; i += blockDim.x) zv[i] = 0.f;  // 256 entries, 192 threads
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

    // Boundary values and tangents of the neighbouring row-block, staged by the
    // one lane that reads them, on sw_linear.cu's schedule: the prologue copies
    // the neighbour's stages 1 and 2 (from step 28 and group 4 on), stage k its
    // stage k+3 once finished, each unless the neighbour pushed it (tag).
    auto copy_stage = [&](int ordinal, int x, int rb) {
        if (W.tag[x & (kHR / 16 - 1)] == ((ordinal << 16) | x)) return;
        const float* const hz = LY.hz + (size_t)rb * hzst;
        const float* const hdz = LY.hdz + (size_t)rb * hzst;
        const float* const hf = LY.hfr + (size_t)rb * hfst;
        const int s0 = x == 1 ? 28 : kCW * x, ns = x == 1 ? 1 : 4, g0 = 4 * x;
        for (int i = 0; i < ns; ++i) {
            cp_async16(W.sv + ((s0 + 4 * i) & (kHR - 1)), hz + s0 + 4 * i, 16);
            cp_async16(W.sdv + ((s0 + 4 * i) & (kHR - 1)), hdz + s0 + 4 * i, 16);
        }
        cp_async16(W.sf + (g0 & (kHR / 4 - 1)), hf + g0, 16);
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
    // past its last stage a row-block's neighbour reads up to 48 steps and 12
    // groups further: zeros, in the final frame (one lane writes them)
    auto write_tail = [&](float* ov, float* odv, float* of, int n, float fr) {
#pragma unroll 4
        for (int i = 0; i < 12; ++i) {
            *reinterpret_cast<float4*>(ov + kCW * n + 4 * i) = make_float4(0.f, 0.f, 0.f, 0.f);
            *reinterpret_cast<float4*>(odv + kCW * n + 4 * i) = make_float4(0.f, 0.f, 0.f, 0.f);
        }
#pragma unroll
        for (int i = 0; i < 3; ++i) *reinterpret_cast<float4*>(of + 4 * n + 4 * i) = make_float4(fr, fr, fr, fr);
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
        C.av = (hasB && lane == 0) ? W.sv : zv;
        C.af = (hasB && lane == 0) ? W.sf : zf;
        C.ov = LY.hz + (size_t)r * hzst;
        C.odv = LY.hdz + (size_t)r * hzst;
        C.of = LY.hfr + (size_t)r * hfst;
        C.pv = (unsigned)__cvta_generic_to_shared(Wn.sv);
        C.zrow = LY.zpl + (size_t)r * zst + lane;
        C.dzrow = LY.dzpl + (size_t)r * zst + lane;
        C.gzrow = BF ? LY.gzpl + (size_t)r * zst + lane : nullptr;
        C.dgzrow = BF ? LY.dgzpl + (size_t)r * zst + lane : nullptr;
        C.erow = LY.efr + (size_t)r * est + lane;
        C.c = c;
        C.G = G;
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
        if (lane == 31) st_release(&progF[warp], r << 16);  // started: the row above may push to this warp
        if (0 < nch) {
            tile_load<4>(tS, 0, L2);
            if (HV && !DOT) tile_load<4>(tV, 0, L2);
        }
        if (hasB) stage_first(prodF, r - 1, r - 1, lane == 0);
        cp_async_commit();
        V.zl = V.zd = V.zsh = V.dzl = V.dzd = V.dzsh = 0.f;
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
            cp_async_wait2();  // everything but this stage's two groups
            __syncwarp();
            V.push = false;
            if (lane == 31 && hasD && !xout) {  // sw_linear.cu's push rule
                const int cw = ld_acquire(&progF[wnext]);
                V.push = (cw >> 16) == r + 1 && (cw & kStageMask) + 8 >= k;
            }
            if (k == 0) {
                if (lane == 0) V.E = C.af[7];
                V.Esent = __shfl_up_sync(kAll, V.E, 1);
                fwd_lookahead(C, V, 0);
            }
            if (kCW * k < 31)
                fwd_stage_start<HV && !DOT, BF>(C, V, k);
            else if (nv == 32 && kCW * k + kCW - 1 <= L2 - 1)
                fwd_stage_full<false, HV && !DOT, BF>(C, V, k, 0);
            else
                fwd_stage_full<true, HV && !DOT, BF>(C, V, k, lane < nv ? L2 + lane - kCW * k : -1);
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
        if (lane == 31) write_tail(C.ov, C.odv, C.of, nst, V.E);
        cp_async_wait0();
        __syncwarp();
        if (lane == 31) {
            st_release(&progF[warp], (r << 16) | kStageMask);
            if (xout) st_release_gpu(gsync + part, (r << 16) | kStageMask);
        }
    }
    const int fwd_out = ((V.ebmin < ((127 - kJMax) << 23) || V.ebmax > ((127 + kJMax) << 23)) ? 1 : 0) |
                        (V.emax > 1000.f ? 8 : 0);
    if (lane < kHR / 16) W.tag[lane] = -1;  // forward pushes are no reverse pushes

    // ---- S (integer + fraction) and dZ_total / Z_total
    {
        float* redf = reinterpret_cast<float*>(red);
        const float abl = block_max(V.ab, redf);
        const double scl = p2d(V.ab - abl);
        const double totl = block_sum_d(V.acc * scl, red);
        const double dtotl = block_sum_d(V.dacc * scl, red);
        if (threadIdx.x == 0) {
            float abmax = abl;
            double tot = totl, dtot = dtotl;
            if (SPLIT && K > 1) {  // every part's partials, after every part's forward
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
            tot += p2d(-abmax);  // alpha[0,0] = 0
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
    for (int q = gw; q < nRB; q += NWt) {
        const int r = nRB - 1 - q;
        const int nv = min(32, L1 - 32 * r);
        const bool hasBelow = r + 1 < nRB, hasAbove = r > 0;
        const float* const zblk = LY.zpl + (size_t)r * zst;
        const float* const dzblk = LY.dzpl + (size_t)r * zst;
        const float* const gzblk = BF ? LY.gzpl + (size_t)r * zst : nullptr;
        const float* const dgzblk = BF ? LY.dgzpl + (size_t)r * zst : nullptr;
        const float* const eblk = LY.efr + (size_t)r * est;
        RevCtx C;
        C.ring = W.ringS + lane * kRW;
        C.vring = W.ringV + lane * kRW;
        C.zr = &W.zr[0][0];
        C.dzr = &W.dzr[0][0];
        C.gzr = &W.gzr[0][0];
        C.dgzr = &W.dgzr[0][0];
        C.er = W.er;
        C.bv = (hasBelow && lane == nv - 1) ? W.sv : zv;
        C.bf = (hasBelow && lane == nv - 1) ? W.sf : zf;
        C.ov = LY.hz + (size_t)r * hzst;
        C.odv = LY.hdz + (size_t)r * hzst;
        C.of = LY.hfr + (size_t)r * hfst;
        C.pv = (unsigned)__cvta_generic_to_shared(Wn.sv);
        C.c = c;
        C.G = G;
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

        // staging for stage kb (M = P/16 + 1 - kb): w and dw rows 16M .. 16M+15
        // and the frames of groups 4M-1 .. 4M+3
        auto batch = [&](int kb) {
            const int M = P / kCW + 1 - kb;
            const size_t o16 = (size_t)(16 * M) * 32;
#pragma unroll
            for (int it = 0; it < 4; ++it) {
                const int e = 4 * (lane + 32 * it);
                cp_async16(&W.zr[M & 1][0] + e, zblk + o16 + e, 16);
                cp_async16(&W.dzr[M & 1][0] + e, dzblk + o16 + e, 16);
                if (BF) {
                    cp_async16(&W.gzr[M & 1][0] + e, gzblk + o16 + e, 16);
                    cp_async16(&W.dgzr[M & 1][0] + e, dgzblk + o16 + e, 16);
                }
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
        if (lane == 0) st_release(&progR[warp], q << 16);  // started: the row-block below may push to this warp
        {
            const int M0 = P / kCW + 1;
            for (int ch = M0; ch >= M0 - 2; --ch) loads(ch);
        }
        batch(0);
        if (hasBelow) stage_first(prodR, q - 1, r + 1, lane == nv - 1);
        cp_async_commit();

        RV.br = RV.pbp = RV.rsh = RV.dbr = RV.dpbp = RV.drsh = 0.f;
        RV.Q = 0.f;
        RV.Qsent = 0.f;
        RV.f.d1 = 0.f;
        for (int k = 0; k < nstR; ++k) {
            const int M = P / kCW + 1 - k;
            __syncwarp();
            if (hasBelow) stage_need(prodR, q - 1, k, r + 1, lane == nv - 1);
            cp_async_commit();
            if (out && M + 1 < nch && M + 1 >= 0) tile_store(tM, M + 1, L2);  // no lane touches it any more
            loads(M - 3);                                                    // for stage k + 1
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
            if (kCW * k <= P + 32 - L2)
                rev_stage_part<HV, DOT, PG, BF>(C, RV, k);
            else if (nv == 32 && kCW * k + kCW - 1 <= P - 1)
                rev_stage_full<false, HV, DOT, PG, BF>(C, RV, k, 0);
            else
                rev_stage_full<true, HV, DOT, PG, BF>(C, RV, k, lane < nv ? 16 * M + 16 - lane : -1);
            if (DOT || PG || BF) RV.dot += (double)RV.sdot;
            if (BF) RV.dot2 += (double)RV.sgap;
            if (RV.push) Wn.tag[k & (kHR / 16 - 1)] = (q << 16) | k;
            __syncwarp();
            if (lane == 0) {
                st_release(&progR[warp], (q << 16) | min(k + 1, kStageMask - 1));
                if (xout) st_release_gpu(gsync + kMaxParts + part, (q << 16) | min(k + 1, kStageMask - 1));
            }
        }
        if (lane == 0) write_tail(C.ov, C.odv, C.of, nstR, RV.Q);
        __syncwarp();
        if (out && nch > 0) tile_store(tM, 0, L2);  // the last stage had M = 0
        cp_async_wait0();
        __syncwarp();
        if (lane == 0) {
            st_release(&progR[warp], (q << 16) | kStageMask);
            if (xout) st_release_gpu(gsync + kMaxParts + part, (q << 16) | kStageMask);
        }
    }

    // a frame step outside the window, a partition or a tangent that is not
    // finite, or a dependency wait that gave up: the caller recomputes this
    // problem with the plane engine (bits as in sw_linear.cu; 16: tangent)
    const bool outside = (fwd_out & 1) || RV.ebmin < ((127 - kJMax) << 23) || RV.ebmax > ((127 + kJMax) << 23);
    const int o_win = __syncthreads_or(outside ? 1 : 0);
    const int o_acc = __syncthreads_or(fwd_out & 8);
    const int o_tan = __syncthreads_or(RV.chk != 0.f ? 1 : 0);
    const int redo = (o_win ? 1 : 0) | (sh_err ? 2 : 0) | (sh_bad ? 4 : 0) | (o_acc ? 8 : 0) | (o_tan ? 16 : 0);
    if (DOT || PG || BF) {
        const double tot = block_sum_d(RV.dot, red);
        const double tot2 = BF ? block_sum_d(RV.dot2, red) : 0.0;
        if (threadIdx.x == 0) {
            // DOT: the weighted sum; PG: dS/dT = (S - sum s mu - gap dS/dgap) / T;
            // BF: d(dS/dgap)[g] and d(dS/dT)[g] = -(sum s H g + gap d(dS/dgap)[g]) / T
            auto finish = [&](double all, double all2) {
                if (DOT && p.dot_out) p.dot_out[b] = (float)all;
                if (PG && p.grad_T) {
                    const double S = ((double)sh_Sint + (double)sh_Sfrac) / (double)c;
                    const double dgap = (double)sh_dSr * (double)T;
                    p.grad_T[b] = (float)((S - all - (double)gapn * dgap) / (double)T);
                }
                if (BF && p.dot_out) {
                    p.dot_out[b] = (float)all2;
                    p.dot_out[p.B + b] = (float)(-(all + (double)gapn * all2) / (double)T);
                }
            };
            if (SPLIT && K > 1) {  // the last part to arrive sums the parts in order
                gpart[kSyncPartDoubles * part + 3] = tot;
                if (BF) gpart[kSyncPartDoubles * part + 4] = tot2;
                if (atom_add_release_gpu(gsync + 2 * kMaxParts + 1, 1) == K - 1) {
                    (void)ld_acquire_gpu(gsync + 2 * kMaxParts + 1);
                    double all = 0.0, all2 = 0.0;
                    for (int k = 0; k < K; ++k) {
                        all += gpart[kSyncPartDoubles * k + 3];
                        if (BF) all2 += gpart[kSyncPartDoubles * k + 4];
                    }
                    finish(all, all2);
                }
            } else {
                finish(tot, tot2);
            }
        }
    }
    if (threadIdx.x == 0 && p.redo) {
        if (SPLIT)
            atomicOr(p.redo + b, redo);  // zeroed by the launcher
        else
            p.redo[b] = redo;
    }
}

}  // namespace ltan

// ------------------------------------------------------------------ host side
size_t lin_tan_workspace_bytes(int B, int L1, int L2, bool bf) {
    if (L1 > 32 * ltan::kMaxRB || L2 % 4 != 0) return 0;
    return ltan::per_problem_bytes(L1, L2, bf) * (size_t)B;
}

int launch_lin_tan(const SwArgs& a, size_t ws_bytes, cudaStream_t st) {
    const bool pg = a.mode == MODE_MARG && (a.grad_gap || a.grad_T);
    if (a.mode != MODE_HVP && a.mode != MODE_PGAP && a.mode != MODE_PT && !pg) return -1;
    if (!a.redo || engine_forced_plane()) return -1;
    if (a.L2 % 4 != 0 || a.L1 > 32 * ltan::kMaxRB || a.L1 == 0 || a.L2 == 0) return -1;
    const bool dot = a.dot_with != nullptr;
    // backward_full in one sweep pair: the HVP along the weights (tangent),
    // with dot_out receiving [B] d(dS/dgap) and [B] d(dS/dT)
    const bool bf = a.mode == MODE_HVP && !dot && a.dot_out != nullptr;
    const bool hv = a.mode == MODE_HVP || dot;
    if (a.mode == MODE_HVP && (dot || !a.tangent)) return -1;
    if (dot && !a.dot_out) return -1;
    if (!dot && !a.out) return -1;
    if (pg && (dot || a.tangent)) return -1;
    auto al16 = [](const void* q) { return (((uintptr_t)q) & 15) == 0; };
    if (!a.scores || !al16(a.scores) || (a.out && !al16(a.out)) || !al16(a.ws) || !a.ws) return -1;
    if ((a.tangent && !al16(a.tangent)) || (dot && !al16(a.dot_with))) return -1;
    if ((((uintptr_t)a.ws) & 255) != 0) return -1;
    if (ws_bytes < ltan::per_problem_bytes(a.L1, a.L2, bf) * (size_t)a.B) return -1;
    const size_t smem = sizeof(ltan::WarpSmem) * ltan::kNW;
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return (int)e;
    static DeviceSetup setup;
    int nsm = 0;
    const int se = device_setup(setup, dev, [smem] {
        const void* ks[10] = {(const void*)ltan::lin_tan_kernel<true, false, false, false, false>,
                              (const void*)ltan::lin_tan_kernel<false, false, false, false, false>,
                              (const void*)ltan::lin_tan_kernel<true, true, false, false, false>,
                              (const void*)ltan::lin_tan_kernel<true, false, true, false, false>,
                              (const void*)ltan::lin_tan_kernel<false, false, true, false, false>,
                              (const void*)ltan::lin_tan_kernel<true, true, true, false, false>,
                              (const void*)ltan::lin_tan_kernel<false, false, false, true, false>,
                              (const void*)ltan::lin_tan_kernel<false, false, true, true, false>,
                              (const void*)ltan::lin_tan_kernel<true, false, false, false, true>,
                              (const void*)ltan::lin_tan_kernel<true, false, true, false, true>};
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
    // value + marginals + parameter gradients: only while one wave of CTAs
    // (one per SM) holds the batch; larger batches run the log-domain kernel
    if (pg && a.B > nsm) return -1;
    // few large problems: several CTAs per problem (sw_linear.cu's rule, with
    // this kernel's 6 warps per CTA)
    const int K = a.sync ? lin_parts_nw(a.B, a.L1, a.L2, nsm, ltan::kNW) : 1;
    if (K > 1) {
        SwArgs s = a;
        s.parts = K;
        e = cudaMemsetAsync(s.sync, 0, kSyncBytes * (size_t)a.B, st);
        if (e == cudaSuccess) e = cudaMemsetAsync(s.redo, 0, sizeof(int) * (size_t)a.B, st);
        if (e != cudaSuccess) return (int)e;
        void* args[1] = {&s};
        const void* k = pg    ? (const void*)ltan::lin_tan_kernel<false, false, true, true, false>
                        : bf  ? (const void*)ltan::lin_tan_kernel<true, false, true, false, true>
                        : dot ? (const void*)ltan::lin_tan_kernel<true, true, true, false, false>
                        : hv  ? (const void*)ltan::lin_tan_kernel<true, false, true, false, false>
                              : (const void*)ltan::lin_tan_kernel<false, false, true, false, false>;
        e = cudaLaunchCooperativeKernel(k, dim3(a.B * K), dim3(ltan::kNW * 32), args, smem, st);
        if (e == cudaSuccess) return 0;
        cudaGetLastError();  // does not fit: one CTA per problem instead
    }
    if (pg)
        ltan::lin_tan_kernel<false, false, false, true, false><<<a.B, ltan::kNW * 32, smem, st>>>(a);
    else if (bf)
        ltan::lin_tan_kernel<true, false, false, false, true><<<a.B, ltan::kNW * 32, smem, st>>>(a);
    else if (dot)
        ltan::lin_tan_kernel<true, true, false, false, false><<<a.B, ltan::kNW * 32, smem, st>>>(a);
    else if (hv)
        ltan::lin_tan_kernel<true, false, false, false, false><<<a.B, ltan::kNW * 32, smem, st>>>(a);
    else
        ltan::lin_tan_kernel<false, false, false, false, false><<<a.B, ltan::kNW * 32, smem, st>>>(a);
    return (int)cudaGetLastError();
}

}  // namespace d2pb
