// sw_linear.cu -- linear-domain fast path for linear-gap soft Smith-Waterman
// value + marginals.
//
// The forward carries Z_ij = 2^a_ij itself (a = alpha log2(e)/T) instead of its
// logarithm.  In that domain the reference's log-sum-exp recurrence
// (src/sw/kernels_cpu.cpp:70-150)
//   Z_ij = P_ij (Z_{i-1,j-1} + 1) + G (Z_{i-1,j} + Z_{i,j-1}),   P = 2^(s c), G = 2^(gap c)
// costs one exponential (P) and a handful of FP operations per cell, and the
// reverse pass (src/sw/kernels_cpu.cpp:156-279) becomes the outside recurrence
//   B_ij = 1 + P_{i+1,j+1} B_{i+1,j+1} + G (B_{i+1,j} + B_{i,j+1}),
//   marginal_ij = B_ij P_ij (Z_{i-1,j-1} + 1) / Z_total,
// with Z_total = 2^S = 1 + sum_ij Z_ij.  Cells outside the problem are 0.
//
// Range.  Every lane (row) keeps its own power-of-two frame, Z = z 2^E and
// B = b 2^Q, one frame per group of 4 steps.  The frame of the next group is
// decided one step early, from the lane's value of the step before (so the
// integer work never sits on the dependency chain), and every factor that
// converts a neighbour's value into the lane's frame is prepared with it.
// Values from the row-block above or below come with their own frames.  If a
// frame step leaves [2^-60, 2^60] (score magnitudes far beyond the usual ones,
// or a temperature far below 1), the problem is flagged and the caller
// recomputes it with the log-domain kernel (sw_wavefront.cu), and what that
// flags in turn with the plane engine (sw_plane.cu).
//
// Dependency chain.  A lane's new value depends on its neighbour's value of
// the previous step through a warp shuffle and ONE fused multiply-add: the
// neighbour's frame conversion is folded into the multiplier (G 2^(E'-E)).
//
// Structure (shared with sw_wavefront.cu): one CTA per problem; warps own
// row-blocks of 32 rows (lane = row) and sweep them along anti-diagonals;
// consecutive row-blocks are ordered by release/acquire progress words.  The
// forward stores each cell's diagonal term w = P (z_diag + 2^-E) in a
// diagonal-major plane (row = forward step, 32 lanes per row) with one
// coalesced 128-byte store per step, and each lane's frame once per group;
// the reverse stages the plane 16 rows at a time through shared memory, each
// lane reading its own column (marginal = b w 2^(Q + E - S)).  Values that
// cross to the next row-block inside a pass (the forward's last lane down, the
// reverse's lane-0 messages up) are written by the boundary lane once per
// group (one 16-byte store) to a per-row-block boundary row in global memory;
// the consumer's reading lane copies each finished producer stage into shared
// memory with cp.async, one to three stages before its look-aheads read it.
// Consumers wait for producers, never the reverse: with warps taking
// row-blocks round-robin, a producer that waited for its consumer could wait
// on a warp still busy with its own earlier row-block, whose progress waits on
// the same chain.
//
// Reverse indexing: reverse step tau of a row-block works on forward
// anti-diagonal tf = P + 31 - tau (P = 16 ceil((L2-1)/16)); lane l is at
// column tf - l.  Stage k (16 steps) covers tf in [16M, 16M + 15] with
// M = P/16 + 1 - k for every row-block height.
#include <stddef.h>
#include <stdint.h>

#include "sw_common.cuh"
#include "sw_internal.h"
#include "sw_lindomain.cuh"
#include "sw_ring.cuh"

namespace d2pb {
namespace lin {
using namespace ring;
using namespace ld;

constexpr int kMaxRB = 512;              // row-blocks per problem (L1 <= 16384)
constexpr int kNW = 6;                   // warps per CTA, two CTAs per SM
constexpr int kNWWide = 12;              // warps per CTA when the batch leaves SMs idle (one CTA per SM)

struct WarpSmem {
    float ringS[32 * kRW];    // scores [rows][64]; reverse: marginals written in place
    float zr[2][16 * 32];     // reverse: the forward's w of 16 anti-diagonals, two slots
    float er[16 * 32];        // reverse: forward frames, 16 group slots
    // staging of the neighbouring row-block's boundary values, by its step,
    // and its frames, by its group (forward: the row above's lane 31 z;
    // reverse: the row-block below's lane 0 messages)
    float sv[kHR];
    float sf[kHR / 4];
    // which neighbour stage each of the 8 stage slots of sv / sf holds when
    // the neighbour pushed it there itself: (ordinal << 16) | stage
    int tag[kHR / 16];
};
static_assert(sizeof(WarpSmem) % 16 == 0, "per-warp shared blocks must stay 16-byte aligned");
static_assert(offsetof(WarpSmem, sf) == offsetof(WarpSmem, sv) + 4 * kHR, "sf follows sv");

struct Layout {  // per-problem workspace
    float* zpl;      // [nRB][ZT][32]   w = P (Z_diag + 1) of forward step t, frame E, at row t
    float* efr;      // [nRB][GT][32]   frame of each lane for each group of 4 forward steps
    float* hz;       // [nRB][ZT]       boundary values of each row-block, by its step
    float* hfr;      // [nRB][GT]       and their frames, by its group
};


__host__ __device__ inline size_t per_problem_bytes(int L1m, int L2m) {
    const size_t nrb = (size_t)(L1m + 31) / 32;
    size_t b = align_up(nrb * zt_rows(L2m) * 32 * 4, 256);
    b += align_up(nrb * gt_rows(L2m) * 32 * 4, 256);
    b += align_up(nrb * hz_stride(L2m) * 4, 256);
    b += align_up(nrb * hf_stride(L2m) * 4, 256);
    return b;
}

__device__ inline Layout carve(float* ws, int b, int L1m, int L2m) {
    const size_t nrb = (size_t)(L1m + 31) / 32;
    char* base = (char*)ws + (size_t)b * per_problem_bytes(L1m, L2m);
    Layout L;
    L.zpl = (float*)base;
    base += align_up(nrb * zt_rows(L2m) * 32 * 4, 256);
    L.efr = (float*)base;
    base += align_up(nrb * gt_rows(L2m) * 32 * 4, 256);
    L.hz = (float*)base;
    base += align_up(nrb * hz_stride(L2m) * 4, 256);
    L.hfr = (float*)base;
    return L;
}


// One group of the boundary lane's (bnd) values and its frame: into the
// staging ring of the consumer row-block's warp while it keeps up (push, pp),
// else to the row-block's boundary row in global memory, from where the
// consumer copies it.
template <class Ctx>
__device__ __forceinline__ void handoff(const Ctx& C, int g, float4 v, float fr, bool bnd, bool pp) {
    stg_group_pred(C.ov + 4 * g, C.of + g, v, fr, bnd && !pp);
    const unsigned sv = C.pv + 16u * (unsigned)(g & (kHR / 4 - 1));  // sf follows sv: 4 kHR bytes on
    sts_group_pred_s(sv, C.pv + 4u * kHR + 4u * (unsigned)(g & (kHR / 4 - 1)), v, fr, pp);
}

// ==========================================================================
// forward sweep of one row-block
// ==========================================================================
struct FwdF {           // one group of 4 forward steps, for frame E
    float d0, d1;       // 2^(E_{l-1} - E) for the up input of the first / other steps (lane 0: 0)
    float Gd0, Gd1;     // G d0, G d1
    float fs;           // 2^-E: the +1 start term in this frame
    float za[4];        // lane 0: the row above's value for each step, in frame E (other lanes: 0)
};

struct FwdVars {
    bool push;          // lane 31, this stage: its values go to the consumer's staging ring
    float zl, zd, zsh;  // own z of the previous step; diagonal input of this step; lane l-1's last z
    float E;            // own frame
    float Esent;        // edge stages: lane l-1's frame of the value in zsh
    FwdF f;
    float nE;           // the next group, decided one step early
    float nfJ;          // 2^(E - nE)
    FwdF nf;
    float gsum;         // this group's sum of z (frame E)
    double acc;         // partition of this lane's cells so far: sum Z 2^-ab
    float ab;           // base (log2) of acc: raised with the frames, so that the
                        // partition may exceed the double range (S > 1023 log2 units)
    int ebmin, ebmax;   // range of the frame steps (exponent fields)
    float emax;         // largest E - ab of a group (must stay inside double range)
};

struct FwdCtx {
    const float* ring;  // this lane's ring row
    const float* av;    // lane 0: the row above's boundary values staged by its step (ring of kHR);
    const float* af;    //   and its frames, by its group.  Other lanes (and r = 0): zeros
    float* ov;          // this row-block's boundary row (global), by step, and its frames by group
    float* of;
    unsigned pv;        // shared address of the staging ring of the warp computing the row-block below
    float* zrow;        // zpl row 0 (forward step 0) of this row-block, this lane
    float* erow;        // efr group 0 of this row-block, this lane
    float c, G;
    float notl0;        // lane != 0 as 1 / 0
    int lane, nv, L2;
    bool l0, l31;       // lane 0 follows the row above's frames; lane 31 hands its values down
};

// Factors of group g for a lane (not lane 0) that starts in frame E; eup0 /
// eup1: lane l-1's frames of the values it receives in the group's first /
// other steps.
__device__ __forceinline__ FwdF fwd_factors(const FwdCtx& C, float E, float eup0, float eup1) {
    FwdF f;
    f.d0 = p2(eup0 - E) * C.notl0;
    f.d1 = p2(eup1 - E) * C.notl0;
    f.Gd0 = C.G * f.d0;
    f.Gd1 = C.G * f.d1;
    f.fs = p2(-E);
    f.za[0] = f.za[1] = f.za[2] = f.za[3] = 0.f;
    return f;
}

// At the last step of a group (before its cell): the next group's frame and
// every factor of group g (the next one).  A lane re-anchors on its previous
// value; lane 0 instead takes the frame of the row above's last lane for the
// steps it receives (its group g + 8: the steps 4g+32 .. 4g+34 of that lane
// are lane 0's inputs 2..4; input 1, step 4g + 31, is converted from group
// g + 7, lane 0's previous frame).  Lane l-1's factors follow by exact
// products: d0' = d1 2^(E - E'), d1' = d0' 2^(E'_{l-1} - E_{l-1}).
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
    const float a0 = C.av[(4 * g + 31) & (kHR - 1)];
    const float4 a = *reinterpret_cast<const float4*>(C.av + ((4 * g + 32) & (kHR - 1)));
    V.nf.za[0] = a0 * w;
    V.nf.za[1] = a.x;
    V.nf.za[2] = a.y;
    V.nf.za[3] = a.z;
}

// group boundary: the finished group's partition in absolute terms, then the new frame
__device__ __forceinline__ void fwd_apply(FwdVars& V) {
    const float dE = V.E - V.ab;
    V.acc = fma((double)V.gsum, p2d(dE), V.acc);
    V.emax = fmaxf(V.emax, dE);
    V.gsum = 0.f;
    V.zl *= V.nfJ;
    V.zd *= V.nfJ;
    V.E = V.nE;
    V.f = V.nf;
}


// one cell, step i of its group; returns z, the up input in this frame (the
// next step's diagonal input) and w = P (z_diag + 2^-E), the cell's diagonal
// term, which is all the reverse needs of the forward: marginal = B P (Z_diag
// + 1) / Z_total = b w 2^(Q + E - S)
__device__ __forceinline__ float fwd_cell(const FwdCtx& C, const FwdVars& V, int i, float sc, float& zuin,
                                          float& w) {
    const float P = ex2f(sc * C.c);
    w = P * (V.zd + V.f.fs);
    const float rest = fmaf(C.G, V.zl + V.f.za[i], w);
    zuin = fmaf(V.zsh, i == 0 ? V.f.d0 : V.f.d1, V.f.za[i]);
    return fmaf(i == 0 ? V.f.Gd0 : V.f.Gd1, V.zsh, rest);
}

// 16 forward steps after every lane has started.  MASK: some lanes are past
// the last column (or beyond nv); thr = first step (u) at which this lane is
// past its last column.
template <bool MASK>
__device__ __forceinline__ void fwd_stage_full(const FwdCtx& C, FwdVars& V, int k, int thr) {
    const int c0 = (kCW * k - C.lane) & (kRW - 1);   // this lane's ring column at u = 0
    const float* const pA = C.ring + c0;
    const float* const pB = pA - kRW;                 // after the wrap past column 63
    float scv[kCW];  // the stage's scores, read before anything else happens
#pragma unroll
    for (int u = 0; u < kCW; ++u) scv[u] = ((u < kRW - c0) ? pA : pB)[u];
    float* const pz = C.zrow + (size_t)(kCW * k) * 32;
    float* const pe = C.erow + (size_t)(kCW * k / 4) * 32;
    float zq[4];
#pragma unroll
    for (int u = 0; u < kCW; ++u) {
        const int i = u & 3;
        if (i == 0) fwd_apply(V);
        if (i == 3) {
            if (u == kCW - 1) cp_async_wait1();  // the last look-ahead's boundary values (copied at stage start)
            fwd_lookahead(C, V, 4 * k + (u >> 2) + 1);
        }
        float zuin, w;
        float z = fwd_cell(C, V, i, scv[u], zuin, w);
        if (MASK) z = (u < thr) ? z : 0.f;
        V.gsum += z;
        pz[(size_t)u * 32] = w;
        zq[i] = z;
        if (i == 3) {
            pe[(u >> 2) * 32] = V.E;
            handoff(C, 4 * k + (u >> 2), make_float4(zq[0], zq[1], zq[2], zq[3]), V.E, C.l31, V.push);
        }
        V.zd = zuin;
        V.zl = z;
        V.zsh = __shfl_up_sync(kAll, z, 1);
    }
}

// the first two stages: lanes start (column 0) and take the frame of the
// value they receive (lane 0 starts in the frame of the row above)
__device__ __forceinline__ void fwd_stage_start(const FwdCtx& C, FwdVars& V, int k) {
    const bool live = C.lane < C.nv;
    float zq[4];
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
            float zuin, w;
            float z = fwd_cell(C, V, i, C.ring[j0 & (kRW - 1)], zuin, w);
            z = act ? z : 0.f;
            V.gsum += z;
            C.zrow[(size_t)t * 32] = w;
            zq[i] = z;
            if (i == 3) {
                const int g = t >> 2;
                C.erow[(size_t)g * 32] = V.E;
                handoff(C, 4 * k + q, make_float4(zq[0], zq[1], zq[2], zq[3]), V.E, C.l31, V.push);
            }
            V.zd = act ? zuin : 0.f;
            V.zl = z;
            V.zsh = __shfl_up_sync(kAll, z, 1);
            V.Esent = __shfl_up_sync(kAll, V.E, 1);
        }
    }
}

// ==========================================================================
// reverse sweep of one row-block
// ==========================================================================
struct RevF {           // one group of 4 reverse steps, for frame Q
    float d0, d1;       // 2^(Q_{l+1} - Q) for the message of the first / other steps (bottom lane: 0)
    float Gd0, Gd1;
    float fb[4];        // 2^-Q, plus for the bottom lane the message from below (frame Q)
    float kE;           // 2^(Q + E - S): E the lane's forward frame of these cells
};

struct RevVars {
    bool push;          // lane 0, this stage: its messages go to the consumer's staging ring
    float br, pbp, rsh; // own b and P*b of column j+1; message from lane l+1
    float Q;            // own frame
    float Qsent;        // edge stages: lane l+1's frame of the message in rsh
    RevF f;
    float nQ;
    float nfJ;          // 2^(Q - nQ)
    RevF nf;
    int ebmin, ebmax;   // range of the frame steps (exponent fields)
};

struct RevCtx {
    float* ring;          // ringS row of this lane
    const float* zr;      // WarpSmem::zr
    const float* er;      // WarpSmem::er
    const float* bv;      // bottom lane: the row-block below's lane-0 messages staged by its step (ring
    const float* bf;      //   of kHR) and its frames, by its group.  Other lanes (and the last row-block): zeros
    float* ov;            // this row-block's boundary row (global) for the row-block above
    float* of;
    unsigned pv;          // shared address of the staging ring of the warp computing the row-block above
    float c, G, cS;       // cS = 2^-Sfrac
    float notBot;         // lane != nv-1 as 1 / 0
    float Sint;
    int lane, nv, L2, P;
    bool l0, bot;         // lane 0 hands its messages up; the bottom lane follows the row-block below's frames
};

// Marginal factor of reverse group h (anti-diagonals tf0 = P + 31 - 4h down
// to tf0 - 3, all in forward group gA = (tf0 - 3) / 4 of this lane) in frame Q.
__device__ __forceinline__ void rev_kfactors(const RevCtx& C, RevF& f, float Q, int h) {
    const int gA = C.P / 4 + 7 - h;
    f.kE = p2(Q + C.er[(gA & 15) * 32 + C.lane] - C.Sint) * C.cS;
}

// Factors of group h for a lane (not the bottom one) that starts in frame Q;
// qdn0 / qdn1: lane l+1's frames of the messages it receives in the group's
// first / other steps.
__device__ __forceinline__ RevF rev_factors(const RevCtx& C, float Q, float qdn0, float qdn1, int h) {
    RevF f;
    f.d0 = p2(qdn0 - Q) * C.notBot;
    f.d1 = p2(qdn1 - Q) * C.notBot;
    f.Gd0 = C.G * f.d0;
    f.Gd1 = C.G * f.d1;
    f.fb[0] = f.fb[1] = f.fb[2] = f.fb[3] = p2(-Q);
    rev_kfactors(C, f, Q, h);
    return f;
}

// At the last step of a group (before its cell): the next group's frame and
// every factor of group h (the next one).  The bottom lane takes the frame
// of lane 0 of the row-block below for the messages it receives: that lane's
// step tau + 31 feeds step tau here, so messages 2..4 of group h come in its
// group h + 8 and message 1 (its step 4h + 31) is converted from group h + 7.
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
    const float e0 = C.bv[(4 * h + 31) & (kHR - 1)];
    const float4 e = *reinterpret_cast<const float4*>(C.bv + ((4 * h + 32) & (kHR - 1)));
    V.nf.fb[0] = fmaf(e0, w, fsq);
    V.nf.fb[1] = fsq + e.x;
    V.nf.fb[2] = fsq + e.y;
    V.nf.fb[3] = fsq + e.z;
    rev_kfactors(C, V.nf, V.nQ, h);
}

__device__ __forceinline__ void rev_apply(RevVars& V) {
    V.br *= V.nfJ;
    V.pbp *= V.nfJ;
    V.Q = V.nQ;
    V.f = V.nf;
}

// one cell, step i of its group: b, P*b, the message to lane l-1 and the marginal
struct RevOut {
    float b, pb, msg, mu;
};
__device__ __forceinline__ RevOut rev_cell(const RevCtx& C, const RevVars& V, int i, float sc, float w) {
    RevOut o;
    const float P = ex2f(sc * C.c);
    const float rest = fmaf(C.G, V.br, V.f.fb[i]);
    o.b = fmaf(i == 0 ? V.f.d0 : V.f.d1, V.rsh, rest);
    o.msg = fmaf(i == 0 ? V.f.Gd0 : V.f.Gd1, V.rsh, fmaf(C.G, rest, V.pbp));
    o.pb = P * o.b;
    o.mu = o.b * (w * V.f.kE);
    return o;
}

// 16 reverse steps after every lane has started.  MASK: some lanes go past
// column 0 (or are beyond nv); thr = first step (u) at which this lane is past
// it.  Their marginals land in ring slots whose chunks were already written
// back (columns -31 .. -1 map to the slots of chunks 2 and 3, stored before
// the last two stages), and their b, P*b and messages are zeroed.
template <bool MASK>
__device__ __forceinline__ void rev_stage_full(const RevCtx& C, RevVars& V, int k, int thr) {
    const int m16 = C.P + 16 - kCW * k;                                   // tf = m16 + 15 - u
    const float* const zb = C.zr + ((m16 >> 4) & 1) * (16 * 32) + C.lane;
    const int cb = (C.P + 31 - kCW * k - C.lane) & (kRW - 1);            // ring column at u = 0
    float* const qA = C.ring + cb;
    float* const qB = qA + kRW;                                            // after the wrap below column 0
    float scv[kCW];
#pragma unroll
    for (int u = 0; u < kCW; ++u) scv[u] = (((u <= cb) ? qA : qB) - u)[0];
    float mq[4];
#pragma unroll
    for (int u = 0; u < kCW; ++u) {
        const int i = u & 3;
        if (i == 0) rev_apply(V);
        if (i == 3) {
            if (u == kCW - 1) cp_async_wait1();
            rev_lookahead(C, V, 4 * k + (u >> 2) + 1);
        }
        const RevOut o = rev_cell(C, V, i, scv[u], zb[(15 - u) * 32]);
        (((u <= cb) ? qA : qB) - u)[0] = o.mu;
        const bool act = !MASK || u < thr;
        const float msg = act ? o.msg : 0.f;
        mq[i] = msg;
        if (i == 3) {
            handoff(C, 4 * k + (u >> 2), make_float4(mq[0], mq[1], mq[2], mq[3]), V.Q, C.l0, V.push);
        }
        V.rsh = __shfl_down_sync(kAll, msg, 1);
        V.br = act ? o.b : 0.f;
        V.pbp = act ? o.pb : 0.f;
    }
}

// edge stages: per-lane activity; a lane that starts (column L2-1, where
// B = 1 + G B_{i+1,j} stays near 1) starts in frame 0 (the bottom lane stays
// on the frames of the row-block below)
__device__ __forceinline__ void rev_stage_part(const RevCtx& C, RevVars& V, int k) {
    const int m16 = C.P + 16 - kCW * k;
    const float* const zb = C.zr + ((m16 >> 4) & 1) * (16 * 32) + C.lane;
    const bool live = C.lane < C.nv;
    float mq[4];
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
            const RevOut o = rev_cell(C, V, i, C.ring[ci], zb[(15 - u) * 32]);
            if (act) C.ring[ci] = o.mu;
            const float msg = act ? o.msg : 0.f;
            mq[i] = msg;
            if (i == 3) {
                handoff(C, 4 * k + q, make_float4(mq[0], mq[1], mq[2], mq[3]), V.Q, C.l0, V.push);
            }
            V.rsh = __shfl_down_sync(kAll, msg, 1);
            V.br = act ? o.b : 0.f;
            V.pbp = act ? o.pb : 0.f;
            V.Qsent = __shfl_down_sync(kAll, V.Q, 1);
        }
    }
}

// ==========================================================================
// kernel
// ==========================================================================
// Progress words: warp w publishes (ordinal << 16 | stages done) for its
// current row-block (ordinal = r forward, nRB-1-r reverse), and
// (ordinal << 16 | kStageMask) when the row-block is complete.  The staging
// for stage k reads the neighbouring row-block up to its stage k + 3, so it
// waits for k + 4 stages there.
// SPLIT: the launch is cooperative and spreads each problem over p.parts CTAs;
// row-block r goes to warp r mod NW of part (r / NW) mod parts, so the
// handoff from a part's last warp to the next part's warp 0 crosses CTAs: it
// takes the global route, with the progress words, the forward -> reverse
// barrier and the partition partials in the problem's p.sync words.
template <int NW, int MINB, bool SPLIT>
__global__ void __launch_bounds__(NW * 32, MINB) lin_fast_kernel(SwArgs p) {
    extern __shared__ __align__(16) unsigned char smem_raw[];
    WarpSmem& W = reinterpret_cast<WarpSmem*>(smem_raw)[threadIdx.x >> 5];
    __shared__ int progF[NW], progR[NW];
    __shared__ __align__(16) float red[4 * 32];
    __shared__ int sh_Sint, sh_err, sh_bad;
    __shared__ float sh_Sfrac;
    __shared__ __align__(16) float zv[kHR];   // handoff ring of a missing neighbour: zeros
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
    const float gapn = p.gap_dev ? __ldg(p.gap_dev) : p.gap;
    const float T = p.temp_dev ? __ldg(p.temp_dev) : p.temp;
    const float c = kLog2e / T;
    const float G = ex2f(gapn * c);
    const size_t plane = (size_t)L1m * L2m;
    const float* __restrict__ S = p.scores + (size_t)b * plane;
    float* __restrict__ out = p.out ? p.out + (size_t)b * plane : nullptr;
    const Layout LY = carve(p.ws, b, L1m, L2m);
    const int nRB = (L1 + 31) / 32;
    const int nch = (L2 + kCW - 1) / kCW;
    const size_t zst = (size_t)zt_rows(L2m) * 32;   // zpl row-block stride (floats)
    const size_t est = (size_t)gt_rows(L2m) * 32;   // efr row-block stride (ints)

    if (out && (L1 < L1m || L2 < L2m)) {  // zero the padded part of the marginals
        for (int i = gw; i < L1m; i += NWt) {
            float* row = out + (size_t)i * L2m;
            for (int j = (i < L1 ? L2 : 0) + lane; j < L2m; j += 32) row[j] = 0.f;
        }
    }
    if (L1 == 0 || L2 == 0) {  // S = log(1) = 0 (alpha[0,0] only)
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
    for (int i = threadIdx.x; i < kHR; i += blockDim.x) zv[i] = 0.f;
    if (threadIdx.x < kHR / 4) zf[threadIdx.x] = 0.f;
    if (lane < kHR / 16) W.tag[lane] = -1;
    if (threadIdx.x == 0) {
        sh_err = 0;
        sh_bad = 0;
    }
    __syncthreads();
    // the warps that compute the neighbouring row-blocks (round-robin
    // assignment): wprev produces this warp's inputs (row-block r-1 forward,
    // r+1 reverse), wnext consumes its outputs
    const int wprev = (warp + NW - 1) % NW, wnext = (warp + 1) % NW;
    WarpSmem& Wn = reinterpret_cast<WarpSmem*>(smem_raw)[wnext];
    const size_t hzst = (size_t)hz_stride(L2m), hfst = (size_t)hf_stride(L2m);

    // Boundary values of the neighbouring row-block (boundary row hz, frames hf),
    // staged into this warp's ring by the one lane that reads them.  Look-ahead
    // q of stage k reads the neighbour's steps 16k+4q+35 .. 16k+4q+39 and groups
    // 4k+q+8, 4k+q+9: look-aheads 0..2 need its stages up to k+2, the last one
    // its stage k+3.  The prologue copies its stages 0..2 (from step 28 and
    // group 4 on).  Stage k then needs the neighbour's stage k+3: unless it is
    // staged already, the stage waits for it and copies it as a copy group of its
    // own, which the stage's last look-ahead waits for.  A neighbour stage that
    // the neighbour pushed into the ring itself (tag) is not copied.
    auto copy_stage = [&](int ordinal, int x, int rb) {  // the reading lane only
        if (W.tag[x & (kHR / 16 - 1)] == ((ordinal << 16) | x)) return;  // pushed
        const float* const hz = LY.hz + (size_t)rb * hzst;
        const float* const hf = LY.hfr + (size_t)rb * hfst;
        const int s0 = kCW * x, g0 = 4 * x;
#pragma unroll
        for (int i = 0; i < 4; ++i) cp_async16(W.sv + ((s0 + 4 * i) & (kHR - 1)), hz + s0 + 4 * i, 16);
        cp_async16(W.sf + (g0 & (kHR / 4 - 1)), hf + g0, 16);
    };
    auto wait_prog = [&](const int* prog, bool global, int need) {
        if (global)
            wait_flag_gpu(prog, need, &sh_err);
        else
            wait_flag(prog, need, &sh_err);
    };
    auto stage_first = [&](const int* prog, int ordinal, int rb, bool reader) {
        wait_prog(prog, xin, (ordinal << 16) + 3);
        if (reader) {
            const float* const hz = LY.hz + (size_t)rb * hzst;
            const float* const hf = LY.hfr + (size_t)rb * hfst;
            if (W.tag[1] != ((ordinal << 16) | 1)) {  // stage 1: steps 28..31, groups 4..7
                cp_async16(W.sv + 28, hz + 28, 16);
                cp_async16(W.sf + 4, hf + 4, 16);
            }
            if (W.tag[2] != ((ordinal << 16) | 2)) {  // stage 2: steps 32..47, groups 8..11
#pragma unroll
                for (int i = 0; i < 4; ++i) cp_async16(W.sv + 32 + 4 * i, hz + 32 + 4 * i, 16);
                cp_async16(W.sf + 8, hf + 8, 16);
            }
        }
    };
    auto stage_need = [&](const int* prog, int ordinal, int k, int rb, bool reader) {
        wait_prog(prog, xin, (ordinal << 16) + min(k + 4, kStageMask));
        if (reader) copy_stage(ordinal, k + 3, rb);
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
        float* const zblk = LY.zpl + (size_t)r * zst;
        FwdCtx C;
        C.ring = W.ringS + lane * kRW;
        C.av = (hasB && lane == 0) ? W.sv : zv;
        C.af = (hasB && lane == 0) ? W.sf : zf;
        C.ov = LY.hz + (size_t)r * hzst;
        C.of = LY.hfr + (size_t)r * hfst;
        C.pv = (unsigned)__cvta_generic_to_shared(Wn.sv);
        C.zrow = zblk + lane;
        C.erow = LY.efr + (size_t)r * est + lane;
        C.c = c;
        C.G = G;
        C.notl0 = lane == 0 ? 0.f : 1.f;
        C.lane = lane;
        C.nv = nv;
        C.L2 = L2;
        C.l0 = lane == 0;
        C.l31 = lane == 31;
        const Tile tS = make_tile(srow, L2m, W.ringS, nv, lane);

        const bool hasD = r + 1 < nRB;
        __syncwarp();
        if (lane == 31) st_release(&progF[warp], r << 16);  // started: the row above may push to this warp
        if (0 < nch) tile_load<4>(tS, 0, L2);
        if (hasB) stage_first(prodF, r - 1, r - 1, lane == 0);
        cp_async_commit();
        V.zl = V.zd = V.zsh = 0.f;
        V.f.d1 = 0.f;  // lane 0 keeps zero neighbour factors; the others set theirs when they start
        for (int k = 0; k < nst; ++k) {
            __syncwarp();
            if (hasB) stage_need(prodF, r - 1, k, r - 1, lane == 0);
            cp_async_commit();
            if (k + 1 < nch) tile_load<4>(tS, k + 1, L2);
            cp_async_commit();
            cp_async_wait2();  // everything but this stage's two groups
            __syncwarp();
            // Push this stage while the row-block below is on its warp and has done
            // at least k - 8 stages: the stage slot then holds a stage it has read
            // (stage c reads stages c+2, c+3), and the slots its prologue copies
            // into (stages 1, 2) are written only with the same stages.
            V.push = false;
            if (lane == 31 && hasD && !xout) {
                const int cw = ld_acquire(&progF[wnext]);
                V.push = (cw >> 16) == r + 1 && (cw & kStageMask) + 8 >= k;
            }
            if (k == 0) {  // lane 0 starts in the frame of the row above; group 0's factors
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
        V.acc = fma((double)V.gsum, p2d(V.E - V.ab), V.acc);  // the last group's partition
        V.emax = fmaxf(V.emax, V.E - V.ab);
        V.gsum = 0.f;
        // past the last stage the row below's look-aheads read up to 48 steps and
        // 12 groups further: zeros, in the final frame
        if (lane == 31) {
#pragma unroll 4
            for (int i = 0; i < 12; ++i)
                *reinterpret_cast<float4*>(C.ov + kCW * nst + 4 * i) = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
            for (int i = 0; i < 3; ++i)
                *reinterpret_cast<float4*>(C.of + 4 * nst + 4 * i) = make_float4(V.E, V.E, V.E, V.E);
        }
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
        // every lane's acc brought to the largest base; alpha[0,0] = 0 adds 2^-abmax
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
            const int e = ef - 1023 + (int)abmax;                             // tot 2^abmax = m 2^e, m in [1, 2)
            const bool fin = ef != 0x7ff && ef != 0;
            const double m = __hiloint2double((hi & 0x800fffff) | 0x3ff00000, __double2loint(tot));
            const float l2 = lg2_rr((float)m);
            sh_Sint = e;
            sh_Sfrac = l2;
            if (!fin) sh_bad = 1;
            if (p.value && part == 0) p.value[b] = ((float)sh_Sint + sh_Sfrac) / c;
        }
        __syncthreads();  // also: every forward read of the handoff rings is done
    }
    // the forward's range checks, folded into one word before the reverse
    const int fwd_out = ((V.ebmin < ((127 - kJMax) << 23) || V.ebmax > ((127 + kJMax) << 23)) ? 1 : 0) |
                        (V.emax > 1000.f ? 8 : 0);

    // ============================== reverse ==============================
    const int P = kCW * ((L2 - 1 + kCW - 1) / kCW);
    const int nstR = P / kCW + 2;  // lane 0 reaches column 0 at step P + 31
    RevVars RV;
    RV.ebmin = RV.ebmax = 0x3f800000;
    for (int q = gw; q < nRB; q += NWt) {
        const int r = nRB - 1 - q;
        const int nv = min(32, L1 - 32 * r);
        const float* srow = S + (size_t)(32 * r) * L2m;
        const bool hasBelow = r + 1 < nRB, hasAbove = r > 0;
        const float* const zblk = LY.zpl + (size_t)r * zst;
        const float* const eblk = LY.efr + (size_t)r * est;
        RevCtx C;
        C.ring = W.ringS + lane * kRW;
        C.zr = &W.zr[0][0];
        C.er = W.er;
        C.bv = (hasBelow && lane == nv - 1) ? W.sv : zv;
        C.bf = (hasBelow && lane == nv - 1) ? W.sf : zf;
        C.ov = LY.hz + (size_t)r * hzst;
        C.of = LY.hfr + (size_t)r * hfst;
        C.pv = (unsigned)__cvta_generic_to_shared(Wn.sv);
        C.c = c;
        C.G = G;
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

        // staging for stage kb (M = P/16 + 1 - kb): w rows 16M .. 16M+15 (2 KB,
        // contiguous) and the frames of groups 4M-1 .. 4M+3, read by the
        // stage's cells and look-aheads
        auto batch = [&](int kb) {
            const int M = P / kCW + 1 - kb;
            float* const zd = &W.zr[M & 1][0];
            const float* const zs = zblk + (size_t)(16 * M) * 32;
#pragma unroll
            for (int it = 0; it < 4; ++it) cp_async16(zd + 4 * (lane + 32 * it), zs + 4 * (lane + 32 * it), 16);
            const int gl = 4 * M - 1;
#pragma unroll
            for (int it = 0; it < 2; ++it) {
                const int cc = lane + 32 * it, g = gl + (cc >> 3), c4 = cc & 7;
                if (cc < 40 && g >= 0) cp_async16(W.er + (g & 15) * 32 + 4 * c4, eblk + (size_t)g * 32 + 4 * c4, 16);
            }
        };

        __syncwarp();
        if (lane == 0) st_release(&progR[warp], q << 16);  // started: the row-block below may push to this warp
        {   // stage 0 reads score chunks M0-2 .. M0 (M0 = P/16 + 1)
            const int M0 = P / kCW + 1;
            for (int ch = M0; ch >= M0 - 2; --ch)
                if (ch >= 0 && ch < nch) tile_load<4>(tS, ch, L2);
        }
        batch(0);
        if (hasBelow) stage_first(prodR, q - 1, r + 1, lane == nv - 1);
        cp_async_commit();

        RV.br = RV.pbp = RV.rsh = 0.f;
        RV.Q = 0.f;
        RV.Qsent = 0.f;
        RV.f.d1 = 0.f;  // the bottom lane keeps zero neighbour factors; the others set theirs when they start
        for (int k = 0; k < nstR; ++k) {
            const int M = P / kCW + 1 - k;
            __syncwarp();
            if (hasBelow) stage_need(prodR, q - 1, k, r + 1, lane == nv - 1);
            cp_async_commit();
            if (out && M + 1 < nch && M + 1 >= 0) tile_store(tM, M + 1, L2);  // no lane touches it any more
            if (M - 3 >= 0 && M - 3 < nch) tile_load<4>(tS, M - 3, L2);       // for stage k + 1
            if (k + 1 < nstR) batch(k + 1);
            cp_async_commit();
            cp_async_wait2();  // everything but this stage's two groups
            __syncwarp();
            RV.push = false;
            if (lane == 0 && hasAbove && !xout) {
                const int cw = ld_acquire(&progR[wnext]);
                RV.push = (cw >> 16) == q + 1 && (cw & kStageMask) + 8 >= k;
            }
            if (k == 0) rev_lookahead(C, RV, 0);
            // full: every lane started before the stage (lane 0 starts at step
            // P - L2 + 32, which must run the start logic); masked when a lane
            // passes column 0 in it (tf - lane < 0 from u = 16M + 16 - lane on)
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
        // past the last stage the row above's look-aheads read up to 48 steps and
        // 12 groups further: zeros, in the final frame
        if (lane == 0) {
#pragma unroll 4
            for (int i = 0; i < 12; ++i)
                *reinterpret_cast<float4*>(C.ov + kCW * nstR + 4 * i) = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
            for (int i = 0; i < 3; ++i)
                *reinterpret_cast<float4*>(C.of + 4 * nstR + 4 * i) = make_float4(RV.Q, RV.Q, RV.Q, RV.Q);
        }
        __syncwarp();
        if (out && nch > 0) tile_store(tM, 0, L2);  // the last stage had M = 0
        cp_async_wait0();
        __syncwarp();
        if (lane == 0) {
            st_release(&progR[warp], (q << 16) | kStageMask);
            if (xout) st_release_gpu(gsync + kMaxParts + part, (q << 16) | kStageMask);
        }
    }

    // a frame step outside the window, a partition that overflowed, or a
    // dependency wait that gave up: the caller recomputes this problem with
    // the log-domain kernel
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

// Problems of a ragged batch by decreasing estimated cost (cells plus the
// row-block pipeline's fill), so that the block scheduler starts the longest
// CTAs first and the last wave is made of short ones.  One CTA: a 1024-bucket
// counting sort.  The order within a bucket does not matter: every problem's
// result is independent of the CTA that computes it.
constexpr int kOrderThreads = 1024;
__global__ void __launch_bounds__(kOrderThreads) lin_order_kernel(const int* __restrict__ lengths, int B, int L1m,
                                                                  int L2m, int* __restrict__ order) {
    __shared__ int cnt[kOrderThreads];
    __shared__ int wsum[kOrderThreads / 32];
    const int t = threadIdx.x;
    cnt[t] = 0;
    __syncthreads();
    const float kmax = (float)L1m * (float)L2m + 48.f * (float)(L1m + L2m);
    auto bucket = [&](int i) {
        const int l1 = min(max(lengths[2 * i], 0), L1m), l2 = min(max(lengths[2 * i + 1], 0), L2m);
        const float key = (float)l1 * (float)l2 + 48.f * (float)(l1 + l2);
        // largest first: bucket 0 holds the most expensive problems
        return kOrderThreads - 1 - min(kOrderThreads - 1, (int)(key * (float)(kOrderThreads - 1) / kmax));
    };
    for (int i = t; i < B; i += kOrderThreads) atomicAdd(&cnt[bucket(i)], 1);
    __syncthreads();
    // exclusive scan of cnt
    const int v = cnt[t];
    int x = v;
    const int lane = t & 31, w = t >> 5;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const int y = __shfl_up_sync(0xffffffffu, x, o);
        if (lane >= o) x += y;
    }
    if (lane == 31) wsum[w] = x;
    __syncthreads();
    if (w == 0) {
        int s = wsum[lane];
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int y = __shfl_up_sync(0xffffffffu, s, o);
            if (lane >= o) s += y;
        }
        wsum[lane] = s;
    }
    __syncthreads();
    cnt[t] = x - v + (w > 0 ? wsum[w - 1] : 0);
    __syncthreads();
    for (int i = t; i < B; i += kOrderThreads) order[atomicAdd(&cnt[bucket(i)], 1)] = i;
}

}  // namespace lin

// ------------------------------------------------------------------ host side
int launch_lin_order(const int* lengths, int B, int L1, int L2, int* order, cudaStream_t st) {
    if (!lengths || !order || B <= 0) return -1;
    int dev = 0, sms = 148;
    if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    if (B <= 2 * sms) return -1;  // one wave: every CTA starts at once
    lin::lin_order_kernel<<<1, lin::kOrderThreads, 0, st>>>(lengths, B, L1, L2, order);
    return (int)cudaGetLastError();
}
size_t lin_fast_workspace_bytes(int B, int L1, int L2) {
    if (L1 > 32 * lin::kMaxRB || L2 % 4 != 0) return 0;
    return lin::per_problem_bytes(L1, L2) * (size_t)B;
}

// Stage times of one pass of the row-block pipeline with nw warps taking
// row-blocks round-robin: a row-block starts once its warp is free and 4
// stages after the one above started, and ends no earlier than 1 stage after
// the one above.
static double pipeline_stages(int n, int st, int nw) {
    double start[lin::kMaxRB], fin[lin::kMaxRB];
    for (int r = 0; r < n; ++r) {
        start[r] = r == 0 ? 0.0 : start[r - 1] + 4.0;
        if (r >= nw) start[r] = fmax(start[r], fin[r - nw]);
        fin[r] = start[r] + st;
        if (r > 0) fin[r] = fmax(fin[r], fin[r - 1] + 1.0);
    }
    return n > 0 ? fin[n - 1] : 0.0;
}
static bool wide_pays(int L1, int L2) {
    const int n = (L1 + 31) / 32, st = (L2 + 31 + lin::kCW - 1) / lin::kCW;
    if (n > lin::kMaxRB) return false;
    return 1.25 * pipeline_stages(n, st, lin::kNWWide) < pipeline_stages(n, st, lin::kNW);
}
bool lin_wide_pays(int L1, int L2) { return wide_pays(L1, L2); }

// CTAs per problem for a batch of B problems of nw warps each, one CTA per SM:
// the smallest part count within 3 % of the best the pipeline model offers
// (parts * B <= SMs; a crossing between parts costs about as much as a
// handoff through global memory, taken into account as 10 % per stage).
int lin_parts_nw(int B, int L1, int L2, int sms, int nw) {
    const int n = (L1 + 31) / 32, st = (L2 + 31 + lin::kCW - 1) / lin::kCW;
    if (B <= 0 || n > lin::kMaxRB || 2 * B > sms) return 1;
    double t[kMaxParts + 1];
    double best = 1e300;
    for (int K = 1; K <= kMaxParts && K * B <= sms; ++K) {
        t[K] = pipeline_stages(n, st, nw * K) * (K > 1 ? 1.1 : 1.0);
        best = fmin(best, t[K]);
    }
    for (int K = 1; K <= kMaxParts && K * B <= sms; ++K)
        if (t[K] <= 1.03 * best) return K;
    return 1;
}

int launch_lin_fast(const SwArgs& a, size_t ws_bytes, cudaStream_t st) {
    if (a.mode != MODE_MARG || !a.redo || a.grad_gap || a.grad_T) return -1;
    if (engine_forced_plane()) return -1;
    if (a.L2 % 4 != 0 || a.L1 > 32 * lin::kMaxRB || a.L1 == 0 || a.L2 == 0) return -1;
    if ((((uintptr_t)a.scores) & 15) != 0 || (a.out && (((uintptr_t)a.out) & 15) != 0)) return -1;
    if ((((uintptr_t)a.ws) & 255) != 0) return -1;
    const size_t need = lin::per_problem_bytes(a.L1, a.L2) * (size_t)a.B;
    if (ws_bytes < need || !a.ws) return -1;
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return (int)e;
    static DeviceSetup setup;
    int nsm = 0;
    const int se = device_setup(setup, dev, [] {
        const size_t s6 = sizeof(lin::WarpSmem) * lin::kNW, s12 = sizeof(lin::WarpSmem) * lin::kNWWide;
        const void* k6 = (const void*)lin::lin_fast_kernel<lin::kNW, 2, false>;
        const void* k12[2] = {(const void*)lin::lin_fast_kernel<lin::kNWWide, 1, false>,
                              (const void*)lin::lin_fast_kernel<lin::kNWWide, 1, true>};
        cudaError_t r = cudaFuncSetAttribute(k6, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)s6);
        if (r == cudaSuccess)
            r = cudaFuncSetAttribute(k6, cudaFuncAttributePreferredSharedMemoryCarveout,
                                     (int)cudaSharedmemCarveoutMaxShared);
        for (int i = 0; i < 2 && r == cudaSuccess; ++i) {
            r = cudaFuncSetAttribute(k12[i], cudaFuncAttributeMaxDynamicSharedMemorySize, (int)s12);
            if (r == cudaSuccess)
                r = cudaFuncSetAttribute(k12[i], cudaFuncAttributePreferredSharedMemoryCarveout,
                                         (int)cudaSharedmemCarveoutMaxShared);
        }
        return (int)r;
    }, &nsm);
    if (se != 0) return se;
    // A batch of at most one problem per SM may run 12 warps per problem,
    // when the pipeline model says that pays (12 warps on one SM run each
    // stage about 25 % slower: measured 1.19 - 1.32 on 256 x 1024 .. 1024 x 1024).
    // A batch that leaves most SMs idle spreads each problem over several
    // CTAs (cooperative launch: every part resident at once).
    const int K = a.sync ? lin_parts_nw(a.B, a.L1, a.L2, nsm, lin::kNWWide) : 1;
    if (K > 1) {
        SwArgs s = a;
        s.parts = K;
        e = cudaMemsetAsync(s.sync, 0, kSyncBytes * (size_t)a.B, st);
        if (e == cudaSuccess) e = cudaMemsetAsync(s.redo, 0, sizeof(int) * (size_t)a.B, st);
        if (e != cudaSuccess) return (int)e;
        void* args[1] = {&s};
        e = cudaLaunchCooperativeKernel((const void*)lin::lin_fast_kernel<lin::kNWWide, 1, true>, dim3(a.B * K),
                                        dim3(lin::kNWWide * 32), args, sizeof(lin::WarpSmem) * lin::kNWWide, st);
        if (e == cudaSuccess) return 0;
        cudaGetLastError();  // a cooperative launch that does not fit: one CTA per problem instead
    }
    if (a.B <= nsm && wide_pays(a.L1, a.L2)) {
        lin::lin_fast_kernel<lin::kNWWide, 1, false>
            <<<a.B, lin::kNWWide * 32, sizeof(lin::WarpSmem) * lin::kNWWide, st>>>(a);
    } else {
        lin::lin_fast_kernel<lin::kNW, 2, false><<<a.B, lin::kNW * 32, sizeof(lin::WarpSmem) * lin::kNW, st>>>(a);
    }
    return (int)cudaGetLastError();
}

}  // namespace d2pb
