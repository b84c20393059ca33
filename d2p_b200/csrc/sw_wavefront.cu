// sw_wavefront.cu -- fast path for soft Smith-Waterman value + marginals (linear gap).
//
// One CTA per problem; warps own row-blocks of 32 rows (lane = row) and sweep
// them left-to-right (forward) and right-to-left (reverse), one cell per lane
// per step, so the 32 lanes of a warp always sit on one anti-diagonal.
// Cross-lane dependencies move by warp shuffles.  Cross-warp dependencies (the
// last row of a row-block feeding the first row of the next) move through
// small L2-resident boundary rows in the workspace, prefetched with cp.async;
// consumers wait on per-warp progress counters in shared memory (release /
// acquire at CTA scope, bounded spins), so no CTA-wide barrier sits on the
// sweep and every warp runs as soon as its inputs exist.
//
// Numerics.  Everything is base-2 scaled (a = alpha*log2(e)/T, one MUFU
// ex2/lg2 per exponential/logarithm).  Every warp keeps an integer "frame" O
// per anti-diagonal: a cell stores a - O, so stored magnitudes stay small even
// when alpha grows to 10^3 along the matrix (the reference carries raw alpha
// in fp32 and loses absolute precision there).  The frame is re-anchored on
// the middle lane every 4 steps and advanced by a predicted integer drift in
// between.  Frame differences are exact integers; the value S is kept as
// (integer part, fraction).  The forward log-sum-exp is max-shifted, so any
// spread of values along an anti-diagonal is exact; every reverse exponent is
// <= 0 by construction (alpha_ij >= alpha_pred + transition).
//
// Memory.  The forward writes the framed alpha plane (4 B/cell) and the frames;
// the reverse reads them back, so each cell costs: scores 4 B read twice, alpha
// 4 B written + read, marginals 4 B written = 20 B/cell.  Every global access
// is a coalesced 16-byte cp.async (loads) or 16-byte store (write-back of
// 16-column tiles staged in shared memory).  Per-warp shared rings are
// [rows][64] floats: lane l touches column j = c - l of row l, so the bank
// (64 l + j) mod 32 = (c - l) mod 32 differs across the warp -- the
// anti-diagonal access pattern is bank-conflict free.  A cell's score slot is
// reused for its output (alpha in the forward, the marginal in the reverse).
//
// Reverse pass: beta is propagated in push form through registers and shuffles
// (no atomics, deterministic).  With N_ij the sum of the cell's four incoming
// weights (1 up to rounding; dividing by it keeps the rounding of the stored
// alpha from scaling the flow, as the reference's softmax does):
//   beta_ij = 2^min(a_ij - S, 0) + sum over successors of beta_succ * w(succ <- ij) / N_succ
//   marginal_ij = beta_ij (w_align + w_sky) / N_ij,  dS/dgap = sum beta (w_up + w_left) / N,
//   dS/dT = path entropy (sum of non-negative terms).
// Semantics follow the reference (src/sw/kernels_cpu.cpp:70-279).
#include <stdint.h>

#include "sw_common.cuh"
#include "sw_internal.h"
#include "sw_ring.cuh"

namespace d2pb {
namespace wf {

using namespace ring;

constexpr int kMaxRB = 512;              // row-blocks per problem (L1 <= 16384)
constexpr int kNW = 6;                   // warps per CTA
constexpr int kRebase = 32;              // partition: rebase when the frame runs this far above R

struct WarpSmem {
    float ringS[32 * kRW];        // scores; forward: alpha written in place; reverse: marginals in place
    float ringA[33 * kRW];        // reverse: framed alpha, row 0 = row above the row-block
    float2 bnd[kRW];              // forward: last row of the previous row-block (a - O, O)
    float bb[kRW];                // reverse: beta pushes from the row below
    float fr[kRW];                // reverse: frames of this row-block
};

struct Layout {  // per-problem workspace
    float* aplane;   // [nRB][33][L2m]: row 0 = row above (in this block's frames), rows 1..32 = alpha - O
    float* frames;   // [nRB][L2m + 64] per-step frame O (exact integers stored as float)
    float2* bnd;     // [nRB][L2m] last row of each row-block: (a - O, O)
    float* bb;       // [nRB][L2m] reverse pushes into the row above
};

__host__ __device__ inline size_t frame_row(int L2m) { return (size_t)L2m + 64; }

__host__ __device__ inline size_t per_problem_bytes(int L1m, int L2m) {
    const size_t nrb = (size_t)(L1m + 31) / 32;
    size_t b = align_up(nrb * 33 * (size_t)L2m * 4, 256);
    b += align_up(nrb * frame_row(L2m) * 4, 256);
    b += align_up(nrb * (size_t)L2m * 8, 256);
    b += align_up(nrb * (size_t)L2m * 4, 256);
    return b;
}

__device__ inline Layout carve(float* ws, int b, int L1m, int L2m) {
    const size_t nrb = (size_t)(L1m + 31) / 32;
    char* base = (char*)ws + (size_t)b * per_problem_bytes(L1m, L2m);
    Layout L;
    L.aplane = (float*)base;
    base += align_up(nrb * 33 * (size_t)L2m * 4, 256);
    L.frames = (float*)base;
    base += align_up(nrb * frame_row(L2m) * 4, 256);
    L.bnd = (float2*)base;
    base += align_up(nrb * (size_t)L2m * 8, 256);
    L.bb = (float*)base;
    return L;
}

// ==========================================================================
// forward sweep of one row-block
// ==========================================================================
struct FwdVars {
    float left, uprev, uprecv;  // own previous output, previous "up", shuffled neighbour output
    float O, pv;                // frame of the current step, middle-lane probe
    float J, inc;               // group: frame jump at its first step, per-step increment
    float gA, gB, dA, dB, dC;   // group offsets: g - J, g - inc, J + inc_prev, inc + J, 2 inc
    float acc, R;               // partition of this lane's cells: sum 2^a = acc * 2^R
};

struct FwdCtx {
    float* ring;             // this lane's ring row (ringS + lane*kRW)
    const float2* bndring;   // last row of the row-block above, (a - O, O); (kNeg, 0) for row-block 0
    float* arow0;            // aplane tile row 0 (row above, kept for the reverse)
    float2* bout;            // boundary row for the next row-block
    float* frow;             // frames of this row-block
    float c, g;
    int lane, nv, L2;
    bool lane0, st31;        // lane == 0; lane == 31 and a row-block follows
};

// Start of a group of 4 steps: move the frame by the rounded middle-lane value
// of the previous step (J), and predict the per-step drift of the next 3 steps
// from the average over the last group (inc), so that stored values a - O stay
// small between probes.  Frames stay exact integers.  pf: frames of the group.
template <bool FULL>
__device__ __forceinline__ void frame_group_start(const FwdCtx& C, FwdVars& V, float* pf) {
    const float J = FULL ? rintf(V.pv) : (V.pv > kNegThresh ? rintf(V.pv) : 0.f);
    const float incp = V.inc;
    V.O += J;
    V.J = J;
    V.inc = fminf(fmaxf(rintf((J + 3.f * incp) * 0.25f), -16.f), 16.f);
    V.gA = C.g - J;
    V.gB = C.g - V.inc;
    V.dA = J + incp;
    V.dB = V.inc + J;
    V.dC = 2.f * V.inc;
    // partition base: keep O - R <= kRebase over the whole group (selects, no branch)
    const float Dg = V.O - V.R;
    const bool reb = Dg + 3.f * fmaxf(V.inc, 0.f) > (float)kRebase;
    V.acc = reb ? V.acc * exp2i(-(int)fminf(Dg, 1.0e6f)) : V.acc;
    V.R = reb ? V.O : V.R;
    if (C.lane0) *reinterpret_cast<float4*>(pf) = make_float4(V.O, V.O + V.inc, V.O + 2.f * V.inc, V.O + 3.f * V.inc);
}

__device__ __forceinline__ float max3f(float a, float b, float c) {
    float r;
    asm("max.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));
    return r;
}

// One forward cell: a = LSE(v0..v3) in max-shifted form (lg2 sees [1, 4],
// where lg2.approx is accurate to an absolute 2^-22), and, for active lanes,
// the cell's term of the partition function added to acc * 2^R.  A lane whose
// term would leave the float range moves its base R up (rare, warp-uniform
// branch).  Must be called by all 32 lanes together (it votes).
__device__ __forceinline__ float fwd_cell(FwdVars& V, float v0, float v1, float v2, float v3, bool act) {
    const float m = fmaxf(max3f(v0, v1, v2), v3);
    const float s = (ex2f(v0 - m) + ex2f(v1 - m)) + (ex2f(v2 - m) + ex2f(v3 - m));
    float t = m + (V.O - V.R);
    const bool big = act && t > 64.f;
    if (__any_sync(kAll, big)) {  // warp-uniform, rarely taken
        const int kk = big ? (int)t - 16 : 0;
        V.acc *= exp2i(-kk);
        V.R += (float)kk;
        t -= (float)kk;
    }
    const float term = ex2f(t);
    V.acc = act ? fmaf(s, term, V.acc) : V.acc;
    return m + lg2f(s);
}

// 16 forward steps with every lane active (nv == 32, all columns inside
// [0, L2)): per-stage base pointers, immediate offsets per step.
__device__ __forceinline__ void fwd_stage_full(const FwdCtx& C, FwdVars& V, int k) {
    const int c0 = (kCW * k - C.lane) & (kRW - 1);      // this lane's ring column at u = 0
    float* const pA = C.ring + c0;                       // columns c0 .. 63
    float* const pB = pA - kRW;                          // after the wrap past column 63
    const float2* const pbnd = C.bndring + ((kCW * k) & (kRW - 1));  // lane 0: column 16k + u
    float2* const pout = C.bout + (kCW * k - 31);        // lane 31: column 16k + u - 31
    float* const prow0 = C.arow0 + kCW * k;              // lane 0: column 16k + u
    float* const pfr = C.frow + kCW * k;
    // the stage's scores, read before any of its alpha stores so that no load
    // waits behind a store to the same ring
    float scv[kCW];
#pragma unroll
    for (int u = 0; u < kCW; ++u) scv[u] = ((u < kRW - c0) ? pA : pB)[u];
    float2 bvg[4];
#pragma unroll
    for (int u = 0; u < kCW; ++u) {
        float* const p = ((u < kRW - c0) ? pA : pB) + u;
        if ((u & 3) == 0) {
#pragma unroll
            for (int i = 0; i < 4; ++i) bvg[i] = pbnd[u + i];
        }
        if ((u & 3) == 0)
            frame_group_start<true>(C, V, pfr + u);
        else
            V.O += V.inc;
        const float dlt = ((u & 3) == 0) ? V.J : V.inc;
        const float dd = ((u & 3) == 0) ? V.dA : (((u & 3) == 1) ? V.dB : V.dC);
        const float g1 = ((u & 3) == 0) ? V.gA : V.gB;
        const float2 bv = bvg[u & 3];
        const float up = C.lane0 ? bv.x + (bv.y - (V.O - dlt)) : V.uprecv;
        const float sc = scv[u];
        const float v0 = fmaf(sc, C.c, V.uprev - dd);
        const float v1 = up + g1;
        const float v2 = V.left + g1;
        const float v3 = fmaf(sc, C.c, -V.O);
        const float aout = fwd_cell(V, v0, v1, v2, v3, true);
        *p = aout;
        if (C.st31) pout[u] = make_float2(aout, V.O);
        if (C.lane0) prow0[u] = up;
        V.left = aout;
        V.uprev = up;
        V.uprecv = __shfl_up_sync(kAll, aout, 1);
        if ((u & 3) == 3) V.pv = __shfl_sync(kAll, aout, 16);
    }
}

// 16 forward steps at the edges of a row-block (lanes not yet started, already
// finished, or beyond nv), with per-lane activity masks.
__device__ __forceinline__ void fwd_stage_part(const FwdCtx& C, FwdVars& V, int k) {
#pragma unroll
    for (int u = 0; u < kCW; ++u) {
        const int tau = kCW * k + u;
        const int j0 = tau - C.lane;
        const bool act = (C.lane < C.nv) & (j0 >= 0) & (j0 < C.L2);
        if ((u & 3) == 0)
            frame_group_start<false>(C, V, C.frow + tau);
        else
            V.O += V.inc;
        const float dlt = ((u & 3) == 0) ? V.J : V.inc;
        const float dd = ((u & 3) == 0) ? V.dA : (((u & 3) == 1) ? V.dB : V.dC);
        const float g1 = ((u & 3) == 0) ? V.gA : V.gB;
        const float2 bv = C.bndring[tau & (kRW - 1)];
        const float up = C.lane0 ? bv.x + (bv.y - (V.O - dlt)) : V.uprecv;
        const int ix = j0 & (kRW - 1);
        const float sc = C.ring[ix];
        const float v0 = fmaf(sc, C.c, V.uprev - dd);
        const float v1 = up + g1;
        const float v2 = V.left + g1;
        const float v3 = fmaf(sc, C.c, -V.O);
        float aout = fwd_cell(V, v0, v1, v2, v3, act);  // all lanes: it votes
        aout = act ? aout : kNeg;
        if (act) {
            C.ring[ix] = aout;
            if (C.st31) C.bout[j0] = make_float2(aout, V.O);
            if (C.lane0) C.arow0[j0] = up;
        }
        V.left = aout;
        V.uprev = up;
        V.uprecv = __shfl_up_sync(kAll, aout, 1);
        if ((u & 3) == 3) {
            const int mid = (max(0, tau - C.L2 + 1) + min(C.nv - 1, tau)) >> 1;
            V.pv = __shfl_sync(kAll, aout, mid);
        }
    }
}

// ==========================================================================
// reverse sweep of one row-block
// ==========================================================================
struct RevVars {
    float anext, adnext;     // own alpha and row-above alpha at this step's column (loaded last step)
    float pleft, pdiag, precv;
    float gs, hs;            // per-stage partial sums (flushed into doubles)
    float f0, f1;            // forward frames of anti-diagonals tf and tf-1
};

struct RevCtx {
    float* ring;             // ringS + lane*kRW; ringA rows sit at fixed offsets from it
    const float* bbring;     // pushes from the row-block below (zeros for the last row-block)
    const float* fr;
    float* bbout;            // pushes into the row above (row-block r-1), or null
    float c, g, Sint, Sfrac;
    int lane, nv, L2, P;
    bool lastLane, push0;    // lane == nv-1; lane 0 of a row-block with a row-block above
};

// ringA rows relative to this lane's ringS row (WarpSmem layout: ringS, then ringA)
constexpr int kUpOff = 32 * kRW;         // ringA row `lane`      (row above)
constexpr int kOwnOff = 33 * kRW;        // ringA row `lane + 1`  (own row)

// one reverse cell; shared by the full and the edge stages
struct RevCell {
    float wsum, send, pd, pl, gs, hs;
};

__device__ __forceinline__ RevCell rev_cell(const RevCtx& C, const RevVars& V, float a, float au, float al,
                                            float ad, float sc, float f0, float d1, float d2, float inc) {
    const float c0 = (f0 - C.Sint) - C.Sfrac;
    const float gg = C.g + d1;
    const float eu = (au - a) + gg;
    const float el = (al - a) + gg;
    const float ea = fmaf(sc, C.c, (ad - a) + d2);
    const float es = fmaf(sc, C.c, -(a + f0));
    const float wu = ex2f(eu), wl = ex2f(el), wa = ex2f(ea), wsk = ex2f(es);
    const float lp = fminf(a + c0, 0.f);
    const float binit = ex2f(lp);
    const float beta = binit + (V.pleft + inc);
    // The cell's incoming weights are divided by their own sum N (1 up to the
    // rounding of the stored alpha, >= 1/4), as the reference's softmax
    // normalises them (src/sw/kernels_cpu.cpp:41-62): the rounding of a large
    // alpha then cancels out of the flow through the cell instead of adding up
    // along the paths (at T = 0.1 it took the marginals to 2.5-3.6x the
    // reference's own fp32 error).
    const float N = (wa + wsk) + (wu + wl);
    const float bn = __fdividef(beta, N);
    RevCell r;
    const float pu = bn * wu;
    r.pd = bn * wa;
    r.pl = bn * wl;
    r.send = pu + V.pdiag;
    r.gs = pu + r.pl;
    // local choice entropy of the normalised weights: h / N + lg2 N
    const float h = -fmaf(wu, eu, fmaf(wl, el, fmaf(wa, ea, wsk * es)));
    r.hs = fmaf(bn, h, fmaf(beta, lg2f(N), -binit * lp));
    r.wsum = bn * (wa + wsk);
    return r;
}

// 16 reverse steps with every lane active (nv == 32, columns in [1, L2)).
// Here tf = P + 31 - 16k - u = 15 - u (mod 16): the stage reads frames
// 16m-2 .. 16m+15 (tfs = 16m+15) once into registers.
__device__ __forceinline__ void rev_stage_full(const RevCtx& C, RevVars& V, int k) {
    const int m16 = (C.P + 16 - kCW * k) & (kRW - 1);  // 16m mod 64
    const float4 q0 = *reinterpret_cast<const float4*>(C.fr + m16);
    const float4 q1 = *reinterpret_cast<const float4*>(C.fr + m16 + 4);
    const float4 q2 = *reinterpret_cast<const float4*>(C.fr + m16 + 8);
    const float4 q3 = *reinterpret_cast<const float4*>(C.fr + m16 + 12);
    const float2 qm = *reinterpret_cast<const float2*>(C.fr + ((m16 - 2) & (kRW - 1)));
    const float F[18] = {qm.x, qm.y, q0.x, q0.y, q0.z, q0.w, q1.x, q1.y, q1.z,
                         q1.w, q2.x, q2.y, q2.z, q2.w, q3.x, q3.y, q3.z, q3.w};
    const int cb = (C.P - kCW * k + 31 - C.lane) & (kRW - 1);  // this lane's column at u = 0
    float* const qA = C.ring + cb;
    float* const qB = qA + kRW;                                  // after the wrap below column 0
    const int b0 = (C.P - kCW * k) & (kRW - 1);                  // lane 31's column at u = 0 (mult. of 16)
    const float* const pb0 = C.bbring + b0;
    const float* const pb1 = C.bbring + (b0 == 0 ? kRW : b0);
    float* const pbo = C.bbout + (C.P - kCW * k + 31);           // lane 0's column at u = 0
    float gs = 0.f, hs = 0.f;
    // per group of 4 steps, every ring value the group reads is loaded before
    // the group's marginal stores
    // this lane's ring column at step u (u = 16: the first of the next stage)
    auto pcol = [&](int u) { return ((u <= cb) ? qA : qB) - u; };
    float alg[4], adg[4], scg[4], bbg[4];
#pragma unroll
    for (int u = 0; u < kCW; ++u) {
        if ((u & 3) == 0) {
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                alg[i] = pcol(u + i + 1)[kOwnOff];
                adg[i] = pcol(u + i + 1)[kUpOff];
                scg[i] = pcol(u + i)[0];
                bbg[i] = (u + i == 0) ? pb0[0] : pb1[-(u + i)];
            }
        }
        float* const pcj = pcol(u);
        const float f0 = F[17 - u];
        const float a = V.anext, au = V.adnext;
        const float al = alg[u & 3], ad = adg[u & 3];
        const float inc = C.lastLane ? bbg[u & 3] : V.precv;
        const RevCell r = rev_cell(C, V, a, au, al, ad, scg[u & 3], f0, F[16 - u] - f0, F[15 - u] - f0, inc);
        *pcj = r.wsum;
        if (C.push0) pbo[-u] = r.send;
        gs += r.gs;
        hs += r.hs;
        V.precv = __shfl_down_sync(kAll, r.send, 1);
        V.pdiag = r.pd;
        V.pleft = r.pl;
        V.anext = al;
        V.adnext = ad;
    }
    V.gs += gs;
    V.hs += hs;
    V.f0 = F[1];
    V.f1 = F[0];
}

// 16 reverse steps at the edges of a row-block, with per-lane activity masks.
__device__ __forceinline__ void rev_stage_part(const RevCtx& C, RevVars& V, int k) {
#pragma unroll
    for (int u = 0; u < kCW; ++u) {
        const int tau = kCW * k + u;
        const int tf = C.P + C.nv - 1 - tau;            // forward step (anti-diagonal) of this step
        const int j0 = C.P - tau + (C.nv - 1 - C.lane);
        const bool act = (C.lane < C.nv) & (j0 >= 0) & (j0 < C.L2);
        // frames of anti-diagonals tf, tf-1, tf-2 (rotated through registers).
        // The forward's lane 0 stores the row above at column 0 in the frame of
        // step 0, so frame indices below 0 read frame 0.
        const float f2 = C.fr[max(tf - 2, 0) & (kRW - 1)];
        const float f0 = V.f0;
        const int cj = j0 & (kRW - 1), cl = (j0 - 1) & (kRW - 1);
        const float a = V.anext;
        const float au = V.adnext;
        const bool hasLeft = j0 >= 1;
        const float al = hasLeft ? C.ring[kOwnOff + cl] : kNeg;
        const float ad = hasLeft ? C.ring[kUpOff + cl] : kNeg;
        const float sc = C.ring[cj];
        const float inc = C.lastLane ? C.bbring[cj] : V.precv;
        const RevCell r = rev_cell(C, V, a, au, al, ad, sc, f0, V.f1 - f0, f2 - f0, inc);
        // inactive lanes push nothing (their inputs may be garbage)
        V.gs += act ? r.gs : 0.f;
        V.hs += act ? r.hs : 0.f;
        const float send = act ? r.send : 0.f;
        if (act) {
            C.ring[cj] = r.wsum;
            if (C.push0) C.bbout[j0] = send;
        }
        V.precv = __shfl_down_sync(kAll, send, 1);
        V.pdiag = act ? r.pd : 0.f;
        V.pleft = act ? r.pl : 0.f;
        V.anext = al;
        V.adnext = ad;
        V.f0 = V.f1;
        V.f1 = f2;
    }
}

// ==========================================================================
// linear gap, value + marginals
// ==========================================================================
// Forward, row-block r (rows 32r .. 32r+nv-1, 0-based), local step tau:
//   lane l works on column j = tau - l.  Stage k (tau = 16k..16k+15): lane 0 is
//   in chunk k, the trailing lane in chunk >= k-2.  At its start chunk k-3
//   (finished) is written back as alpha and chunk k+1 of the scores is
//   prefetched into the same ring slot.
// Reverse, row-block r, local step tau, P = 16*ceil((L2-1)/16):
//   lane l works on column j = P - tau + (nv-1-l) (real work only for j <= L2-1);
//   forward frame index tf = P + nv - 1 - tau.  At stage k the leading lane
//   enters chunk n = P/16 - k - 1; chunks n..n+2 are read, chunk n+3 (finished)
//   is written back as marginals and chunk n-1 is prefetched.
// Progress: warp w publishes (ordinal << 16 | stages done) after every stage of
// its current row-block (ordinal = r forward, nRB-1-r reverse), and
// (ordinal << 16 | kStageMask) when the row-block is complete.
// problems this kernel recomputed after a linear-domain kernel flagged them
// (cumulative on the device; d2p_engine_counts reads it)
__device__ unsigned long long g_fixups;

__global__ void __launch_bounds__(kNW * 32) lin_marg_kernel(SwArgs p) {
    extern __shared__ __align__(16) unsigned char smem_raw[];
    WarpSmem& W = reinterpret_cast<WarpSmem*>(smem_raw)[threadIdx.x >> 5];
    __shared__ int progF[kNW], progR[kNW];
    __shared__ __align__(16) float red[4 * 32];
    __shared__ int sh_Sint, sh_err;
    __shared__ float sh_Sfrac;

    const int b = blockIdx.x;
    if (p.only) {   // fix-up launch: only the problems a linear-domain kernel flagged
        if (p.only[b] == 0) {
            if (p.redo && threadIdx.x == 0) p.redo[b] = 0;
            return;
        }
        if (threadIdx.x == 0) atomicAdd(&g_fixups, 1ull);
    }
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int L1m = p.L1, L2m = p.L2;
    const int L1 = p.lengths ? min(max(p.lengths[2 * b], 0), L1m) : L1m;
    const int L2 = p.lengths ? min(max(p.lengths[2 * b + 1], 0), L2m) : L2m;
    const float gapn = p.gap_dev ? __ldg(p.gap_dev) : p.gap;
    const float T = p.temp_dev ? __ldg(p.temp_dev) : p.temp;
    const float c = kLog2e / T;
    const float g = gapn * c;
    const size_t plane = (size_t)L1m * L2m;
    const float* __restrict__ S = p.scores + (size_t)b * plane;
    float* __restrict__ out = p.out ? p.out + (size_t)b * plane : nullptr;
    const Layout LY = carve(p.ws, b, L1m, L2m);
    const int nRB = (L1 + 31) / 32;
    const int nch = (L2 + kCW - 1) / kCW;
    const size_t abs_ = (size_t)33 * L2m;       // aplane row-block stride
    const size_t fst = frame_row(L2m);          // frames row stride

    if (out && (L1 < L1m || L2 < L2m)) {  // zero the padded part of the marginals
        for (int i = warp; i < L1m; i += kNW) {
            float* row = out + (size_t)i * L2m;
            for (int j = (i < L1 ? L2 : 0) + lane; j < L2m; j += 32) row[j] = 0.f;
        }
    }
    if (L1 == 0 || L2 == 0) {  // S = log(1) = 0 (alpha[0,0] only), zero gradients
        if (threadIdx.x == 0) {
            if (p.value) p.value[b] = 0.f;
            if (p.grad_gap) p.grad_gap[b] = 0.f;
            if (p.grad_T) p.grad_T[b] = 0.f;
            if (p.redo) p.redo[b] = 0;
        }
        return;
    }
    if (threadIdx.x < kNW) {
        progF[threadIdx.x] = -1;
        progR[threadIdx.x] = -1;
    }
    if (threadIdx.x == 0) sh_err = 0;
    __syncthreads();

    // ============================== forward ==============================
    FwdVars V;
    V.acc = 0.f;
    V.R = 0.f;
    bool haveR = false;
    for (int r = warp; r < nRB; r += kNW) {
        const int nv = min(32, L1 - 32 * r);
        const int nst = (L2 + nv - 1 + kCW - 1) / kCW;
        const float* srow = S + (size_t)(32 * r) * L2m;
        const float2* brow = LY.bnd + (size_t)(r - 1) * L2m;
        float* arow = LY.aplane + (size_t)r * abs_;
        const bool hasB = r > 0, hasD = r + 1 < nRB;
        FwdCtx C;
        C.ring = W.ringS + lane * kRW;
        C.bndring = W.bnd;
        C.arow0 = arow;
        C.bout = LY.bnd + (size_t)r * L2m;
        C.frow = LY.frames + (size_t)r * fst;
        C.c = c;
        C.g = g;
        C.lane = lane;
        C.nv = nv;
        C.L2 = L2;
        C.lane0 = lane == 0;
        C.st31 = (lane == 31) && hasD;
        const int* upflag = &progF[(warp + kNW - 1) % kNW];
        const int upbase = (r - 1) << 16;

        const Tile tS = make_tile(srow, L2m, W.ringS, nv, lane);        // scores -> ring
        const Tile tA = make_tile(arow + L2m, L2m, W.ringS, nv, lane);  // ring (alpha) -> plane
        __syncwarp();
        if (!hasB) {  // no row above: the boundary ring reads as -inf
            W.bnd[lane] = make_float2(kNeg, 0.f);
            W.bnd[lane + 32] = make_float2(kNeg, 0.f);
        }
        int ld = 0, sta = 0;
        for (; ld < 2 && ld < nch; ++ld) {
            if (hasB) wait_flag(upflag, upbase + min(ld + 3, kStageMask), &sh_err);
            tile_load<4>(tS, ld, L2);
            if (hasB) load_row_chunk8(W.bnd, brow, L2, ld, lane);
            cp_async_commit();
        }
        V.O = 0.f;
        if (hasB) {  // start the frame at the row above, column 0
            cp_async_wait0();
            __syncwarp();
            const float2 bv = W.bnd[0];
            V.O = bv.y + rintf(bv.x);
        }
        if (!haveR) {
            V.R = V.O;
            haveR = true;
        }
        V.inc = 0.f;  // the first group start sets J, inc and the offsets
        V.left = V.uprev = V.uprecv = kNeg;
        V.pv = kNeg;

        for (int k = 0; k < nst; ++k) {
            if (k > 0) {
                __syncwarp();
                // alpha write-back of finished chunks (rows 1..nv of this row-block's tile)
                while (sta < nch && (sta + 1) * kCW <= kCW * k - (nv - 1)) {
                    tile_store(tA, sta, L2);
                    ++sta;
                }
                if (ld <= k + 1 && ld < nch) {
                    if (hasB) wait_flag(upflag, upbase + min(ld + 3, kStageMask), &sh_err);
                    tile_load<4>(tS, ld, L2);
                    if (hasB) load_row_chunk8(W.bnd, brow, L2, ld, lane);
                    ++ld;
                }
            }
            cp_async_commit();
            cp_async_wait1();
            __syncwarp();
            if ((nv == 32) && (kCW * k >= 31) && (kCW * k + kCW - 1 <= L2 - 1))
                fwd_stage_full(C, V, k);
            else
                fwd_stage_part(C, V, k);
            // lane 31 wrote this stage's boundary cells: publish them
            if (C.st31) st_release(&progF[warp], (r << 16) | min(k + 1, kStageMask - 1));
        }
        __syncwarp();
        while (sta < nch) {
            tile_store(tA, sta, L2);
            ++sta;
        }
        cp_async_wait0();
        __syncwarp();
        if (lane == 31) st_release(&progF[warp], (r << 16) | kStageMask);
    }

    // ---- S = log2(sum_lanes acc*2^R + 2^0), kept as integer + fraction
    {
        const bool has = haveR && V.acc > 0.f;
        const int Rm = (int)block_max(has ? fmaxf(V.R, 0.f) : 0.f, red);
        float part = has ? V.acc * exp2i((int)V.R - Rm) : 0.f;
        if (threadIdx.x == 0) part += exp2i(-Rm);  // alpha[0,0] = 0
        const float tot = block_sum(part, red);
        if (threadIdx.x == 0) {
            const float l2 = lg2_rr(tot);
            const float fl = floorf(l2);
            sh_Sint = Rm + (int)fl;
            sh_Sfrac = l2 - fl;
            if (p.value) p.value[b] = ((float)sh_Sint + sh_Sfrac) / c;
        }
        __syncthreads();
    }

    // ============================== reverse ==============================
    const int P = kCW * ((L2 - 1 + kCW - 1) / kCW);
    double gsum = 0.0, hsum = 0.0;
    {
        RevVars RV;
        for (int q = warp; q < nRB; q += kNW) {
            const int r = nRB - 1 - q;
            const int nv = min(32, L1 - 32 * r);
            const int nst = (P + nv + kCW - 1) / kCW;
            const int nfr = L2 + nv - 1;           // frames recorded for this row-block
            const float* atile = LY.aplane + (size_t)r * abs_;
            const float* srow = S + (size_t)(32 * r) * L2m;
            const float* frow = LY.frames + (size_t)r * fst;
            const float* bbrow = LY.bb + (size_t)(r + 1) * L2m;
            const bool hasBelow = r + 1 < nRB;
            RevCtx C;
            C.ring = W.ringS + lane * kRW;
            C.bbring = W.bb;
            C.fr = W.fr;
            C.bbout = r > 0 ? LY.bb + (size_t)r * L2m : LY.bb;
            C.c = c;
            C.g = g;
            C.Sint = (float)sh_Sint;
            C.Sfrac = sh_Sfrac;
            C.lane = lane;
            C.nv = nv;
            C.L2 = L2;
            C.P = P;
            C.lastLane = lane == nv - 1;
            C.push0 = (lane == 0) && (r > 0);
            const int nvB = hasBelow ? min(32, L1 - 32 * (r + 1)) : 0;
            const int* dnflag = &progR[(warp + kNW - 1) % kNW];
            const int dnbase = (q - 1) << 16;
            // stages of row-block r+1 that must be complete before bb chunk ch is
            // read: its lane 0 pushes into column j at its step P + nvB - 1 - j
            auto bb_need = [&](int ch) {
                return dnbase + min(max(P + nvB - 1 - kCW * ch, 0) / kCW + 1, kStageMask);
            };

            const Tile tA = make_tile(atile, L2m, W.ringA, nv + 1, lane);  // alpha tile -> ringA
            const Tile tS = make_tile(srow, L2m, W.ringS, nv, lane);       // scores -> ringS
            const Tile tM = make_tile(out ? out + (size_t)(32 * r) * L2m : S, L2m, W.ringS, nv, lane);
            __syncwarp();
            if (!hasBelow) {  // no row-block below: its pushes read as zero
                W.bb[lane] = 0.f;
                W.bb[lane + 32] = 0.f;
            }
            int ldn = nch, stm = nch - 1;
            int ldf = (min(P + nv - 1, nfr - 1) >> 4) + 1;
            const int n0 = P / kCW - 1;
            while (ldn > max(n0, 0)) {  // chunks n..n+2 for stage 0
                --ldn;
                tile_load<5>(tA, ldn, L2);
                tile_load<4>(tS, ldn, L2);
                if (hasBelow) {
                    wait_flag(dnflag, bb_need(ldn), &sh_err);
                    load_row_chunk4(W.bb, bbrow, L2, ldn, lane);
                }
            }
            while (ldf > (max(P + nv - 1 - 17, 0) >> 4)) {
                --ldf;
                load_row_chunk4(W.fr, frow, nfr, ldf, lane);
            }
            cp_async_commit();
            RV.pleft = RV.pdiag = RV.precv = 0.f;

            for (int k = 0; k < nst; ++k) {
                const int n = P / kCW - k - 1;       // chunk the leading lane enters
                const int tfs = P + nv - 1 - kCW * k; // frame index at the stage start
                __syncwarp();
                if (k > 0) {
                    while (stm >= 0 && stm >= n + 3) {  // finished marginal chunks
                        if (out) tile_store(tM, stm, L2);
                        --stm;
                    }
                }
                while (ldn > max(n - 1, 0)) {  // prefetch for the next stage
                    --ldn;
                    tile_load<5>(tA, ldn, L2);
                    tile_load<4>(tS, ldn, L2);
                    if (hasBelow) {
                        wait_flag(dnflag, bb_need(ldn), &sh_err);
                        load_row_chunk4(W.bb, bbrow, L2, ldn, lane);
                    }
                }
                while (ldf > (max(tfs - 33, 0) >> 4)) {
                    --ldf;
                    load_row_chunk4(W.fr, frow, nfr, ldf, lane);
                }
                cp_async_commit();
                cp_async_wait1();
                __syncwarp();
                if (k == 0) {  // own alpha, row-above alpha and frames at the first step
                    const int j0 = P + nv - 1 - lane;
                    RV.anext = C.ring[kOwnOff + (j0 & (kRW - 1))];
                    RV.adnext = C.ring[kUpOff + (j0 & (kRW - 1))];
                    RV.f0 = W.fr[(P + nv - 1) & (kRW - 1)];
                    RV.f1 = W.fr[max(P + nv - 2, 0) & (kRW - 1)];
                }
                RV.gs = 0.f;
                RV.hs = 0.f;
                if ((nv == 32) && (kCW * k >= P + 32 - L2) && (kCW * k + kCW - 1 <= P - 1))
                    rev_stage_full(C, RV, k);
                else
                    rev_stage_part(C, RV, k);
                gsum += (double)RV.gs;
                hsum += (double)RV.hs;
                // lane 0 wrote this stage's pushes into the row above: publish them
                if (C.push0) st_release(&progR[warp], (q << 16) | min(k + 1, kStageMask - 1));
            }
            __syncwarp();
            while (stm >= 0) {
                if (out) tile_store(tM, stm, L2);
                --stm;
            }
            cp_async_wait0();
            __syncwarp();
            if (lane == 0) st_release(&progR[warp], (q << 16) | kStageMask);
        }
    }

    if (threadIdx.x == 0) {  // origin alpha[0,0] = 0 as an end state
        const float lp0 = fminf(-sh_Sfrac - (float)sh_Sint, 0.f);
        hsum += (double)ex2f(lp0) * (double)(-lp0);
    }
    const double G = block_sum_d(gsum, reinterpret_cast<double*>(red));
    const double H = block_sum_d(hsum, reinterpret_cast<double*>(red));
    // a dependency wait that gave up: the general engine recomputes this problem
    // (the caller launches it)
    const int redo = __syncthreads_or(sh_err);
    if (threadIdx.x == 0) {
        if (p.redo) p.redo[b] = redo;
        if (sh_err && p.status) atomicOr(p.status, 1);
        if (p.grad_gap) p.grad_gap[b] = (float)G;
        if (p.grad_T) p.grad_T[b] = (float)(H * (double)kLn2);
    }
}

}  // namespace wf

// ------------------------------------------------------------------ host side
int wavefront_fixup_count(unsigned long long* n) {
    return (int)cudaMemcpyFromSymbol(n, wf::g_fixups, sizeof(unsigned long long));
}

size_t wavefront_workspace_bytes(int family, int B, int L1, int L2) {
    if (family != 0) return 0;
    if (L1 > 32 * wf::kMaxRB || L2 % 4 != 0) return 0;
    return wf::per_problem_bytes(L1, L2) * (size_t)B;
}

int launch_wavefront(const SwArgs& a, int family, size_t ws_bytes, cudaStream_t st) {
    if (family != 0 || a.mode != MODE_MARG || !a.redo) return -1;
    if (engine_forced_plane()) return -1;
    if (a.L2 % 4 != 0 || a.L1 > 32 * wf::kMaxRB || a.L1 == 0 || a.L2 == 0) return -1;
    if ((((uintptr_t)a.scores) & 15) != 0 || (a.out && (((uintptr_t)a.out) & 15) != 0)) return -1;
    if ((((uintptr_t)a.ws) & 255) != 0) return -1;
    const size_t need = wf::per_problem_bytes(a.L1, a.L2) * (size_t)a.B;
    if (ws_bytes < need || !a.ws) return -1;
    const size_t smem = sizeof(wf::WarpSmem) * wf::kNW;
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return (int)e;
    static DeviceSetup setup;
    int nsm = 0;
    const int se = device_setup(setup, dev, [smem] {
        return (int)cudaFuncSetAttribute(wf::lin_marg_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    }, &nsm);
    if (se != 0) return se;
    wf::lin_marg_kernel<<<a.B, wf::kNW * 32, smem, st>>>(a);
    return (int)cudaGetLastError();
}

}  // namespace d2pb
