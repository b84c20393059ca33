// sw_linear.cu -- linear-domain fast path for linear-gap soft Smith-Waterman
// value + marginals.
//
// The forward carries Z_ij = 2^a_ij itself (a = alpha log2(e)/T) instead of its
// logarithm.  In that domain the reference's log-sum-exp recurrence
// (src/sw/kernels_cpu.cpp:70-150)
//   Z_ij = P_ij (Z_{i-1,j-1} + 1) + G (Z_{i-1,j} + Z_{i,j-1}),   P = 2^(s c), G = 2^(gap c)
// costs one exponential (P) and four FP operations per cell, and the reverse
// pass (src/sw/kernels_cpu.cpp:156-279) becomes the outside recurrence
//   B_ij = 1 + P_{i+1,j+1} B_{i+1,j+1} + G (B_{i+1,j} + B_{i,j+1}),
//   marginal_ij = B_ij P_ij (Z_{i-1,j-1} + 1) / Z_total,
// with Z_total = 2^S = 1 + sum_ij Z_ij.  Cells outside the problem are 0.
//
// Range.  Every lane (row) keeps its own power-of-two frame, Z = z 2^E and
// B = b 2^Q, re-anchored every 4 steps on the lane's own last value, so z and
// b stay near 1; values from a neighbour lane or from the next row-block are
// converted by exact 2^k factors, and a lane that starts inherits its
// neighbour's frame.  If a value of a problem still leaves [2^-60, 2^60]
// (score magnitudes far beyond the usual ones), the problem is flagged and the
// caller recomputes it with the log-domain kernel (sw_wavefront.cu).
//
// Structure (shared with sw_wavefront.cu): one CTA per problem; warps own
// row-blocks of 32 rows (lane = row) and sweep them along anti-diagonals;
// consecutive row-blocks hand their boundary rows over through L2-resident
// workspace rows guarded by release/acquire progress words.  The forward
// stores z in a diagonal-major plane (row = forward step + 2, 32 lanes per
// row) so that both passes move it with one coalesced 128-byte access per
// step; the reverse stages it 16 rows (2 KB) at a time through shared memory.
//
// Reverse indexing: reverse step tau of a row-block works on forward
// anti-diagonal tf = P + 31 - tau (P = 16 ceil((L2-1)/16)); lane l is at
// column tf - l.  Stage k (16 steps) covers tf in [16M, 16M + 15] with
// M = P/16 + 1 - k for every row-block height.
#include <stdint.h>

#include "sw_common.cuh"
#include "sw_internal.h"
#include "sw_ring.cuh"

namespace d2pb {
namespace lin {
using namespace ring;

constexpr int kMaxRB = 512;              // row-blocks per problem (L1 <= 16384)
constexpr int kNW = 6;                   // warps per CTA
constexpr int kRebase = 32;              // partition: rebase when the frame runs this far above R
constexpr float kWinLo = 8.673617380e-19f;   // 2^-60
constexpr float kWinHi = 1.152921505e18f;    // 2^60

struct WarpSmem {
    float ringS[32 * kRW];   // scores [rows][64]; reverse: marginals written in place
    float zr[2][16 * 32];    // reverse: z plane, one 16-step block per slot
    int er[16 * 32];         // reverse: forward frames, 16 group slots (4 blocks of 4 groups)
    float rr[kRW];           // reverse: row above the row-block (lane 0's diagonal input)
    float2 bnd[kRW];         // forward: last row of the row-block above (z, frame bits)
    float2 bbr[kRW];         // reverse: pushes from the row-block below (value, frame bits)
};

struct Layout {  // per-problem workspace
    float* zpl;      // [nRB][ZT][32]   z of forward step t at row t + 2 (rows 0, 1: zeros)
    int* efr;        // [nRB][GT][32]   frame of each lane for each group of 4 forward steps
    float* rab;      // [nRB][L2m + 64] lane 0's up input (row above) of column j at j + 1
    float2* bnd;     // [nRB][L2m]      last row of each row-block: (z, frame bits)
    float2* bbv;     // [nRB][L2m + 64] reverse pushes of lane 0 into the row above, at column + 15
};

// Row lengths leave room for the reverse's 16-entry staging blocks, which run
// up to 31 entries past the last column.
__host__ __device__ inline int zt_rows(int L2m) { return L2m + 64; }
__host__ __device__ inline int gt_rows(int L2m) { return (L2m + 64) / 4; }
__host__ __device__ inline int rb_len(int L2m) { return L2m + 64; }

__host__ __device__ inline size_t per_problem_bytes(int L1m, int L2m) {
    const size_t nrb = (size_t)(L1m + 31) / 32;
    size_t b = align_up(nrb * zt_rows(L2m) * 32 * 4, 256);
    b += align_up(nrb * gt_rows(L2m) * 32 * 4, 256);
    b += align_up(nrb * (size_t)rb_len(L2m) * 4, 256);
    b += align_up(nrb * (size_t)L2m * 8, 256);
    b += align_up(nrb * (size_t)rb_len(L2m) * 8, 256);
    return b;
}

__device__ inline Layout carve(float* ws, int b, int L1m, int L2m) {
    const size_t nrb = (size_t)(L1m + 31) / 32;
    char* base = (char*)ws + (size_t)b * per_problem_bytes(L1m, L2m);
    Layout L;
    L.zpl = (float*)base;
    base += align_up(nrb * zt_rows(L2m) * 32 * 4, 256);
    L.efr = (int*)base;
    base += align_up(nrb * gt_rows(L2m) * 32 * 4, 256);
    L.rab = (float*)base;
    base += align_up(nrb * (size_t)rb_len(L2m) * 4, 256);
    L.bnd = (float2*)base;
    base += align_up(nrb * (size_t)L2m * 8, 256);
    L.bbv = (float2*)base;
    return L;
}

// 2^k for integer k, exact; 0 below 2^-126, clamped at 2^127
__device__ __forceinline__ float p2(int k) { return exp2i(k); }
// exponent of a positive normal float (0 for zero)
__device__ __forceinline__ int expo(float v) { return v > 0.f ? (__float_as_int(v) >> 23) - 127 : 0; }

// ==========================================================================
// forward sweep of one row-block
// ==========================================================================
struct FwdVars {
    float zl, zu, zd;   // own previous output, up input (as received), diag input (this lane's frame)
    int E;              // this lane's frame
    int Eup_last;       // lane l-1's frame when it produced the up input received next
    float d0, d1;       // 2^(E_{l-1} - E) for outputs lane l-1 sent in the previous / this group
    float fs;           // 2^-E: the +1 start term in this frame
    float acc, ps;      // partition of this lane's cells: sum Z = acc 2^R; ps = 2^(E - R)
    int R;
    float mn, mx;       // range of this lane's outputs
};

struct FwdCtx {
    const float* ring;   // this lane's ring row
    const float2* bndring;
    float* zrow;         // zpl row 2 (forward step 0) of this row-block, this lane
    int* erow;           // efr group 0 of this row-block, this lane
    float* rab;          // rab of this row-block
    float2* bout;        // bnd of this row-block
    float c, G;
    int lane, nv, L2;
    bool lane0, st31;
};

// partition base and start term after a change of E
__device__ __forceinline__ void fwd_frame_factors(FwdVars& V) {
    int D = V.E - V.R;
    const bool reb = D > kRebase;
    V.acc = reb ? V.acc * p2(-D) : V.acc;
    V.R = reb ? V.E : V.R;
    D = reb ? 0 : D;
    V.ps = p2(D);
    V.fs = p2(-V.E);
}

// group start (every 4 steps): re-anchor this lane's frame on its last output
// and set the conversion factors for lane l-1's outputs (d0: the one it sent
// in the previous step, d1: those it sends in this group).  Returns lane
// l-1's frame of the previous step (needed by a lane that starts right now).
__device__ __forceinline__ int fwd_group_start(FwdVars& V) {
    const int J = expo(V.zl);
    V.E += J;
    const float fJ = p2(-J);
    V.zl *= fJ;
    V.zd *= fJ;
    const int Eup = __shfl_up_sync(kAll, V.E, 1);
    const int before = V.Eup_last;
    V.d0 = p2(V.Eup_last - V.E);
    V.d1 = p2(Eup - V.E);
    V.Eup_last = Eup;
    fwd_frame_factors(V);
    return before;
}

// lane 0's up input: the row-block above's last row, (z, frame) -> frame E
__device__ __forceinline__ float from_above(float2 bv, int E) { return bv.x * p2(__float_as_int(bv.y) - E); }

// 16 forward steps with every lane active: per-stage pointers, immediate offsets
__device__ __forceinline__ void fwd_stage_full(const FwdCtx& C, FwdVars& V, int k) {
    const int c0 = (kCW * k - C.lane) & (kRW - 1);   // this lane's ring column at u = 0
    const float* const pA = C.ring + c0;
    const float* const pB = pA - kRW;                 // after the wrap past column 63
    float scv[kCW];  // the stage's scores, read before anything else happens
#pragma unroll
    for (int u = 0; u < kCW; ++u) scv[u] = ((u < kRW - c0) ? pA : pB)[u];
    const float2* const pbnd = C.bndring + ((kCW * k) & (kRW - 1));  // lane 0: column 16k + u
    float* const pz = C.zrow + (size_t)(kCW * k) * 32;
    float2* const pout = C.bout + (kCW * k - 31);                     // lane 31: column 16k + u - 31
    float* const prab = C.rab + kCW * k + 1;
    int* const pe = C.erow + (size_t)(kCW * k / 4) * 32;
#pragma unroll
    for (int u = 0; u < kCW; ++u) {
        if ((u & 3) == 0) fwd_group_start(V);
        const float zu_n = V.zu * (((u & 3) == 0) ? V.d0 : V.d1);
        const float zu_in = C.lane0 ? from_above(pbnd[u], V.E) : zu_n;
        const float P = ex2f(scv[u] * C.c);
        const float z = fmaf(C.G, zu_in + V.zl, P * (V.zd + V.fs));
        V.acc = fmaf(z, V.ps, V.acc);
        V.mn = fminf(V.mn, z);
        V.mx = fmaxf(V.mx, z);
        pz[(size_t)u * 32] = z;
        if (C.st31) pout[u] = make_float2(z, __int_as_float(V.E));
        if (C.lane0) prab[u] = zu_in;
        if ((u & 3) == 3) pe[(u >> 2) * 32] = V.E;
        V.zd = zu_in;
        V.zl = z;
        V.zu = __shfl_up_sync(kAll, z, 1);
    }
}

// edge stages: per-lane activity masks; a lane that starts (column 0) takes
// lane l-1's frame (lane 0: the frame of the row above) so that its first
// value is near 1
__device__ __forceinline__ void fwd_stage_part(const FwdCtx& C, FwdVars& V, int k) {
#pragma unroll 4
    for (int u = 0; u < kCW; ++u) {
        const int tau = kCW * k + u;
        const int j0 = tau - C.lane;
        const bool act = (C.lane < C.nv) & (j0 >= 0) & (j0 < C.L2);
        int Eup_before = V.Eup_last;  // lane l-1's frame at the previous step
        if ((u & 3) == 0) Eup_before = fwd_group_start(V);
        const int Eup = __shfl_up_sync(kAll, V.E, 1);
        const float2 bv = C.bndring[tau & (kRW - 1)];
        if ((C.lane < C.nv) && j0 == 0) {  // this lane starts: adopt the neighbour's frame
            V.E = C.lane0 ? __float_as_int(bv.y) : Eup;
            V.d0 = p2(Eup_before - V.E);
            V.d1 = 1.f;
            V.zl = V.zd = 0.f;
            fwd_frame_factors(V);
        }
        const float zu_n = V.zu * (((u & 3) == 0) ? V.d0 : V.d1);
        const float zu_in = C.lane0 ? from_above(bv, V.E) : zu_n;
        const float P = ex2f(C.ring[j0 & (kRW - 1)] * C.c);
        float z = fmaf(C.G, zu_in + V.zl, P * (V.zd + V.fs));
        z = act ? z : 0.f;
        V.acc = fmaf(z, V.ps, V.acc);
        V.mn = act ? fminf(V.mn, z) : V.mn;
        V.mx = act ? fmaxf(V.mx, z) : V.mx;
        C.zrow[(size_t)tau * 32] = z;
        if (act && C.st31) C.bout[j0] = make_float2(z, __int_as_float(V.E));
        if (act && C.lane0) C.rab[j0 + 1] = zu_in;
        if ((u & 3) == 3) C.erow[(size_t)(tau >> 2) * 32] = V.E;
        V.zd = act ? zu_in : 0.f;
        V.zl = z;
        V.zu = __shfl_up_sync(kAll, z, 1);
        // lane l-1's frame for the output just received (it may have started this step)
        V.Eup_last = __shfl_up_sync(kAll, V.E, 1);
    }
}

// ==========================================================================
// reverse sweep of one row-block
// ==========================================================================
struct RevVars {
    float br, recv, pbp;  // own b of column j+1, message from lane l+1, own P*b of column j+1
    int Q;                // this lane's reverse frame
    int Qdn_last;         // lane l+1's frame when it sent the message received next
    float d0, d1;         // 2^(Q_{l+1} - Q) for messages lane l+1 sent in the previous / this group
    float fsq;            // 2^-Q: the +1 end term in this frame
    float k2;             // 2^(Q - S)
    float kA, kB;         // 2^(Q + E_diag - S) for the two forward groups a reverse group reads
    float mn, mx;
};

struct RevCtx {
    float* ring;          // ringS row of this lane
    const float* zr;      // WarpSmem::zr
    const int* er;        // WarpSmem::er
    const float* rr;      // WarpSmem::rr
    const float2* bbr;    // WarpSmem::bbr
    float2* bbout;        // bbv of this row-block (pushes into the row above), index column + 15
    float c, G, cS;       // cS = 2^-Sfrac
    int Sint, lane, nv, L2, P;
    int ecol;             // er column of this lane's diagonal input: lane l-1 (lane 0: 0)
    bool lane0, lastLane, push0;
};

// k factors of the reverse group starting at anti-diagonal tf0 (tf0 = 3 mod 4).
// The diagonal input of lane l at anti-diagonal tf is lane l-1's z of forward
// group (tf-2)/4 (lane 0: the row above, kept in lane 0's frame of group
// (tf-1)/4); over tf0, tf0-1, tf0-2, tf0-3 that is group A = (tf0-3)/4 + ... :
//   lanes >= 1: A for the first two steps, B = A - 1 for the last two;
//   lane 0:     A for the first three steps, B for the last.
__device__ __forceinline__ void rev_k_factors(const RevCtx& C, RevVars& V, int tf0) {
    const int gA = (tf0 - 3) >> 2;
    const int EA = C.er[(gA & 15) * 32 + C.ecol];
    const int EB = C.er[((gA - 1) & 15) * 32 + C.ecol];
    V.kA = p2(V.Q + EA - C.Sint) * C.cS;
    V.kB = p2(V.Q + EB - C.Sint) * C.cS;
    V.fsq = p2(-V.Q);
    V.k2 = p2(V.Q - C.Sint) * C.cS;
}

__device__ __forceinline__ int rev_group_start(const RevCtx& C, RevVars& V, int tf0) {
    const int J = expo(V.br);
    V.Q += J;
    const float fJ = p2(-J);
    V.br *= fJ;
    V.pbp *= fJ;
    const int Qdn = __shfl_down_sync(kAll, V.Q, 1);
    const int before = V.Qdn_last;
    V.d0 = p2(V.Qdn_last - V.Q);
    V.d1 = p2(Qdn - V.Q);
    V.Qdn_last = Qdn;
    rev_k_factors(C, V, tf0);
    return before;
}

__device__ __forceinline__ float kdiag(const RevCtx& C, const RevVars& V, int w) {
    if (w < 2) return V.kA;
    if (w == 3) return V.kB;
    return C.lane0 ? V.kA : V.kB;
}

__device__ __forceinline__ float from_below(float2 bv, int Q) { return bv.x * p2(__float_as_int(bv.y) - Q); }

// 16 reverse steps with every lane active
__device__ __forceinline__ void rev_stage_full(const RevCtx& C, RevVars& V, int k) {
    const int m16 = C.P + 16 - kCW * k;                              // tf = m16 + 15 - u
    const float* const zb = C.zr + ((m16 >> 4) & 1) * (16 * 32) + C.ecol;   // lane l-1's column
    const int cb = (C.P + 31 - kCW * k - C.lane) & (kRW - 1);       // ring column at u = 0
    float* const qA = C.ring + cb;
    float* const qB = qA + kRW;                                       // after the wrap below column 0
    float scv[kCW];
#pragma unroll
    for (int u = 0; u < kCW; ++u) scv[u] = (((u <= cb) ? qA : qB) - u)[0];
    const int b0 = (C.P - kCW * k + 15) & (kRW - 1);                 // bbr index of lane 31 at u = 0
    float2* const pbo = C.bbout + (C.P - kCW * k + 31 + 15);          // lane 0: column P - 16k + 31 - u
#pragma unroll
    for (int u = 0; u < kCW; ++u) {
        const int tf = m16 + 15 - u;
        if ((u & 3) == 0) rev_group_start(C, V, tf);
        const float ad = C.lane0 ? C.rr[tf & (kRW - 1)] : zb[(15 - u) * 32];
        const float rc = V.recv * (((u & 3) == 0) ? V.d0 : V.d1);
        const float inc = C.lastLane ? from_below(C.bbr[(b0 - u) & (kRW - 1)], V.Q) : rc;
        const float P = ex2f(scv[u] * C.c);
        const float b = fmaf(C.G, V.br, inc) + V.fsq;
        const float pb = P * b;
        const float msg = fmaf(C.G, b, V.pbp);
        const float mu = P * fmaf(b * ad, kdiag(C, V, u & 3), b * V.k2);
        (((u <= cb) ? qA : qB) - u)[0] = mu;
        if (C.push0) pbo[-u] = make_float2(msg, __int_as_float(V.Q));
        V.mn = fminf(V.mn, b);
        V.mx = fmaxf(V.mx, b);
        V.recv = __shfl_down_sync(kAll, msg, 1);
        V.br = b;
        V.pbp = pb;
    }
}

// edge stages: per-lane activity; a lane that starts (column L2-1) takes lane
// l+1's frame (the bottom lane: the frame of the pushes from below)
__device__ __forceinline__ void rev_stage_part(const RevCtx& C, RevVars& V, int k) {
    const int m16 = C.P + 16 - kCW * k;
    const float* const zb = C.zr + ((m16 >> 4) & 1) * (16 * 32) + C.ecol;
#pragma unroll 4
    for (int u = 0; u < kCW; ++u) {
        const int tf = m16 + 15 - u;
        const int j0 = tf - C.lane;
        const bool act = (C.lane < C.nv) & (j0 >= 0) & (j0 < C.L2);
        int Qdn_before = V.Qdn_last;
        if ((u & 3) == 0) Qdn_before = rev_group_start(C, V, tf);
        const int Qdn = __shfl_down_sync(kAll, V.Q, 1);
        const float2 bv = C.bbr[(j0 + 15) & (kRW - 1)];
        if ((C.lane < C.nv) && j0 == C.L2 - 1) {  // this lane starts: adopt the neighbour's frame
            V.Q = C.lastLane ? __float_as_int(bv.y) : Qdn;
            V.d0 = p2(Qdn_before - V.Q);
            V.d1 = 1.f;
            V.br = V.pbp = 0.f;
            rev_k_factors(C, V, m16 + 15 - (u & ~3));
        }
        const float adz = (C.lane0 ? C.rr[tf & (kRW - 1)] : zb[(15 - u) * 32]);
        const float ad = (j0 >= 1) ? adz : 0.f;
        const float rc = V.recv * (((u & 3) == 0) ? V.d0 : V.d1);
        const float inc = C.lastLane ? from_below(bv, V.Q) : rc;
        const int ci = j0 & (kRW - 1);
        const float P = ex2f(C.ring[ci] * C.c);
        float b = fmaf(C.G, V.br, inc) + V.fsq;
        const float mu = P * fmaf(b * ad, kdiag(C, V, u & 3), b * V.k2);
        b = act ? b : 0.f;
        const float pb = P * b;
        float msg = fmaf(C.G, b, V.pbp);
        msg = act ? msg : 0.f;
        if (act) {
            C.ring[ci] = mu;
            if (C.push0) C.bbout[j0 + 15] = make_float2(msg, __int_as_float(V.Q));
            V.mn = fminf(V.mn, b);
            V.mx = fmaxf(V.mx, b);
        }
        V.recv = __shfl_down_sync(kAll, msg, 1);
        V.br = b;
        V.pbp = act ? pb : 0.f;
        // lane l+1's frame for the message just received (it may have started this step)
        V.Qdn_last = __shfl_down_sync(kAll, V.Q, 1);
    }
}

// ==========================================================================
// kernel
// ==========================================================================
// Progress words: warp w publishes (ordinal << 16 | stages done) for its
// current row-block (ordinal = r forward, nRB-1-r reverse), and
// (ordinal << 16 | kStageMask) when the row-block is complete.
__global__ void __launch_bounds__(kNW * 32) lin_fast_kernel(SwArgs p) {
    extern __shared__ __align__(16) unsigned char smem_raw[];
    WarpSmem& W = reinterpret_cast<WarpSmem*>(smem_raw)[threadIdx.x >> 5];
    __shared__ int progF[kNW], progR[kNW];
    __shared__ __align__(16) float red[4 * 32];
    __shared__ int sh_Sint, sh_err;
    __shared__ float sh_Sfrac;

    const int b = blockIdx.x;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
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
        for (int i = warp; i < L1m; i += kNW) {
            float* row = out + (size_t)i * L2m;
            for (int j = (i < L1 ? L2 : 0) + lane; j < L2m; j += 32) row[j] = 0.f;
        }
    }
    if (L1 == 0 || L2 == 0) {  // S = log(1) = 0 (alpha[0,0] only)
        if (threadIdx.x == 0) {
            if (p.value) p.value[b] = 0.f;
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

    float wmn = 1.f, wmx = 1.f;  // range of every z and b this lane produced

    // ============================== forward ==============================
    FwdVars V;
    V.acc = 0.f;
    V.R = 0;
    for (int r = warp; r < nRB; r += kNW) {
        const int nv = min(32, L1 - 32 * r);
        const int nst = (L2 + nv - 1 + kCW - 1) / kCW;
        const float* srow = S + (size_t)(32 * r) * L2m;
        const float2* brow = LY.bnd + (size_t)(r - 1) * L2m;
        const bool hasB = r > 0, hasD = r + 1 < nRB;
        float* const zblk = LY.zpl + (size_t)r * zst;
        FwdCtx C;
        C.ring = W.ringS + lane * kRW;
        C.bndring = W.bnd;
        C.zrow = zblk + 2 * 32 + lane;
        C.erow = LY.efr + (size_t)r * est + lane;
        C.rab = LY.rab + (size_t)r * rb_len(L2m);
        C.bout = LY.bnd + (size_t)r * L2m;
        C.c = c;
        C.G = G;
        C.lane = lane;
        C.nv = nv;
        C.L2 = L2;
        C.lane0 = lane == 0;
        C.st31 = (lane == 31) && hasD;
        const int* upflag = &progF[(warp + kNW - 1) % kNW];
        const int upbase = (r - 1) << 16;
        const Tile tS = make_tile(srow, L2m, W.ringS, nv, lane);

        __syncwarp();
        if (!hasB) {  // no row above: its values are zero
            W.bnd[lane] = make_float2(0.f, __int_as_float(0));
            W.bnd[lane + 32] = make_float2(0.f, __int_as_float(0));
        }
        // rows 0, 1 of the z plane (steps -2, -1) and the row above at column -1 are zero
        zblk[lane] = 0.f;
        zblk[32 + lane] = 0.f;
        if (lane == 0) C.rab[0] = 0.f;
        int ld = 0;
        for (; ld < 2 && ld < nch; ++ld) {
            if (hasB) wait_flag(upflag, upbase + min(ld + 3, kStageMask), &sh_err);
            tile_load<4>(tS, ld, L2);
            if (hasB) load_row_chunk8(W.bnd, brow, L2, ld, lane);
            cp_async_commit();
        }
        V.E = 0;
        if (hasB) {
            cp_async_wait0();
            __syncwarp();
            V.E = __float_as_int(W.bnd[0].y);
        }
        V.Eup_last = V.E;
        V.zl = V.zu = V.zd = 0.f;
        V.d0 = V.d1 = 1.f;
        V.mn = V.mx = 1.f;
        fwd_frame_factors(V);

        for (int k = 0; k < nst; ++k) {
            if (k > 0 && ld <= k + 1 && ld < nch) {
                __syncwarp();
                if (hasB) wait_flag(upflag, upbase + min(ld + 3, kStageMask), &sh_err);
                tile_load<4>(tS, ld, L2);
                if (hasB) load_row_chunk8(W.bnd, brow, L2, ld, lane);
                ++ld;
            }
            cp_async_commit();
            cp_async_wait1();
            __syncwarp();
            if ((nv == 32) && (kCW * k >= 31) && (kCW * k + kCW - 1 <= L2 - 1))
                fwd_stage_full(C, V, k);
            else
                fwd_stage_part(C, V, k);
            if (C.st31) st_release(&progF[warp], (r << 16) | min(k + 1, kStageMask - 1));
        }
        cp_async_wait0();
        __syncwarp();
        if (lane == 31) st_release(&progF[warp], (r << 16) | kStageMask);
        wmn = fminf(wmn, V.mn);
        wmx = fmaxf(wmx, V.mx);
    }

    // ---- S = log2(1 + sum_lanes acc 2^R), kept as integer + fraction
    {
        const bool has = V.acc > 0.f;
        const int Rm = (int)block_max(has ? (float)max(V.R, 0) : 0.f, red);
        float part = has ? V.acc * exp2i(V.R - Rm) : 0.f;
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
    const int nstR = P / kCW + 2;  // lane 0 reaches column 0 at step P + 31
    for (int q = warp; q < nRB; q += kNW) {
        const int r = nRB - 1 - q;
        const int nv = min(32, L1 - 32 * r);
        const float* srow = S + (size_t)(32 * r) * L2m;
        const bool hasBelow = r + 1 < nRB;
        const float* zblk = LY.zpl + (size_t)r * zst;
        const int* eblk = LY.efr + (size_t)r * est;
        const float* rblk = LY.rab + (size_t)r * rb_len(L2m);
        const float2* bbrow = LY.bbv + (size_t)(r + 1) * rb_len(L2m);
        RevCtx C;
        C.ring = W.ringS + lane * kRW;
        C.zr = &W.zr[0][0];
        C.er = W.er;
        C.rr = W.rr;
        C.bbr = W.bbr;
        C.bbout = LY.bbv + (size_t)r * rb_len(L2m);
        C.c = c;
        C.G = G;
        C.cS = ex2f(-sh_Sfrac);
        C.Sint = sh_Sint;
        C.lane = lane;
        C.nv = nv;
        C.L2 = L2;
        C.P = P;
        C.ecol = lane > 0 ? lane - 1 : 0;
        C.lane0 = lane == 0;
        C.lastLane = lane == nv - 1;
        C.push0 = (lane == 0) && (r > 0);
        const int* dnflag = &progR[(warp + kNW - 1) % kNW];
        const int dnbase = (q - 1) << 16;
        const Tile tS = make_tile(srow, L2m, W.ringS, nv, lane);
        const Tile tM = make_tile(out ? out + (size_t)(32 * r) * L2m : srow, L2m, W.ringS, nv, lane);

        // staging for stage kk (M = P/16 + 1 - kk, anti-diagonals 16M .. 16M+15)
        auto stage_z = [&](int kk) {  // z plane rows 16M .. 16M+15 (lane l-1's diagonal inputs)
            const int M = P / kCW + 1 - kk;
            if (kk >= nstR || M < 0) return;
            const float* src = zblk + (size_t)(16 * M) * 32;
            float* dst = &W.zr[M & 1][0];
            for (int i = lane; i < 16 * 32 / 4; i += 32) cp_async16(dst + 4 * i, src + 4 * i, 16);
        };
        auto stage_e = [&](int kk) {  // forward frames of groups 4M .. 4M+3
            const int M = P / kCW + 1 - kk;
            if (kk >= nstR || M < 0) return;
            const int g0 = 4 * M;
            cp_async16(W.er + (g0 & 15) * 32 + 4 * lane, eblk + (size_t)g0 * 32 + 4 * lane, 16);
        };
        auto stage_r = [&](int kk) {  // row above (lane 0) and pushes from below (bottom lane)
            const int M = P / kCW + 1 - kk;
            if (kk >= nstR || M < 0) return;
            if (lane < 4) cp_async16(W.rr + ((16 * M + 4 * lane) & (kRW - 1)), rblk + 16 * M + 4 * lane, 16);
            if (hasBelow && M >= 1) {
                // bbv indices 16M-16 .. 16M-1 = columns 16M-31 .. 16M-16, pushed by row-block
                // r+1's lane 0 at its steps P + 31 - column
                wait_flag(dnflag, dnbase + min((P + 31 - (16 * M - 31)) / kCW + 1, kStageMask), &sh_err);
                if (lane < 8)
                    cp_async16(W.bbr + ((16 * M - 16 + 2 * lane) & (kRW - 1)), bbrow + 16 * M - 16 + 2 * lane, 16);
            }
        };

        __syncwarp();
        if (!hasBelow) {  // no row-block below: its pushes are zero
            W.bbr[lane] = make_float2(0.f, __int_as_float(0));
            W.bbr[lane + 32] = make_float2(0.f, __int_as_float(0));
        }
        {   // stage 0 reads score chunks M0-2 .. M0 (M0 = P/16 + 1)
            const int M0 = P / kCW + 1;
            for (int ch = M0; ch >= M0 - 2; --ch)
                if (ch >= 0 && ch < nch) tile_load<4>(tS, ch, L2);
        }
        stage_z(0);
        stage_e(0);
        stage_e(1);
        stage_r(0);
        cp_async_commit();

        RevVars RV;
        RV.recv = RV.pbp = RV.br = 0.f;
        RV.mn = RV.mx = 1.f;
        bool started = false;
        for (int k = 0; k < nstR; ++k) {
            const int M = P / kCW + 1 - k;
            __syncwarp();
            if (out && M + 1 < nch && M + 1 >= 0) tile_store(tM, M + 1, L2);  // no lane touches it any more
            if (M - 3 >= 0 && M - 3 < nch) tile_load<4>(tS, M - 3, L2);       // for stage k + 1
            stage_z(k + 1);
            stage_e(k + 2);
            stage_r(k + 1);
            cp_async_commit();
            cp_async_wait1();
            __syncwarp();
            if (!started) {  // lanes adopt a neighbour's frame when they start
                RV.Q = 0;
                RV.Qdn_last = 0;
                RV.d0 = RV.d1 = 1.f;
                rev_k_factors(C, RV, P + 31);
                started = true;
            }
            if ((nv == 32) && (kCW * k >= P + 32 - L2) && (kCW * k + kCW - 1 <= P - 1))
                rev_stage_full(C, RV, k);
            else
                rev_stage_part(C, RV, k);
            if (C.push0) st_release(&progR[warp], (q << 16) | min(k + 1, kStageMask - 1));
        }
        __syncwarp();
        if (out && nch > 0) tile_store(tM, 0, L2);  // the last stage had M = 0
        cp_async_wait0();
        __syncwarp();
        if (lane == 0) st_release(&progR[warp], (q << 16) | kStageMask);
        wmn = fminf(wmn, RV.mn);
        wmx = fmaxf(wmx, RV.mx);
    }

    // a value outside the frame window, or a dependency wait that gave up: the
    // caller recomputes this problem with the log-domain kernel
    const bool outside = !(wmn >= kWinLo && wmx <= kWinHi);
    const int redo = __syncthreads_or(outside ? 1 : 0) || sh_err;
    if (threadIdx.x == 0 && p.redo) p.redo[b] = redo;
}

}  // namespace lin

// ------------------------------------------------------------------ host side
size_t lin_fast_workspace_bytes(int B, int L1, int L2) {
    if (L1 > 32 * lin::kMaxRB || L2 % 4 != 0) return 0;
    return lin::per_problem_bytes(L1, L2) * (size_t)B;
}

int launch_lin_fast(const SwArgs& a, size_t ws_bytes, cudaStream_t st) {
    if (a.mode != MODE_MARG || !a.redo || a.grad_gap || a.grad_T) return -1;
    if (engine_forced_plane()) return -1;
    if (a.L2 % 4 != 0 || a.L1 > 32 * lin::kMaxRB || a.L1 == 0 || a.L2 == 0) return -1;
    if ((((uintptr_t)a.scores) & 15) != 0 || (a.out && (((uintptr_t)a.out) & 15) != 0)) return -1;
    if ((((uintptr_t)a.ws) & 255) != 0) return -1;
    const size_t need = lin::per_problem_bytes(a.L1, a.L2) * (size_t)a.B;
    if (ws_bytes < need || !a.ws) return -1;
    const size_t smem = sizeof(lin::WarpSmem) * lin::kNW;
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return (int)e;
    static bool attr_set[64] = {false};
    if (dev < 64 && !attr_set[dev]) {
        e = cudaFuncSetAttribute(lin::lin_fast_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return (int)e;
        attr_set[dev] = true;
    }
    lin::lin_fast_kernel<<<a.B, lin::kNW * 32, smem, st>>>(a);
    return (int)cudaGetLastError();
}

}  // namespace d2pb
