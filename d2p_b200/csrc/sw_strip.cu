// sw_strip.cu -- linear-gap soft Smith-Waterman value + marginals for problems of
// up to 512 rows: each lane holds a strip of 4 consecutive rows, a warp 128
// rows; a CTA (one problem) runs a forward set of warps sweeping the columns
// left to right and, at the same time, a reverse set sweeping them right to
// left.
//
// Recurrences (linear domain, as in sw_linear.cu; src/sw/kernels_cpu.cpp:70-279
// restated): with P = 2^(s c), G = 2^(gap c), c = log2(e) / T,
//   Z_ij = P_ij (Z_{i-1,j-1} + 1) + G (Z_{i-1,j} + Z_{i,j-1}),
//   B_ij = 1 + P_{i+1,j+1} B_{i+1,j+1} + G (B_{i+1,j} + B_{i,j+1}),
//   marginal_ij = B_ij w_ij / Z_total,  w_ij = P_ij (Z_{i-1,j-1} + 1).
// B (the outside weights) does not depend on Z, and the partition splits at
// any column cut m | m+1: counting each alignment path by its last cell left
// of the cut, by its first cell right of it, or by the move that crosses it,
//   Z_total = 1 + sum_{j<=m} Z_ij + sum_{j>m} P_ij B_ij
//               + sum_i Z_{i,m} (G B_{i,m+1} + P_{i+1,m+1} B_{i+1,m+1}).
// So the two sweeps run at once: phase 1 takes the forward over the left half
// (keeping w there) and the reverse over the right half (keeping B there);
// at the cut they assemble Z_total; phase 2 takes each sweep on through the
// other half, where it meets the values the other kept and writes the
// marginals.  Each problem's columns are swept once per direction, in half the
// time of a forward pass followed by a reverse pass.
//
// Column sweep.  Within column j, Z_ij = a_i + G Z_{i-1,j} with a_i = w_ij +
// G Z_{i,j-1} known from column j-1: a first-order linear recurrence with a
// constant coefficient.  A lane forms the prefix of its 4 rows in registers,
// the 32 lanes combine their last rows with a 5-level shuffle scan
// (multipliers G^(4 2^k), each lane in its own frame), the row above the warp
// enters every lane through one more multiply-add, and each row then adds
// G^(r+1) times the row above its strip.  The reverse is the same sweep
// mirrored (right to left, bottom to top).  Cells outside the problem (rows
// past its length, columns past its width) are forced to zero by selects, so
// every column runs the same code.
//
// Warps.  Forward warp w (rows 128w .. 128w+127) needs forward warp w-1's last
// row, column by column; reverse warp w needs reverse warp w+1's first row.  A
// warp publishes them one block of 8 columns at a time into a ring in shared
// memory (a release of its progress word), so the warps of a set run one block
// apart.  Only consumers wait for producers (and a producer for ring space 16
// blocks back); every wait is bounded.
//
// Range.  Each lane keeps a power-of-two frame for its rows, decided at the
// start of every block from the largest of its values (forward Z, reverse B).
// Frames are integer-valued floats; conversions between lanes and warps are
// exact powers of two folded into the multipliers.  A frame step outside
// 2^+-60, a wait that gave up, or a partition that is not finite flags the
// problem; the caller recomputes flagged problems with the plane engine.
//
// Memory.  Scores arrive by TMA in tiles of 8 columns x 128 rows per warp,
// laid out [row in strip][lane][8 columns] (a view of the score plane as
// columns x strips x rows in strip) with the 32-byte swizzle, so that the 32
// lanes read their rows' 4 columns with conflict-free 16-byte loads.  The
// values kept across the cut (w left of it, B right of it) go to a plane in
// the workspace, each lane's 4 rows of a column as one coalesced 16-byte
// store, with each lane's frame per block; phase 2 reads them back one group
// of 4 columns ahead of use.  The marginals leave through a staging tile of
// the score layout, stored by TMA.  HBM traffic per cell: scores read twice
// (8 B), the kept plane written and read (8 B), marginals written (4 B).
//
// Occupancy.  A block is worked in two groups of 4 columns, so that a lane
// holds P for 4 columns and the kept values for 8 (this group's and the
// next's); with the handoff values read and written in shared memory column
// by column this fits 128 registers, two CTAs (two problems) per SM.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <stddef.h>
#include <stdint.h>

#include "sw_common.cuh"
#include "sw_internal.h"
#include "sw_lindomain.cuh"
#include "sw_ring.cuh"

namespace d2pb {
namespace strip {
using ring::kAll;
using ring::kSpinLimit;

constexpr int kR = 4;                  // rows per lane
constexpr int kWR = 32 * kR;           // rows per warp
constexpr int kMaxW = 4;               // warps per direction: problems of at most 512 rows
constexpr int kBC = 8;                 // columns per block = per TMA tile
constexpr int kQC = 4;                 // columns per group (half a block)
constexpr int kNS = 2;                 // score tiles resident per warp
constexpr int kTileFloats = kBC * kWR;
constexpr int kTileBytes = kTileFloats * 4;
constexpr int kHB = 16;                // blocks in a handoff ring

struct alignas(256) WarpSmem {         // 256-byte aligned: TMA tiles and the 32-byte swizzle pattern
    float sc[kNS][kTileFloats];        // score tiles, [r][lane][8] with the 32-byte swizzle; in phase 2
                                       // the marginals replace the scores they came from, and leave by TMA
    float4 kr[2][kQC * 32];            // phase 2: kept values of two groups of 4 columns, [column][lane]
    unsigned long long bar[kNS];       // TMA arrival barrier of each score slot
    unsigned long long kbar[2];        // bulk-copy arrival barrier of each kept slot
};

struct Hand {                          // handoffs between the warps of a set, by block (ring of kHB)
    float fv[kHB][kBC];                // forward: Z of the warp's last row, per column
    float fe[kHB];                     //   and the frame of its lane 31
    float rv[kHB][kBC];                // reverse: B of the warp's first row, per column
    float rp[kHB][kBC];                //   P B of that row
    float re[kHB];                     //   and the frame of its lane 0
};

struct Meet {                          // the reverse's values at the cut, per row block
    float B[kWR], PB[kWR];
    float Q[32];
    float b0;                          // NW, row block 0: B of the boundary row 0 (lane 0's frame)
};

// The warps' tiles come last, so that a CTA of W warps per direction
// allocates 2W of them.
// A CTA has Wc slots, each a forward and a reverse warp on one row block of a
// problem; a problem's row blocks take consecutive slots o .. o + Wp - 1.
struct CtaSmem {
    Hand h[kMaxW];                     // by slot
    Meet meet[kMaxW];
    int progF[kMaxW], progR[kMaxW];    // blocks published (forward / reverse ordinal)
    int consF[kMaxW], consR[kMaxW];    // blocks read by the slot's consumer
    float pbase[3 * kMaxW];            // partition partials: base (log2) ...
    double psum[3 * kMaxW];            //   ... and sum: forward, reverse, crossing per slot
    unsigned long long pbar[kMaxW];    // by a problem's first slot: its barrier at the column cut
    int err[kMaxW];                    //   and its flags
    int slot[kMaxW];                   // problem * 4 + row block of each slot (-1: none)
    int slot_ok[kMaxW];                // the slot's problem passed the table check
    WarpSmem w[2 * kMaxW];             // by warp: forward warps 0..Wc-1, reverse warps Wc..2Wc-1
};
__host__ __device__ constexpr size_t smem_bytes_for(int W) {
    return offsetof(CtaSmem, w) + 2 * (size_t)W * sizeof(WarpSmem) + 256;   // + alignment slack
}

// the plane kept across the cut: [W][nT][8 columns][32 lanes] float4 (a
// lane's 4 rows), and each lane's frame per block [W][nT][32]
__host__ __device__ inline size_t plane_bytes_of(int W, int L2m) {
    const size_t nT = (size_t)(L2m + kBC - 1) / kBC;
    return ring::align_up((size_t)W * nT * kBC * 32 * sizeof(float4), 256);
}
__host__ __device__ inline size_t frames_bytes_of(int W, int L2m) {
    const size_t nT = (size_t)(L2m + kBC - 1) / kBC;
    return ring::align_up((size_t)W * nT * 32 * sizeof(float), 256);
}
__host__ __device__ inline int warps_for(int L1m) { return (L1m + kWR - 1) / kWR; }
__host__ __device__ inline size_t per_problem_bytes(int L1m, int L2m) {
    const int W = warps_for(L1m);
    return plane_bytes_of(W, L2m) + frames_bytes_of(W, L2m);
}

// float offset of the 16-byte chunk h (columns 4h..4h+3) of row r of lane l in
// a tile: TMA's 32-byte swizzle exchanges the two chunks of a 32-byte row when
// bit 2 of the row index (r * 32 + l) is set
__device__ __forceinline__ int sw_off(int r, int l, int h) { return ((r * 32 + l) << 3) + ((h ^ ((l >> 2) & 1)) << 2); }

__device__ __forceinline__ unsigned smem_u32(const void* p) { return (unsigned)__cvta_generic_to_shared(p); }

__device__ __forceinline__ void tma_load_tile(const CUtensorMap* tm, float* dst, unsigned long long* bar, int x, int y,
                                              int b) {
    const unsigned d = smem_u32(dst), m = smem_u32(bar);
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(m), "r"(kTileBytes) : "memory");
    asm volatile(
        "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4, "
        "%5}], [%6];" ::"r"(d),
        "l"((unsigned long long)tm), "r"(x), "r"(y), "r"(0), "r"(b), "r"(m)
        : "memory");
}

// Marginal tiles are written once and not read again in the launch: evict
// them from L2 first, so that the scores and kept values read a second time
// stay.
__device__ __forceinline__ void tma_store_tile(const CUtensorMap* tm, const float* src, int x, int y, int b) {
    unsigned long long pol;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
    asm volatile(
        "cp.async.bulk.tensor.4d.global.shared::cta.tile.bulk_group.L2::cache_hint [%0, {%1, %2, %3, %4}], [%5], "
        "%6;" ::"l"((unsigned long long)tm),
        "r"(x), "r"(y), "r"(0), "r"(b), "r"(smem_u32(src)), "l"(pol)
        : "memory");
    asm volatile("cp.async.bulk.commit_group;" ::: "memory");
}
// n bytes (a multiple of 16) from global src to shared dst (both 16-byte aligned), arriving on bar
__device__ __forceinline__ void bulk_load(void* dst, const void* src, unsigned n, unsigned long long* bar) {
    const unsigned d = smem_u32(dst), m = smem_u32(bar);
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(m), "r"(n) : "memory");
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(d),
                 "l"(src), "r"(n), "r"(m)
                 : "memory");
}
__device__ __forceinline__ void tma_store_wait_read0() { asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory"); }
__device__ __forceinline__ void tma_store_wait0() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }
__device__ __forceinline__ void fence_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

// bounded wait for phase `parity` of a TMA barrier; false when it gave up
__device__ __forceinline__ bool bar_wait(unsigned long long* bar, unsigned parity) {
    const unsigned m = smem_u32(bar);
    for (int it = 0; it < kSpinLimit; ++it) {
        unsigned done;
        asm volatile(
            "{\n .reg .pred p;\n mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
            : "=r"(done)
            : "r"(m), "r"(parity)
            : "memory");
        if (done) return true;
        __nanosleep(32);
    }
    return false;
}

struct Args {
    const int* lengths;
    int B, L1, L2;      // the planes' layout (rows of whole 16-byte units)
    int L1v, L2v;       // the problems' padded shape inside it (lengths are clamped to it)
    float gap, temp;
    const float* gap_dev;
    const float* temp_dev;
    float* value;
    float* ws;
    int* redo;
    const int* order;
    const int* pack;    // [B][kMaxW] or null: problem * 4 + row block of each slot of each CTA (-1: none)
    size_t ws_stride;   // bytes of workspace per problem
};

// Per-problem constants, and this lane's place in it.
struct Prob {
    float c, gl, G, G2;
    int L1, L2, nv;     // nv: rows of this lane inside the problem (0..4)
    int rend;           // NW: the end row's place in this lane's strip (0..3), -1 when another lane holds it
};

__device__ __forceinline__ void prob_init(const Args& A, int b, int w, int lane, Prob& p) {
    const float gapn = A.gap_dev ? __ldg(A.gap_dev) : A.gap;
    const float T = A.temp_dev ? __ldg(A.temp_dev) : A.temp;
    p.c = kLog2e / T;
    p.gl = gapn * p.c;
    p.G = ex2f(p.gl);
    p.G2 = ex2f(2.f * p.gl);
    p.L1 = A.lengths ? min(max(A.lengths[2 * b], 0), A.L1v) : A.L1v;
    p.L2 = A.lengths ? min(max(A.lengths[2 * b + 1], 0), A.L2v) : A.L2v;
    p.nv = min(max(p.L1 - kWR * w - kR * lane, 0), kR);
    const int er = p.L1 - 1 - kWR * w - kR * lane;   // the end row (0-based) relative to this strip
    p.rend = (er >= 0 && er < kR) ? er : -1;
}

// Constants of one lane for one block (forward): from its frame E, its upper
// neighbours' frames, and the frame Ein of the row above the warp.
struct FwdK {
    float fs;           // 2^-E: the "+1" start term in this frame
    float m1;           // 2^(E_{l-1} - E): the row above the strip into this frame (0 when there is none)
    float Gm[kR];       // G^(r+1) m1
    float M[5];         // G^(4 2^k) 2^(E_{l-2^k} - E) (0 where l < 2^k)
    float Min;          // G^(4 (l+1)) 2^(Ein - E): the row above the warp into this lane's last row
};

__device__ __forceinline__ void fwd_consts(const Prob& p, float E, float Ein, bool above, int lane, FwdK& k) {
    float e1 = __shfl_up_sync(kAll, E, 1);
    const float e2 = __shfl_up_sync(kAll, E, 2), e4 = __shfl_up_sync(kAll, E, 4);
    const float e8 = __shfl_up_sync(kAll, E, 8), e16 = __shfl_up_sync(kAll, E, 16);
    if (lane == 0) e1 = Ein;
    const bool has1 = lane >= 1 || above;
    k.fs = ex2f(-E);
    const float d1 = e1 - E;
    k.m1 = has1 ? ex2f(d1) : 0.f;
#pragma unroll
    for (int r = 0; r < kR; ++r) k.Gm[r] = has1 ? ex2f(fmaf((float)(r + 1), p.gl, d1)) : 0.f;
    k.M[0] = lane >= 1 ? ex2f(fmaf(4.f, p.gl, d1)) : 0.f;
    k.M[1] = lane >= 2 ? ex2f(fmaf(8.f, p.gl, e2 - E)) : 0.f;
    k.M[2] = lane >= 4 ? ex2f(fmaf(16.f, p.gl, e4 - E)) : 0.f;
    k.M[3] = lane >= 8 ? ex2f(fmaf(32.f, p.gl, e8 - E)) : 0.f;
    k.M[4] = lane >= 16 ? ex2f(fmaf(64.f, p.gl, e16 - E)) : 0.f;
    k.Min = above ? ex2f(fmaf((float)(kR * (lane + 1)), p.gl, Ein - E)) : 0.f;
}

// The reverse's: lower neighbours and the row below the warp (frame Qin) feed rows above.
struct RevK {
    float fsq;          // 2^-Q: the "+1" term in this frame
    float m1;           // 2^(Q_{l+1} - Q) (0 when there is nothing below)
    float Gm[kR];       // G^(4-r) m1
    float M[5];         // G^(4 2^k) 2^(Q_{l+2^k} - Q) (0 where l + 2^k > 31)
    float Min;          // G^(4 (32-l)) 2^(Qin - Q): the row below the warp into this lane's first row
};

// lv: the last lane with rows of the problem (31 when the warp is full).  Lanes
// below it hold zeros in frame 0; NW frames can lie far below 0, and a
// conversion factor from such a lane would overflow (inf x 0), so NW passes lv
// and takes nothing from them.
__device__ __forceinline__ void rev_consts(const Prob& p, float Q, float Qin, bool below, int lane, RevK& k,
                                           int lv = 31) {
    float q1 = __shfl_down_sync(kAll, Q, 1);
    const float q2 = __shfl_down_sync(kAll, Q, 2), q4 = __shfl_down_sync(kAll, Q, 4);
    const float q8 = __shfl_down_sync(kAll, Q, 8), q16 = __shfl_down_sync(kAll, Q, 16);
    if (lane == 31) q1 = Qin;
    const bool has1 = lane + 1 <= lv || (lane == 31 && below);
    k.fsq = ex2f(-Q);
    const float d1 = q1 - Q;
    k.m1 = has1 ? ex2f(d1) : 0.f;
#pragma unroll
    for (int r = 0; r < kR; ++r) k.Gm[r] = has1 ? ex2f(fmaf((float)(kR - r), p.gl, d1)) : 0.f;
    k.M[0] = lane + 1 <= lv ? ex2f(fmaf(4.f, p.gl, d1)) : 0.f;
    k.M[1] = lane + 2 <= lv ? ex2f(fmaf(8.f, p.gl, q2 - Q)) : 0.f;
    k.M[2] = lane + 4 <= lv ? ex2f(fmaf(16.f, p.gl, q4 - Q)) : 0.f;
    k.M[3] = lane + 8 <= lv ? ex2f(fmaf(32.f, p.gl, q8 - Q)) : 0.f;
    k.M[4] = lane + 16 <= lv ? ex2f(fmaf(64.f, p.gl, q16 - Q)) : 0.f;
    k.Min = below ? ex2f(fmaf((float)(kR * (32 - lane)), p.gl, Qin - Q)) : 0.f;
}

// One forward column: z (this lane's rows, column j-1 -> j), dc (the row
// above the strip at column j-1 -> j, in this lane's frame), P of column j,
// yin: the row above the warp at column j (frame Ein; 0 when there is none),
// nvc: rows of this lane inside the problem at column j (MASK only).  Returns
// the inclusive scan value (lane 31: the warp's last row); adds the column's Z
// to gs; w receives the diagonal terms.  MASK: cells outside the problem are 0
// (Z and w; w is selected, not multiplied, since the row above a lane past the
// problem may reach it as inf in that lane's frame).
template <bool MASK>
__device__ __forceinline__ float fwd_column(const Prob& p, const FwdK& k, float (&z)[kR], float& dc,
                                            const float (&P)[kR], float yin, int nvc, int lane, float (&w)[kR],
                                            float& gs) {
    float a[kR];
#pragma unroll
    for (int r = 0; r < kR; ++r) {
        const float d = r == 0 ? dc : z[r - 1];
        const float wr = P[r] * (d + k.fs);
        w[r] = (!MASK || r < nvc) ? wr : 0.f;
        a[r] = fmaf(p.G, z[r], wr);
    }
    // prefix of the strip: a[r] <- sum_{q <= r} G^(r-q) a[q]
#pragma unroll
    for (int r = kR - 1; r >= 1; --r) a[r] = fmaf(p.G, a[r - 1], a[r]);
#pragma unroll
    for (int r = kR - 1; r >= 2; --r) a[r] = fmaf(p.G2, a[r - 2], a[r]);
    // the strips' last rows, scanned over the lanes, then the row above the warp
    float y = a[kR - 1];
    y = fmaf(k.M[0], __shfl_up_sync(kAll, y, 1), y);
    y = fmaf(k.M[1], __shfl_up_sync(kAll, y, 2), y);
    y = fmaf(k.M[2], __shfl_up_sync(kAll, y, 4), y);
    y = fmaf(k.M[3], __shfl_up_sync(kAll, y, 8), y);
    y = fmaf(k.M[4], __shfl_up_sync(kAll, y, 16), y);
    y = fmaf(k.Min, yin, y);
    float yp = __shfl_up_sync(kAll, y, 1);   // the row above the strip (lane l-1's frame)
    if (lane == 0) yp = yin;
    float s = 0.f;
#pragma unroll
    for (int r = 0; r < kR; ++r) {
        float v = fmaf(k.Gm[r], yp, a[r]);
        if (MASK) v = r < nvc ? v : 0.f;
        z[r] = v;
        s += v;
    }
    gs += s;
    dc = yp * k.m1;
    return y;
}

// One reverse column: B, PB (this lane's rows at column j+1 -> j; PB = P B),
// P and w of column j; bin: B of the row below the warp at column j (frame
// Qin), pbn: P B of that row at column j+1 (lane 31, already in its frame).  w
// is replaced by the marginals (before the frame factor).  MASK: cells outside
// the problem are 0 (B, and so P B, and the marginals).
template <bool MASK, bool NW>
__device__ __forceinline__ void rev_column(const Prob& p, const RevK& k, float (&Bv)[kR], float (&PB)[kR],
                                           const float (&P)[kR], float (&w)[kR], float bin, float pbn, int nvc,
                                           int lane, int onerow, float k1 = 1.f, float k2 = 1.f) {
    float pbd = __shfl_down_sync(kAll, PB[0], 1) * k.m1;   // lane l+1's top row, column j+1
    if (lane == 31) pbd = pbn;
    float cc[kR];
#pragma unroll
    for (int r = 0; r < kR; ++r) {
        // SW: a path may end at any cell; NW: only at the end cell (onerow of this lane)
        const float one = NW ? (r == onerow ? k.fsq : 0.f) : ((!MASK || r < nvc) ? k.fsq : 0.f);
        cc[r] = fmaf(p.G, Bv[r], one + (r + 1 < kR ? PB[r + 1] : pbd));
    }
    // suffix of the strip: cc[r] <- sum_{q >= r} G^(q-r) cc[q]
#pragma unroll
    for (int r = 0; r < kR - 1; ++r) cc[r] = fmaf(p.G, cc[r + 1], cc[r]);
#pragma unroll
    for (int r = 0; r < kR - 2; ++r) cc[r] = fmaf(p.G2, cc[r + 2], cc[r]);
    float y = cc[0];
    y = fmaf(k.M[0], __shfl_down_sync(kAll, y, 1), y);
    y = fmaf(k.M[1], __shfl_down_sync(kAll, y, 2), y);
    y = fmaf(k.M[2], __shfl_down_sync(kAll, y, 4), y);
    y = fmaf(k.M[3], __shfl_down_sync(kAll, y, 8), y);
    y = fmaf(k.M[4], __shfl_down_sync(kAll, y, 16), y);
    y = fmaf(k.Min, bin, y);
    float yn = __shfl_down_sync(kAll, y, 1);   // the row below the strip (lane l+1's frame)
    if (lane == 31) yn = bin;
#pragma unroll
    for (int r = 0; r < kR; ++r) {
        const float b = fmaf(k.Gm[r], yn, cc[r]);
        Bv[r] = b;
        PB[r] = P[r] * b;
        const float m = NW ? (b * k1) * (w[r] * k2) : b * w[r];
        w[r] = (!MASK || r < nvc) ? m : 0.f;
    }
}

// NW: log2 C(n + 4, 4), the growth of the number of paths over the first four
// columns next to an edge n rows away (the frames at the grid's edges start
// half a block ahead, so that the first block's combinatorial growth stays
// inside the frame window)
__device__ __forceinline__ float nw_lead(int n) {
    const float f = (float)(n + 1) * (float)(n + 2) * (float)(n + 3) * (float)(n + 4) * (1.f / 24.f);
    return log2f(f);
}
// NW frame steps may reach this (the edges' combinatorial growth); marginals
// are then formed as (b 2^xa) (w 2^(x - xa)) so that b w cannot overflow
constexpr int kJMaxNW = 90;
__device__ __forceinline__ void split_scale(float x, float& k1, float& k2) {
    const float xa = fminf(fmaxf(floorf(0.5f * x), -126.f), 126.f);
    k1 = ex2f(xa);
    k2 = ex2f(fminf(fmaxf(x - xa, -126.f), 126.f));
}

// Largest value of the strip -> the frame step J (new frame E + J) and 2^-J.
__device__ __forceinline__ float frame_step(const float (&v)[kR], float& inv) {
    float m = fmaxf(fmaxf(v[0], v[1]), fmaxf(v[2], v[3]));
    const int eb = ld::efield(m);
    inv = __int_as_float(0x7f000000 - eb);
    return ld::efield_j(eb);
}

// P = 2^(s c) of group q (columns 4q..4q+3) of a block starting at column j0,
// from the score tile (MASK: 0 outside the problem)
template <bool MASK>
__device__ __forceinline__ void group_P(const Prob& p, const float* tile, int lane, int q, int j0,
                                        float (&P)[kQC][kR]) {
#pragma unroll
    for (int r = 0; r < kR; ++r) {
        const float4 s = *reinterpret_cast<const float4*>(tile + sw_off(r, lane, q));
        if (MASK) {
            const bool ok = r < p.nv;
            P[0][r] = ok && j0 < p.L2 ? ex2f(s.x * p.c) : 0.f;
            P[1][r] = ok && j0 + 1 < p.L2 ? ex2f(s.y * p.c) : 0.f;
            P[2][r] = ok && j0 + 2 < p.L2 ? ex2f(s.z * p.c) : 0.f;
            P[3][r] = ok && j0 + 3 < p.L2 ? ex2f(s.w * p.c) : 0.f;
        } else {
            P[0][r] = ex2f(s.x * p.c);
            P[1][r] = ex2f(s.y * p.c);
            P[2][r] = ex2f(s.z * p.c);
            P[3][r] = ex2f(s.w * p.c);
        }
    }
}

__device__ __forceinline__ float4 f4(float a, float b, float c, float d) { return make_float4(a, b, c, d); }
__device__ __forceinline__ float f4at(const float4& v, int r) { return r == 0 ? v.x : r == 1 ? v.y : r == 2 ? v.z : v.w; }

// One problem's barrier at the column cut: each of its 2 Wact warps arrives
// once per phase (0, then 1) on the mbarrier its first slot holds, and every
// lane polls for the phase (a wait polled by one lane while the others sit in
// __syncwarp measured 0.14 ms per barrier at C2, against a few microseconds).
// The wait is bounded; one that gives up flags the problem (bit 2).
__device__ __forceinline__ void prob_barrier(unsigned long long* bar, unsigned phase, int* err, int lane) {
    __syncwarp();
    const unsigned m = smem_u32(bar);
    if (lane == 0) asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(m) : "memory");
    bool ok = false;
    for (int it = 0; it < (1 << 22) && !ok; ++it) {
        unsigned done;
        asm volatile(
            "{\n .reg .pred p;\n mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
            : "=r"(done)
            : "r"(m), "r"(phase)
            : "memory");
        ok = done != 0;
    }
    if (!ok && lane == 0) atomicOr(err, 2);
    __syncwarp();
}

// The partition partials (log2 base, sum) of one warp -> the CTA's table.
__device__ __forceinline__ void put_partial(CtaSmem& S, int slot, float base, double sum, int lane) {
    float m = base;
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) m = fmaxf(m, __shfl_xor_sync(kAll, m, o));
    double t = sum * ld::p2d(base - m);
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) t += __shfl_xor_sync(kAll, t, o);
    if (lane == 0) {
        S.pbase[slot] = m;
        S.psum[slot] = t;
    }
}

// S = log2(1 + sum of the partials of slots o .. o + n - 1), as integer +
// fraction; false when not finite
template <bool NW>
__device__ __forceinline__ bool partition(const CtaSmem& S, int o, int n, float& Sint, float& Sfrac) {
    float m = -3.0e38f;
    for (int g = 0; g < 3; ++g)
        for (int v = o; v < o + n; ++v) m = fmaxf(m, S.pbase[g * kMaxW + v]);
    double tot = 0.0;
    for (int g = 0; g < 3; ++g)
        for (int v = o; v < o + n; ++v) tot = fma(S.psum[g * kMaxW + v], ld::p2d(S.pbase[g * kMaxW + v] - m), tot);
    if (!NW) tot += ld::p2d(-m);   // SW: alpha[0,0] = 0 adds 1 (the empty path)
    const int hi = __double2hiint(tot);
    const int ef = (hi >> 20) & 0x7ff;
    Sint = (float)(ef - 1023 + (int)m);
    const double mant = __hiloint2double((hi & 0x800fffff) | 0x3ff00000, __double2loint(tot));
    Sfrac = ring::lg2_rr((float)mant);
    return ef != 0x7ff && ef != 0;
}

// group q of a block's marginals (mu[c], times k) -> the staging tile
__device__ __forceinline__ void stage_group(float* mu_tile, int lane, int q, const float4 (&mu)[kQC], float k) {
#pragma unroll
    for (int r = 0; r < kR; ++r)
        *reinterpret_cast<float4*>(mu_tile + sw_off(r, lane, q)) =
            f4(f4at(mu[0], r) * k, f4at(mu[1], r) * k, f4at(mu[2], r) * k, f4at(mu[3], r) * k);
}

// What a warp needs across its blocks.  The kept plane of its row block holds
// column j's float4 of lane l at kb[32 j + l] (kp = kb + lane); its frames are
// pfr[32 bk] (this lane's).
struct Sweep {
    const CUtensorMap* tmS;
    const CUtensorMap* tmO;
    CtaSmem* S;
    WarpSmem* WS;
    const float4* kb;
    float4* kp;
    float* pfr;
    int* err;           // the problem's flags
    unsigned long long* pbar;
    int b, w, lane, nT, nL, y0;
    int s, o, Wp;       // slot, the problem's first slot, its slots
    bool above, below;
};

// phase 2: group g's kept values (block bk, group q: 4 columns x 32 lanes, 2 KB
// contiguous) -> kept slot g % 2
__device__ __forceinline__ void load_kept(const Sweep& sw, int g, int bk, int q) {
    bulk_load(sw.WS->kr[g & 1], sw.kb + 32 * (kBC * bk + kQC * q), kQC * 32 * sizeof(float4), &sw.WS->kbar[g & 1]);
}

// ------------------------------------------------------------------ forward
struct FwdState {
    float z[kR];
    float dc, E;
    double acc;         // partition of this lane's cells left of the cut: sum Z 2^-ab
    float ab;
    int jmax;
    float Qn;           // phase 2: the reverse's frame of the block
    float endz, endE;   // NW: Z of the end cell (in the lane that holds it) and its frame
    int nf;             // NW: a marginal came out non-finite
};

// One forward block bk.  Phase 1 (!P2): keeps w and adds the block's Z to the
// partition.  Phase 2: forms the marginals from the kept B, writes them over
// the block's scores in shared memory and stores that tile.
template <bool MASK, bool P2, bool NW>
__device__ __forceinline__ void fwd_block(const Sweep& sw, const Prob& p, FwdState& st, int bk, float Sint,
                                          float Sfrac) {
    CtaSmem& S = *sw.S;
    WarpSmem& WS = *sw.WS;
    const Hand& Hup = S.h[sw.above ? sw.s - 1 : sw.s];
    Hand& Hme = S.h[sw.s];
    const int lane = sw.lane, slot = bk % kHB, nT = sw.nT, nL = sw.nL;
    int* const err = sw.err;
    if (!bar_wait(&WS.bar[bk % kNS], (unsigned)(bk / kNS) & 1u)) *err = 1;
    float* const tile = WS.sc[bk % kNS];
    if (bk > 0) {   // the block's frame, from the strip's values
        float inv;
        const float J = frame_step(st.z, inv);
        st.jmax = max(st.jmax, abs((int)J));
#pragma unroll
        for (int r = 0; r < kR; ++r) st.z[r] *= inv;
        st.dc *= inv;
        st.E += J;
        if (!P2) ld::acc_rebase(st.acc, st.ab, st.E);
    }
    float Ein = 0.f;   // the row above the warp for this block: its frame
    if (sw.above) {
        ring::wait_flag(&S.progF[sw.s - 1], bk + 1, err);
        Ein = Hup.fe[slot];
    } else if (NW) {   // NW, warp 0: the boundary row 0 (Z_0j = G^j) is the row above
        Ein = rintf((float)(kBC * bk) * p.gl);
    }
    if (sw.below && bk >= kHB) ring::wait_flag(&S.consF[sw.s + 1], bk - kHB + 1, err);   // ring space
    FwdK K;
    fwd_consts(p, st.E, Ein, sw.above || NW, lane, K);
    if (NW) K.fs = 0.f;   // no path starts inside the grid
    float kE = 0.f, k1 = 1.f, k2 = 1.f;
    if (P2) {   // marginals = B w 2^(Q + E - S)
        const float x = (st.Qn + st.E - Sint) - Sfrac;
        if (NW) {
            split_scale(x, k1, k2);
            kE = 1.f;
        } else {
            // (clamped: a lane with no cells of the problem has B w = 0, and 0 x
            // inf would be NaN)
            kE = fminf(ex2f(x), 3.0e38f);
        }
        if (bk + 1 < nT) st.Qn = sw.pfr[32 * (bk + 1)];
    }
    float gs = 0.f;
#pragma unroll 1
    for (int q = 0; q < 2; ++q) {
        const int j0 = kBC * bk + kQC * q;
        float P[kQC][kR];
        group_P<MASK>(p, tile, lane, q, j0, P);
        if (!P2) {
            if (q == 1) {
                __syncwarp();
                if (lane == 0 && bk + kNS < nT) {   // every lane has read the tile: refill its slot
                    fence_async_smem();
                    tma_load_tile(sw.tmS, tile, &WS.bar[bk % kNS], kBC * (bk + kNS), sw.y0, sw.b);
                }
            }
        } else if (q == 0 && bk > nL && lane == 0) {
            // the previous block's marginals have left its slot: refill it with tile bk + 1
            tma_store_wait_read0();
            if (bk + 1 < nT)
                tma_load_tile(sw.tmS, WS.sc[(bk + 1) % kNS], &WS.bar[(bk + 1) % kNS], kBC * (bk + 1), sw.y0, sw.b);
        }
        const int g = 2 * (bk - nL) + q;   // phase 2: the group's ordinal
        if (P2 && !bar_wait(&WS.kbar[g & 1], (unsigned)(g >> 1) & 1u)) *err = 1;
        const float4* const kr = WS.kr[g & 1];
        float4 mu[kQC];
#pragma unroll
        for (int c = 0; c < kQC; ++c) {
            const int j = j0 + c;
            const int nvc = MASK ? (j < p.L2 ? p.nv : 0) : kR;
            const float yin = sw.above ? Hup.fv[slot][kQC * q + c]
                                       : (NW ? ex2f(fmaf((float)(j + 1), p.gl, -Ein)) : 0.f);
            float wv[kR];
            const float y = fwd_column<MASK>(p, K, st.z, st.dc, P[c], yin, nvc, lane, wv, gs);
            if (NW && !P2 && j == p.L2 - 1 && p.rend >= 0) {   // the end cell: the partition when no cut crosses
                st.endz = p.rend == 0 ? st.z[0] : p.rend == 1 ? st.z[1] : p.rend == 2 ? st.z[2] : st.z[3];
                st.endE = st.E;
            }
            if (sw.below && lane == 31) Hme.fv[slot][kQC * q + c] = y;
            if (!P2) {
                sw.kp[32 * j] = f4(wv[0], wv[1], wv[2], wv[3]);
            } else {
                const float4 bv = kr[32 * c + lane];
                if (NW) {
                    mu[c] = f4((bv.x * k1) * (wv[0] * k2), (bv.y * k1) * (wv[1] * k2), (bv.z * k1) * (wv[2] * k2),
                               (bv.w * k1) * (wv[3] * k2));
                    const float t = (mu[c].x + mu[c].y) + (mu[c].z + mu[c].w);
                    if (!(fabsf(t) <= 3.0e38f)) st.nf = 1;
                } else {
                    mu[c] = f4(bv.x * wv[0], bv.y * wv[1], bv.z * wv[2], bv.w * wv[3]);
                }
            }
        }
        if (P2) {
            stage_group(tile, lane, q, mu, kE);   // over the group's scores, which no lane reads again
            __syncwarp();
            if (lane == 0 && g + 2 < 2 * (nT - nL)) {   // every lane has read kept slot g % 2: refill it
                fence_async_smem();
                load_kept(sw, g, nL + ((g + 2) >> 1), g & 1);
            }
        }
    }
    if (sw.above) {
        __syncwarp();
        if (lane == 0) ring::st_release(&S.consF[sw.s], bk + 1);
    }
    if (sw.below && lane == 31) {   // the warp's last row of this block, for the warp below
        Hme.fe[slot] = st.E;
        ring::st_release(&S.progF[sw.s], bk + 1);
    }
    if (!P2) {
        st.acc = fma((double)gs, ld::p2d(st.E - st.ab), st.acc);
        sw.pfr[32 * bk] = st.E;
    } else {
        fence_async_smem();
        __syncwarp();
        if (lane == 0) tma_store_tile(sw.tmO, tile, kBC * bk, sw.y0, sw.b);
    }
}

template <bool MASK, bool NW>
__device__ void run_fwd(const Sweep& sw, const Args& A) {
    CtaSmem& S = *sw.S;
    const int lane = sw.lane, w = sw.w, nT = sw.nT, nL = sw.nL;
    Prob p;
    prob_init(A, sw.b, w, lane, p);
    // score tiles 0..nT-1: tile t goes to slot t % kNS, phase (t / kNS) & 1
    if (lane == 0)
        for (int n = 0; n < kNS && n < nT; ++n)
            tma_load_tile(sw.tmS, sw.WS->sc[n % kNS], &sw.WS->bar[n % kNS], kBC * n, sw.y0, sw.b);

    FwdState st;
#pragma unroll
    for (int r = 0; r < kR; ++r) st.z[r] = 0.f;
    st.dc = st.E = st.ab = 0.f;
    st.acc = 0.0;
    st.jmax = 0;
    st.Qn = 0.f;
    st.endz = 0.f;
    st.endE = -3.0e38f;
    st.nf = 0;
    if (NW && p.nv > 0) {
        // the boundary column 0: Z_i0 = G^i for this strip's rows, and Z of the
        // row above the strip as the first column's diagonal predecessor
        const int i0 = kWR * w + kR * lane + 1;   // the strip's first row (1-based)
        st.E = rintf(fmaf((float)i0, p.gl, nw_lead(i0)));
#pragma unroll
        for (int r = 0; r < kR; ++r) st.z[r] = r < p.nv ? ex2f(fmaf((float)(i0 + r), p.gl, -st.E)) : 0.f;
        st.dc = ex2f(fmaf((float)(i0 - 1), p.gl, -st.E));
    }

    for (int bk = 0; bk < nL; ++bk) fwd_block<MASK, false, NW>(sw, p, st, bk, 0.f, 0.f);

    // the cut
    if (NW) {   // every column left of the cut (nL == nT): the partition is the end cell's Z
        const bool e = nL == nT && p.rend >= 0;
        put_partial(S, sw.s, e ? st.endE : -3.0e38f, e ? (double)st.endz : 0.0, lane);
    } else {
        put_partial(S, sw.s, st.ab, st.acc, lane);
    }
    prob_barrier(sw.pbar, 0, sw.err, lane);   // phase 1 done: every partial and the reverse's values at the cut are in
    if (nL < nT) {   // the moves across the cut: Z_{i,m} (G B_{i,m+1} + P_{i+1,m+1} B_{i+1,m+1})
        const Meet& M = S.meet[sw.s];
        const float Ql = M.Q[lane];
        float pn, Qb;   // the row below the strip: P B at the cut and its frame
        if (lane < 31) {
            pn = M.PB[kR * (lane + 1)];
            Qb = M.Q[lane + 1];
        } else if (sw.below) {
            pn = S.meet[sw.s + 1].PB[0];
            Qb = S.meet[sw.s + 1].Q[0];
        } else {
            pn = 0.f;
            Qb = Ql;
        }
        float s1 = 0.f;
#pragma unroll
        for (int r = 0; r < kR; ++r)
            s1 = fmaf(st.z[r], fmaf(p.G, M.B[kR * lane + r], r + 1 < kR ? M.PB[kR * lane + r + 1] : 0.f), s1);
        double cr = (double)s1 + (double)(st.z[kR - 1] * pn) * ld::p2d(Qb - Ql);
        if (NW && w == 0 && lane == 0) {
            // the moves out of the boundary row 0 at the cut column m: Z_0m = G^m,
            // to (0, m+1) and to (1, m+1)
            const float x = fmaf((float)(kBC * nL), p.gl, -st.E);   // log2 of G^m in this lane's frame
            const float xi = floorf(x);
            cr += (double)(fmaf(p.G, M.b0, M.PB[0]) * ex2f(x - xi)) * ld::p2d(xi);
        }
        put_partial(S, 2 * kMaxW + sw.s, st.E + Ql, cr, lane);
    }
    prob_barrier(sw.pbar, 1, sw.err, lane);
    float Sint, Sfrac;
    const bool fin = partition<NW>(S, sw.o, sw.Wp, Sint, Sfrac);
    if (w == 0 && lane == 0 && A.value) A.value[sw.b] = (Sint + Sfrac) / p.c;

    if (nL < nT) {
        if (lane == 0) {   // the zero tiles stored from the kept slots have left them
            tma_store_wait_read0();
            load_kept(sw, 0, nL, 0);
            load_kept(sw, 1, nL, 1);
        }
        st.Qn = sw.pfr[32 * nL];
    }
    for (int bk = nL; bk < nT; ++bk) fwd_block<MASK, true, NW>(sw, p, st, bk, Sint, Sfrac);

    const bool bad = __any_sync(kAll, st.jmax > (NW ? kJMaxNW : ld::kJMax));
    const bool nf = NW && __any_sync(kAll, st.nf != 0);
    if (lane == 0 && (bad || !fin || nf)) atomicOr(sw.err, bad ? 4 : 8);
}

// ------------------------------------------------------------------ reverse
struct RevState {
    float Bv[kR], PB[kR];
    float Q;
    float pbin;         // lane 31: P B of the row below the warp, one column right of the block
    double acc;         // sum of P B right of the cut: paths counted by their first cell
    float ab;
    int jmax;
    float En;           // phase 2: the forward's frame of the block
    float b0;           // NW, warp 0 lane 0: B of the boundary row 0 at the current column
    int nf;             // NW: a marginal came out non-finite
};

// One reverse block bk (ordinal rb).  Phase 1 (!P2): keeps B and adds the
// block's P B to the partition.  Phase 2: forms the marginals from the kept w,
// over the block's scores, and stores them.
template <bool MASK, bool P2, bool NW>
__device__ __forceinline__ void rev_block(const Sweep& sw, const Prob& p, RevState& st, int rb, float Sint,
                                          float Sfrac) {
    CtaSmem& S = *sw.S;
    WarpSmem& WS = *sw.WS;
    const Hand& Hdn = S.h[sw.below ? sw.s + 1 : sw.s];
    Hand& Hme = S.h[sw.s];
    const int lane = sw.lane, slot = rb % kHB, nT = sw.nT, bk = nT - 1 - rb, r0 = nT - sw.nL;
    int* const err = sw.err;
    if (!bar_wait(&WS.bar[rb % kNS], (unsigned)(rb / kNS) & 1u)) *err = 1;
    float* const tile = WS.sc[rb % kNS];
    if (rb > 0) {   // the block's reverse frame
        float inv;
        const float J = frame_step(st.Bv, inv);
        st.jmax = max(st.jmax, abs((int)J));
#pragma unroll
        for (int r = 0; r < kR; ++r) {
            st.Bv[r] *= inv;
            st.PB[r] *= inv;
        }
        st.pbin *= inv;
        if (NW) st.b0 *= inv;
        st.Q += J;
        if (!P2) ld::acc_rebase(st.acc, st.ab, st.Q);
    }
    float Qin = 0.f;   // the row below the warp for this block: its frame
    if (sw.below) {
        ring::wait_flag(&S.progR[sw.s + 1], rb + 1, err);
        Qin = Hdn.re[slot];
    }
    if (sw.above && rb >= kHB) ring::wait_flag(&S.consR[sw.s - 1], rb - kHB + 1, err);   // ring space
    RevK K;
    rev_consts(p, st.Q, Qin, sw.below, lane, K, NW ? min(31, (p.L1 - 1 - kWR * sw.w) / kR) : 31);
    float kE = 0.f, k1 = 1.f, k2 = 1.f;
    if (P2) {   // marginals = B w 2^(Q + E - S)
        const float x = (st.Q + st.En - Sint) - Sfrac;
        if (NW) {
            split_scale(x, k1, k2);
            kE = 1.f;
        } else {
            kE = fminf(ex2f(x), 3.0e38f);
        }
        if (bk > 0) st.En = sw.pfr[32 * (bk - 1)];
    }
    float gs = 0.f;
#pragma unroll 1
    for (int q = 1; q >= 0; --q) {
        const int j0 = kBC * bk + kQC * q;
        float P[kQC][kR];
        group_P<MASK>(p, tile, lane, q, j0, P);
        if (!P2) {
            if (q == 0) {
                __syncwarp();
                if (lane == 0 && rb + kNS < nT) {
                    fence_async_smem();
                    tma_load_tile(sw.tmS, tile, &WS.bar[rb % kNS], kBC * (nT - 1 - rb - kNS), sw.y0, sw.b);
                }
            }
        } else if (q == 1 && rb > r0 && lane == 0) {
            // the previous block's marginals have left its slot: refill it with the next tile
            tma_store_wait_read0();
            if (rb + 1 < nT)
                tma_load_tile(sw.tmS, WS.sc[(rb + 1) % kNS], &WS.bar[(rb + 1) % kNS], kBC * (bk - 1), sw.y0, sw.b);
        }
        const int g = 2 * (rb - r0) + (1 - q);   // phase 2: the group's ordinal
        if (P2 && !bar_wait(&WS.kbar[g & 1], (unsigned)(g >> 1) & 1u)) *err = 1;
        const float4* const kr = WS.kr[g & 1];
        float4 mu[kQC];
#pragma unroll
        for (int c = kQC - 1; c >= 0; --c) {
            const int j = j0 + c, cb = kQC * q + c;
            const int nvc = MASK ? (j < p.L2 ? p.nv : 0) : kR;
            const float bin = sw.below ? Hdn.rv[slot][cb] : 0.f;
            const float pbn = cb + 1 < kBC ? (sw.below ? Hdn.rp[slot][cb + 1] : 0.f) * K.m1 : st.pbin;
            float wk[kR];
            if (P2) {
                const float4 wv = kr[32 * c + lane];
                wk[0] = wv.x;
                wk[1] = wv.y;
                wk[2] = wv.z;
                wk[3] = wv.w;
            } else {
                wk[0] = wk[1] = wk[2] = wk[3] = 0.f;
            }
            const float pbprev = st.PB[0];
            rev_column<MASK, NW>(p, K, st.Bv, st.PB, P[c], wk, bin, pbn, nvc, lane,
                                 (NW && j == p.L2 - 1) ? p.rend : -1, k1, k2);
            if (NW && P2) {
                const float t = (wk[0] + wk[1]) + (wk[2] + wk[3]);
                if (!(fabsf(t) <= 3.0e38f)) st.nf = 1;
            }
            // NW, warp 0 (lane 0's value is used): B of the boundary row 0 at this
            // column, from row 1 here (down) and one column right (diagonal), and
            // row 0 one column right
            if (NW && !P2 && sw.w == 0) st.b0 = fmaf(p.G, st.b0 + st.Bv[0], pbprev);
            if (sw.above && lane == 0) {
                Hme.rv[slot][cb] = st.Bv[0];
                Hme.rp[slot][cb] = st.PB[0];
            }
            if (P2) {
                mu[c] = f4(wk[0], wk[1], wk[2], wk[3]);
            } else {
                sw.kp[32 * j] = f4(st.Bv[0], st.Bv[1], st.Bv[2], st.Bv[3]);
                gs += (st.PB[0] + st.PB[1]) + (st.PB[2] + st.PB[3]);
            }
        }
        if (P2) {
            stage_group(tile, lane, q, mu, kE);
            __syncwarp();
            if (lane == 0 && g + 2 < 2 * sw.nL) {
                fence_async_smem();
                const int g2 = g + 2;
                load_kept(sw, g, nT - 1 - (r0 + (g2 >> 1)), 1 - (g2 & 1));
            }
        }
    }
    st.pbin = (sw.below ? Hdn.rp[slot][0] : 0.f) * K.m1;
    if (sw.below) {
        __syncwarp();
        if (lane == 0) ring::st_release(&S.consR[sw.s], rb + 1);
    }
    if (sw.above && lane == 0) {   // the warp's first row of this block, for the warp above
        Hme.re[slot] = st.Q;
        ring::st_release(&S.progR[sw.s], rb + 1);
    }
    if (!P2) {
        st.acc = fma((double)gs, ld::p2d(st.Q - st.ab), st.acc);
        sw.pfr[32 * bk] = st.Q;
    } else {
        fence_async_smem();
        __syncwarp();
        if (lane == 0) tma_store_tile(sw.tmO, tile, kBC * bk, sw.y0, sw.b);
    }
}

template <bool MASK, bool NW>
__device__ void run_rev(const Sweep& sw, const Args& A) {
    CtaSmem& S = *sw.S;
    const int lane = sw.lane, w = sw.w, nT = sw.nT, nL = sw.nL;
    Prob p;
    prob_init(A, sw.b, w, lane, p);
    // score tiles nT-1..0: ordinal n (tile nT-1-n) goes to slot n % kNS
    if (lane == 0)
        for (int n = 0; n < kNS && n < nT; ++n)
            tma_load_tile(sw.tmS, sw.WS->sc[n % kNS], &sw.WS->bar[n % kNS], kBC * (nT - 1 - n), sw.y0, sw.b);

    RevState st;
#pragma unroll
    for (int r = 0; r < kR; ++r) st.Bv[r] = st.PB[r] = 0.f;
    st.Q = st.pbin = st.ab = 0.f;
    st.acc = 0.0;
    st.jmax = 0;
    st.En = 0.f;
    st.b0 = 0.f;
    st.nf = 0;
    if (NW && p.nv > 0) {
        // NW weights scale like G^(rows below): at the right edge B_iL2 = G^(L1 - i).
        // Start each lane's frame there (and half a block ahead), so that lanes
        // far above the end row do not begin as zeros that no frame step can
        // bring back.
        const int ilast = kWR * w + kR * lane + p.nv;   // the strip's last row inside the problem (1-based)
        st.Q = rintf(fmaf((float)(p.L1 - ilast), p.gl, nw_lead(p.L1 - ilast)));
    }

    for (int rb = 0; rb < nT - nL; ++rb) rev_block<MASK, false, NW>(sw, p, st, rb, 0.f, 0.f);

    // the cut: B and P B at its right column (zero when nothing is right of it)
    Meet& M = S.meet[sw.s];
#pragma unroll
    for (int r = 0; r < kR; ++r) {
        M.B[kR * lane + r] = st.Bv[r];
        M.PB[kR * lane + r] = st.PB[r];
    }
    M.Q[lane] = st.Q;
    if (NW && sw.w == 0 && lane == 0) M.b0 = st.b0;
    // NW: no path starts right of the cut, nothing to add there
    put_partial(S, kMaxW + sw.s, NW ? -3.0e38f : st.ab, NW ? 0.0 : st.acc, lane);
    prob_barrier(sw.pbar, 0, sw.err, lane);
    prob_barrier(sw.pbar, 1, sw.err, lane);   // the forward warps have added the moves across the cut
    float Sint, Sfrac;
    partition<NW>(S, sw.o, sw.Wp, Sint, Sfrac);

    if (lane == 0) {   // the kept w of the last block left of the cut: group 1, then group 0
        load_kept(sw, 0, nL - 1, 1);
        load_kept(sw, 1, nL - 1, 0);
    }
    st.En = sw.pfr[32 * (nL - 1)];
    for (int rb = nT - nL; rb < nT; ++rb) rev_block<MASK, true, NW>(sw, p, st, rb, Sint, Sfrac);

    const bool bad = __any_sync(kAll, st.jmax > (NW ? kJMaxNW : ld::kJMax));
    const bool nf = NW && __any_sync(kAll, st.nf != 0);
    if (lane == 0 && (bad || nf)) atomicOr(sw.err, bad ? 4 : 8);
}

// rows and columns of problem b inside the padded shape
__device__ __forceinline__ void prob_shape(const Args& A, int b, int& L1, int& L2) {
    L1 = A.lengths ? min(max(A.lengths[2 * b], 0), A.L1v) : A.L1v;
    L2 = A.lengths ? min(max(A.lengths[2 * b + 1], 0), A.L2v) : A.L2v;
}

// Without a packing table a CTA is one problem: Wc = row blocks of the padded
// plane, slot = row block.  With one (ragged batches), a CTA has kMaxW slots
// and the table gives each slot's problem and row block; a problem holds
// max(Wact, 1) consecutive slots, and the last of them also writes the zeros
// of the padded plane's row blocks past them.
// NW: soft Needleman-Wunsch (global alignment): no start term, the boundary row
// and column of gaps, the end cell's weight, the partition from the crossing
// terms alone.
template <bool NW>
__global__ void __launch_bounds__(64 * kMaxW, 2) lin_strip_kernel(const __grid_constant__ CUtensorMap tmS,
                                                                const __grid_constant__ CUtensorMap tmO,
                                                                const Args A) {
    extern __shared__ unsigned char smem_raw[];
    CtaSmem& S = *reinterpret_cast<CtaSmem*>((reinterpret_cast<uintptr_t>(smem_raw) + 255) & ~(uintptr_t)255);
    const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
    const int Wall = warps_for(A.L1);                // row blocks of the padded plane
    const int Wc = A.pack ? kMaxW : Wall;            // slots of this CTA
    const bool fwd = wid < Wc;
    const int s = fwd ? wid : wid - Wc;              // slot
    WarpSmem& WS = S.w[wid];                         // this warp's tiles (2 Wc of them are allocated)
    if (lane == 0) {
        for (int i = 0; i < kNS; ++i)
            asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(smem_u32(&WS.bar[i])) : "memory");
        for (int i = 0; i < 2; ++i)
            asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(smem_u32(&WS.kbar[i])) : "memory");
    }
    if (threadIdx.x < kMaxW) {
        S.progF[threadIdx.x] = S.progR[threadIdx.x] = 0;
        S.consF[threadIdx.x] = S.consR[threadIdx.x] = 0;
        S.err[threadIdx.x] = 0;
        S.slot_ok[threadIdx.x] = 0;
        S.slot[threadIdx.x] = -1;
    }
    if (threadIdx.x < 3 * kMaxW) {   // partials of slots without rows: nothing
        S.pbase[threadIdx.x] = -3.0e38f;
        S.psum[threadIdx.x] = 0.0;
    }
    __syncwarp();
    if (threadIdx.x == 0) {
        // the slots' problems; a problem whose slots do not match the table is
        // left to the fix-up engines (flag 1), and none of its warps runs
        const int cb = A.order ? A.order[blockIdx.x] : (int)blockIdx.x;
        for (int q = 0; q < Wc; ++q) S.slot[q] = A.pack ? A.pack[(size_t)kMaxW * blockIdx.x + q] : cb * 4 + q;
        for (int o = 0; o < Wc; ++o) {
            const int e = S.slot[o];
            if (e < 0 || (e & 3) != 0) continue;   // not a problem's first slot
            int L1, L2;
            prob_shape(A, e >> 2, L1, L2);
            const int Wact = (L1 > 0 && L2 > 0) ? warps_for(L1) : 0;
            const int Wp = A.pack ? max(Wact, 1) : Wall;
            bool ok = o + Wp <= Wc;
            for (int q = o; ok && q < o + Wp; ++q) ok = S.slot[q] == e + (q - o);
            S.err[o] = ok ? 0 : 1;
            if (!ok) continue;
            for (int q = o; q < o + Wp; ++q) S.slot_ok[q] = 1;
            if (Wact > 0)
                asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(&S.pbar[o])), "r"(2 * Wact)
                             : "memory");
        }
    }
    if (lane == 0) asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    __syncthreads();

    if (S.slot_ok[s]) {
        const int e = S.slot[s];
        const int b = e >> 2, w = e & 3, o = s - w;
        int L1, L2;
        prob_shape(A, b, L1, L2);
        const int Wact = (L1 > 0 && L2 > 0) ? warps_for(L1) : 0;   // row blocks with rows of the problem
        const int Wp = A.pack ? max(Wact, 1) : Wall;
        char* const base = reinterpret_cast<char*>(A.ws) + (size_t)b * A.ws_stride;
        const int nT = (L2 + kBC - 1) / kBC;
        const int nTall = (A.L2 + kBC - 1) / kBC;
        Sweep sw;
        sw.tmS = &tmS;
        sw.tmO = &tmO;
        sw.S = &S;
        sw.WS = &WS;
        sw.kb = reinterpret_cast<const float4*>(base) + (size_t)w * nT * kBC * 32;
        sw.kp = reinterpret_cast<float4*>(base) + (size_t)w * nT * kBC * 32 + lane;
        sw.pfr = reinterpret_cast<float*>(base + plane_bytes_of(Wall, A.L2)) + (size_t)w * nT * 32 + lane;
        sw.err = &S.err[o];
        sw.pbar = &S.pbar[o];
        sw.b = b;
        sw.w = w;
        sw.s = s;
        sw.o = o;
        sw.Wp = Wp;
        sw.lane = lane;
        sw.nT = nT;
        sw.nL = (nT + 1) / 2;                        // blocks left of the cut
        sw.y0 = 32 * w;
        sw.above = w > 0;
        sw.below = w + 1 < Wact;
        // output tiles that no sweep writes (past the problem's columns, rows
        // of a row block without rows of the problem, and -- from the problem's
        // last slot -- the padded plane's row blocks past its slots): zeros,
        // stored by the forward warp from its kept slots (4 KB, free until its
        // phase 2)
        const int zfrom = w < Wact ? nT : 0;
        const int zrb = w == Wp - 1 ? Wall : w + 1;  // row blocks w .. zrb - 1
        if (fwd && (zfrom < nTall || zrb > w + 1)) {
            float4* zt = &WS.kr[0][0];
            for (int i = lane; i < kTileFloats / 4; i += 32) zt[i] = f4(0.f, 0.f, 0.f, 0.f);
            fence_async_smem();
            __syncwarp();
            if (lane == 0) {
                for (int t = zfrom; t < nTall; ++t) tma_store_tile(&tmO, reinterpret_cast<float*>(zt), kBC * t, sw.y0, b);
                for (int r = w + 1; r < zrb; ++r)
                    for (int t = 0; t < nTall; ++t) tma_store_tile(&tmO, reinterpret_cast<float*>(zt), kBC * t, 32 * r, b);
            }
        }
        if (w < Wact) {
            // cells outside the problem in this row block: rows past L1, or a last block cut by L2
            const bool mask = L1 < kWR * (w + 1) || L2 % kBC != 0;
            if (fwd) {
                if (mask)
                    run_fwd<true, NW>(sw, A);
                else
                    run_fwd<false, NW>(sw, A);
            } else {
                if (mask)
                    run_rev<true, NW>(sw, A);
                else
                    run_rev<false, NW>(sw, A);
            }
        }
        if (lane == 0) tma_store_wait0();
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        for (int o = 0; o < Wc; ++o) {
            const int e = S.slot[o];
            if (e < 0 || (e & 3) != 0) continue;
            const int b = e >> 2;
            int L1, L2;
            prob_shape(A, b, L1, L2);
            if ((L1 == 0 || L2 == 0) && A.value && S.err[o] == 0) {
                // SW: the empty path; NW: the one all-gap path
                const float g = A.gap_dev ? *A.gap_dev : A.gap;
                A.value[b] = NW ? (float)(L1 + L2) * g : 0.f;
            }
            if (A.redo) A.redo[b] = S.err[o];
        }
    }
}

// The packing table of a ragged batch (one CTA of 1024 threads).  A problem
// takes max(Wact, 1) slots (its class, 1..4); CTAs are filled class by class,
// each class in the given order (largest cost first): one 4-slot problem; a
// 3-slot problem with a 1-slot one; two 2-slot problems (the last, if their
// number is odd, with two 1-slot ones); the remaining 1-slot problems four by
// four.  pack[kMaxW c + q] = problem * 4 + row block of slot q of CTA c (-1:
// none); *ncta = CTAs used.  Deterministic: ranks come from ballots in order.
__global__ void __launch_bounds__(1024) strip_pack_kernel(const int* __restrict__ lengths, int B, int L1v, int L2v,
                                                          const int* __restrict__ order, int* __restrict__ pack,
                                                          int* __restrict__ ncta) {
    __shared__ int cnt[5], run[5], wtot[32][5], wpre[32][5];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    for (int i = tid; i < kMaxW * B; i += blockDim.x) pack[i] = -1;
    if (tid < 5) cnt[tid] = run[tid] = 0;
    __syncthreads();
    auto cls_of = [&](int k, int& b) {
        if (k >= B) return 0;
        b = order ? order[k] : k;
        const int l1 = min(max(lengths[2 * b], 0), L1v), l2 = min(max(lengths[2 * b + 1], 0), L2v);
        return (l1 > 0 && l2 > 0) ? min(warps_for(l1), kMaxW) : 1;
    };
    for (int k0 = 0; k0 < B; k0 += blockDim.x) {
        int b = 0;
        const int c = cls_of(k0 + tid, b);
        if (c > 0) atomicAdd(&cnt[c], 1);
    }
    __syncthreads();
    const int n1 = cnt[1], n2 = cnt[2], n3 = cnt[3], n4 = cnt[4];
    const int m13 = min(n1, n3);                      // 1-slot problems beside 3-slot ones
    const int n2h = (n2 + 1) / 2;
    const int m2 = (n2 & 1) ? min(2, n1 - m13) : 0;   // 1-slot problems in the odd 2-slot CTA
    const int rem1 = n1 - m13 - m2;
    if (tid == 0) *ncta = n4 + n3 + n2h + (rem1 + kMaxW - 1) / kMaxW;
    for (int k0 = 0; k0 < B; k0 += blockDim.x) {
        int b = 0;
        const int c = cls_of(k0 + tid, b);
        int lpre[5];
#pragma unroll
        for (int q = 1; q <= 4; ++q) {
            const unsigned m = __ballot_sync(0xffffffffu, c == q);
            lpre[q] = __popc(m & ((1u << lane) - 1u));
            if (lane == 0) wtot[warp][q] = __popc(m);
        }
        __syncthreads();
        if (tid < 4) {
            const int q = tid + 1;
            int acc = run[q];
            for (int v = 0; v < (int)(blockDim.x >> 5); ++v) {
                wpre[v][q] = acc;
                acc += wtot[v][q];
            }
            run[q] = acc;
        }
        __syncthreads();
        if (c > 0) {
            const int r = wpre[warp][c] + lpre[c];    // rank within the class, in order
            int cta, q0;
            if (c == 4) {
                cta = r;
                q0 = 0;
            } else if (c == 3) {
                cta = n4 + r;
                q0 = 0;
            } else if (c == 2) {
                cta = n4 + n3 + r / 2;
                q0 = 2 * (r & 1);
            } else if (r < m13) {
                cta = n4 + r;
                q0 = 3;
            } else if (r < m13 + m2) {
                cta = n4 + n3 + n2h - 1;
                q0 = 2 + (r - m13);
            } else {
                const int r1 = r - m13 - m2;
                cta = n4 + n3 + n2h + r1 / kMaxW;
                q0 = r1 % kMaxW;
            }
            for (int j = 0; j < c; ++j) pack[(size_t)kMaxW * cta + q0 + j] = b * 4 + j;
        }
        __syncthreads();
    }
}

}  // namespace strip

// ------------------------------------------------------------------ host side
namespace {
PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = [] {
        void* f = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) != cudaSuccess ||
            q != cudaDriverEntryPointSuccess)
            f = nullptr;
        return reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(f);
    }();
    return fn;
}

// The score / marginal plane [B][L1][L2] as a 4-D tensor (columns, strip, row
// in strip, problem), boxes of 8 columns x 32 strips x 4 rows (one warp's).
bool strip_tensor_map(CUtensorMap* tm, const float* base, int B, int L1, int L2) {
    auto fn = encode_fn();
    if (!fn) return false;
    const cuuint64_t dims[4] = {(cuuint64_t)L2, (cuuint64_t)(L1 / strip::kR), (cuuint64_t)strip::kR, (cuuint64_t)B};
    const cuuint64_t strides[3] = {(cuuint64_t)L2 * 4 * strip::kR, (cuuint64_t)L2 * 4, (cuuint64_t)L1 * L2 * 4};
    const cuuint32_t box[4] = {(cuuint32_t)strip::kBC, 32, (cuuint32_t)strip::kR, 1};
    const cuuint32_t es[4] = {1, 1, 1, 1};
    return fn(tm, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, const_cast<float*>(base), dims, strides, box, es,
              CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_32B, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}
}  // namespace

// Any problem of at most 512 rows.  Planes whose rows are not whole 16-byte
// units (L2 % 4 != 0), or whose row count is not a multiple of 4, cannot be
// TMA tensors: they are copied into padded planes in the workspace, and the
// marginals copied back (8 + 8 bytes per cell, at HBM rate).
static bool strip_shape_ok(int L1, int L2) { return L1 > 0 && L2 > 0 && L1 <= strip::kWR * strip::kMaxW; }
static int round4(int x) { return (x + 3) & ~3; }
static size_t align256z(size_t x) { return (x + 255) & ~(size_t)255; }
static bool strip_repack(int L1, int L2) { return L1 % strip::kR != 0 || L2 % 4 != 0; }
// [kept planes][padded scores][padded marginals]
static size_t strip_plane_area(int B, int L1, int L2) {
    return align256z(strip::per_problem_bytes(round4(L1), round4(L2)) * (size_t)B);
}
static size_t strip_padded_bytes(int B, int L1, int L2) {
    return align256z((size_t)B * round4(L1) * round4(L2) * sizeof(float));
}
// the packing table of a ragged batch and its CTA count
static size_t strip_pack_bytes(int B) { return align256z((size_t)strip::kMaxW * B * sizeof(int)) + 256; }
static size_t strip_main_bytes(int B, int L1, int L2) {
    return strip_repack(L1, L2) ? strip_plane_area(B, L1, L2) + 2 * strip_padded_bytes(B, L1, L2)
                                : strip_plane_area(B, L1, L2);
}

size_t lin_strip_workspace_bytes(int B, int L1, int L2) {
    if (!strip_shape_ok(L1, L2)) return 0;
    return strip_main_bytes(B, L1, L2) + strip_pack_bytes(B);
}

int launch_lin_strip(const SwArgs& a, size_t ws_bytes, cudaStream_t st, bool nw) {
    if (a.mode != MODE_MARG || !a.redo || a.grad_gap || a.grad_T || !a.out || !a.scores) return -1;
    if (engine_forced_plane() || engine_forced_pipeline()) return -1;
    if (!strip_shape_ok(a.L1, a.L2)) return -1;
    if ((((uintptr_t)a.ws) & 255) != 0 || !a.ws) return -1;
    const bool repack = strip_repack(a.L1, a.L2);
    const int L1p = round4(a.L1), L2p = round4(a.L2);
    const size_t per = strip::per_problem_bytes(L1p, L2p);
    if (ws_bytes < lin_strip_workspace_bytes(a.B, a.L1, a.L2)) return -1;
    const float* sc = a.scores;
    float* out = a.out;
    if (repack) {
        float* ps = (float*)((char*)a.ws + strip_plane_area(a.B, a.L1, a.L2));
        sc = ps;
        out = (float*)((char*)ps + strip_padded_bytes(a.B, a.L1, a.L2));
    } else if ((((uintptr_t)a.scores) & 15) != 0 || (((uintptr_t)a.out) & 15) != 0) {
        return -1;
    }
    CUtensorMap tmS, tmO;
    if (!strip_tensor_map(&tmS, sc, a.B, L1p, L2p) || !strip_tensor_map(&tmO, out, a.B, L1p, L2p)) return -1;
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return (int)e;
    static DeviceSetup setup;
    int nsm = 0;
    const int se = device_setup(setup, dev, [] {
        const int bytes = (int)strip::smem_bytes_for(strip::kMaxW);
        cudaError_t e = cudaFuncSetAttribute(strip::lin_strip_kernel<false>,
                                             cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
        if (e == cudaSuccess)
            e = cudaFuncSetAttribute(strip::lin_strip_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     bytes);
        return (int)e;
    }, &nsm);
    if (se != 0) return se;
    strip::Args A;
    A.lengths = a.lengths;
    A.B = a.B;
    A.L1 = L1p;
    A.L2 = L2p;
    A.L1v = a.L1;
    A.L2v = a.L2;
    A.gap = a.gap;
    A.temp = a.temp;
    A.gap_dev = a.gap_dev;
    A.temp_dev = a.temp_dev;
    A.value = a.value;
    A.ws = a.ws;
    A.redo = a.redo;
    A.order = a.order;
    A.pack = nullptr;
    A.ws_stride = per;
    const int W = strip::warps_for(L1p);
    if (repack) {
        const int rc = launch_pad_rows(a.scores, a.B, a.L1, a.L2, const_cast<float*>(sc), L1p, L2p, st);
        if (rc) return rc;
    }
    // ragged batches of problems over 128 rows: several problems per CTA,
    // by the packing table (CTAs past the table's count find no slot and exit)
    const bool pack = a.lengths && W > 1 && a.B > 1;
    if (pack) {
        int* const tab = (int*)((char*)a.ws + strip_main_bytes(a.B, a.L1, a.L2));
        int* const ncta = (int*)((char*)tab + align256z((size_t)strip::kMaxW * a.B * sizeof(int)));
        strip::strip_pack_kernel<<<1, 1024, 0, st>>>(a.lengths, a.B, a.L1, a.L2, a.order, tab, ncta);
        const cudaError_t pe = cudaGetLastError();
        if (pe != cudaSuccess) return (int)pe;
        A.pack = tab;
        A.order = nullptr;
        if (nw)
            strip::lin_strip_kernel<true><<<a.B, 64 * strip::kMaxW, strip::smem_bytes_for(strip::kMaxW), st>>>(tmS, tmO, A);
        else
            strip::lin_strip_kernel<false><<<a.B, 64 * strip::kMaxW, strip::smem_bytes_for(strip::kMaxW), st>>>(tmS, tmO, A);
    } else if (nw) {
        strip::lin_strip_kernel<true><<<a.B, 64 * W, strip::smem_bytes_for(W), st>>>(tmS, tmO, A);
    } else {
        strip::lin_strip_kernel<false><<<a.B, 64 * W, strip::smem_bytes_for(W), st>>>(tmS, tmO, A);
    }
    cudaError_t e2 = cudaGetLastError();
    if (e2 != cudaSuccess || !repack) return (int)e2;
    return launch_unpad_rows(out, L1p, L2p, a.out, a.B, a.L1, a.L2, st);
}

}  // namespace d2pb
