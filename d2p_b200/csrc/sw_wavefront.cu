// sw_wavefront.cu -- fast path for soft Smith-Waterman value + marginals (linear gap).
//
// One CTA per problem; warps own row-blocks of 32 rows (lane = row) and sweep
// them left-to-right (forward) and right-to-left (reverse), one cell per lane
// per step, so the 32 lanes of a warp always sit on one anti-diagonal.
// Cross-lane dependencies move by warp shuffles; cross-warp dependencies (the
// last row of a row-block feeding the first row of the next) move through small
// global boundary rows (L2-resident) prefetched with cp.async, with a CTA barrier
// every kSync steps and a fixed minimum skew between consecutive row-blocks.
//
// Numerics.  Everything is base-2 scaled (a = alpha*log2(e)/T, one MUFU
// ex2/lg2 per exponential/logarithm) and every warp keeps its own integer
// "frame" O per anti-diagonal: a cell stores a - O, so stored magnitudes stay
// small even when alpha grows to 10^3 along the matrix (the reference carries
// raw alpha in fp32 and loses absolute precision there).  Frame differences are
// exact integers; the value S is kept as (integer part, fraction).
//
// Memory.  The forward writes the framed alpha plane (4 B/cell) and the per-step
// frames; the reverse pass reads them back, so each cell costs: scores 4 B read
// twice, alpha 4 B written + read, marginals 4 B written = 20 B/cell.  Every
// global access is a coalesced 16-byte cp.async (loads) or 16-byte store
// (write-back of 16-column tiles staged in shared memory).  Per-warp shared
// rings are [rows][64] floats: lane l touches column j = c - l of row l, so the
// bank (64 l + j) mod 32 = (c - l) mod 32 differs across the warp -- the
// anti-diagonal access pattern is bank-conflict free.  A cell's score slot is
// reused for its output (alpha in the forward, the marginal in the reverse),
// so the forward needs one ring per warp and the reverse two.
//
// Reverse pass: beta is propagated in gather/push form through registers and
// shuffles (no atomics, deterministic):
//   beta_ij = 2^min(a_ij - S, 0) + sum over successors of beta_succ * w(succ <- ij)
//   marginal_ij = beta_ij * (w_align + w_sky),  dS/dgap = sum beta*(w_up + w_left),
//   dS/dT = path entropy (sum of non-negative terms).
// Semantics follow the reference (src/sw/kernels_cpu.cpp:70-279).
#include <stdint.h>

#include "sw_common.cuh"
#include "sw_internal.h"

namespace d2pb {
namespace wf {

constexpr int kCW = 16;                 // chunk width (columns): unit of loads, write-backs and stages
constexpr int kRW = 64;                 // ring width (columns) = row stride of the rings (4 chunks)
constexpr int kSync = 16;               // steps between CTA barriers (= one stage)
constexpr int kSkew = 80;               // minimum step skew between consecutive row-blocks (> 63, multiple of 16)
constexpr int kMaxRB = 512;             // row-blocks per problem (L1 <= 16384)
constexpr int kNW = 6;                  // warps per CTA

struct WarpSmem {
    float ringS[32 * kRW];        // scores; forward: alpha written in place; reverse: marginals in place
    float ringA[33 * kRW];        // reverse: framed alpha, row 0 = row above the row-block
    float2 bnd[kRW];              // forward: last row of the previous row-block (a - O, O)
    float bb[kRW];                // reverse: beta pushes from the row below
    float fr[kRW];                // reverse: frames of this row-block
};

struct Layout {  // per-problem workspace
    float* aplane;   // [nRB][33][L2m]: row 0 = row above (in this block's frames), rows 1..32 = alpha - O
    float* frames;   // [nRB][L2m + 32] per-step frame O (exact integers stored as float)
    float2* bnd;     // [nRB][L2m] last row of each row-block: (a - O, O)
    float* bb;       // [nRB][L2m] reverse pushes into the row above
};

__host__ __device__ inline size_t align_up(size_t x, size_t a) { return (x + a - 1) / a * a; }

__host__ __device__ inline size_t per_problem_bytes(int L1m, int L2m) {
    const size_t nrb = (size_t)(L1m + 31) / 32;
    size_t b = align_up(nrb * 33 * (size_t)L2m * 4, 256);
    b += align_up(nrb * (size_t)(L2m + 32) * 4, 256);
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
    base += align_up(nrb * (size_t)(L2m + 32) * 4, 256);
    L.bnd = (float2*)base;
    base += align_up(nrb * (size_t)L2m * 8, 256);
    L.bb = (float*)base;
    return L;
}

// ---------------------------------------------------------------- cp.async
__device__ __forceinline__ void cp_async16(void* smem, const void* gmem, int src_bytes) {
    const unsigned s = (unsigned)__cvta_generic_to_shared(smem);
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(s), "l"(gmem), "r"(src_bytes));
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::); }
__device__ __forceinline__ void cp_async_wait1() { asm volatile("cp.async.wait_group 1;\n" ::); }
__device__ __forceinline__ void cp_async_wait0() { asm volatile("cp.async.wait_group 0;\n" ::); }

__device__ __forceinline__ float exp2i(int k) {  // exact 2^k (0 below 2^-126)
    return k < -126 ? 0.f : __int_as_float((127 + min(k, 127)) << 23);
}

// Load chunk `ch` (0-based columns [16ch, 16ch+16)) of `nrows` rows of a
// row-major fp32 plane (row stride ld) into a [rows][64] ring; columns >= ncols
// are zero-filled without being read.
__device__ __forceinline__ void load_chunk(float* ring, const float* plane, int ld, int nrows, int ncols,
                                           int ch, int lane) {
    const int col0 = ch * kCW;
    const int rc = col0 & (kRW - 1);
    for (int p = lane; p < nrows * 4; p += 32) {
        const int row = p >> 2, pc = p & 3;
        const int c = col0 + pc * 4;
        const bool in = c < ncols;
        cp_async16(ring + row * kRW + rc + pc * 4, plane + (size_t)row * ld + (in ? c : 0), in ? 16 : 0);
    }
}

// Write back chunk `ch` of a ring (rows < nrows, columns < ncols) to a plane.
__device__ __forceinline__ void store_chunk(const float* ring, float* plane, int ld, int nrows, int ncols,
                                            int ch, int lane) {
    const int col0 = ch * kCW;
    const int rc = col0 & (kRW - 1);
    for (int p = lane; p < nrows * 4; p += 32) {
        const int row = p >> 2, pc = p & 3;
        const int c = col0 + pc * 4;
        if (c < ncols) {
            const float4 v = *reinterpret_cast<const float4*>(ring + row * kRW + rc + pc * 4);
            float* dst = plane + (size_t)row * ld + c;
            if (c + 4 <= ncols) {
                __stcs(reinterpret_cast<float4*>(dst), v);
            } else {
                const int rem = ncols - c;
                dst[0] = v.x;
                if (rem > 1) dst[1] = v.y;
                if (rem > 2) dst[2] = v.z;
            }
        }
    }
}

// one row, one chunk: 16 elements of 4 or 8 bytes
__device__ __forceinline__ void load_row_chunk4(float* ring, const float* row, int ncols, int ch, int lane) {
    if (lane < 4) {
        const int c = ch * kCW + lane * 4;
        const bool in = c < ncols;
        cp_async16(ring + ((ch * kCW) & (kRW - 1)) + lane * 4, row + (in ? c : 0), in ? 16 : 0);
    }
}
__device__ __forceinline__ void load_row_chunk8(float2* ring, const float2* row, int ncols, int ch, int lane) {
    if (lane < 8) {
        const int c = ch * kCW + lane * 2;
        const bool in = c < ncols;
        cp_async16(ring + ((ch * kCW) & (kRW - 1)) + lane * 2, row + (in ? c : 0), in ? 16 : 0);
    }
}

__device__ __forceinline__ int round16(int x) { return (x + 15) & ~15; }

// Start step of each row-block in processing order q (multiples of 16 so that
// every row-block stage coincides with one barrier interval):
//   S(q) = max(S(q-1) + kSkew, S(q-NW) + dur16(q-NW));  sched[nRB] = total steps.
__device__ void build_schedule(int* sched, int nRB, int L1, int dur_base, bool reverse) {
    if (threadIdx.x == 0) {
        int prev = -kSkew, total = 0;
        for (int q = 0; q < nRB; ++q) {
            int s = prev + kSkew;
            if (q >= kNW) {
                const int qq = q - kNW;
                const int rr = reverse ? nRB - 1 - qq : qq;
                s = max(s, sched[qq] + round16(dur_base + min(32, L1 - 32 * rr)));
            }
            sched[q] = s;
            prev = s;
            const int r = reverse ? nRB - 1 - q : q;
            total = max(total, s + round16(dur_base + min(32, L1 - 32 * r)));
        }
        sched[nRB] = total;
    }
    __syncthreads();
}

// ==========================================================================
// linear gap, value + marginals
// ==========================================================================
// Forward, row-block r (rows 32r .. 32r+nv-1, 0-based), local step tau:
//   lane l works on column j = tau - l; all lanes share the frame O[tau].
//   Stage k (tau = 16k..16k+15): lane 0 is in chunk k, the trailing lane in
//   chunk >= k-2.  At its start chunk k-3 (finished) is written back as alpha
//   and chunk k+1 of the scores is prefetched into the same ring slot.
// Reverse, row-block r, local step tau, P = 16*ceil((L2-1)/16):
//   lane l works on column j = P - tau + (nv-1-l) (real work only for j <= L2-1);
//   forward frame index tf = P + nv - 1 - tau.  At stage k the leading lane
//   enters chunk n = P/16 - k - 1; chunks n..n+2 are read, chunk n+3 (finished)
//   is written back as marginals and chunk n-1 is prefetched.
__global__ void __launch_bounds__(kNW * 32) lin_marg_kernel(SwArgs p) {
    extern __shared__ __align__(16) unsigned char smem_raw[];
    WarpSmem& W = reinterpret_cast<WarpSmem*>(smem_raw)[threadIdx.x >> 5];
    __shared__ int sched[kMaxRB + 1];
    __shared__ __align__(16) float red[4 * 32];
    __shared__ int sh_Sint;
    __shared__ float sh_Sfrac;

    const int b = blockIdx.x;
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
    const size_t fst = (size_t)L2m + 32;        // frames row stride

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
        }
        return;
    }

    // ============================== forward ==============================
    build_schedule(sched, nRB, L1, L2 - 1, false);
    float acc = 0.f, R = 0.f;   // per-lane partition: sum 2^a = acc * 2^R
    bool haveR = false;
    {
        const int Tf = sched[nRB];
        int q = warp, nv = 0, ld = 0, sta = 0;
        float O = 0.f, dlt = 0.f, dltp = 0.f;
        float left = kNeg, uprev = kNeg, uprecv = kNeg;
        for (int T0 = 0; T0 < Tf; T0 += kSync) {
            if (q < nRB && T0 >= sched[q]) {
                const int r = q;
                const int k = (T0 - sched[q]) >> 4;
                const float* srow = S + (size_t)(32 * r) * L2m;
                const float2* brow = LY.bnd + (size_t)(r - 1) * L2m;
                float* arow = LY.aplane + (size_t)r * abs_;
                if (k == 0) {  // row-block prologue
                    nv = min(32, L1 - 32 * r);
                    O = dlt = dltp = 0.f;
                    left = uprev = uprecv = kNeg;
                    ld = sta = 0;
                    __syncwarp();
                    for (; ld < 2 && ld < nch; ++ld) {
                        load_chunk(W.ringS, srow, L2m, nv, L2, ld, lane);
                        if (r > 0) load_row_chunk8(W.bnd, brow, L2, ld, lane);
                        cp_async_commit();
                    }
                    if (r > 0) {  // start the frame at the row above, column 0
                        cp_async_wait0();
                        __syncwarp();
                        const float2 bv = W.bnd[0];
                        O = bv.y + rintf(bv.x);
                    }
                } else {
                    __syncwarp();
                    // alpha write-back of finished chunks (rows 1..nv of this row-block's tile)
                    while (sta < nch && (sta + 1) * kCW <= 16 * k - (nv - 1)) {
                        store_chunk(W.ringS, arow + L2m, L2m, nv, L2, sta, lane);
                        ++sta;
                    }
                }
                if (ld <= k + 1 && ld < nch) {
                    load_chunk(W.ringS, srow, L2m, nv, L2, ld, lane);
                    if (r > 0) load_row_chunk8(W.bnd, brow, L2, ld, lane);
                    ++ld;
                }
                cp_async_commit();
                cp_async_wait1();
                __syncwarp();

                const bool hasB = r > 0, hasD = r + 1 < nRB;
                float* frow = LY.frames + (size_t)r * fst;
#pragma unroll
                for (int u = 0; u < kCW; ++u) {
                    const int tau = 16 * k + u;
                    const int j0 = tau - lane;
                    const bool act = (lane < nv) & (j0 >= 0) & (j0 < L2);
                    const int ix = lane * kRW + (j0 & (kRW - 1));
                    const float Oprev = O - dlt;
                    float up = uprecv;
                    if (lane == 0) {
                        const float2 bv = W.bnd[j0 & (kRW - 1)];
                        up = hasB ? bv.x + (bv.y - Oprev) : kNeg;  // into frame O[tau-1]
                        if (act) arow[j0] = up;                     // row above, kept for the reverse
                    }
                    const float x = W.ringS[ix] * c;
                    const Lse4 rr = lse4(uprev + x - (dlt + dltp), up + g - dlt, left + g - dlt, x - O);
                    const float aout = act ? rr.a : kNeg;
                    if (act) {
                        W.ringS[ix] = aout;
                        if (!haveR) {
                            R = O;
                            haveR = true;
                        }
                        acc += ex2f(aout + (O - R));
                        if (lane == 31 && hasD) LY.bnd[(size_t)r * L2m + j0] = make_float2(aout, O);
                    }
                    if (lane == 0 && tau < L2 + nv - 1) frow[tau] = O;
                    left = aout;
                    uprev = up;
                    uprecv = __shfl_up_sync(0xffffffffu, aout, 1);
                    // next frame: round the value of the middle active lane
                    const int lo = max(0, tau - L2 + 1), hi = min(nv - 1, tau);
                    const float pv = __shfl_sync(0xffffffffu, aout, (lo + hi) >> 1);
                    const float nd = (pv > kNegThresh) ? rintf(pv) : 0.f;
                    dltp = dlt;
                    dlt = nd;
                    O += nd;
                    if (haveR && O - R > 32.f) {
                        acc *= exp2i((int)(R - O));
                        R = O;
                    }
                }
                if (16 * (k + 1) >= L2 + nv - 1) {  // last stage of this row-block
                    __syncwarp();
                    while (sta < nch) {
                        store_chunk(W.ringS, arow + L2m, L2m, nv, L2, sta, lane);
                        ++sta;
                    }
                    cp_async_wait0();
                    __syncwarp();
                    q += kNW;
                }
            }
            __syncthreads();
        }
    }

    // ---- S = log2(sum_lanes acc*2^R + 2^0), kept as integer + fraction
    {
        const int Rm = (int)block_max(haveR ? fmaxf(R, 0.f) : 0.f, red);
        float part = haveR ? acc * exp2i((int)R - Rm) : 0.f;
        if (threadIdx.x == 0) part += exp2i(-Rm);  // alpha[0,0] = 0
        const float tot = block_sum(part, red);
        if (threadIdx.x == 0) {
            const float l2 = lg2f(tot);
            const float fl = floorf(l2);
            sh_Sint = Rm + (int)fl;
            sh_Sfrac = l2 - fl;
            if (p.value) p.value[b] = ((float)sh_Sint + sh_Sfrac) / c;
        }
        __syncthreads();
    }
    const float Sint = (float)sh_Sint;
    const float Sfrac = sh_Sfrac;

    // ============================== reverse ==============================
    const int P = kCW * ((L2 - 1 + kCW - 1) / kCW);
    build_schedule(sched, nRB, L1, P + 1, true);
    double gsum = 0.0, hsum = 0.0;
    {
        const int Tb = sched[nRB];
        int q = warp, nv = 0, ldn = 0, ldf = 0, stm = 0;
        float pleft = 0.f, pdiag = 0.f, precv = 0.f;
        float f0 = 0.f, f1 = 0.f;
        for (int T0 = 0; T0 < Tb; T0 += kSync) {
            if (q < nRB && T0 >= sched[q]) {
                const int r = nRB - 1 - q;
                const int k = (T0 - sched[q]) >> 4;
                if (k == 0) nv = min(32, L1 - 32 * r);
                const int n = P / kCW - k - 1;       // chunk the leading lane enters
                const int tfs = P + nv - 1 - 16 * k; // frame index at the stage start
                const int nfr = L2 + nv - 1;         // frames recorded for this row-block
                const float* atile = LY.aplane + (size_t)r * abs_;
                const float* srow = S + (size_t)(32 * r) * L2m;
                const float* frow = LY.frames + (size_t)r * fst;
                const float* bbrow = LY.bb + (size_t)(r + 1) * L2m;
                const bool hasBelow = r + 1 < nRB;
                __syncwarp();
                if (k == 0) {
                    pleft = pdiag = precv = 0.f;
                    ldn = nch;
                    ldf = (min(tfs, nfr - 1) >> 4) + 1;
                    stm = nch - 1;
                    while (ldn > max(n, 0)) {  // chunks n..n+2 for this stage
                        --ldn;
                        load_chunk(W.ringA, atile, L2m, nv + 1, L2, ldn, lane);
                        load_chunk(W.ringS, srow, L2m, nv, L2, ldn, lane);
                        if (hasBelow) load_row_chunk4(W.bb, bbrow, L2, ldn, lane);
                    }
                    while (ldf > (max(tfs - 17, 0) >> 4)) {
                        --ldf;
                        load_row_chunk4(W.fr, frow, nfr, ldf, lane);
                    }
                    cp_async_commit();
                } else {
                    while (stm >= 0 && stm >= n + 3) {  // finished marginal chunks
                        if (out) store_chunk(W.ringS, out + (size_t)(32 * r) * L2m, L2m, nv, L2, stm, lane);
                        --stm;
                    }
                }
                while (ldn > max(n - 1, 0)) {  // prefetch for the next stage
                    --ldn;
                    load_chunk(W.ringA, atile, L2m, nv + 1, L2, ldn, lane);
                    load_chunk(W.ringS, srow, L2m, nv, L2, ldn, lane);
                    if (hasBelow) load_row_chunk4(W.bb, bbrow, L2, ldn, lane);
                }
                while (ldf > (max(tfs - 33, 0) >> 4)) {
                    --ldf;
                    load_row_chunk4(W.fr, frow, nfr, ldf, lane);
                }
                cp_async_commit();
                cp_async_wait1();
                __syncwarp();
                if (k == 0) {
                    f0 = W.fr[max(tfs, 0) & (kRW - 1)];
                    f1 = W.fr[max(tfs - 1, 0) & (kRW - 1)];
                }

                float gs = 0.f, hs = 0.f;
#pragma unroll
                for (int u = 0; u < kCW; ++u) {
                    const int tau = 16 * k + u;
                    const int tf = tfs - u;
                    const float f2 = W.fr[max(tf - 2, 0) & (kRW - 1)];
                    const int j0 = P - tau + (nv - 1 - lane);
                    const bool act = (lane < nv) & (j0 >= 0) & (j0 < L2);
                    const int cj = j0 & (kRW - 1), cl = (j0 - 1) & (kRW - 1);
                    const float a = W.ringA[(lane + 1) * kRW + cj];
                    const float al = j0 >= 1 ? W.ringA[(lane + 1) * kRW + cl] : kNeg;
                    const float au = W.ringA[lane * kRW + cj];
                    const float ad = j0 >= 1 ? W.ringA[lane * kRW + cl] : kNeg;
                    const float sc = W.ringS[lane * kRW + cj];
                    const float x = sc * c;
                    const float vs = x - f0, vu = au + (f1 - f0) + g, vl = al + (f1 - f0) + g;
                    const float va = ad + (f2 - f0) + x;
                    const float wu = ex2f(vu - a), wl = ex2f(vl - a), wa = ex2f(va - a), wsk = ex2f(vs - a);
                    const float lp = fminf((a - Sfrac) + (f0 - Sint), 0.f);
                    const float binit = ex2f(lp);
                    float incoming = pleft + precv;
                    if (lane == nv - 1) incoming = pleft + (hasBelow ? W.bb[cj] : 0.f);
                    const float beta = binit + incoming;
                    float send = 0.f, pushdiag = 0.f, pushleft = 0.f;
                    if (act) {
                        W.ringS[lane * kRW + cj] = beta * (wa + wsk);
                        const float pushup = beta * wu;
                        pushdiag = beta * wa;
                        pushleft = beta * wl;
                        send = pushup + pdiag;
                        gs += pushup + pushleft;
                        float h = wsk * (a - vs);
                        if (va > kNegThresh) h += wa * (a - va);
                        if (vu > kNegThresh) h += wu * (a - vu);
                        if (vl > kNegThresh) h += wl * (a - vl);
                        hs += beta * h - binit * lp;
                        if (lane == 0 && r > 0) LY.bb[(size_t)r * L2m + j0] = send;
                    }
                    precv = __shfl_down_sync(0xffffffffu, send, 1);
                    pdiag = pushdiag;
                    pleft = pushleft;
                    f0 = f1;
                    f1 = f2;
                }
                gsum += (double)gs;
                hsum += (double)hs;
                if (16 * (k + 1) >= P + nv) {  // last stage of this row-block
                    __syncwarp();
                    while (stm >= 0) {
                        if (out) store_chunk(W.ringS, out + (size_t)(32 * r) * L2m, L2m, nv, L2, stm, lane);
                        --stm;
                    }
                    cp_async_wait0();
                    __syncwarp();
                    q += kNW;
                }
            }
            __syncthreads();
        }
    }

    if (threadIdx.x == 0) {  // origin alpha[0,0] = 0 as an end state
        const float lp0 = fminf(-Sfrac - Sint, 0.f);
        hsum += (double)ex2f(lp0) * (double)(-lp0);
    }
    const double G = block_sum_d(gsum, reinterpret_cast<double*>(red));
    const double H = block_sum_d(hsum, reinterpret_cast<double*>(red));
    if (threadIdx.x == 0) {
        if (p.grad_gap) p.grad_gap[b] = (float)G;
        if (p.grad_T) p.grad_T[b] = (float)(H * (double)kLn2);
    }
}

}  // namespace wf

// ------------------------------------------------------------------ host side
size_t wavefront_workspace_bytes(int family, int B, int L1, int L2) {
    if (family != 0) return 0;
    if (L1 > 32 * wf::kMaxRB || L2 % 4 != 0) return 0;
    return wf::per_problem_bytes(L1, L2) * (size_t)B;
}

int launch_wavefront(const SwArgs& a, int family, size_t ws_bytes, cudaStream_t st) {
    if (family != 0 || a.mode != MODE_MARG) return -1;
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
    static bool attr_set[64] = {false};
    if (dev < 64 && !attr_set[dev]) {
        e = cudaFuncSetAttribute(wf::lin_marg_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return (int)e;
        attr_set[dev] = true;
    }
    wf::lin_marg_kernel<<<a.B, wf::kNW * 32, smem, st>>>(a);
    return (int)cudaGetLastError();
}

}  // namespace d2pb
