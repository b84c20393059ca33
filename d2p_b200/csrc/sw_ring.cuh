// sw_ring.cuh -- building blocks shared by the row-block wavefront kernels
// (sw_wavefront.cu: log-domain; sw_linear.cu: linear-domain fast path).
//
//  * cp.async helpers and per-row-block tile copies between a row-major plane
//    and a per-warp [rows][64] shared ring (one 16-column chunk at a time);
//  * CTA-scope release/acquire progress words with bounded waits;
//  * exact power-of-two construction and a range-reduced lg2.
#pragma once
#include <stdint.h>

#include "sw_common.cuh"

namespace d2pb {
namespace ring {

constexpr int kCW = 16;                  // chunk width (columns) = steps per stage
constexpr int kRW = 64;                  // ring width (columns) = row stride of the rings (4 chunks)
constexpr int kStageMask = 0xffff;       // progress word = (row-block ordinal << 16) | stages done
constexpr int kSpinLimit = 1 << 20;      // bounded waits (polls of ~40 ns)
constexpr unsigned kAll = 0xffffffffu;

__host__ __device__ inline size_t align_up(size_t x, size_t a) { return (x + a - 1) / a * a; }

// ---------------------------------------------------------------- cp.async
__device__ __forceinline__ void cp_async16(void* smem, const void* gmem, int src_bytes) {
    const unsigned s = (unsigned)__cvta_generic_to_shared(smem);
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(s), "l"(gmem), "r"(src_bytes));
}
__device__ __forceinline__ void cp_async4(void* smem, const void* gmem) {
    const unsigned s = (unsigned)__cvta_generic_to_shared(smem);
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4;\n" ::"r"(s), "l"(gmem));
}
// 4 bytes, or zeros when src_bytes is 0 (gmem must still be a valid address)
__device__ __forceinline__ void cp_async4_zfill(float* smem, const float* gmem, int src_bytes) {
    const unsigned s = (unsigned)__cvta_generic_to_shared(smem);
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4, %2;\n" ::"r"(s), "l"(gmem), "r"(src_bytes));
}
// bring a 128-byte line into L2 ahead of a cp.async that will read it
__device__ __forceinline__ void prefetch_l2(const void* gmem) {
    asm volatile("prefetch.global.L2 [%0];\n" ::"l"(gmem));
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::); }
// The waits are compiler memory barriers as well: shared-memory reads of the
// copied data must not be moved above them.
__device__ __forceinline__ void cp_async_wait1() { asm volatile("cp.async.wait_group 1;\n" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait2() { asm volatile("cp.async.wait_group 2;\n" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait0() { asm volatile("cp.async.wait_group 0;\n" ::: "memory"); }

// ---------------------------------------------------------------- progress flags
__device__ __forceinline__ int ld_acquire(const int* p) {
    int v;
    asm volatile("ld.acquire.cta.shared::cta.b32 %0, [%1];\n"
                 : "=r"(v)
                 : "r"((unsigned)__cvta_generic_to_shared(p))
                 : "memory");
    return v;
}
__device__ __forceinline__ void st_release(int* p, int v) {
    asm volatile("st.release.cta.shared::cta.b32 [%0], %1;\n" ::"r"((unsigned)__cvta_generic_to_shared(p)), "r"(v)
                 : "memory");
}
// Wait (all lanes) until *flag >= need.  Gives up after kSpinLimit polls and
// records the failure in *err, so a broken dependency can never hang the GPU.
__device__ __forceinline__ void wait_flag(const int* flag, int need, int* err) {
    int it = 0;
    if (*(volatile int*)err) {  // an earlier wait already gave up: do not stall again
        __syncwarp();
        return;
    }
    while (ld_acquire(flag) < need) {
        if (++it > kSpinLimit) {
            *err = 1;
            break;
        }
        __nanosleep(40);
    }
    __syncwarp();
}

// The same progress words in global memory, at GPU scope: between the CTAs
// that share one problem (every CTA of such a launch is resident at once: it
// is a cooperative launch).
__device__ __forceinline__ int ld_acquire_gpu(const int* p) {
    int v;
    asm volatile("ld.acquire.gpu.global.b32 %0, [%1];\n" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ void st_release_gpu(int* p, int v) {
    asm volatile("st.release.gpu.global.b32 [%0], %1;\n" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ int atom_add_release_gpu(int* p, int v) {
    int old;
    asm volatile("atom.add.release.gpu.global.s32 %0, [%1], %2;\n" : "=r"(old) : "l"(p), "r"(v) : "memory");
    return old;
}
// wait_flag on a global word (all lanes; bounded like wait_flag)
__device__ __forceinline__ void wait_flag_gpu(const int* flag, int need, int* err) {
    int it = 0;
    if (*(volatile int*)err) {
        __syncwarp();
        return;
    }
    while (ld_acquire_gpu(flag) < need) {
        if (++it > kSpinLimit) {
            *err = 1;
            break;
        }
        __nanosleep(64);
    }
    __syncwarp();
}

// One lane's group handoff into shared memory: four values and a frame word,
// stored under a predicate (no branch) so the other lanes only pay one issue.
__device__ __forceinline__ void sts_group_pred_s(unsigned a, unsigned b, float4 v, float fr, bool pr) {
    asm volatile(
        "{\n .reg .pred q;\n setp.ne.b32 q, %6, 0;\n"
        " @q st.shared.v4.f32 [%0], {%2, %3, %4, %5};\n"
        " @q st.shared.f32 [%1], %7;\n}\n" ::"r"(a),
        "r"(b), "f"(v.x), "f"(v.y), "f"(v.z), "f"(v.w), "r"((int)pr), "f"(fr)
        : "memory");
}
__device__ __forceinline__ void sts_v4_pred_s(unsigned a, float4 v, bool pr) {
    asm volatile(
        "{\n .reg .pred q;\n setp.ne.b32 q, %5, 0;\n"
        " @q st.shared.v4.f32 [%0], {%1, %2, %3, %4};\n}\n" ::"r"(a),
        "f"(v.x), "f"(v.y), "f"(v.z), "f"(v.w), "r"((int)pr)
        : "memory");
}
__device__ __forceinline__ void sts_group_pred(float* v4, float* f, float4 v, float fr, bool pr) {
    const unsigned a = (unsigned)__cvta_generic_to_shared(v4);
    const unsigned b = (unsigned)__cvta_generic_to_shared(f);
    asm volatile(
        "{\n .reg .pred q;\n setp.ne.b32 q, %6, 0;\n"
        " @q st.shared.v4.f32 [%0], {%2, %3, %4, %5};\n"
        " @q st.shared.f32 [%1], %7;\n}\n" ::"r"(a),
        "r"(b), "f"(v.x), "f"(v.y), "f"(v.z), "f"(v.w), "r"((int)pr), "f"(fr));
}

// The same handoff into global memory (the neighbouring row-block stages it
// with cp.async one stage ahead)
__device__ __forceinline__ void stg_group_pred(float* v4, float* f, float4 v, float fr, bool pr) {
    asm volatile(
        "{\n .reg .pred q;\n setp.ne.b32 q, %6, 0;\n"
        " @q st.global.v4.f32 [%0], {%2, %3, %4, %5};\n"
        " @q st.global.f32 [%1], %7;\n}\n" ::"l"(v4),
        "l"(f), "f"(v.x), "f"(v.y), "f"(v.z), "f"(v.w), "r"((int)pr), "f"(fr)
        : "memory");
}
// two values per step and one frame (the affine kernel's handoff)
__device__ __forceinline__ void stg_pair_pred(float* a4, float* b4, float* f, float4 a, float4 b, float fr, bool pr) {
    asm volatile(
        "{\n .reg .pred q;\n setp.ne.b32 q, %11, 0;\n"
        " @q st.global.v4.f32 [%0], {%3, %4, %5, %6};\n"
        " @q st.global.v4.f32 [%1], {%7, %8, %9, %10};\n"
        " @q st.global.f32 [%2], %12;\n}\n" ::"l"(a4),
        "l"(b4), "l"(f), "f"(a.x), "f"(a.y), "f"(a.z), "f"(a.w), "f"(b.x), "f"(b.y), "f"(b.z), "f"(b.w),
        "r"((int)pr), "f"(fr)
        : "memory");
}

// log2 of a positive normal float, with the exponent split off exactly so that
// lg2.approx only sees the mantissa in [1, 2), where its error is absolute.
__device__ __forceinline__ float lg2_rr(float s) {
    const int bits = __float_as_int(s);
    const float m = __int_as_float((bits & 0x007fffff) | 0x3f800000);
    return (float)((bits >> 23) - 127) + lg2f(m);
}

__device__ __forceinline__ float exp2i(int k) {  // exact 2^k for k in [-126, 127]; 0 below
    return __int_as_float((127 + min(max(k, -127), 127)) << 23);
}

// A lane's share of copying a [rows][16] chunk between a row-major plane and a
// [rows][64] ring: rows lane/4 + 8i (i < nit), columns 4*(lane%4) .. +3.
// Addresses are set up once per row-block; a chunk copy is then a few
// cp.async / vector loads and stores at immediate offsets.
struct Tile {
    const char* g0;   // plane element (row lane/4, column 4*(lane%4))
    size_t g8;        // bytes from row r to row r + 8
    unsigned s0;      // shared address of ring element (row lane/4, column 4*(lane%4))
    int c0;           // 4*(lane%4)
    int nit;          // rows lane/4 + 8i exist for i < nit
};

__device__ __forceinline__ Tile make_tile(const float* plane, int ld, const float* ring, int nrows, int lane) {
    Tile t;
    const int r0 = lane >> 2;
    t.c0 = 4 * (lane & 3);
    t.g0 = reinterpret_cast<const char*>(plane + (size_t)r0 * ld + t.c0);
    t.g8 = (size_t)8 * ld * sizeof(float);
    t.s0 = (unsigned)__cvta_generic_to_shared(ring + r0 * kRW + t.c0);
    t.nit = nrows > r0 ? (nrows - r0 + 7) / 8 : 0;
    return t;
}

__device__ __forceinline__ void cp_async16_s(unsigned s, const void* g, int src_bytes) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(s), "l"(g), "r"(src_bytes));
}

// chunk ch (columns [16ch, 16ch+16)) plane -> ring; columns >= ncols zero-filled, not read
template <int NI>
__device__ __forceinline__ void tile_load(const Tile& t, int ch, int ncols) {
    const bool in = kCW * ch + t.c0 < ncols;
    const char* g = t.g0 + (in ? (size_t)(kCW * ch) * sizeof(float) : 0);
    const unsigned s = t.s0 + (unsigned)(((kCW * ch) & (kRW - 1)) * sizeof(float));
    const int nb = in ? 16 : 0;
#pragma unroll
    for (int i = 0; i < NI; ++i)
        if (i < t.nit) cp_async16_s(s + i * 8 * kRW * sizeof(float), g + i * t.g8, nb);
}

// chunk ch ring -> plane (columns < ncols only)
__device__ __forceinline__ void tile_store(const Tile& t, int ch, int ncols) {
    const int c = kCW * ch + t.c0;
    if (c >= ncols) return;
    char* g = const_cast<char*>(t.g0) + (size_t)(kCW * ch) * sizeof(float);
    const unsigned s = t.s0 + (unsigned)(((kCW * ch) & (kRW - 1)) * sizeof(float));
    const bool whole = c + 4 <= ncols;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        if (i < t.nit) {
            float4 v;
            asm volatile("ld.shared.v4.f32 {%0, %1, %2, %3}, [%4];\n"
                         : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
                         : "r"(s + i * 8 * kRW * (unsigned)sizeof(float)));
            float* dst = reinterpret_cast<float*>(g + i * t.g8);
            if (whole) {
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

}  // namespace ring
}  // namespace d2pb
