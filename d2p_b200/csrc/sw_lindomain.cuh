// sw_lindomain.cuh -- pieces shared by the linear-domain kernels
// (sw_linear.cu, sw_affine_fast.cu, sw_tangent.cu): power-of-two frames held
// as integer-valued floats, the partition accumulator's base, and the row
// counts of the per-row-block workspace planes.
#pragma once

#include "sw_common.cuh"
#include "sw_ring.cuh"

namespace d2pb {
namespace ld {

constexpr int kJMax = 60;   // largest frame step (log2) a problem may take per group of 4 steps
constexpr int kHR = 128;    // staging ring of a neighbour's boundary values (steps; 8 stage slots)

// Row counts cover every row the staging reaches past the last step (up to 46
// rows past L2, and 12 frame groups).
__host__ __device__ inline int zt_rows(int L2m) { return L2m + 96; }
__host__ __device__ inline int gt_rows(int L2m) { return (L2m + 96) / 4; }
// boundary rows are stored and staged in 16-byte pieces: strides in whole float4s
__host__ __device__ inline int hz_stride(int L2m) { return (zt_rows(L2m) + 3) & ~3; }
__host__ __device__ inline int hf_stride(int L2m) { return (gt_rows(L2m) + 3) & ~3; }

// Frames are integer-valued floats: 2^k is one MUFU ex2, exact for integer k
// in [-126, 127] (0 below, +inf above; checked on the B200 for |k| <= 150).
__device__ __forceinline__ float p2(float k) { return ex2f(k); }

// Frame steps come from the exponent field of the lane's previous value: for
// v = m 2^J (m in [1, 2)) the field is the bit pattern of 2^J, so 2^J, 2^-J
// and J cost one integer operation each.  Zero (a lane that has not started)
// reads as J = 0.
__device__ __forceinline__ int efield(float v) {
    const int b = __float_as_int(v) & 0x7f800000;
    return b ? b : 0x3f800000;
}
__device__ __forceinline__ float inv_p2(float w) { return __int_as_float(0x7f000000 - __float_as_int(w)); }
// 2^E as a double (|E| <= 1022; larger frames flag the problem)
__device__ __forceinline__ double p2d(float E) {
    return __hiloint2double((min(max(__float2int_rn(E), -1022), 1023) + 1023) << 20, 0);
}
// J of an exponent field (eb = bits of 2^J) as a float: exact
__device__ __forceinline__ float efield_j(int eb) { return fmaf((float)eb, 1.0f / 8388608.0f, -127.f); }

// Once per stage: move the partition's base up with the frames (a group's
// frame moves by at most kJMax, so E - ab stays below 700 + 4 kJMax until the
// next check).  Frames far below the base add nothing visible to acc.
__device__ __forceinline__ void acc_rebase(double& acc, float& ab, float E) {
    if (E - ab > 700.f) {
        acc *= p2d(ab - E);
        ab = E;
    }
}

}  // namespace ld
}  // namespace d2pb
