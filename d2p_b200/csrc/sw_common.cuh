// sw_common.cuh -- shared device numerics for the d2p_b200 soft Smith-Waterman kernels.
//
// All DP arithmetic runs in a base-2 scaled log domain: a value alpha (natural
// units, as in the reference) is carried as a = alpha * log2(e) / T, so that
//   LSE_T(x_1..x_n) = T * ln(sum_k exp(x_k / T))        (reference numerics.cuh:45-76)
// becomes
//   a = m + log2(sum_k 2^(v_k - m)),   v_k = x_k * log2(e) / T,   m = max_k v_k
// and every exponential / logarithm is one MUFU instruction (ex2.approx.ftz /
// lg2.approx.ftz).  The reference's safe_exp clamp at -88 (numerics.cuh:34-39)
// maps to 2^-126.96; ex2.approx.ftz already flushes results below 2^-126 to 0,
// so the clamp is implicit.  The reference's NINF = -1e30 sentinel is kept as a
// sentinel in the scaled domain.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

namespace d2pb {

constexpr float kNeg = -1e30f;            // "-inf" sentinel (reference NINF)
constexpr float kNegThresh = -1e29f;      // anything below is treated as -inf
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLn2 = 0.6931471805599453f;

__device__ __forceinline__ float ex2f(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

__device__ __forceinline__ float lg2f(float x) {
    float y;
    asm("lg2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

__device__ __forceinline__ float rcpf(float x) {
    float y;
    asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

// 4-way scaled logsumexp; also returns the unnormalised terms t_k = 2^(v_k - m)
// and their sum so that callers can form softmax weights w_k = t_k / sum.
struct Lse4 {
    float a, t0, t1, t2, t3, sum;
};

__device__ __forceinline__ Lse4 lse4(float v0, float v1, float v2, float v3) {
    Lse4 r;
    float m = fmaxf(fmaxf(v0, v1), fmaxf(v2, v3));
    r.t0 = ex2f(v0 - m);
    r.t1 = ex2f(v1 - m);
    r.t2 = ex2f(v2 - m);
    r.t3 = ex2f(v3 - m);
    r.sum = (r.t0 + r.t1) + (r.t2 + r.t3);
    r.a = m + lg2f(r.sum);
    if (m <= kNegThresh) r.a = kNeg;
    return r;
}

struct Lse2 {
    float a, t0, t1, sum;
};

__device__ __forceinline__ Lse2 lse2(float v0, float v1) {
    Lse2 r;
    float m = fmaxf(v0, v1);
    r.t0 = ex2f(v0 - m);
    r.t1 = ex2f(v1 - m);
    r.sum = r.t0 + r.t1;
    r.a = m + lg2f(r.sum);
    if (m <= kNegThresh) {
        r.a = kNeg;
        r.t0 = r.t1 = 0.f;
        r.sum = 1.f;
    }
    return r;
}

// ---------------------------------------------------------------------------
// Block reductions (deterministic: fixed shuffle tree, fixed warp order).
// ---------------------------------------------------------------------------
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

// Sum over the block; every thread gets the result.  `scratch` needs one
// float per warp.  Contains the trailing barrier that makes back-to-back
// calls safe (the write-after-read hazard the reference fixed in
// src/common/reduce.cuh:179-183 cannot occur).
__device__ __forceinline__ float block_sum(float v, float* scratch) {
    const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5, nw = (blockDim.x + 31) >> 5;
    v = warp_sum(v);
    if (lane == 0) scratch[wid] = v;
    __syncthreads();
    float r = 0.f;
    for (int w = 0; w < nw; ++w) r += scratch[w];
    __syncthreads();
    return r;
}

__device__ __forceinline__ double warp_sum_d(double v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

// Double-precision block sum (scratch: one double per warp).  Used for the
// per-problem expectation sums behind dS/dgap and dS/dT, which feed a
// cancellation (S - E[score]) / T.
__device__ __forceinline__ double block_sum_d(double v, double* scratch) {
    const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5, nw = (blockDim.x + 31) >> 5;
    v = warp_sum_d(v);
    if (lane == 0) scratch[wid] = v;
    __syncthreads();
    double r = 0.0;
    for (int w = 0; w < nw; ++w) r += scratch[w];
    __syncthreads();
    return r;
}

__device__ __forceinline__ float block_max(float v, float* scratch) {
    const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5, nw = (blockDim.x + 31) >> 5;
    v = warp_max(v);
    if (lane == 0) scratch[wid] = v;
    __syncthreads();
    float r = kNeg;
    for (int w = 0; w < nw; ++w) r = fmaxf(r, scratch[w]);
    __syncthreads();
    return r;
}

// Online base-2 log-sum-exp accumulator: represents sum_k 2^(a_k) as
// s * 2^m, plus optional companion sums  sum_k 2^(a_k) * y_k  (same scale).
struct OnlineLse {
    float m, s, y1, y2;
    __device__ __forceinline__ void init() { m = kNeg; s = 0.f; y1 = 0.f; y2 = 0.f; }
    __device__ __forceinline__ void add(float a, float ya = 0.f, float yb = 0.f) {
        if (a <= kNegThresh) return;
        if (a > m) {
            float f = ex2f(m - a);
            s = s * f + 1.f;
            y1 = y1 * f + ya;
            y2 = y2 * f + yb;
            m = a;
        } else {
            float e = ex2f(a - m);
            s += e;
            y1 += e * ya;
            y2 += e * yb;
        }
    }
    __device__ __forceinline__ void merge(const OnlineLse& o) {
        if (o.m <= kNegThresh) return;
        if (m <= kNegThresh) { *this = o; return; }
        if (o.m > m) {
            float f = ex2f(m - o.m);
            s = s * f + o.s; y1 = y1 * f + o.y1; y2 = y2 * f + o.y2; m = o.m;
        } else {
            float f = ex2f(o.m - m);
            s += o.s * f; y1 += o.y1 * f; y2 += o.y2 * f;
        }
    }
};

__device__ __forceinline__ OnlineLse shfl_xor_lse(const OnlineLse& v, int o) {
    OnlineLse r;
    r.m = __shfl_xor_sync(0xffffffffu, v.m, o);
    r.s = __shfl_xor_sync(0xffffffffu, v.s, o);
    r.y1 = __shfl_xor_sync(0xffffffffu, v.y1, o);
    r.y2 = __shfl_xor_sync(0xffffffffu, v.y2, o);
    return r;
}

// Block-wide merge of OnlineLse; all threads receive the result.
// `scratch` must hold 4 floats per warp.
__device__ __forceinline__ OnlineLse block_lse(OnlineLse v, float* scratch) {
    const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5, nw = (blockDim.x + 31) >> 5;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v.merge(shfl_xor_lse(v, o));
    if (lane == 0) {
        scratch[4 * wid + 0] = v.m;
        scratch[4 * wid + 1] = v.s;
        scratch[4 * wid + 2] = v.y1;
        scratch[4 * wid + 3] = v.y2;
    }
    __syncthreads();
    OnlineLse r;
    r.init();
    for (int w = 0; w < nw; ++w) {
        OnlineLse q;
        q.m = scratch[4 * w + 0];
        q.s = scratch[4 * w + 1];
        q.y1 = scratch[4 * w + 2];
        q.y2 = scratch[4 * w + 3];
        r.merge(q);
    }
    __syncthreads();
    return r;
}

}  // namespace d2pb
