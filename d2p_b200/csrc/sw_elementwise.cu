// sw_elementwise.cu -- the value-branch backward and small deterministic reductions.
//
// value backward (replaces the torch ops in the reference's
// SoftSWRegularCUDAFunction::backward value branch, src/sw/torch_cuda.cpp:292-321,
// which re-ran the whole reverse DP; d2p/_pt2_ops.py:180 shows that reusing the
// saved marginals is the same gradient):
//     grad_scores[b,i,j] = grad_value[b] * marginals[b,i,j]
//     grad_param[p]      = sum_b grad_value[b] * dvalue_dparam[p,b]
// HBM-bound: 8 bytes per cell (read marginals, write grad), 128-bit accesses,
// grid sized to a multiple of the SM count.
#include "sw_common.cuh"
#include "sw_internal.h"

namespace d2pb {

__global__ void __launch_bounds__(256) value_backward_kernel(const float* __restrict__ g,
                                                             const float* __restrict__ marg,
                                                             const float* __restrict__ dparams,
                                                             int n_params, int B, size_t plane,
                                                             float* __restrict__ out,
                                                             float* __restrict__ gparams) {
    const size_t total = (size_t)B * plane;
    const size_t tid = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    const size_t stride = (size_t)gridDim.x * blockDim.x;
    const bool vec = ((plane & 3) == 0) && ((((uintptr_t)marg) | ((uintptr_t)out)) & 15) == 0;
    if (vec) {
        const size_t n4 = total >> 2;
        const float4* __restrict__ m4 = reinterpret_cast<const float4*>(marg);
        float4* __restrict__ o4 = reinterpret_cast<float4*>(out);
        for (size_t q = tid; q < n4; q += stride) {
            const size_t b = (q << 2) / plane;
            const float gb = __ldg(g + b);
            float4 v = __ldcs(m4 + q);  // streamed: read once
            v.x *= gb; v.y *= gb; v.z *= gb; v.w *= gb;
            __stcs(o4 + q, v);
        }
    } else {
        for (size_t q = tid; q < total; q += stride) out[q] = __ldg(g + q / plane) * marg[q];
    }
    if (blockIdx.x == 0 && threadIdx.x < 32 && n_params > 0 && gparams) {
        // fixed-order reduction: lane-strided partial sums, then a shuffle tree
        for (int pi = 0; pi < n_params; ++pi) {
            float acc = 0.f;
            for (int b = threadIdx.x; b < B; b += 32) acc += g[b] * dparams[(size_t)pi * B + b];
            acc = warp_sum(acc);
            if (threadIdx.x == 0) gparams[pi] = acc;
        }
    }
}

// The same with per-problem lengths: one warp per row; cells outside the
// problem (marginals 0 there) are written as 0 without being read, which saves
// the read of a ragged batch's padding.
__global__ void __launch_bounds__(256) value_backward_rows_kernel(const float* __restrict__ g,
                                                                  const float* __restrict__ marg,
                                                                  const int* __restrict__ lengths, int B, int L1,
                                                                  int L2, float* __restrict__ out,
                                                                  const float* __restrict__ dparams, int n_params,
                                                                  float* __restrict__ gparams) {
    const int lane = threadIdx.x & 31;
    const long long rows = (long long)B * L1;
    const long long w0 = ((long long)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const long long nw = ((long long)gridDim.x * blockDim.x) >> 5;
    const bool vec = (L2 & 3) == 0 && ((((uintptr_t)marg) | ((uintptr_t)out)) & 15) == 0;
    for (long long row = w0; row < rows; row += nw) {
        const int b = (int)(row / L1), i = (int)(row - (long long)b * L1);
        const int l1 = min(max(lengths[2 * b], 0), L1), l2 = min(max(lengths[2 * b + 1], 0), L2);
        const int valid = i < l1 ? l2 : 0;  // columns [0, valid) hold marginals
        const float gb = __ldg(g + b);
        const size_t base = (size_t)row * L2;
        if (vec) {
            const float4* __restrict__ m4 = reinterpret_cast<const float4*>(marg + base);
            float4* __restrict__ o4 = reinterpret_cast<float4*>(out + base);
            for (int c = lane; c < (L2 >> 2); c += 32) {
                float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
                if (4 * c < valid) {
                    v = __ldcs(m4 + c);
                    v.x *= gb;
                    v.y = 4 * c + 1 < valid ? v.y * gb : 0.f;
                    v.z = 4 * c + 2 < valid ? v.z * gb : 0.f;
                    v.w = 4 * c + 3 < valid ? v.w * gb : 0.f;
                }
                __stcs(o4 + c, v);
            }
        } else {
            for (int c = lane; c < L2; c += 32) out[base + c] = c < valid ? gb * marg[base + c] : 0.f;
        }
    }
    if (blockIdx.x == 0 && threadIdx.x < 32 && n_params > 0 && gparams) {  // as value_backward_kernel
        for (int pi = 0; pi < n_params; ++pi) {
            float acc = 0.f;
            for (int b = threadIdx.x; b < B; b += 32) acc += g[b] * dparams[(size_t)pi * B + b];
            acc = warp_sum(acc);
            if (threadIdx.x == 0) gparams[pi] = acc;
        }
    }
}

// out[p] (+)= sum_b partials[p*B + b], deterministic (one warp).
__global__ void sum_batches_kernel(const float* __restrict__ partials, int P, int B,
                                   float* __restrict__ out, int accumulate) {
    for (int pi = 0; pi < P; ++pi) {
        float acc = 0.f;
        for (int b = threadIdx.x; b < B; b += 32) acc += partials[(size_t)pi * B + b];
        acc = warp_sum(acc);
        if (threadIdx.x == 0) out[pi] = accumulate ? out[pi] + acc : acc;
    }
}

// Row repacking for kernels that move rows by TMA (16-byte row strides): one
// warp per row, 4-byte coalesced loads and stores.  pad: in [B][L1][L2] ->
// out [B][L1p][L2p] with zeros in the added rows and columns; unpad: the
// [L1][L2] corner of each padded problem back to [B][L1][L2].
__global__ void __launch_bounds__(256) pad_rows_kernel(const float* __restrict__ in, int L1, int L2,
                                                       float* __restrict__ out, int L1p, int L2p,
                                                       long long rows) {
    const int lane = threadIdx.x & 31;
    const long long w0 = (long long)blockIdx.x * 8 + (threadIdx.x >> 5), ws = (long long)gridDim.x * 8;
    for (long long r = w0; r < rows; r += ws) {
        const long long b = r / L1p;
        const int i = (int)(r - b * L1p);
        float* __restrict__ o = out + r * L2p;
        const float* __restrict__ s = in + (b * L1 + i) * (long long)L2;
        const int n = i < L1 ? L2 : 0;
#pragma unroll 4
        for (int j = lane; j < L2p; j += 32) o[j] = j < n ? __ldg(s + j) : 0.f;
    }
}

__global__ void __launch_bounds__(256) unpad_rows_kernel(const float* __restrict__ in, int L1p, int L2p,
                                                         float* __restrict__ out, int L1, int L2,
                                                         long long rows) {
    const int lane = threadIdx.x & 31;
    const long long w0 = (long long)blockIdx.x * 8 + (threadIdx.x >> 5), ws = (long long)gridDim.x * 8;
    for (long long r = w0; r < rows; r += ws) {
        const long long b = r / L1;
        const int i = (int)(r - b * L1);
        const float* __restrict__ s = in + (b * L1p + i) * (long long)L2p;
        float* __restrict__ o = out + r * L2;
#pragma unroll 4
        for (int j = lane; j < L2; j += 32) __stcs(o + j, __ldcs(s + j));
    }
}

static int grid_for(size_t work_items) {
    int dev = 0, sms = 148;
    if (cudaGetDevice(&dev) == cudaSuccess) {
        int v = 0;
        if (cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev) == cudaSuccess && v > 0) sms = v;
    }
    size_t want = (work_items + 255) / 256;
    size_t cap = (size_t)sms * 8;  // 8 resident CTAs of 256 threads per SM
    if (want > cap) want = cap;
    if (want < 1) want = 1;
    return (int)want;
}

int launch_value_backward_rows(const float* grad_value, const float* marginals, const int* lengths,
                               const float* dparams, int n_params, int B, int L1, int L2,
                               float* grad_scores, float* grad_params, cudaStream_t st) {
    if (!lengths || (long long)B * L1 == 0 || L2 == 0)
        return launch_value_backward(grad_value, marginals, dparams, n_params, B, L1, L2, grad_scores,
                                     grad_params, st);
    const int grid = grid_for((size_t)B * L1 * 32);
    value_backward_rows_kernel<<<grid, 256, 0, st>>>(grad_value, marginals, lengths, B, L1, L2, grad_scores,
                                                     dparams, n_params, grad_params);
    return (int)cudaGetLastError();
}

int launch_value_backward(const float* grad_value, const float* marginals, const float* dparams,
                          int n_params, int B, int L1, int L2, float* grad_scores,
                          float* grad_params, cudaStream_t st) {
    const size_t plane = (size_t)L1 * L2;
    const size_t total = (size_t)B * plane;
    if (total == 0 && n_params == 0) return 0;
    const int grid = grid_for(total / 4 + 1);
    value_backward_kernel<<<grid, 256, 0, st>>>(grad_value, marginals, dparams, n_params, B,
                                                plane > 0 ? plane : 1, grad_scores, grad_params);
    return (int)cudaGetLastError();
}

int launch_pad_rows(const float* in, int B, int L1, int L2, float* out, int L1p, int L2p, cudaStream_t st) {
    const long long rows = (long long)B * L1p;
    if (rows == 0 || L2p == 0) return 0;
    pad_rows_kernel<<<grid_for((size_t)rows * 32), 256, 0, st>>>(in, L1, L2, out, L1p, L2p, rows);
    return (int)cudaGetLastError();
}

int launch_unpad_rows(const float* in, int L1p, int L2p, float* out, int B, int L1, int L2, cudaStream_t st) {
    const long long rows = (long long)B * L1;
    if (rows == 0 || L2 == 0) return 0;
    unpad_rows_kernel<<<grid_for((size_t)rows * 32), 256, 0, st>>>(in, L1p, L2p, out, L1, L2, rows);
    return (int)cudaGetLastError();
}

__global__ void or_flags_kernel(int* __restrict__ a, const int* __restrict__ b, int n) {
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) a[i] |= b[i];
}

int launch_or_flags(int* a, const int* b, int n, cudaStream_t st) {
    if (n <= 0) return 0;
    or_flags_kernel<<<(n + 255) / 256 < 148 ? (n + 255) / 256 : 148, 256, 0, st>>>(a, b, n);
    return (int)cudaGetLastError();
}

int launch_sum_batches(const float* partials, int P, int B, float* out, int accumulate,
                       cudaStream_t st) {
    sum_batches_kernel<<<1, 32, 0, st>>>(partials, P, B, out, accumulate);
    return (int)cudaGetLastError();
}

}  // namespace d2pb
