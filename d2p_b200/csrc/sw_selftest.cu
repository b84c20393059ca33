// sw_selftest.cu -- diagnostic entry point for the bounded device waits.
//
// Every wait of the kernels on a progress word gives up after kSpinLimit polls
// (sw_ring.cuh) and records that in an error word. wait_flag waits on a word in
// shared memory, written by another warp of the same CTA. wait_flag_gpu waits on
// a global word written by another CTA of a cooperative launch. The kernel then
// flags its problem, and the caller recomputes the problem with the plane
// engine.
//
// d2p_wait_selftest runs those same helpers on a word that nothing ever sets.
// A test can then check, on a real device, that the wait ends, that the error
// is reported, and that the context stays usable afterwards.
//
// d2p_mufu_probe measures the throughput of the MUFU pipe's ex2.approx, the
// denominator of the kernels' transcendental roofline: every thread runs
// kProbeChains independent ex2 chains, so the pipe, not their latency, limits it.
#include "../../include/d2p_b200.h"
#include "sw_common.cuh"
#include "sw_internal.h"
#include "sw_ring.cuh"

namespace d2pb {

__global__ void __launch_bounds__(64) wait_selftest_kernel(int scope, const int* __restrict__ word,
                                                           int* __restrict__ status) {
    __shared__ int sh_flag, sh_err;
    if (threadIdx.x == 0) {
        sh_flag = 0;  // never set
        sh_err = 0;
    }
    __syncthreads();
    if (threadIdx.x < 32) {  // one warp waits, as a kernel's reading warp does
        if (scope == 0)
            ring::wait_flag(&sh_flag, 1, &sh_err);
        else
            ring::wait_flag_gpu(word, 1, &sh_err);
    }
    __syncthreads();
    if (threadIdx.x == 0) *status = sh_err;
}

constexpr int kProbeThreads = D2P_MUFU_PROBE_THREADS;
constexpr int kProbeChains = D2P_MUFU_PROBE_CHAINS;

__global__ void __launch_bounds__(kProbeThreads) mufu_probe_kernel(float* __restrict__ out, int iters) {
    float x[kProbeChains];
#pragma unroll
    for (int k = 0; k < kProbeChains; ++k) x[k] = -1e-7f * (float)(threadIdx.x * kProbeChains + k);
    for (int i = 0; i < iters; ++i) {
#pragma unroll
        for (int k = 0; k < kProbeChains; ++k) x[k] = ex2f(-x[k]);  // stays in (0.5, 1]
    }
    float acc = 0.f;
#pragma unroll
    for (int k = 0; k < kProbeChains; ++k) acc += x[k];
    out[(size_t)blockIdx.x * kProbeThreads + threadIdx.x] = acc;
}

}  // namespace d2pb

extern "C" int d2p_mufu_probe(float* out, int blocks, int iters, void* stream) {
    if (!out || blocks <= 0 || iters <= 0) return D2P_ERR_INVALID_ARGUMENT;
    d2pb::mufu_probe_kernel<<<blocks, d2pb::kProbeThreads, 0, (cudaStream_t)stream>>>(out, iters);
    return (int)cudaGetLastError();
}

extern "C" int d2p_wait_selftest(int scope, const int* word, int* status, void* stream) {
    if ((scope != 0 && scope != 1) || !status || (scope == 1 && !word)) return D2P_ERR_INVALID_ARGUMENT;
    d2pb::wait_selftest_kernel<<<1, 64, 0, (cudaStream_t)stream>>>(scope, word, status);
    return (int)cudaGetLastError();
}
