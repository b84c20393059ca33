// sw_noalloc.cu -- linear value + marginals with library-owned scratch.
//
// d2p_sw_forward_backward needs a caller workspace.  Some callers cannot
// provide one: a host program with no device allocator of its own (a plain C,
// cgo or FFI caller) would have to cudaMalloc/cudaFree around every call, and
// those calls synchronize the whole device and cost more than the kernel for
// small batches; a process whose device memory is already handed out to a
// fixed pool has nothing left to allocate from.  This entry point serves them:
// its scratch is a fixed-size array in the library's own device image, so a
// call allocates nothing.
//
// Rules for callers:
//   * the scratch is one array per device, shared by every call on that device:
//     calls that overlap on the GPU (on different streams, or from different
//     host threads) race on it and produce wrong results.  Order them on one
//     stream, or use d2p_sw_forward_backward with separate workspaces;
//   * the first call on a device looks up the array's address on that device
//     (cudaGetSymbolAddress with the caller's device current); make that first
//     call before any stream capture;
//   * sizes whose workspace (d2p_sw_workspace_bytes for the linear
//     forward/backward) exceeds D2P_STATIC_SCRATCH_BYTES are rejected with
//     D2P_ERR_WORKSPACE_TOO_SMALL before any device work.
// What must start at zero is cleared inside each call: when the call spreads
// a few large problems over several CTAs, the launcher zeroes their cross-CTA
// progress words, barrier counters and recompute flags with cudaMemsetAsync
// on the caller's stream; every other scratch word is written before it is read.
#include <mutex>

#include "../../include/d2p_b200.h"
#include "sw_internal.h"

namespace d2pb {

static __device__ __align__(256) unsigned char g_static_scratch[D2P_STATIC_SCRATCH_BYTES];

constexpr int kMaxDevices = 64;
static void* g_scratch_ptr[kMaxDevices];
static std::mutex g_scratch_mu;

// Address of this device's scratch array; set up once per device.
static int static_scratch(int dev, void** out) {
    if (dev < 0 || dev >= kMaxDevices) return D2P_ERR_INVALID_ARGUMENT;
    std::lock_guard<std::mutex> lk(g_scratch_mu);
    if (!g_scratch_ptr[dev]) {
        void* p = nullptr;
        const cudaError_t e = cudaGetSymbolAddress(&p, g_static_scratch);
        if (e != cudaSuccess) return (int)e;
        if (!p) return D2P_ERR_INVALID_ARGUMENT;
        g_scratch_ptr[dev] = p;
    }
    *out = g_scratch_ptr[dev];
    return D2P_OK;
}

}  // namespace d2pb

extern "C" int d2p_sw_forward_backward_static(const float* scores, const int* lengths, int B, int L1,
                                              int L2, float gap, float temperature,
                                              const float* gap_dev, const float* temperature_dev,
                                              float* value, float* marginals, float* grad_gap,
                                              float* grad_temperature, void* stream) {
    const size_t need = d2p_sw_workspace_bytes(D2P_FAMILY_LINEAR, D2P_OP_FORWARD_BACKWARD, B, L1, L2);
    if (need == (size_t)-1) return D2P_ERR_TOO_LARGE;
    if (need > (size_t)D2P_STATIC_SCRATCH_BYTES) return D2P_ERR_WORKSPACE_TOO_SMALL;
    if (B == 0) return D2P_OK;
    int dev = -1;
    const cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return (int)e;
    void* ws = nullptr;
    const int rc = d2pb::static_scratch(dev, &ws);
    if (rc != D2P_OK) return rc;
    return d2p_sw_forward_backward(scores, lengths, B, L1, L2, gap, temperature, gap_dev,
                                   temperature_dev, value, marginals, grad_gap, grad_temperature,
                                   ws, (size_t)D2P_STATIC_SCRATCH_BYTES, stream);
}
