// sw_internal.h -- internal launch descriptors shared by the d2p_b200 CUDA sources.
// Not part of the public C ABI (that is include/d2p_b200.h).
#pragma once
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stddef.h>

#include <atomic>
#include <mutex>

namespace d2pb {

// One-time set-up of a launcher on a device (kernel attributes), safe when
// several host threads make their first call at once.  `setup()` runs once
// per device under the lock and returns a cudaError_t; the device's SM count
// is published with release ordering only after it, so a thread that reads a
// nonzero count has also seen the attributes set.  Devices past the cache
// run the set-up on every call.  Returns a cudaError_t and the SM count
// through *sms.
constexpr int kMaxSetupDevices = 64;
struct DeviceSetup {
    std::atomic<int> sms[kMaxSetupDevices];
    std::mutex mu;
};
template <class F>
inline int device_setup(DeviceSetup& ds, int dev, F&& setup, int* sms) {
    if (dev >= 0 && dev < kMaxSetupDevices) {
        const int n = ds.sms[dev].load(std::memory_order_acquire);
        if (n > 0) {
            *sms = n;
            return 0;
        }
    }
    std::lock_guard<std::mutex> lk(ds.mu);
    if (dev >= 0 && dev < kMaxSetupDevices) {
        const int n = ds.sms[dev].load(std::memory_order_relaxed);
        if (n > 0) {
            *sms = n;
            return 0;
        }
    }
    cudaError_t e = (cudaError_t)setup();
    int n = 0;
    if (e == cudaSuccess) e = cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    if (e != cudaSuccess) return (int)e;
    if (dev >= 0 && dev < kMaxSetupDevices) ds.sms[dev].store(n, std::memory_order_release);
    *sms = n;
    return 0;
}

// operator modes (one kernel instantiation each)
enum SwMode : int {
    MODE_MARG = 0,  // value + marginals (+ dS/dgap, dS/dT)
    MODE_HVP = 1,   // Hessian-vector product  H = d(marginals)/d(scores) . V
    MODE_PGAP = 2,  // dP/d(gap)          (affine: dP/d(gap_open))
    MODE_PGE = 3,   // affine only: dP/d(gap_ext)
    MODE_PT = 4,    // dP/d(temperature)
};

// DP planes (each B*L1*L2 floats) the plane engine needs per mode; planes are
// ordered so that a mode uses a prefix of the full layout.
__host__ __device__ constexpr int lin_planes(int mode) {
    return mode == MODE_MARG ? 2 : (mode == MODE_PT ? 5 : 4);
}
__host__ __device__ constexpr int aff_planes(int mode) {
    return mode == MODE_MARG ? 6 : (mode == MODE_PT ? 15 : 12);
}

// The plane engine keeps one integer frame per anti-diagonal (k = i + j, k in
// [0, L1 + L2 + 2]) per problem after its planes.
__host__ __device__ inline size_t frame_stride(int L1, int L2) { return (size_t)L1 + (size_t)L2 + 4; }

// library error codes (cudaError_t values are passed through unchanged)
constexpr int kErrInvalid = 1001;
constexpr int kErrWorkspace = 1002;
constexpr int kErrTooLarge = 1003;
constexpr int kErrDeviceStatus = 1004;

struct SwArgs {
    const float* scores;                // [B, L1, L2] fp32 (may be null if scores_bf16 set)
    const __nv_bfloat16* scores_bf16;   // [B, L1, L2] bf16 (affine fast/plane paths)
    const float* tangent;               // [B, L1, L2] HVP direction
    const int* lengths;                 // [B, 2] or null (full lengths)
    int B, L1, L2;                      // padded dims
    float gap, gap2, temp;              // linear: gap; affine: gap=open, gap2=ext
    const float* gap_dev;               // optional device scalars (override host values)
    const float* gap2_dev;
    const float* temp_dev;
    int mode;
    float* value;                       // [B]
    float* out;                         // [B, L1, L2]: marginals / H / dP
    float* grad_gap;                    // [B]  (affine: d/d gap_open)
    float* grad_gap2;                   // [B]  (affine: d/d gap_ext)
    float* grad_T;                      // [B]
    float* ws;                          // workspace
    int* status;                        // device status word (optional)
    const float* dot_with;              // [B, L1, L2] optional: param modes accumulate
    float* dot_out;                     //   dot_out[b] = sum_ij dot_with[b,i,j] * dP[b,i,j]
    int* redo;                          // [B] out: set for problems the kernel could not finish
    const int* only;                    // [B] in, optional: run only the problems whose entry is set
    const int* order;                   // [B] in, optional: problem of each CTA (largest first)
    int parts;                          // CTAs per problem (1 unless a kernel spreads problems);
                                        //   soft DTW: the Sakoe-Chiba bandwidth (< 0: no band)
    int* sync;                          // [B][kSyncBytes / 4], zeroed: cross-CTA words of each problem
};

// A problem spread over several CTAs (a cooperative launch) keeps its
// cross-CTA progress words, barrier counters and per-part partials here:
// ints [0, kMaxParts) forward progress of each part's last warp, [kMaxParts,
// 2 kMaxParts) reverse progress, 2 kMaxParts + 0 / + 1 two arrival counters;
// from byte 256 on, kSyncPartDoubles doubles per part (frame base, partition
// partial, its tangent, two dot-product partials).
constexpr int kMaxParts = 16;
constexpr int kSyncPartDoubles = 5;
constexpr size_t kSyncBytes = 256 + 8 * kSyncPartDoubles * kMaxParts;

// linear-domain fast path (sw_linear.cu): value + marginals without parameter
// gradients; returns -1 when the shape or arguments are not covered
size_t lin_fast_workspace_bytes(int B, int L1, int L2);
// whether a batch of at most one problem per SM runs the linear-domain
// kernels with 12 warps per problem rather than 6 (shape L1 x L2)
bool lin_wide_pays(int L1, int L2);
int launch_lin_fast(const SwArgs& a, size_t ws_bytes, cudaStream_t st);
// column-sweep strip kernel (sw_strip.cu): value + marginals without parameter
// gradients for problems of at most 512 rows (planes whose rows are not whole
// 16-byte units go through padded copies in the workspace); returns -1 when
// the shape or arguments are not covered
size_t lin_strip_workspace_bytes(int B, int L1, int L2);
// nw: soft Needleman-Wunsch instead of Smith-Waterman (value + marginals)
int launch_lin_strip(const SwArgs& a, size_t ws_bytes, cudaStream_t st, bool nw = false);
// affine-gap linear-domain fast path (sw_affine_fast.cu): value + marginals
// without parameter gradients, fp32 or bf16 scores (bf16 widened into the
// workspace first); returns -1 when the shape or arguments are not covered
size_t aff_fast_workspace_bytes(int B, int L1, int L2, bool bf16);
int launch_aff_fast(const SwArgs& a, size_t ws_bytes, cudaStream_t st);
// bf16 -> fp32 copy of n scores (both pointers 16-byte aligned; exact)
int launch_bf16_widen(const __nv_bfloat16* in, float* out, size_t n, cudaStream_t st);
// order[B]: problems by decreasing estimated cost, for batches of uneven
// lengths that take more than one wave; returns -1 when ordering cannot help
int launch_lin_order(const int* lengths, int B, int L1, int L2, int* order, cudaStream_t st);

int launch_lin_plane(const SwArgs& a, cudaStream_t st);
// soft Needleman-Wunsch (sw_nw.cu): workspace of one operator, and one sweep
// pair in a.mode (MODE_MARG, MODE_HVP, MODE_PGAP, MODE_PT)
size_t nw_workspace_bytes(int op, int B, int L1, int L2);
int launch_nw(const SwArgs& a, cudaStream_t st);
// soft Needleman-Wunsch with affine gaps (sw_nw_affine.cu): the same, in
// a.mode MODE_MARG, MODE_HVP, MODE_PGAP (open), MODE_PGE (ext), MODE_PT
size_t nwa_workspace_bytes(int op, int B, int L1, int L2);
int launch_nwa(const SwArgs& a, cudaStream_t st);
// affine NW value pass in wavefront form (sw_nw_affine_wave.cu): its
// workspace, and the launch (MODE_MARG, a.redo a zeroed flag per problem; -1:
// shape not covered, nothing launched)
size_t nwa_wave_area(int B, int L1, int L2);
int launch_nwa_wave(const SwArgs& a, cudaStream_t st);
// soft DTW (sw_dtw.cu): workspace of one operator
size_t dtw_workspace_bytes(int op, int B, int L1, int L2);
// soft DTW value pass in wavefront form (sw_dtw_wave.cu): its workspace, and
// the launch (MODE_MARG, a.redo a zeroed flag per problem; -1: shape not
// covered, nothing launched)
size_t dtw_wave_area(int B, int L1, int L2);
int launch_dtw_wave(const SwArgs& a, cudaStream_t st);
size_t dtw_wave_tan_area(int B, int L1, int L2);
// soft NW tangent operators in wavefront form (sw_nw_wave_tan.cu)
size_t nw_wave_tan_area(int B, int L1, int L2);
int launch_nw_wave_tan(const SwArgs& a, cudaStream_t st);
int launch_dtw_wave_tan(const SwArgs& a, cudaStream_t st);
// engine counters of the current device (cumulative, read synchronously):
// problems the plane engine computed [linear, affine], and problems the
// log-domain kernel recomputed after a linear-domain kernel flagged them
int plane_problem_counts(unsigned long long* n2);
int wavefront_fixup_count(unsigned long long* n);

// D2P_B200_ENGINE=plane selects the general plane engine for every operator,
// D2P_B200_ENGINE=pipeline the anti-diagonal row-block pipeline
// (lin_fast_kernel) for linear value + marginals at every size (the engines
// compute the same results; used to cross-check and time them).
bool engine_forced_plane();
bool engine_forced_pipeline();

// linear-domain tangent sweeps (sw_tangent.cu): HVP, dP/dgap, dP/dT, and the
// dot mode (dot_with / dot_out) of the param modes; sets redo[b] for problems
// the plane engine must recompute.  Returns -1 when the shape is not covered.
// bf: the fused backward_full sweep, which also keeps the gap part of Z and
// its tangent per cell
size_t lin_tan_workspace_bytes(int B, int L1, int L2, bool bf = false);
// the affine counterpart (sw_affine_tangent.cu): HVP, dP/d(gap_open),
// dP/d(gap_ext), dP/dT and their dot mode
// pg: value + marginals + parameter gradients (keeps I and D per cell too)
size_t aff_tan_workspace_bytes(int B, int L1, int L2, bool pg = false);
int launch_aff_tan(const SwArgs& a, size_t ws_bytes, cudaStream_t st);
// CTAs per problem for B problems of nw warps per CTA, one CTA per SM (the
// row-block pipeline model; 1 = one CTA per problem)
int lin_parts_nw(int B, int L1, int L2, int sms, int nw);
int launch_lin_tan(const SwArgs& a, size_t ws_bytes, cudaStream_t st);
int launch_aff_plane(const SwArgs& a, cudaStream_t st);

// elementwise / reduction kernels (sw_elementwise.cu)
int launch_value_backward(const float* grad_value, const float* marginals, const float* dparams,
                          int n_params, int B, int L1, int L2, float* grad_scores,
                          float* grad_params, cudaStream_t st);
// the same with per-problem lengths (null: as launch_value_backward): cells
// outside each problem are written as 0 without reading the marginals
int launch_value_backward_rows(const float* grad_value, const float* marginals, const int* lengths,
                               const float* dparams, int n_params, int B, int L1, int L2,
                               float* grad_scores, float* grad_params, cudaStream_t st);
int launch_sum_batches(const float* partials, int P, int B, float* out, int accumulate,
                       cudaStream_t st);
// a[i] |= b[i] for n problem flags
int launch_or_flags(int* a, const int* b, int n, cudaStream_t st);
// [B][L1][L2] <-> [B][L1p][L2p] (L1p >= L1, L2p >= L2; zeros in the padding)
int launch_pad_rows(const float* in, int B, int L1, int L2, float* out, int L1p, int L2p, cudaStream_t st);
int launch_unpad_rows(const float* in, int L1p, int L2p, float* out, int B, int L1, int L2, cudaStream_t st);

}  // namespace d2pb
