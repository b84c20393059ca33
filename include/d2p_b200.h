/*
 * d2p_b200.h -- C ABI of the B200-native soft Smith-Waterman operator family.
 *
 * Plain pointers and sizes only (no torch types).  Every pointer argument is a
 * device pointer on the current CUDA device unless stated otherwise; `stream`
 * is a cudaStream_t passed as void* (NULL = legacy default stream).  All entry
 * points are asynchronous with respect to the host (no stream synchronisation)
 * and capturable in a CUDA graph once the workspace is allocated.
 *
 * Layouts follow the reference operators (d2p, src/sw/registry.cpp:30-44):
 *   scores, tangent, marginals, hvp, jacobian, grad_* planes : [B, L1, L2] row-major
 *   lengths : [B, 2] int32 (L1_b, L2_b) with 0 <= L1_b <= L1, 0 <= L2_b <= L2,
 *             or NULL for full lengths.  Out-of-range lengths are clamped on the
 *             device; callers wanting the reference's error messages validate
 *             on the host first (the torch binding does).
 *   value, grad_gap, grad_temperature, ... (per problem) : [B] fp32
 * Padded cells (i >= L1_b or j >= L2_b) of every [B,L1,L2] output are written
 * as exact zeros.
 *
 * Return value: 0 on success; a cudaError_t value (1..999) when a CUDA call
 * fails; or one of the D2P_ERR_* codes below.  d2p_error_string() describes a code.
 *
 * Workspace: each operator needs a device scratch buffer of at least
 * d2p_sw_workspace_bytes(family, op, B, L1, L2) bytes (256-byte aligned).
 */
#ifndef D2P_B200_H
#define D2P_B200_H

#include <stddef.h>

#if defined(__GNUC__)
#define D2P_API __attribute__((visibility("default")))
#else
#define D2P_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

#define D2P_OK 0
#define D2P_ERR_INVALID_ARGUMENT 1001
#define D2P_ERR_WORKSPACE_TOO_SMALL 1002
#define D2P_ERR_TOO_LARGE 1003
#define D2P_ERR_DEVICE_STATUS 1004

#define D2P_DTYPE_F32 0
#define D2P_DTYPE_BF16 1

#define D2P_FAMILY_LINEAR 0
#define D2P_FAMILY_AFFINE 1
#define D2P_FAMILY_NW 2 /* soft Needleman-Wunsch, linear gap (d2p_nw_*) */
#define D2P_FAMILY_NW_AFFINE 3 /* soft Needleman-Wunsch, affine gaps (d2p_nw_affine_*) */
#define D2P_FAMILY_DTW 4 /* soft dynamic time warping (d2p_dtw_*) */

#define D2P_OP_FORWARD_BACKWARD 0
#define D2P_OP_HVP 1
#define D2P_OP_PARAM_JACOBIAN 2
#define D2P_OP_BACKWARD_FULL 3

/* Library version (major*10000 + minor*100 + patch). */
D2P_API int d2p_version(void);

/* Human-readable description of a return code (static storage). */
D2P_API const char* d2p_error_string(int code);

/* Scratch bytes needed by operator `op` of `family` at this problem size
 * (0 if none).  Returns (size_t)-1 when the size is not supported. */
D2P_API size_t d2p_sw_workspace_bytes(int family, int op, int B, int L1, int L2);

/* ------------------------------------------------------------------------
 * Linear gap (reference family src/sw)
 * --------------------------------------------------------------------- */

/* value[b] = S_b (log partition), marginals = dS/dscores, grad_gap[b] = dS/dgap,
 * grad_temperature[b] = dS/dT.  Any output pointer may be NULL.  gap_dev /
 * temperature_dev, when non-NULL, are device scalars that override the host
 * values (graph-capturable learnable parameters).
 * Replaces: sw_regular_forward / sw_regular_forward_warp + sw_regular_backward /
 * sw_regular_backward_warp (reference src/sw/kernels.cuh:139-235) as driven by
 * soft_sw_regular_cuda_with_grads (src/sw/torch_cuda.cpp:450-504). */
D2P_API int d2p_sw_forward_backward(const float* scores, const int* lengths, int B, int L1, int L2,
                            float gap, float temperature, const float* gap_dev,
                            const float* temperature_dev, float* value, float* marginals,
                            float* grad_gap, float* grad_temperature, void* workspace,
                            size_t workspace_bytes, void* stream);

/* Size of the library-owned device scratch behind d2p_sw_forward_backward_static
 * (one array per device). */
#define D2P_STATIC_SCRATCH_BYTES (64u * 1024u * 1024u)

/* Same results as d2p_sw_forward_backward, but the call allocates nothing and
 * takes no workspace: it runs in a fixed scratch array built into the library.
 * For callers that cannot allocate device memory per call -- a host with no
 * device allocator of its own (C, cgo, FFI), where cudaMalloc/cudaFree around
 * each call would synchronize the device, or a process whose device memory is
 * already handed out to a fixed pool.
 * Limits: problems whose d2p_sw_workspace_bytes(D2P_FAMILY_LINEAR,
 * D2P_OP_FORWARD_BACKWARD, B, L1, L2) exceeds D2P_STATIC_SCRATCH_BYTES return
 * D2P_ERR_WORKSPACE_TOO_SMALL.  The scratch is shared by all calls on a device:
 * calls that overlap on the GPU (different streams or host threads) race on it.
 * The first call on a device looks up the scratch address with that device
 * current; make it before any stream capture.
 * No counterpart in the reference (its CUDA path allocates through torch). */
D2P_API int d2p_sw_forward_backward_static(const float* scores, const int* lengths, int B, int L1,
                                           int L2, float gap, float temperature,
                                           const float* gap_dev, const float* temperature_dev,
                                           float* value, float* marginals, float* grad_gap,
                                           float* grad_temperature, void* stream);

/* hvp = d(marginals)/d(scores) . tangent.
 * Replaces: sw_regular_forward + sw_regular_hvp (src/sw/kernels.cuh:237-270) as
 * driven by soft_sw_regular_hvp_cuda (src/sw/torch_cuda.cpp:507-570). */
D2P_API int d2p_sw_hvp(const float* scores, const float* tangent, const int* lengths, int B, int L1,
               int L2, float gap, float temperature, float* hvp, void* workspace,
               size_t workspace_bytes, void* stream);

/* jacobian = d(marginals)/d(theta), theta = gap (param_type 0) or temperature (1).
 * Replaces: sw_regular_forward + sw_regular_backward + sw_regular_param_grad
 * (src/sw/kernels.cuh:272-285) as driven by soft_sw_regular_param_jacobian_cuda
 * (src/sw/torch_cuda.cpp:573-662). */
D2P_API int d2p_sw_param_jacobian(const float* scores, const int* lengths, int B, int L1, int L2,
                          int param_type, float gap, float temperature, float* jacobian,
                          void* workspace, size_t workspace_bytes, void* stream);

/* Gradient of <grad_marginals, marginals> w.r.t. scores, gap and temperature:
 * grad_scores [B,L1,L2], grad_gap [1], grad_temperature [1] (device).
 * Replaces: soft_sw_backward_full_cuda (src/sw/torch_cuda.cpp:665-771). */
D2P_API int d2p_sw_backward_full(const float* scores, const float* grad_marginals, const int* lengths,
                         int B, int L1, int L2, float gap, float temperature, float* grad_scores,
                         float* grad_gap, float* grad_temperature, void* workspace,
                         size_t workspace_bytes, void* stream);

/* Value-branch backward shared by both families:
 * grad_scores[b,i,j] = grad_value[b] * marginals[b,i,j];
 * grad_params[p] = sum_b grad_value[b] * dvalue_dparams[p*B + b], p < n_params.
 * grad_params / dvalue_dparams may be NULL when n_params == 0.
 * Replaces: the value branch of SoftSWRegularCUDAFunction::backward
 * (src/sw/torch_cuda.cpp:292-321) and SoftSWAffineCUDAFunction::backward
 * (src/sw_affine/torch_cuda.cpp:250-290). */
D2P_API int d2p_sw_value_backward(const float* grad_value, const float* marginals,
                          const float* dvalue_dparams, int n_params, int B, int L1, int L2,
                          float* grad_scores, float* grad_params, void* stream);

/* d2p_sw_value_backward for a ragged batch: lengths [B, 2] (NULL: full
 * problems).  Cells outside each problem (where the marginals are 0) get 0
 * without the marginals being read.  Same replacement as above. */
D2P_API int d2p_sw_value_backward_lengths(const float* grad_value, const float* marginals,
                                          const int* lengths, const float* dvalue_dparams,
                                          int n_params, int B, int L1, int L2, float* grad_scores,
                                          float* grad_params, void* stream);

/* ------------------------------------------------------------------------
 * Affine gap (reference family src/sw_affine); parameters (gap_open, gap_ext, T)
 * --------------------------------------------------------------------- */

/* scores_dtype: D2P_DTYPE_F32 or D2P_DTYPE_BF16 (bf16 scores are upcast in
 * registers; all arithmetic is fp32).
 * Replaces: sw_affine_forward + sw_affine_backward (src/sw_affine/kernels.cuh:165-223)
 * as driven by soft_sw_affine_cuda_with_grads (src/sw_affine/torch_cuda.cpp:445-505). */
D2P_API int d2p_sw_affine_forward_backward(const void* scores, int scores_dtype, const int* lengths,
                                   int B, int L1, int L2, float gap_open, float gap_ext,
                                   float temperature, const float* gap_open_dev,
                                   const float* gap_ext_dev, const float* temperature_dev,
                                   float* value, float* marginals, float* grad_gap_open,
                                   float* grad_gap_ext, float* grad_temperature, void* workspace,
                                   size_t workspace_bytes, void* stream);

/* Replaces: sw_affine_forward + sw_affine_hvp (src/sw_affine/kernels.cuh:225-254) as
 * driven by soft_sw_affine_hvp_cuda (src/sw_affine/torch_cuda.cpp:508-577). */
D2P_API int d2p_sw_affine_hvp(const float* scores, const float* tangent, const int* lengths, int B,
                      int L1, int L2, float gap_open, float gap_ext, float temperature,
                      float* hvp, void* workspace, size_t workspace_bytes, void* stream);

/* param_type 0 = gap_open, 1 = gap_ext, 2 = temperature.
 * Replaces: sw_affine_forward + sw_affine_backward + sw_affine_param_grad
 * (src/sw_affine/kernels.cuh:256-269) as driven by soft_sw_affine_param_jacobian_cuda
 * (src/sw_affine/torch_cuda.cpp:580-677). */
D2P_API int d2p_sw_affine_param_jacobian(const float* scores, const int* lengths, int B, int L1, int L2,
                                 int param_type, float gap_open, float gap_ext,
                                 float temperature, float* jacobian, void* workspace,
                                 size_t workspace_bytes, void* stream);

/* grad_scores [B,L1,L2], grad_gap_open [1], grad_gap_ext [1], grad_temperature [1].
 * Replaces: soft_sw_affine_backward_full_cuda (src/sw_affine/torch_cuda.cpp:680-817). */
D2P_API int d2p_sw_affine_backward_full(const float* scores, const float* grad_marginals,
                                const int* lengths, int B, int L1, int L2, float gap_open,
                                float gap_ext, float temperature, float* grad_scores,
                                float* grad_gap_open, float* grad_gap_ext,
                                float* grad_temperature, void* workspace,
                                size_t workspace_bytes, void* stream);

/* Diagnostic: runs the kernels' bounded wait on a progress word that nothing
 * ever sets, on `stream`, and writes 1 to *status (device int) once the wait
 * has given up (0 would mean it saw the word set).  scope 0: a word in shared
 * memory (the wait between warps of one CTA); scope 1: the global word `word`
 * (device int, 0 and left untouched by the caller; the wait between the CTAs
 * of a problem spread over several CTAs).  The wait ends after its poll limit
 * (well under a second to a few seconds, depending on the scope) and the
 * context stays usable.  No counterpart in the reference. */
D2P_API int d2p_wait_selftest(int scope, const int* word, int* status, void* stream);

/* Diagnostic: MUFU (ex2.approx) throughput probe, for the transcendental
 * roofline.  Launches `blocks` CTAs of D2P_MUFU_PROBE_THREADS threads on
 * `stream`; each thread runs D2P_MUFU_PROBE_CHAINS independent ex2 chains of
 * `iters` steps and writes one float to out[blocks * D2P_MUFU_PROBE_THREADS]
 * (device).  ex2 operations per launch = blocks * threads * chains * iters; the
 * caller times the launch.  No counterpart in the reference. */
#define D2P_MUFU_PROBE_THREADS 512
#define D2P_MUFU_PROBE_CHAINS 8
D2P_API int d2p_mufu_probe(float* out, int blocks, int iters, void* stream);

/* ---- soft Needleman-Wunsch (global alignment, linear gap) ----
 * The same operator set as the linear soft Smith-Waterman entry points above,
 * with S = alpha[L1, L2] and marginal = P(the path's diagonal move into
 * (i, j)); workspace from d2p_sw_workspace_bytes(D2P_FAMILY_NW, op, ...).
 * They replace the reference's nw launchers (src/nw/kernels.cuh) behind its
 * soft_nw operators (src/nw/torch_cuda.cpp, src/nw/registry.cpp:35-49). */
D2P_API int d2p_nw_forward_backward(const float* scores, const int* lengths, int B, int L1, int L2, float gap,
                                    float temperature, const float* gap_dev, const float* temperature_dev,
                                    float* value, float* marginals, float* grad_gap, float* grad_temperature,
                                    void* workspace, size_t workspace_bytes, void* stream);
D2P_API int d2p_nw_hvp(const float* scores, const float* tangent, const int* lengths, int B, int L1, int L2,
                       float gap, float temperature, float* hvp, void* workspace, size_t workspace_bytes,
                       void* stream);
D2P_API int d2p_nw_param_jacobian(const float* scores, const int* lengths, int B, int L1, int L2, int param_type,
                                  float gap, float temperature, float* jacobian, void* workspace,
                                  size_t workspace_bytes, void* stream);
D2P_API int d2p_nw_backward_full(const float* scores, const float* grad_marginals, const int* lengths, int B,
                                 int L1, int L2, float gap, float temperature, float* grad_scores,
                                 float* grad_gap, float* grad_temperature, void* workspace,
                                 size_t workspace_bytes, void* stream);

/* ---- soft Needleman-Wunsch with affine gaps (states M, I, D) ----
 * M(0,0) = 0, I(i,0) = gap_open + (i-1) gap_ext, D(0,j) = gap_open + (j-1)
 * gap_ext; S = the logsumexp of the three states at (L1, L2); marginal = the
 * probability that the path visits M at (i, j).  fp32 scores.  Workspace from
 * d2p_sw_workspace_bytes(D2P_FAMILY_NW_AFFINE, op, ...); param_type 0 =
 * gap_open, 1 = gap_ext, 2 = temperature; the gradient outputs of
 * forward_backward may be NULL.  They replace the reference's nw_affine
 * launchers (src/nw_affine/kernels.cuh) behind its soft_nw_affine operators
 * (src/nw_affine/torch_cuda.cpp, src/nw_affine/registry.cpp:35-50). */
D2P_API int d2p_nw_affine_forward_backward(const float* scores, const int* lengths, int B, int L1, int L2,
                                           float gap_open, float gap_ext, float temperature,
                                           const float* gap_open_dev, const float* gap_ext_dev,
                                           const float* temperature_dev, float* value, float* marginals,
                                           float* grad_gap_open, float* grad_gap_ext, float* grad_temperature,
                                           void* workspace, size_t workspace_bytes, void* stream);
D2P_API int d2p_nw_affine_hvp(const float* scores, const float* tangent, const int* lengths, int B, int L1,
                              int L2, float gap_open, float gap_ext, float temperature, float* hvp,
                              void* workspace, size_t workspace_bytes, void* stream);
D2P_API int d2p_nw_affine_param_jacobian(const float* scores, const int* lengths, int B, int L1, int L2,
                                         int param_type, float gap_open, float gap_ext, float temperature,
                                         float* jacobian, void* workspace, size_t workspace_bytes, void* stream);
D2P_API int d2p_nw_affine_backward_full(const float* scores, const float* grad_marginals, const int* lengths,
                                        int B, int L1, int L2, float gap_open, float gap_ext, float temperature,
                                        float* grad_scores, float* grad_gap_open, float* grad_gap_ext,
                                        float* grad_temperature, void* workspace, size_t workspace_bytes,
                                        void* stream);

/* ---- soft dynamic time warping (softmin over the three predecessors) ----
 * alpha[0,0] = 0; alpha[i,j] = costs[i,j] + softmin_T of the three
 * predecessors for cells inside the Sakoe-Chiba band |j - i L2 / L1| <=
 * bandwidth (bandwidth < 0: no band); S = alpha[L1, L2] (the sentinel 1e30
 * when a sequence is empty or the end cannot be reached); marginal = the
 * probability that the warping path visits (i, j).  fp32 costs; lengths may
 * be NULL (full lengths).  Workspace from
 * d2p_sw_workspace_bytes(D2P_FAMILY_DTW, op, ...).  They replace the
 * reference's dtw launchers (src/dtw/kernels.cuh) behind its soft_dtw
 * operators (src/dtw/torch_cuda.cpp, src/dtw/registry.cpp:35-40). */
D2P_API int d2p_dtw_forward_backward(const float* costs, const int* lengths, int B, int L1, int L2,
                                     float temperature, const float* temperature_dev, int bandwidth, float* value,
                                     float* marginals, float* grad_temperature, void* workspace,
                                     size_t workspace_bytes, void* stream);
D2P_API int d2p_dtw_hvp(const float* costs, const float* tangent, const int* lengths, int B, int L1, int L2,
                        float temperature, int bandwidth, float* hvp, void* workspace, size_t workspace_bytes,
                        void* stream);
D2P_API int d2p_dtw_param_jacobian(const float* costs, const int* lengths, int B, int L1, int L2, float temperature,
                                   int bandwidth, float* jacobian, void* workspace, size_t workspace_bytes,
                                   void* stream);
D2P_API int d2p_dtw_backward_full(const float* costs, const float* grad_marginals, const int* lengths, int B, int L1,
                                  int L2, float temperature, int bandwidth, float* grad_costs,
                                  float* grad_temperature, void* workspace, size_t workspace_bytes, void* stream);

/* Score producer: scores[b] = scale * x[b] y[b]^T for bf16 embeddings x [B, L1,
 * D] and y [B, L2, D] (contiguous, 16-byte aligned), fp32 scores [B, L1, L2],
 * on the tcgen05 tensor cores.  D a multiple of 64, at most 256 (pad the
 * embeddings with zeros: a zero column adds nothing to a dot product).
 * status (optional, device int): incremented for each output tile whose copy
 * or product did not arrive within the kernel's bounded waits (the tile is
 * then computed on the CUDA cores; nothing is wrong with its values).  No
 * operator of the reference corresponds: it takes the score plane as input
 * (d2p/sw.py:247) and its examples build it with an einsum of embeddings
 * (docs/examples.md:9-23). */
D2P_API int d2p_embed_scores(const void* x, const void* y, int B, int L1, int L2, int D, float scale, float* scores,
                             int* status, void* stream);
/* The scores' gradient for a loss of the values only, in bf16 for the
 * embeddings' gradient GEMMs: grad_scores[b] = bf16(scale * grad_value[b] *
 * marginals[b]) (any size; 8 elements per thread when L1 * L2 is a multiple
 * of 8 and both planes are 16-byte aligned).  No reference counterpart (see
 * d2p_embed_scores). */
D2P_API int d2p_embed_grad_scores(const float* marginals, const float* grad_value, int B, int L1, int L2, float scale,
                                  void* grad_scores_bf16, void* stream);

/* Engine selection for the whole process (all devices): D2P_ENGINE_AUTO picks
 * per shape (the default, or what D2P_B200_ENGINE names at load: "plane",
 * "pipeline"); D2P_ENGINE_PLANE runs the general plane engine for every
 * operator; D2P_ENGINE_PIPELINE runs the anti-diagonal row-block pipeline for
 * linear value + marginals at every size.  The engines compute the same
 * results; the switch exists to cross-check and time them.  *previous (may
 * be NULL) receives the setting before the call.  Takes effect for launches
 * issued after it returns.  No reference counterpart. */
#define D2P_ENGINE_AUTO 0
#define D2P_ENGINE_PLANE 1
#define D2P_ENGINE_PIPELINE 2
D2P_API int d2p_set_engine(int engine, int* previous);

/* Engine counters of the current device, cumulative since the library was
 * loaded: counts[0] = linear problems the log-domain kernel recomputed after a
 * linear-domain kernel flagged them (low temperatures, extreme scores);
 * counts[1] = linear problems the plane engine computed (shapes no fast
 * kernel covers, and problems both fast kernels flagged); counts[2] = affine
 * problems the plane engine computed.  n: entries to fill (at most 3).
 * Synchronises with the device.  No reference counterpart: the reference has
 * one engine per family. */
D2P_API int d2p_engine_counts(unsigned long long* counts, int n);

#ifdef __cplusplus
}
#endif

#endif /* D2P_B200_H */
