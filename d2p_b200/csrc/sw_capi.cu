// sw_capi.cu -- extern "C" entry points of libd2p_b200.so (declared in include/d2p_b200.h).
//
// Argument checking, workspace carving and kernel selection live here; the
// kernels themselves are in sw_linear.cu / sw_affine_fast.cu (linear-domain
// value + marginals), sw_tangent.cu / sw_affine_tangent.cu (linear-domain
// tangent sweeps), sw_wavefront.cu (log-domain value + marginals + parameter
// gradients for batches over one wave), sw_plane.cu (general engine and fix-up)
// and sw_elementwise.cu.
#include <limits.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#include <atomic>

#include "../../include/d2p_b200.h"
#include "sw_internal.h"

namespace d2pb {

// fast path hooks (sw_wavefront.cu); return kNotHandled when the shape is not
// covered so that the plane engine runs instead.
size_t wavefront_workspace_bytes(int family, int B, int L1, int L2);
int launch_wavefront(const SwArgs& a, int family, size_t ws_bytes, cudaStream_t st);
constexpr int kNotHandled = -1;

static size_t align256(size_t x) { return (x + 255) & ~(size_t)255; }

// Engine selection: 0 automatic, 1 the plane engine for every operator, 2 the
// row-block pipeline for linear value + marginals.  Starts from
// D2P_B200_ENGINE ("plane", "pipeline"); d2p_set_engine changes it.
static std::atomic<int> g_engine{-1};
static int engine_mode() {
    const int v = g_engine.load(std::memory_order_acquire);
    if (v >= 0) return v;
    const char* e = getenv("D2P_B200_ENGINE");
    const int m = e && strcmp(e, "plane") == 0 ? 1 : e && strcmp(e, "pipeline") == 0 ? 2 : 0;
    int unset = -1;
    g_engine.compare_exchange_strong(unset, m, std::memory_order_acq_rel);
    return g_engine.load(std::memory_order_acquire);
}
bool engine_forced_plane() { return engine_mode() == 1; }
bool engine_forced_pipeline() { return engine_mode() == 2; }

static bool dims_ok(int B, int L1, int L2) {
    if (B < 0 || L1 < 0 || L2 < 0) return false;
    // per-problem cell indices are 32-bit inside the kernels (the reference's
    // "(L1 + 1) * (L2 + 1) <= INT_MAX" rule, src/sw/torch_cuda.cpp:49-65)
    if ((long long)(L1 + 1) * (long long)(L2 + 1) > (long long)INT_MAX) return false;
    return true;
}

static size_t plane_bytes(int family, int mode, int B, int L1, int L2) {
    const size_t plane = (size_t)L1 * (size_t)L2;
    const int np = family == D2P_FAMILY_AFFINE ? aff_planes(mode) : lin_planes(mode);
    // planes, then one frame per anti-diagonal per problem
    return align256(((size_t)B * plane * np + (size_t)B * frame_stride(L1, L2)) * sizeof(float));
}

// the shared area of the tangent ops: the linear tangent kernel's workspace
// (linear family, covered shapes) or the plane engine's, whichever is larger
static size_t tan_area(int family, int op, int B, int L1, int L2) {
    size_t pe = plane_bytes(family, op == D2P_OP_HVP ? MODE_HVP : MODE_PT, B, L1, L2);
    const size_t tf = family == D2P_FAMILY_LINEAR ? lin_tan_workspace_bytes(B, L1, L2, op == D2P_OP_BACKWARD_FULL)
                                                  : aff_tan_workspace_bytes(B, L1, L2);
    pe = pe > tf ? pe : tf;
    return align256(pe);
}

static size_t op_bytes(int family, int op, int B, int L1, int L2) {
    switch (op) {
        case D2P_OP_FORWARD_BACKWARD: {
            // the fast kernels' workspace, or the plane engine's (which also serves as
            // the fix-up for problems the fast kernels flag), then one flag per problem
            size_t pe = plane_bytes(family, MODE_MARG, B, L1, L2);
            const size_t wf = family == D2P_FAMILY_LINEAR ? wavefront_workspace_bytes(family, B, L1, L2)
                                                          : aff_fast_workspace_bytes(B, L1, L2, true);
            const size_t lf = family == D2P_FAMILY_LINEAR ? lin_fast_workspace_bytes(B, L1, L2) : 0;
            const size_t sf = family == D2P_FAMILY_LINEAR ? lin_strip_workspace_bytes(B, L1, L2) : 0;
            const size_t tf = family == D2P_FAMILY_LINEAR ? lin_tan_workspace_bytes(B, L1, L2)
                                                          : aff_tan_workspace_bytes(B, L1, L2, true);
            if (wf == 0 && lf == 0 && sf == 0 && tf == 0) return pe;
            pe = pe > wf ? pe : wf;
            pe = pe > lf ? pe : lf;
            pe = pe > sf ? pe : sf;
            pe = pe > tf ? pe : tf;
            if (family == D2P_FAMILY_AFFINE && tf > 0) {
                // bf16 scores with parameter gradients: the tangent kernel's
                // area, then the widened scores
                const size_t tw = align256(tf) + align256((size_t)B * L1 * L2 * sizeof(float));
                pe = pe > tw ? pe : tw;
            }
            // flags, the CTA order of ragged batches, the log-domain fix-up's
            // flags, the cross-CTA words of problems spread over several CTAs
            return align256(pe) + 3 * align256((size_t)(B > 0 ? B : 1) * sizeof(int)) +
                   align256((size_t)(B > 0 ? B : 1) * kSyncBytes);
        }
        case D2P_OP_HVP:
        case D2P_OP_PARAM_JACOBIAN:
            // the tangent kernel's workspace or the plane engine's (its fix-up),
            // then one flag per problem and the cross-CTA words of problems
            // spread over several CTAs
            return tan_area(family, op, B, L1, L2) + align256((size_t)(B > 0 ? B : 1) * sizeof(int)) +
                   align256((size_t)(B > 0 ? B : 1) * kSyncBytes);
        case D2P_OP_BACKWARD_FULL:
            // the tangent area, per-problem partials, flags, cross-CTA words,
            // and a second flag array (affine: the gap_ext dot sweep's)
            return tan_area(family, op, B, L1, L2) + align256((size_t)4 * (B > 0 ? B : 1) * sizeof(float)) +
                   2 * align256((size_t)(B > 0 ? B : 1) * sizeof(int)) +
                   align256((size_t)(B > 0 ? B : 1) * kSyncBytes);
        default:
            return (size_t)-1;
    }
}

static SwArgs base_args(const float* scores, const int* lengths, int B, int L1, int L2) {
    SwArgs a{};
    a.scores = scores;
    a.lengths = lengths;
    a.B = B;
    a.L1 = L1;
    a.L2 = L2;
    return a;
}

}  // namespace d2pb

using namespace d2pb;

extern "C" {

int d2p_version(void) { return 100; }

int d2p_set_engine(int engine, int* previous) {
    if (engine < D2P_ENGINE_AUTO || engine > D2P_ENGINE_PIPELINE) return D2P_ERR_INVALID_ARGUMENT;
    const int prev = engine_mode();
    g_engine.store(engine, std::memory_order_release);
    if (previous) *previous = prev;
    return D2P_OK;
}

int d2p_engine_counts(unsigned long long* counts, int n) {
    if (!counts || n < 0 || n > 3) return D2P_ERR_INVALID_ARGUMENT;
    unsigned long long c[3] = {0, 0, 0};
    int rc = wavefront_fixup_count(&c[0]);
    if (rc == D2P_OK) rc = plane_problem_counts(&c[1]);
    if (rc != D2P_OK) return rc;
    for (int i = 0; i < n; ++i) counts[i] = c[i];
    return D2P_OK;
}

const char* d2p_error_string(int code) {
    switch (code) {
        case D2P_OK: return "success";
        case D2P_ERR_INVALID_ARGUMENT: return "d2p_b200: invalid argument";
        case D2P_ERR_WORKSPACE_TOO_SMALL: return "d2p_b200: workspace too small";
        case D2P_ERR_TOO_LARGE: return "d2p_b200: problem too large for 32-bit cell indexing";
        case D2P_ERR_DEVICE_STATUS: return "d2p_b200: device-side status error";
        default: break;
    }
    if (code > 0 && code < 1000) return cudaGetErrorString((cudaError_t)code);
    return "d2p_b200: unknown error";
}

size_t d2p_sw_workspace_bytes(int family, int op, int B, int L1, int L2) {
    if (family != D2P_FAMILY_LINEAR && family != D2P_FAMILY_AFFINE && family != D2P_FAMILY_NW &&
        family != D2P_FAMILY_NW_AFFINE && family != D2P_FAMILY_DTW)
        return (size_t)-1;
    if (!dims_ok(B, L1, L2)) return (size_t)-1;
    if (family == D2P_FAMILY_DTW) {
        if (op < D2P_OP_FORWARD_BACKWARD || op > D2P_OP_BACKWARD_FULL) return (size_t)-1;
        return dtw_workspace_bytes(op, B, L1, L2);
    }
    if (family == D2P_FAMILY_NW || family == D2P_FAMILY_NW_AFFINE) {
        if (op < D2P_OP_FORWARD_BACKWARD || op > D2P_OP_BACKWARD_FULL) return (size_t)-1;
        if (family == D2P_FAMILY_NW_AFFINE && 3LL * (L1 + 1LL) * (L2 + 1LL) > (long long)INT_MAX) return (size_t)-1;
        return family == D2P_FAMILY_NW ? nw_workspace_bytes(op, B, L1, L2) : nwa_workspace_bytes(op, B, L1, L2);
    }
    return op_bytes(family, op, B, L1, L2);
}

// ---------------------------------------------------------------- linear
int d2p_sw_forward_backward(const float* scores, const int* lengths, int B, int L1, int L2,
                            float gap, float temperature, const float* gap_dev,
                            const float* temperature_dev, float* value, float* marginals,
                            float* grad_gap, float* grad_temperature, void* workspace,
                            size_t workspace_bytes, void* stream) {
    if (!dims_ok(B, L1, L2)) return D2P_ERR_TOO_LARGE;
    if (B == 0) return D2P_OK;
    if (!scores && L1 > 0 && L2 > 0) return D2P_ERR_INVALID_ARGUMENT;
    const size_t need = op_bytes(D2P_FAMILY_LINEAR, D2P_OP_FORWARD_BACKWARD, B, L1, L2);
    if (need > 0 && (!workspace || workspace_bytes < need)) return D2P_ERR_WORKSPACE_TOO_SMALL;
    cudaStream_t st = (cudaStream_t)stream;
    SwArgs a = base_args(scores, lengths, B, L1, L2);
    a.gap = gap;
    a.temp = temperature;
    a.gap_dev = gap_dev;
    a.temp_dev = temperature_dev;
    a.mode = MODE_MARG;
    a.value = value;
    a.out = marginals;
    a.grad_gap = grad_gap;
    a.grad_T = grad_temperature;
    a.ws = (float*)workspace;
    size_t pe = plane_bytes(D2P_FAMILY_LINEAR, MODE_MARG, B, L1, L2);
    const size_t wf = wavefront_workspace_bytes(D2P_FAMILY_LINEAR, B, L1, L2);
    const size_t lf = lin_fast_workspace_bytes(B, L1, L2);
    const size_t sf = lin_strip_workspace_bytes(B, L1, L2);
    const size_t tf = lin_tan_workspace_bytes(B, L1, L2);
    if (wf > 0 || lf > 0 || sf > 0 || tf > 0) {
        // Fast kernels, each later one recomputing what the earlier flagged:
        //   value + marginals: the column-sweep strip kernel (at most 512
        //   rows) or the anti-diagonal row-block pipeline (sw_linear.cu) ->
        //   the normalised log-domain kernel (sw_wavefront.cu) -> plane engine;
        //   with parameter gradients: the tangent kernel's gap sweep
        //   (sw_tangent.cu) -> plane engine;
        //   shapes no linear-domain kernel covers: log-domain -> plane engine.
        pe = pe > wf ? pe : wf;
        pe = pe > lf ? pe : lf;
        pe = pe > sf ? pe : sf;
        pe = pe > tf ? pe : tf;
        const size_t fb = align256((size_t)B * sizeof(int));
        int* flags = (int*)((char*)workspace + align256(pe));
        int* order = (int*)((char*)flags + fb);
        int* flags2 = (int*)((char*)order + fb);
        a.redo = flags;
        a.only = nullptr;
        a.order = nullptr;
        a.sync = (int*)((char*)flags2 + fb);
        const bool pgrad = grad_gap || grad_temperature;
        if (lengths && !pgrad) {
            const int ro = launch_lin_order(lengths, B, L1, L2, order, st);
            if (ro == D2P_OK) a.order = order;
            else if (ro != kNotHandled) return ro;
        }
        int rc;
        if (pgrad) {
            rc = launch_lin_tan(a, workspace_bytes, st);
        } else {
            rc = launch_lin_strip(a, workspace_bytes, st);
            if (rc == kNotHandled) rc = launch_lin_fast(a, workspace_bytes, st);
        }
        a.order = nullptr;
        a.sync = nullptr;
        if (rc == D2P_OK && !pgrad) {
            // flagged problems (low temperatures, extreme scores): the log-domain
            // kernel, then the plane engine (the reference's score-unit
            // arithmetic) for any it flags in turn
            SwArgs w = a;
            w.only = flags;
            w.redo = flags2;
            const int rw = launch_wavefront(w, D2P_FAMILY_LINEAR, workspace_bytes, st);
            if (rw != D2P_OK && rw != kNotHandled) return rw;
            a.only = rw == D2P_OK ? flags2 : flags;
            a.redo = nullptr;
            return launch_lin_plane(a, st);
        }
        if (rc == D2P_OK) {
            a.only = flags;
            a.redo = nullptr;
            return launch_lin_plane(a, st);
        }
        if (rc != kNotHandled) return rc;
        rc = launch_wavefront(a, D2P_FAMILY_LINEAR, workspace_bytes, st);
        if (rc == D2P_OK) {
            a.only = flags;
            a.redo = nullptr;
            return launch_lin_plane(a, st);
        }
        if (rc != kNotHandled) return rc;
        a.redo = nullptr;
        a.only = nullptr;
    }
    return launch_lin_plane(a, st);
}

// One tangent op: the linear-domain tangent kernel of the family, then the
// plane engine for the problems it flagged (or for all, if the shape is not
// covered).  flags: the op's per-problem flag array in the workspace, followed
// by the cross-CTA words.
static int run_tangent(int family, SwArgs a, size_t ws_bytes, int* flags, cudaStream_t st) {
    a.redo = flags;
    a.only = nullptr;
    a.sync = (int*)((char*)flags + align256((size_t)a.B * sizeof(int)));
    int rc = family == D2P_FAMILY_LINEAR ? launch_lin_tan(a, ws_bytes, st) : launch_aff_tan(a, ws_bytes, st);
    a.redo = nullptr;
    a.sync = nullptr;
    if (rc == D2P_OK) a.only = flags;
    else if (rc != kNotHandled) return rc;
    return family == D2P_FAMILY_LINEAR ? launch_lin_plane(a, st) : launch_aff_plane(a, st);
}
static int run_lin_tangent(SwArgs a, size_t ws_bytes, int* flags, cudaStream_t st) {
    return run_tangent(D2P_FAMILY_LINEAR, a, ws_bytes, flags, st);
}

int d2p_sw_hvp(const float* scores, const float* tangent, const int* lengths, int B, int L1,
               int L2, float gap, float temperature, float* hvp, void* workspace,
               size_t workspace_bytes, void* stream) {
    if (!dims_ok(B, L1, L2)) return D2P_ERR_TOO_LARGE;
    if (B == 0) return D2P_OK;
    if ((!scores || !tangent || !hvp) && L1 > 0 && L2 > 0) return D2P_ERR_INVALID_ARGUMENT;
    const size_t need = op_bytes(D2P_FAMILY_LINEAR, D2P_OP_HVP, B, L1, L2);
    if (need > 0 && (!workspace || workspace_bytes < need)) return D2P_ERR_WORKSPACE_TOO_SMALL;
    SwArgs a = base_args(scores, lengths, B, L1, L2);
    a.tangent = tangent;
    a.gap = gap;
    a.temp = temperature;
    a.mode = MODE_HVP;
    a.out = hvp;
    a.ws = (float*)workspace;
    int* flags = (int*)((char*)workspace + tan_area(D2P_FAMILY_LINEAR, D2P_OP_HVP, B, L1, L2));
    return run_lin_tangent(a, workspace_bytes, flags, (cudaStream_t)stream);
}

int d2p_sw_param_jacobian(const float* scores, const int* lengths, int B, int L1, int L2,
                          int param_type, float gap, float temperature, float* jacobian,
                          void* workspace, size_t workspace_bytes, void* stream) {
    if (param_type != 0 && param_type != 1) return D2P_ERR_INVALID_ARGUMENT;
    if (!dims_ok(B, L1, L2)) return D2P_ERR_TOO_LARGE;
    if (B == 0) return D2P_OK;
    if ((!scores || !jacobian) && L1 > 0 && L2 > 0) return D2P_ERR_INVALID_ARGUMENT;
    const size_t need = op_bytes(D2P_FAMILY_LINEAR, D2P_OP_PARAM_JACOBIAN, B, L1, L2);
    if (need > 0 && (!workspace || workspace_bytes < need)) return D2P_ERR_WORKSPACE_TOO_SMALL;
    SwArgs a = base_args(scores, lengths, B, L1, L2);
    a.gap = gap;
    a.temp = temperature;
    a.mode = param_type == 0 ? MODE_PGAP : MODE_PT;
    a.out = jacobian;
    a.ws = (float*)workspace;
    int* flags = (int*)((char*)workspace + tan_area(D2P_FAMILY_LINEAR, D2P_OP_PARAM_JACOBIAN, B, L1, L2));
    return run_lin_tangent(a, workspace_bytes, flags, (cudaStream_t)stream);
}

int d2p_sw_backward_full(const float* scores, const float* grad_marginals, const int* lengths,
                         int B, int L1, int L2, float gap, float temperature, float* grad_scores,
                         float* grad_gap, float* grad_temperature, void* workspace,
                         size_t workspace_bytes, void* stream) {
    if (!dims_ok(B, L1, L2)) return D2P_ERR_TOO_LARGE;
    if (!grad_scores || !grad_gap || !grad_temperature) return D2P_ERR_INVALID_ARGUMENT;
    const size_t need = op_bytes(D2P_FAMILY_LINEAR, D2P_OP_BACKWARD_FULL, B, L1, L2);
    if (!workspace || workspace_bytes < need) return D2P_ERR_WORKSPACE_TOO_SMALL;
    cudaStream_t st = (cudaStream_t)stream;
    if (B == 0) {
        cudaError_t e1 = cudaMemsetAsync(grad_gap, 0, sizeof(float), st);
        cudaError_t e2 = cudaMemsetAsync(grad_temperature, 0, sizeof(float), st);
        return (int)(e1 != cudaSuccess ? e1 : e2);
    }
    // grad_scores = H . grad_marginals (the Hessian of S is symmetric);
    // grad_gap / grad_T = sum grad_marginals * dP/dgap, dP/dT
    const size_t area = tan_area(D2P_FAMILY_LINEAR, D2P_OP_BACKWARD_FULL, B, L1, L2);
    float* planes = (float*)workspace;
    float* partials = (float*)((char*)workspace + area);
    int* flags = (int*)((char*)partials + align256((size_t)4 * B * sizeof(float)));
    SwArgs a = base_args(scores, lengths, B, L1, L2);
    a.gap = gap;
    a.temp = temperature;
    a.ws = planes;
    a.tangent = grad_marginals;
    a.mode = MODE_HVP;
    a.out = grad_scores;
    // one sweep pair of the tangent kernel: H . grad_marginals, and the
    // parameter parts as tangents of dS/dgap and dS/dT (sw_tangent.cu); the
    // problems it flags get the plane engine's three sweeps
    a.dot_out = partials;
    a.redo = flags;
    a.sync = (int*)((char*)flags + align256((size_t)B * sizeof(int)));
    int rc = launch_lin_tan(a, workspace_bytes, st);
    a.redo = nullptr;
    a.sync = nullptr;
    a.dot_out = nullptr;
    if (rc == D2P_OK) {
        a.only = flags;
        rc = launch_lin_plane(a, st);
        if (rc) return rc;
        a.tangent = nullptr;
        a.out = nullptr;
        a.dot_with = grad_marginals;
        a.mode = MODE_PGAP;
        a.dot_out = partials;
        rc = launch_lin_plane(a, st);
        if (rc) return rc;
        a.mode = MODE_PT;
        a.dot_out = partials + B;
        rc = launch_lin_plane(a, st);
        if (rc) return rc;
        rc = launch_sum_batches(partials, 1, B, grad_gap, 0, st);
        if (rc) return rc;
        return launch_sum_batches(partials + B, 1, B, grad_temperature, 0, st);
    }
    if (rc != kNotHandled) return rc;
    rc = run_lin_tangent(a, workspace_bytes, flags, st);
    if (rc) return rc;
    a.tangent = nullptr;
    a.out = nullptr;
    a.dot_with = grad_marginals;
    a.mode = MODE_PGAP;
    a.dot_out = partials;
    rc = run_lin_tangent(a, workspace_bytes, flags, st);
    if (rc) return rc;
    a.mode = MODE_PT;
    a.dot_out = partials + B;
    rc = run_lin_tangent(a, workspace_bytes, flags, st);
    if (rc) return rc;
    rc = launch_sum_batches(partials, 1, B, grad_gap, 0, st);
    if (rc) return rc;
    return launch_sum_batches(partials + B, 1, B, grad_temperature, 0, st);
}

int d2p_sw_value_backward(const float* grad_value, const float* marginals,
                          const float* dvalue_dparams, int n_params, int B, int L1, int L2,
                          float* grad_scores, float* grad_params, void* stream) {
    if (B < 0 || L1 < 0 || L2 < 0 || n_params < 0) return D2P_ERR_INVALID_ARGUMENT;
    if (B == 0) {
        if (n_params > 0 && grad_params)
            return (int)cudaMemsetAsync(grad_params, 0, sizeof(float) * n_params, (cudaStream_t)stream);
        return D2P_OK;
    }
    if (!grad_value || (!marginals && L1 > 0 && L2 > 0) || (!grad_scores && L1 > 0 && L2 > 0))
        return D2P_ERR_INVALID_ARGUMENT;
    if (n_params > 0 && (!dvalue_dparams || !grad_params)) return D2P_ERR_INVALID_ARGUMENT;
    return launch_value_backward(grad_value, marginals, dvalue_dparams, n_params, B, L1, L2,
                                 grad_scores, grad_params, (cudaStream_t)stream);
}
int d2p_sw_value_backward_lengths(const float* grad_value, const float* marginals, const int* lengths,
                                  const float* dvalue_dparams, int n_params, int B, int L1, int L2,
                                  float* grad_scores, float* grad_params, void* stream) {
    if (!lengths || B <= 0)
        return d2p_sw_value_backward(grad_value, marginals, dvalue_dparams, n_params, B, L1, L2, grad_scores,
                                     grad_params, stream);
    if (L1 < 0 || L2 < 0 || n_params < 0) return D2P_ERR_INVALID_ARGUMENT;
    if (!grad_value || (!marginals && L1 > 0 && L2 > 0) || (!grad_scores && L1 > 0 && L2 > 0))
        return D2P_ERR_INVALID_ARGUMENT;
    if (n_params > 0 && (!dvalue_dparams || !grad_params)) return D2P_ERR_INVALID_ARGUMENT;
    return launch_value_backward_rows(grad_value, marginals, lengths, dvalue_dparams, n_params, B, L1, L2,
                                      grad_scores, grad_params, (cudaStream_t)stream);
}

// ---------------------------------------------------------------- affine
int d2p_sw_affine_forward_backward(const void* scores, int scores_dtype, const int* lengths,
                                   int B, int L1, int L2, float gap_open, float gap_ext,
                                   float temperature, const float* gap_open_dev,
                                   const float* gap_ext_dev, const float* temperature_dev,
                                   float* value, float* marginals, float* grad_gap_open,
                                   float* grad_gap_ext, float* grad_temperature, void* workspace,
                                   size_t workspace_bytes, void* stream) {
    if (scores_dtype != D2P_DTYPE_F32 && scores_dtype != D2P_DTYPE_BF16) return D2P_ERR_INVALID_ARGUMENT;
    if (!dims_ok(B, L1, L2)) return D2P_ERR_TOO_LARGE;
    if (B == 0) return D2P_OK;
    if (!scores && L1 > 0 && L2 > 0) return D2P_ERR_INVALID_ARGUMENT;
    const size_t need = op_bytes(D2P_FAMILY_AFFINE, D2P_OP_FORWARD_BACKWARD, B, L1, L2);
    if (need > 0 && (!workspace || workspace_bytes < need)) return D2P_ERR_WORKSPACE_TOO_SMALL;
    cudaStream_t st = (cudaStream_t)stream;
    SwArgs a = base_args(scores_dtype == D2P_DTYPE_F32 ? (const float*)scores : nullptr, lengths, B, L1, L2);
    a.scores_bf16 = scores_dtype == D2P_DTYPE_BF16 ? (const __nv_bfloat16*)scores : nullptr;
    a.gap = gap_open;
    a.gap2 = gap_ext;
    a.temp = temperature;
    a.gap_dev = gap_open_dev;
    a.gap2_dev = gap_ext_dev;
    a.temp_dev = temperature_dev;
    a.mode = MODE_MARG;
    a.value = value;
    a.out = marginals;
    a.grad_gap = grad_gap_open;
    a.grad_gap2 = grad_gap_ext;
    a.grad_T = grad_temperature;
    a.ws = (float*)workspace;
    const size_t af = aff_fast_workspace_bytes(B, L1, L2, true);
    if (af > 0) {
        // linear-domain kernels -- value + marginals: sw_affine_fast.cu; with
        // parameter gradients: the tangent kernel's gap sweep pair,
        // sw_affine_tangent.cu -- then the plane engine for the problems they
        // flagged
        const bool grads = grad_gap_open || grad_gap_ext || grad_temperature;
        size_t pe = plane_bytes(D2P_FAMILY_AFFINE, MODE_MARG, B, L1, L2);
        const size_t tf = aff_tan_workspace_bytes(B, L1, L2, true);
        pe = pe > af ? pe : af;
        pe = pe > tf ? pe : tf;
        if (tf > 0) {
            const size_t tw = align256(tf) + align256((size_t)B * L1 * L2 * sizeof(float));
            pe = pe > tw ? pe : tw;
        }
        int* flags = (int*)((char*)workspace + align256(pe));
        int* order = (int*)((char*)flags + align256((size_t)B * sizeof(int)));
        a.redo = flags;
        a.only = nullptr;
        a.order = nullptr;
        int rc;
        if (grads) {
            a.sync = (int*)((char*)order + align256((size_t)B * sizeof(int)));
            rc = kNotHandled;
            SwArgs t = a;
            if (a.scores_bf16 && tf > 0) {
                // the tangent kernel reads fp32: widen bf16 scores (exactly) into
                // the workspace after its area; a flagged problem's plane-engine
                // fix-up reads the bf16 input itself (scores_bf16 stays set)
                float* wide = (float*)((char*)workspace + align256(tf));
                const int wr = launch_bf16_widen(a.scores_bf16, wide, (size_t)B * L1 * L2, st);
                if (wr == D2P_OK) t.scores = wide;
                else if (wr != kNotHandled) return wr;
            }
            if (t.scores) rc = launch_aff_tan(t, align256(tf), st);
            a.sync = nullptr;
        } else {
            if (lengths) {
                const int ro = launch_lin_order(lengths, B, L1, L2, order, st);
                if (ro == D2P_OK) a.order = order;
                else if (ro != kNotHandled) return ro;
            }
            a.sync = (int*)((char*)order + align256((size_t)B * sizeof(int)));
            rc = launch_aff_fast(a, workspace_bytes, st);
            a.sync = nullptr;
        }
        a.order = nullptr;
        a.redo = nullptr;
        if (rc == D2P_OK) {
            a.only = flags;
            return launch_aff_plane(a, st);
        }
        if (rc != kNotHandled) return rc;
        a.only = nullptr;
    }
    return launch_aff_plane(a, st);
}

int d2p_sw_affine_hvp(const float* scores, const float* tangent, const int* lengths, int B,
                      int L1, int L2, float gap_open, float gap_ext, float temperature,
                      float* hvp, void* workspace, size_t workspace_bytes, void* stream) {
    if (!dims_ok(B, L1, L2)) return D2P_ERR_TOO_LARGE;
    if (B == 0) return D2P_OK;
    if ((!scores || !tangent || !hvp) && L1 > 0 && L2 > 0) return D2P_ERR_INVALID_ARGUMENT;
    const size_t need = op_bytes(D2P_FAMILY_AFFINE, D2P_OP_HVP, B, L1, L2);
    if (need > 0 && (!workspace || workspace_bytes < need)) return D2P_ERR_WORKSPACE_TOO_SMALL;
    SwArgs a = base_args(scores, lengths, B, L1, L2);
    a.tangent = tangent;
    a.gap = gap_open;
    a.gap2 = gap_ext;
    a.temp = temperature;
    a.mode = MODE_HVP;
    a.out = hvp;
    a.ws = (float*)workspace;
    int* flags = (int*)((char*)workspace + tan_area(D2P_FAMILY_AFFINE, D2P_OP_HVP, B, L1, L2));
    return run_tangent(D2P_FAMILY_AFFINE, a, workspace_bytes, flags, (cudaStream_t)stream);
}

int d2p_sw_affine_param_jacobian(const float* scores, const int* lengths, int B, int L1, int L2,
                                 int param_type, float gap_open, float gap_ext,
                                 float temperature, float* jacobian, void* workspace,
                                 size_t workspace_bytes, void* stream) {
    if (param_type < 0 || param_type > 2) return D2P_ERR_INVALID_ARGUMENT;
    if (!dims_ok(B, L1, L2)) return D2P_ERR_TOO_LARGE;
    if (B == 0) return D2P_OK;
    if ((!scores || !jacobian) && L1 > 0 && L2 > 0) return D2P_ERR_INVALID_ARGUMENT;
    const size_t need = op_bytes(D2P_FAMILY_AFFINE, D2P_OP_PARAM_JACOBIAN, B, L1, L2);
    if (need > 0 && (!workspace || workspace_bytes < need)) return D2P_ERR_WORKSPACE_TOO_SMALL;
    SwArgs a = base_args(scores, lengths, B, L1, L2);
    a.gap = gap_open;
    a.gap2 = gap_ext;
    a.temp = temperature;
    a.mode = param_type == 0 ? MODE_PGAP : (param_type == 1 ? MODE_PGE : MODE_PT);
    a.out = jacobian;
    a.ws = (float*)workspace;
    int* flags = (int*)((char*)workspace + tan_area(D2P_FAMILY_AFFINE, D2P_OP_PARAM_JACOBIAN, B, L1, L2));
    return run_tangent(D2P_FAMILY_AFFINE, a, workspace_bytes, flags, (cudaStream_t)stream);
}

int d2p_sw_affine_backward_full(const float* scores, const float* grad_marginals,
                                const int* lengths, int B, int L1, int L2, float gap_open,
                                float gap_ext, float temperature, float* grad_scores,
                                float* grad_gap_open, float* grad_gap_ext,
                                float* grad_temperature, void* workspace,
                                size_t workspace_bytes, void* stream) {
    if (!dims_ok(B, L1, L2)) return D2P_ERR_TOO_LARGE;
    if (!grad_scores || !grad_gap_open || !grad_gap_ext || !grad_temperature) return D2P_ERR_INVALID_ARGUMENT;
    const size_t need = op_bytes(D2P_FAMILY_AFFINE, D2P_OP_BACKWARD_FULL, B, L1, L2);
    if (!workspace || workspace_bytes < need) return D2P_ERR_WORKSPACE_TOO_SMALL;
    cudaStream_t st = (cudaStream_t)stream;
    if (B == 0) {
        float* outs[3] = {grad_gap_open, grad_gap_ext, grad_temperature};
        for (float* o : outs) {
            cudaError_t e = cudaMemsetAsync(o, 0, sizeof(float), st);
            if (e != cudaSuccess) return (int)e;
        }
        return D2P_OK;
    }
    // grad_scores = H . grad_marginals (the Hessian of S is symmetric);
    // grad_gap_open / _ext / T = sum grad_marginals * dP/dgo, dP/dge, dP/dT
    const size_t area = tan_area(D2P_FAMILY_AFFINE, D2P_OP_BACKWARD_FULL, B, L1, L2);
    float* planes = (float*)workspace;
    float* partials = (float*)((char*)workspace + area);
    int* flags = (int*)((char*)partials + align256((size_t)4 * B * sizeof(float)));
    SwArgs a = base_args(scores, lengths, B, L1, L2);
    a.gap = gap_open;
    a.gap2 = gap_ext;
    a.temp = temperature;
    a.ws = planes;
    a.tangent = grad_marginals;
    a.mode = MODE_HVP;
    a.out = grad_scores;
    const int modes[3] = {MODE_PGAP, MODE_PGE, MODE_PT};
    float* outs[3] = {grad_gap_open, grad_gap_ext, grad_temperature};
    int* const sync = (int*)((char*)flags + align256((size_t)B * sizeof(int)));
    int* const flags2 = (int*)((char*)sync + align256((size_t)B * kSyncBytes));
    // Two sweep pairs of the tangent kernel (sw_affine_tangent.cu): the dot
    // sweep along gap_ext (d(dS/dge)[g] per problem), then the BF sweep (H . g,
    // d(dS/dgo)[g], and d(dS/dT)[g] by Euler's identity from the first).
    // Problems either flags get the plane engine's HVP and three dot sweeps.
    SwArgs d = a;
    d.mode = MODE_PGE;
    d.tangent = nullptr;
    d.out = nullptr;
    d.dot_with = grad_marginals;
    d.dot_out = partials + (size_t)B;
    d.redo = flags2;
    d.sync = sync;
    int rc = launch_aff_tan(d, workspace_bytes, st);
    if (rc == D2P_OK) {
        a.dot_out = partials;
        a.redo = flags;
        a.sync = sync;
        rc = launch_aff_tan(a, workspace_bytes, st);
        a.redo = nullptr;
        a.sync = nullptr;
        a.dot_out = nullptr;
        if (rc == D2P_OK) rc = launch_or_flags(flags, flags2, B, st);
        if (rc) return rc;
        a.only = flags;
        rc = launch_aff_plane(a, st);
        if (rc) return rc;
        a.tangent = nullptr;
        a.out = nullptr;
        a.dot_with = grad_marginals;
        for (int q = 0; q < 3; ++q) {
            a.mode = modes[q];
            a.dot_out = partials + (size_t)q * B;
            rc = launch_aff_plane(a, st);
            if (rc) return rc;
        }
        for (int q = 0; q < 3; ++q) {
            rc = launch_sum_batches(partials + (size_t)q * B, 1, B, outs[q], 0, st);
            if (rc) return rc;
        }
        return D2P_OK;
    }
    if (rc != kNotHandled) return rc;
    // shapes the tangent kernel does not take: the HVP and three dot sweep pairs
    rc = run_tangent(D2P_FAMILY_AFFINE, a, workspace_bytes, flags, st);
    if (rc) return rc;
    a.tangent = nullptr;
    a.out = nullptr;
    a.dot_with = grad_marginals;
    for (int q = 0; q < 3; ++q) {
        a.mode = modes[q];
        a.dot_out = partials + (size_t)q * B;
        rc = run_tangent(D2P_FAMILY_AFFINE, a, workspace_bytes, flags, st);
        if (rc) return rc;
        rc = launch_sum_batches(partials + (size_t)q * B, 1, B, outs[q], 0, st);
        if (rc) return rc;
    }
    return D2P_OK;
}

}  // extern "C"
