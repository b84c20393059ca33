// torch_bindings.cpp -- the reference's dispatcher surface (torch.ops.d2p.*) for the
// soft Smith-Waterman family, the soft Needleman-Wunsch operators (linear and
// affine gaps) and soft DTW,
// implemented on top of the C ABI in
// include/d2p_b200.h (libd2p_b200.so).
//
// Schemas are the reference's, verbatim (src/sw/registry.cpp:30-44,
// src/sw_affine/registry.cpp:27-42, src/nw/registry.cpp:35-49,
// src/nw_affine/registry.cpp:35-50, src/dtw/registry.cpp:35-40), so code written against d2p's ops binds
// unchanged.  CUDA and AutogradCUDA keys are registered exactly as the reference
// does (src/sw/torch_cuda.cpp:857-883, src/sw_affine/torch_cuda.cpp:914-948);
// there is no CPU kernel and no fallback: CPU tensors are rejected with the
// reference's "must be a CUDA tensor" message.
//
// Differences from the reference host glue, all behaviour-preserving:
//  * no cudaStreamSynchronize after launches, no DP planes cloned into the
//    autograd context (the value backward reuses the saved marginals, as the
//    reference's PT2 path does, d2p/_pt2_ops.py:178-206);
//  * tensor gap/temperature on the scores' device are read on the device
//    (no .item() host sync on the forward path);
//  * lengths=None is passed down as "full lengths" instead of materialising a
//    [B,2] tensor with a host->device copy.
#include <ATen/ATen.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/csrc/autograd/custom_function.h>
#include <torch/library.h>
#include <torch/types.h>

#include <limits>
#include <vector>

#include "../../include/d2p_b200.h"

namespace {

using torch::Tensor;
using torch::autograd::AutogradContext;
using torch::autograd::tensor_list;

#define D2PB_CHECK_CUDA(x) TORCH_CHECK((x).is_cuda(), #x " must be a CUDA tensor")
#define D2PB_CHECK_CONTIGUOUS(x) TORCH_CHECK((x).is_contiguous(), #x " must be contiguous")
#define D2PB_CHECK_FLOAT(x) \
    TORCH_CHECK((x).scalar_type() == torch::kFloat32, #x " must be float32, got ", (x).scalar_type())
#define D2PB_CHECK_INPUT(x) \
    D2PB_CHECK_CUDA(x);     \
    D2PB_CHECK_CONTIGUOUS(x); \
    D2PB_CHECK_FLOAT(x)

inline void check_rc(int rc, const char* what) {
    TORCH_CHECK(rc == 0, what, " failed: ", d2p_error_string(rc), " (code ", rc, ")");
}

inline void* cur_stream() { return (void*)at::cuda::getCurrentCUDAStream().stream(); }

struct Shape {
    int B, L1, L2;
};

// src/sw/torch_cuda.cpp:41-65 (messages kept)
int checked_dim(int64_t value, const char* name) {
    TORCH_CHECK(value >= 0 && value <= static_cast<int64_t>(std::numeric_limits<int>::max()),
                name, " must fit int32 CUDA kernel indexing, got ", value);
    return static_cast<int>(value);
}

Shape checked_shape(const Tensor& scores, int fam = D2P_FAMILY_LINEAR) {
    TORCH_CHECK(scores.dim() == 3, "scores must be 3D (B, L1, L2)");
    Shape s{checked_dim(scores.size(0), "scores batch dimension"),
            checked_dim(scores.size(1), "scores L1 dimension"),
            checked_dim(scores.size(2), "scores L2 dimension")};
    const int64_t cells = (static_cast<int64_t>(s.L1) + 1) * (static_cast<int64_t>(s.L2) + 1);
    TORCH_CHECK(cells <= static_cast<int64_t>(std::numeric_limits<int>::max()),
                fam == D2P_FAMILY_NW ? "NW" : "SW", " CUDA DP table is too large for 32-bit kernel indexing: ",
                "(L1 + 1) * (L2 + 1) = ", cells, " exceeds ", std::numeric_limits<int>::max());
    return s;
}

// src/sw_affine/torch_cuda.cpp:35-67: the affine family's limit counts its three
// state tables, 3 (L1 + 1) (L2 + 1) <= INT_MAX, with the reference's messages.
Shape checked_affine_shape(const Tensor& scores) {
    TORCH_CHECK(scores.dim() == 3, "scores must be 3D (B, L1, L2)");
    Shape s{checked_dim(scores.size(0), "scores batch dimension"),
            checked_dim(scores.size(1), "scores L1 dimension"),
            checked_dim(scores.size(2), "scores L2 dimension")};
    TORCH_CHECK(s.L1 <= std::numeric_limits<int>::max() - s.L2,
                "sw_affine dimensions too large: L1 + L2 exceeds CUDA int index range");
    const int64_t cells = 3 * (static_cast<int64_t>(s.L1) + 1) * (static_cast<int64_t>(s.L2) + 1);
    TORCH_CHECK(cells <= static_cast<int64_t>(std::numeric_limits<int>::max()),
                "sw_affine DP table too large: 3 * (L1 + 1) * (L2 + 1) exceeds CUDA int index range");
    return s;
}

// src/sw/torch_cuda.cpp:67-97: same checks and messages.  The range check needs
// the values on the host (one small device->host copy), as in the reference.
void validate_lengths(const Tensor& lengths, const Shape& s, const torch::Device& device) {
    D2PB_CHECK_CUDA(lengths);
    D2PB_CHECK_CONTIGUOUS(lengths);
    TORCH_CHECK(lengths.dim() == 2 && lengths.size(0) == s.B && lengths.size(1) == 2);
    TORCH_CHECK(lengths.dtype() == torch::kInt32, "lengths must be int32");
    TORCH_CHECK(lengths.device() == device, "lengths must be on same device as scores, got ",
                lengths.device(), " vs ", device);
    auto h = lengths.to(torch::kCPU);
    auto acc = h.accessor<int32_t, 2>();
    for (int b = 0; b < s.B; ++b) {
        const int l1 = acc[b][0], l2 = acc[b][1];
        TORCH_CHECK(l1 >= 0 && l1 <= s.L1, "lengths[", b, ",0] must be between 0 and ", s.L1, ", got ", l1);
        TORCH_CHECK(l2 >= 0 && l2 <= s.L2, "lengths[", b, ",1] must be between 0 and ", s.L2, ", got ", l2);
    }
}

// Returns an undefined tensor for "full lengths".
Tensor resolve_lengths(const c10::optional<Tensor>& lengths, const Shape& s, const torch::Device& dev) {
    if (!lengths.has_value() || !lengths->defined()) return Tensor();
    validate_lengths(*lengths, s, dev);
    return *lengths;
}

inline const int* len_ptr(const Tensor& t) { return t.defined() ? t.data_ptr<int>() : nullptr; }

Tensor workspace(int family, int op, const Shape& s, const torch::Device& dev, size_t* bytes) {
    size_t n = d2p_sw_workspace_bytes(family, op, s.B, s.L1, s.L2);
    TORCH_CHECK(n != static_cast<size_t>(-1), "SW CUDA problem size not supported");
    *bytes = n;
    return torch::empty({static_cast<int64_t>(n > 0 ? n : 1)},
                        torch::TensorOptions().dtype(torch::kUInt8).device(dev));
}

// A scalar parameter either as a device pointer (no sync) or a host float.
struct Param {
    float host = 0.f;
    const float* dev = nullptr;
    Tensor keep;
};

Param read_param(const Tensor& t, const Tensor& scores, const char* name) {
    TORCH_CHECK(t.numel() == 1, name, " must be a scalar tensor");
    Param p;
    if (t.is_cuda() && t.device() == scores.device()) {
        p.keep = t.to(torch::kFloat32).contiguous();
        p.dev = p.keep.data_ptr<float>();
    } else {
        p.host = t.to(torch::kCPU).to(torch::kFloat32).item<float>();
    }
    return p;
}

float host_value(const Tensor& t) { return t.to(torch::kCPU).to(torch::kFloat32).item<float>(); }

Tensor prep_grad(Tensor g, const Tensor& scores, const char* what) {
    TORCH_CHECK(g.sizes() == scores.sizes(), what, " shape mismatch: expected ", scores.sizes(),
                " but got ", g.sizes());
    TORCH_CHECK(g.is_cuda(), what, " must be on CUDA, got ", g.device());
    if (g.scalar_type() != torch::kFloat32) g = g.to(torch::kFloat32);
    if (g.device() != scores.device()) g = g.to(scores.device());
    return g.contiguous();
}

// =============================================================================
// linear gap: raw computations
// =============================================================================
struct LinFwd {
    Tensor value, marginals, dparams;  // dparams [2,B]: dS/dgap, dS/dT (undefined if not requested)
};

// want_params: also compute dS/dgap and dS/dT (needed by soft_sw_with_grads and
// when gap or temperature require grad); without them the linear-domain fast
// path can run.
LinFwd lin_forward(int fam, const Tensor& scores, const Param& gap, const Param& T, const Tensor& lengths,
                   const Shape& s, bool want_params) {
    auto opt = scores.options();
    LinFwd r;
    r.value = torch::empty({s.B}, opt);
    r.marginals = torch::empty({s.B, s.L1, s.L2}, opt);
    float* gg = nullptr;
    float* gt = nullptr;
    if (want_params) {
        r.dparams = torch::empty({2, s.B}, opt);
        gg = r.dparams.data_ptr<float>();
        gt = gg + s.B;
    }
    size_t wb = 0;
    Tensor ws = workspace(fam, D2P_OP_FORWARD_BACKWARD, s, scores.device(), &wb);
    const bool nw = fam == D2P_FAMILY_NW;
    check_rc((nw ? d2p_nw_forward_backward : d2p_sw_forward_backward)(
                 scores.data_ptr<float>(), len_ptr(lengths), s.B, s.L1, s.L2, gap.host, T.host, gap.dev, T.dev,
                 r.value.data_ptr<float>(), r.marginals.data_ptr<float>(), gg, gt, ws.data_ptr(), wb, cur_stream()),
             nw ? "d2p_nw_forward_backward" : "d2p_sw_forward_backward");
    return r;
}

Tensor lin_hvp_raw(int fam, const Tensor& scores, const Tensor& tangent, float gap, float T,
                   const Tensor& lengths, const Shape& s) {
    Tensor H = torch::empty({s.B, s.L1, s.L2}, scores.options());
    size_t wb = 0;
    Tensor ws = workspace(fam, D2P_OP_HVP, s, scores.device(), &wb);
    const bool nw = fam == D2P_FAMILY_NW;
    check_rc((nw ? d2p_nw_hvp : d2p_sw_hvp)(scores.data_ptr<float>(), tangent.data_ptr<float>(), len_ptr(lengths),
                                            s.B, s.L1, s.L2, gap, T, H.data_ptr<float>(), ws.data_ptr(), wb,
                                            cur_stream()),
             nw ? "d2p_nw_hvp" : "d2p_sw_hvp");
    return H;
}

Tensor lin_jac_raw(int fam, const Tensor& scores, int param_type, float gap, float T, const Tensor& lengths,
                   const Shape& s) {
    Tensor J = torch::empty({s.B, s.L1, s.L2}, scores.options());
    size_t wb = 0;
    Tensor ws = workspace(fam, D2P_OP_PARAM_JACOBIAN, s, scores.device(), &wb);
    const bool nw = fam == D2P_FAMILY_NW;
    check_rc((nw ? d2p_nw_param_jacobian : d2p_sw_param_jacobian)(scores.data_ptr<float>(), len_ptr(lengths), s.B,
                                                                  s.L1, s.L2, param_type, gap, T,
                                                                  J.data_ptr<float>(), ws.data_ptr(), wb,
                                                                  cur_stream()),
             nw ? "d2p_nw_param_jacobian" : "d2p_sw_param_jacobian");
    return J;
}

std::tuple<Tensor, Tensor, Tensor> lin_backward_full_raw(int fam, const Tensor& scores, const Tensor& G,
                                                         float gap, float T, const Tensor& lengths,
                                                         const Shape& s) {
    auto opt = scores.options();
    Tensor gs = torch::empty({s.B, s.L1, s.L2}, opt);
    Tensor gg = torch::empty({1}, opt), gT = torch::empty({1}, opt);
    size_t wb = 0;
    Tensor ws = workspace(fam, D2P_OP_BACKWARD_FULL, s, scores.device(), &wb);
    const bool nw = fam == D2P_FAMILY_NW;
    check_rc((nw ? d2p_nw_backward_full : d2p_sw_backward_full)(
                 scores.data_ptr<float>(), G.data_ptr<float>(), len_ptr(lengths), s.B, s.L1, s.L2, gap, T,
                 gs.data_ptr<float>(), gg.data_ptr<float>(), gT.data_ptr<float>(), ws.data_ptr(), wb, cur_stream()),
             nw ? "d2p_nw_backward_full" : "d2p_sw_backward_full");
    return {gs, gg, gT};
}

// =============================================================================
// linear gap: autograd function (reference SoftSWRegularCUDAFunction,
// src/sw/torch_cuda.cpp:178-411; for FAM = D2P_FAMILY_NW SoftNWCUDAFunction,
// src/nw/torch_cuda.cpp:115-330, which has the same outputs and gradients)
// =============================================================================
template <int FAM>
class LinFamilyFunction : public torch::autograd::Function<LinFamilyFunction<FAM>> {
   public:
    // lengths travels as an optional non-variable argument: autograd records
    // metadata (device, dtype) for every Tensor input, which an undefined
    // "full lengths" tensor does not have.
    static tensor_list forward(AutogradContext* ctx, Tensor scores, Tensor gap, Tensor temperature,
                               c10::optional<Tensor> lengths_opt) {
        Tensor lengths = lengths_opt.has_value() ? *lengths_opt : Tensor();
        ctx->set_materialize_grads(false);
        D2PB_CHECK_INPUT(scores);
        const Shape s = checked_shape(scores, FAM);
        c10::cuda::CUDAGuard guard(scores.device());
        Param pg = read_param(gap, scores, "gap");
        Param pT = read_param(temperature, scores, "temperature");
        if (lengths.defined()) validate_lengths(lengths, s, scores.device());
        LinFwd r = lin_forward(FAM, scores, pg, pT, lengths, s, gap.requires_grad() || temperature.requires_grad());
        ctx->save_for_backward({scores, r.marginals, r.dparams, gap, temperature});
        ctx->saved_data["lengths"] = lengths.defined() ? c10::IValue(lengths) : c10::IValue();
        return {r.value, r.marginals};
    }

    static tensor_list backward(AutogradContext* ctx, tensor_list grad_outputs) {
        auto saved = ctx->get_saved_variables();
        Tensor scores = saved[0], marginals = saved[1], dparams = saved[2];
        Tensor gap = saved[3], temperature = saved[4];
        Tensor lengths;
        if (!ctx->saved_data["lengths"].isNone()) lengths = ctx->saved_data["lengths"].toTensor();
        const Shape s = checked_shape(scores, FAM);
        c10::cuda::CUDAGuard guard(scores.device());
        auto opt = scores.options();
        Tensor gv = grad_outputs[0], gm = grad_outputs[1];
        // parameters that need no gradient get none (no zero-filled tensors)
        Tensor grad_scores;
        Tensor grad_gap = ctx->needs_input_grad(1) ? torch::zeros({1}, opt) : Tensor();
        Tensor grad_T = ctx->needs_input_grad(2) ? torch::zeros({1}, opt) : Tensor();
        bool have = false;
        if (gv.defined() && gv.numel() > 0) {
            Tensor g = gv.to(torch::kFloat32).contiguous();
            if (g.device() != scores.device()) g = g.to(scores.device());
            grad_scores = torch::empty({s.B, s.L1, s.L2}, opt);
            const bool params = dparams.defined();
            Tensor gp = params ? torch::empty({2}, opt) : Tensor();
            check_rc(d2p_sw_value_backward_lengths(g.data_ptr<float>(), marginals.data_ptr<float>(),
                                                   lengths.defined() ? lengths.data_ptr<int>() : nullptr,
                                                   params ? dparams.data_ptr<float>() : nullptr, params ? 2 : 0,
                                                   s.B, s.L1, s.L2, grad_scores.data_ptr<float>(),
                                                   params ? gp.data_ptr<float>() : nullptr, cur_stream()),
                     "d2p_sw_value_backward_lengths");
            if (params) {
                grad_gap = gp.narrow(0, 0, 1);
                grad_T = gp.narrow(0, 1, 1);
            }
            have = true;
        }
        if (gm.defined() && gm.numel() > 0) {
            Tensor G = prep_grad(gm, scores, "grad_posteriors");
            auto r = lin_backward_full_raw(FAM, scores, G, host_value(gap), host_value(temperature), lengths, s);
            grad_scores = have ? grad_scores + std::get<0>(r) : std::get<0>(r);
            if (ctx->needs_input_grad(1)) grad_gap = grad_gap + std::get<1>(r);
            if (ctx->needs_input_grad(2)) grad_T = grad_T + std::get<2>(r);
            have = true;
        }
        if (!have) grad_scores = torch::zeros({s.B, s.L1, s.L2}, opt);
        if (!ctx->needs_input_grad(1)) grad_gap = Tensor();
        if (!ctx->needs_input_grad(2)) grad_T = Tensor();
        return {grad_scores, grad_gap, grad_T, Tensor()};
    }
};

template <int FAM>
std::vector<Tensor> soft_lin_cuda(Tensor scores, Tensor gap, Tensor temperature, Tensor lengths) {
    return LinFamilyFunction<FAM>::apply(scores, gap, temperature, c10::optional<Tensor>(lengths));
}

template <int FAM>
std::vector<Tensor> soft_lin_float_cuda(Tensor scores, double gap, double temperature,
                                       c10::optional<Tensor> lengths) {
    D2PB_CHECK_INPUT(scores);
    const Shape s = checked_shape(scores, FAM);
    c10::cuda::CUDAGuard guard(scores.device());
    Tensor len = resolve_lengths(lengths, s, scores.device());
    auto cpu = torch::TensorOptions().dtype(torch::kFloat32);
    return LinFamilyFunction<FAM>::apply(scores, torch::full({1}, (float)gap, cpu),
                                 torch::full({1}, (float)temperature, cpu),
                                 len.defined() ? c10::optional<Tensor>(len) : c10::nullopt);
}

template <int FAM>
std::tuple<Tensor, Tensor, Tensor, Tensor> soft_lin_with_grads_cuda(Tensor scores, double gap,
                                                                   double temperature,
                                                                   c10::optional<Tensor> lengths) {
    D2PB_CHECK_INPUT(scores);
    const Shape s = checked_shape(scores, FAM);
    c10::cuda::CUDAGuard guard(scores.device());
    Tensor len = resolve_lengths(lengths, s, scores.device());
    Param pg, pT;
    pg.host = (float)gap;
    pT.host = (float)temperature;
    LinFwd r = lin_forward(FAM, scores, pg, pT, len, s, true);
    // the schema's outputs are independent tensors: no views of one buffer
    return {r.value, r.marginals, r.dparams[0].clone(), r.dparams[1].clone()};
}

template <int FAM>
Tensor soft_lin_hvp_cuda(Tensor scores, Tensor tangent, double gap, double temperature,
                        c10::optional<Tensor> lengths) {
    D2PB_CHECK_INPUT(scores);
    D2PB_CHECK_INPUT(tangent);
    TORCH_CHECK(scores.dim() == 3, "scores must be 3D");
    TORCH_CHECK(scores.sizes() == tangent.sizes(), "scores and tangent must have same shape");
    TORCH_CHECK(tangent.device() == scores.device(), "tangent must be on same device as scores, got ",
                tangent.device(), " vs ", scores.device());
    const Shape s = checked_shape(scores, FAM);
    c10::cuda::CUDAGuard guard(scores.device());
    Tensor len = resolve_lengths(lengths, s, scores.device());
    return lin_hvp_raw(FAM, scores, tangent, (float)gap, (float)temperature, len, s);
}

template <int FAM>
Tensor soft_lin_param_jacobian_cuda(Tensor scores, int64_t param_type, double gap, double temperature,
                                   c10::optional<Tensor> lengths) {
    D2PB_CHECK_INPUT(scores);
    TORCH_CHECK(scores.dim() == 3, "scores must be 3D");
    TORCH_CHECK(param_type >= 0 && param_type <= 1, "param_type must be 0 or 1");
    const Shape s = checked_shape(scores, FAM);
    c10::cuda::CUDAGuard guard(scores.device());
    Tensor len = resolve_lengths(lengths, s, scores.device());
    return lin_jac_raw(FAM, scores, (int)param_type, (float)gap, (float)temperature, len, s);
}

template <int FAM>
std::tuple<Tensor, Tensor, Tensor> soft_lin_backward_full_cuda(Tensor scores, Tensor grad_alignment,
                                                              double gap, double temperature,
                                                              c10::optional<Tensor> lengths) {
    D2PB_CHECK_INPUT(scores);
    TORCH_CHECK(scores.dim() == 3, "scores must be 3D (B, L1, L2)");
    TORCH_CHECK(grad_alignment.sizes() == scores.sizes(), "grad_alignment must have same shape as scores");
    TORCH_CHECK(grad_alignment.is_cuda(), "grad_alignment must be a CUDA tensor");
    TORCH_CHECK(grad_alignment.device() == scores.device(),
                "grad_alignment must be on same device as scores, got ", grad_alignment.device(), " vs ",
                scores.device());
    const Shape s = checked_shape(scores, FAM);
    c10::cuda::CUDAGuard guard(scores.device());
    Tensor len = resolve_lengths(lengths, s, scores.device());
    Tensor G = grad_alignment.contiguous();
    if (G.scalar_type() != torch::kFloat32) G = G.to(torch::kFloat32);
    return lin_backward_full_raw(FAM, scores, G, (float)gap, (float)temperature, len, s);
}

// namespaced aliases (src/sw/torch_cuda.cpp:778-848; src/nw/torch_cuda.cpp:700-785)
template <int FAM>
std::vector<Tensor> lin_forward_alias(Tensor scores, double gap, double temp, c10::optional<Tensor> lengths) {
    return soft_lin_float_cuda<FAM>(scores, gap, temp, lengths);
}
template <int FAM>
std::vector<Tensor> lin_forward_t_alias(Tensor scores, Tensor gap, Tensor temp, Tensor lengths) {
    return soft_lin_cuda<FAM>(scores, gap, temp, lengths);
}
template <int FAM>
std::tuple<Tensor, Tensor> lin_value_grad_params_alias(Tensor scores, double gap, double temp,
                                                       c10::optional<Tensor> lengths) {
    auto r = soft_lin_with_grads_cuda<FAM>(scores, gap, temp, lengths);
    return {std::get<2>(r), std::get<3>(r)};
}
template <int FAM>
std::tuple<Tensor, Tensor, Tensor> lin_marginals_backward_alias(Tensor scores, Tensor grad_marginals, double gap,
                                                                double temp, c10::optional<Tensor> lengths) {
    return soft_lin_backward_full_cuda<FAM>(scores, grad_marginals, gap, temp, lengths);
}
template <int FAM>
Tensor lin_marginals_hvp_alias(Tensor scores, Tensor v, double gap, double temp, c10::optional<Tensor> lengths) {
    return soft_lin_hvp_cuda<FAM>(scores, v, gap, temp, lengths);
}
template <int FAM>
Tensor lin_marginals_grad_gap_alias(Tensor scores, double gap, double temp, c10::optional<Tensor> lengths) {
    return soft_lin_param_jacobian_cuda<FAM>(scores, 0, gap, temp, lengths);
}
template <int FAM>
Tensor lin_marginals_grad_temp_alias(Tensor scores, double gap, double temp, c10::optional<Tensor> lengths) {
    return soft_lin_param_jacobian_cuda<FAM>(scores, 1, gap, temp, lengths);
}

constexpr int kSW = D2P_FAMILY_LINEAR;
constexpr int kNW = D2P_FAMILY_NW;

// =============================================================================
// affine gap
// =============================================================================
// The affine forward accepts bf16 scores directly (read as bf16, upcast in
// registers).  The reference requires fp32 (bf16 only via autocast,
// d2p/_compile.py:886-891); accepting bf16 is an extension that halves the
// score bytes of the bf16 workload and changes no fp32 behaviour.
#define D2PB_CHECK_AFF_SCORES(x)                                                        \
    D2PB_CHECK_CUDA(x);                                                                 \
    D2PB_CHECK_CONTIGUOUS(x);                                                           \
    TORCH_CHECK((x).scalar_type() == torch::kFloat32 || (x).scalar_type() == torch::kBFloat16, \
                #x " must be float32, got ", (x).scalar_type())

// SW affine reads fp32 or bf16 scores; NW affine fp32, as the reference
// (src/nw_affine/torch_cuda.cpp:57-58)
void check_aff_scores(const Tensor& scores, int fam) {
    if (fam == D2P_FAMILY_NW_AFFINE) {
        D2PB_CHECK_INPUT(scores);
    } else {
        D2PB_CHECK_AFF_SCORES(scores);
    }
}

struct AffFwd {
    Tensor value, marginals, dparams;  // dparams [3,B]: dS/dgap_open, dS/dgap_ext, dS/dT
};

// want_params: also compute the three parameter gradients (soft_sw_affine_with_grads,
// or parameters that require grad); without them the linear-domain fast path can run.
AffFwd aff_forward(int fam, const Tensor& scores, const Param& go, const Param& ge, const Param& T,
                   const Tensor& lengths, const Shape& s, bool want_params) {
    auto opt = scores.options().dtype(torch::kFloat32);
    AffFwd r;
    r.value = torch::empty({s.B}, opt);
    r.marginals = torch::empty({s.B, s.L1, s.L2}, opt);
    float* dp = nullptr;
    if (want_params) {
        r.dparams = torch::empty({3, s.B}, opt);
        dp = r.dparams.data_ptr<float>();
    }
    size_t wb = 0;
    Tensor ws = workspace(fam, D2P_OP_FORWARD_BACKWARD, s, scores.device(), &wb);
    if (fam == D2P_FAMILY_NW_AFFINE) {
        check_rc(d2p_nw_affine_forward_backward(scores.data_ptr<float>(), len_ptr(lengths), s.B, s.L1, s.L2,
                                                go.host, ge.host, T.host, go.dev, ge.dev, T.dev,
                                                r.value.data_ptr<float>(), r.marginals.data_ptr<float>(), dp,
                                                dp ? dp + s.B : nullptr, dp ? dp + 2 * s.B : nullptr,
                                                ws.data_ptr(), wb, cur_stream()),
                 "d2p_nw_affine_forward_backward");
        return r;
    }
    const int dt = scores.scalar_type() == torch::kBFloat16 ? D2P_DTYPE_BF16 : D2P_DTYPE_F32;
    check_rc(d2p_sw_affine_forward_backward(scores.data_ptr(), dt, len_ptr(lengths), s.B, s.L1, s.L2,
                                            go.host, ge.host, T.host, go.dev, ge.dev, T.dev,
                                            r.value.data_ptr<float>(), r.marginals.data_ptr<float>(), dp,
                                            dp ? dp + s.B : nullptr, dp ? dp + 2 * s.B : nullptr, ws.data_ptr(),
                                            wb, cur_stream()),
             "d2p_sw_affine_forward_backward");
    return r;
}

Tensor aff_hvp_raw(int fam, const Tensor& scores, const Tensor& tangent, float go, float ge, float T,
                   const Tensor& lengths, const Shape& s) {
    Tensor H = torch::empty({s.B, s.L1, s.L2}, scores.options());
    size_t wb = 0;
    Tensor ws = workspace(fam, D2P_OP_HVP, s, scores.device(), &wb);
    const bool nw = fam == D2P_FAMILY_NW_AFFINE;
    check_rc((nw ? d2p_nw_affine_hvp : d2p_sw_affine_hvp)(scores.data_ptr<float>(), tangent.data_ptr<float>(),
                                                          len_ptr(lengths), s.B, s.L1, s.L2, go, ge, T,
                                                          H.data_ptr<float>(), ws.data_ptr(), wb, cur_stream()),
             nw ? "d2p_nw_affine_hvp" : "d2p_sw_affine_hvp");
    return H;
}

Tensor aff_jac_raw(int fam, const Tensor& scores, int param_type, float go, float ge, float T,
                   const Tensor& lengths, const Shape& s) {
    Tensor J = torch::empty({s.B, s.L1, s.L2}, scores.options());
    size_t wb = 0;
    Tensor ws = workspace(fam, D2P_OP_PARAM_JACOBIAN, s, scores.device(), &wb);
    const bool nw = fam == D2P_FAMILY_NW_AFFINE;
    check_rc((nw ? d2p_nw_affine_param_jacobian : d2p_sw_affine_param_jacobian)(
                 scores.data_ptr<float>(), len_ptr(lengths), s.B, s.L1, s.L2, param_type, go, ge, T,
                 J.data_ptr<float>(), ws.data_ptr(), wb, cur_stream()),
             nw ? "d2p_nw_affine_param_jacobian" : "d2p_sw_affine_param_jacobian");
    return J;
}

std::tuple<Tensor, Tensor, Tensor, Tensor> aff_backward_full_raw(int fam, const Tensor& scores, const Tensor& G,
                                                                 float go, float ge, float T,
                                                                 const Tensor& lengths, const Shape& s) {
    auto opt = scores.options();
    Tensor gs = torch::empty({s.B, s.L1, s.L2}, opt);
    Tensor a = torch::empty({1}, opt), b = torch::empty({1}, opt), c = torch::empty({1}, opt);
    size_t wb = 0;
    Tensor ws = workspace(fam, D2P_OP_BACKWARD_FULL, s, scores.device(), &wb);
    const bool nw = fam == D2P_FAMILY_NW_AFFINE;
    check_rc((nw ? d2p_nw_affine_backward_full : d2p_sw_affine_backward_full)(
                 scores.data_ptr<float>(), G.data_ptr<float>(), len_ptr(lengths), s.B, s.L1, s.L2, go, ge, T,
                 gs.data_ptr<float>(), a.data_ptr<float>(), b.data_ptr<float>(), c.data_ptr<float>(), ws.data_ptr(),
                 wb, cur_stream()),
             nw ? "d2p_nw_affine_backward_full" : "d2p_sw_affine_backward_full");
    return {gs, a, b, c};
}

// reference SoftSWAffineCUDAFunction (src/sw_affine/torch_cuda.cpp:126-400); for
// FAM = D2P_FAMILY_NW_AFFINE SoftNWAffineCUDAFunction
// (src/nw_affine/torch_cuda.cpp:170-420), same outputs and gradients, fp32 scores
template <int FAM>
class AffFamilyFunction : public torch::autograd::Function<AffFamilyFunction<FAM>> {
   public:
    static tensor_list forward(AutogradContext* ctx, Tensor scores, Tensor gap_open, Tensor gap_ext,
                               Tensor temperature, c10::optional<Tensor> lengths_opt) {
        Tensor lengths = lengths_opt.has_value() ? *lengths_opt : Tensor();
        ctx->set_materialize_grads(false);
        check_aff_scores(scores, FAM);
        const Shape s = checked_affine_shape(scores);
        c10::cuda::CUDAGuard guard(scores.device());
        Param po = read_param(gap_open, scores, "gap_open");
        Param pe = read_param(gap_ext, scores, "gap_ext");
        Param pT = read_param(temperature, scores, "temperature");
        if (lengths.defined()) validate_lengths(lengths, s, scores.device());
        const bool want = gap_open.requires_grad() || gap_ext.requires_grad() || temperature.requires_grad();
        AffFwd r = aff_forward(FAM, scores, po, pe, pT, lengths, s, want);
        ctx->save_for_backward({scores, r.marginals, r.dparams, gap_open, gap_ext, temperature});
        ctx->saved_data["lengths"] = lengths.defined() ? c10::IValue(lengths) : c10::IValue();
        return {r.value, r.marginals};
    }

    static tensor_list backward(AutogradContext* ctx, tensor_list grad_outputs) {
        auto saved = ctx->get_saved_variables();
        Tensor scores = saved[0], marginals = saved[1], dparams = saved[2];
        Tensor go = saved[3], ge = saved[4], temperature = saved[5];
        Tensor lengths;
        if (!ctx->saved_data["lengths"].isNone()) lengths = ctx->saved_data["lengths"].toTensor();
        const Shape s = checked_affine_shape(scores);
        c10::cuda::CUDAGuard guard(scores.device());
        auto opt = scores.options().dtype(torch::kFloat32);
        Tensor gv = grad_outputs[0], gm = grad_outputs[1];
        // parameters that need no gradient get none (no zero-filled tensors)
        Tensor grad_scores;
        Tensor g_o = ctx->needs_input_grad(1) ? torch::zeros({1}, opt) : Tensor();
        Tensor g_e = ctx->needs_input_grad(2) ? torch::zeros({1}, opt) : Tensor();
        Tensor g_T = ctx->needs_input_grad(3) ? torch::zeros({1}, opt) : Tensor();
        bool have = false;
        if (gv.defined() && gv.numel() > 0) {
            Tensor g = gv.to(torch::kFloat32).contiguous();
            if (g.device() != scores.device()) g = g.to(scores.device());
            grad_scores = torch::empty({s.B, s.L1, s.L2}, opt);
            const bool params = dparams.defined();
            Tensor gp = params ? torch::empty({3}, opt) : Tensor();
            check_rc(d2p_sw_value_backward_lengths(g.data_ptr<float>(), marginals.data_ptr<float>(),
                                                   lengths.defined() ? lengths.data_ptr<int>() : nullptr,
                                                   params ? dparams.data_ptr<float>() : nullptr, params ? 3 : 0,
                                                   s.B, s.L1, s.L2, grad_scores.data_ptr<float>(),
                                                   params ? gp.data_ptr<float>() : nullptr, cur_stream()),
                     "d2p_sw_value_backward_lengths");
            if (params) {
                g_o = gp.narrow(0, 0, 1);
                g_e = gp.narrow(0, 1, 1);
                g_T = gp.narrow(0, 2, 1);
            }
            have = true;
        }
        if (gm.defined() && gm.numel() > 0) {
            Tensor G = prep_grad(gm, scores, "grad_posteriors");
            Tensor sf = scores.scalar_type() == torch::kFloat32 ? scores : scores.to(torch::kFloat32);
            auto r = aff_backward_full_raw(FAM, sf, G, host_value(go), host_value(ge), host_value(temperature),
                                           lengths, s);
            grad_scores = have ? grad_scores + std::get<0>(r) : std::get<0>(r);
            if (ctx->needs_input_grad(1)) g_o = g_o + std::get<1>(r);
            if (ctx->needs_input_grad(2)) g_e = g_e + std::get<2>(r);
            if (ctx->needs_input_grad(3)) g_T = g_T + std::get<3>(r);
            have = true;
        }
        if (!have) grad_scores = torch::zeros({s.B, s.L1, s.L2}, opt);
        if (!ctx->needs_input_grad(1)) g_o = Tensor();
        if (!ctx->needs_input_grad(2)) g_e = Tensor();
        if (!ctx->needs_input_grad(3)) g_T = Tensor();
        return {grad_scores, g_o, g_e, g_T, Tensor()};
    }
};

template <int FAM>
std::vector<Tensor> soft_aff_cuda(Tensor scores, Tensor gap_open, Tensor gap_ext, Tensor temperature,
                                  Tensor lengths) {
    return AffFamilyFunction<FAM>::apply(scores, gap_open, gap_ext, temperature, c10::optional<Tensor>(lengths));
}

template <int FAM>
std::vector<Tensor> soft_aff_float_cuda(Tensor scores, double gap_open, double gap_ext,
                                        double temperature, c10::optional<Tensor> lengths) {
    check_aff_scores(scores, FAM);
    const Shape s = checked_affine_shape(scores);
    c10::cuda::CUDAGuard guard(scores.device());
    Tensor len = resolve_lengths(lengths, s, scores.device());
    auto cpu = torch::TensorOptions().dtype(torch::kFloat32);
    return AffFamilyFunction<FAM>::apply(scores, torch::full({1}, (float)gap_open, cpu),
                                       torch::full({1}, (float)gap_ext, cpu),
                                       torch::full({1}, (float)temperature, cpu),
                                       len.defined() ? c10::optional<Tensor>(len) : c10::nullopt);
}

template <int FAM>
std::tuple<Tensor, Tensor, Tensor, Tensor, Tensor> soft_aff_with_grads_cuda(
    Tensor scores, double gap_open, double gap_ext, double temperature, c10::optional<Tensor> lengths) {
    check_aff_scores(scores, FAM);
    const Shape s = checked_affine_shape(scores);
    c10::cuda::CUDAGuard guard(scores.device());
    Tensor len = resolve_lengths(lengths, s, scores.device());
    Param po, pe, pT;
    po.host = (float)gap_open;
    pe.host = (float)gap_ext;
    pT.host = (float)temperature;
    AffFwd r = aff_forward(FAM, scores, po, pe, pT, len, s, true);
    return {r.value, r.marginals, r.dparams[0].clone(), r.dparams[1].clone(), r.dparams[2].clone()};
}

template <int FAM>
Tensor soft_aff_hvp_cuda(Tensor scores, Tensor tangent, double gap_open, double gap_ext,
                               double temperature, c10::optional<Tensor> lengths) {
    D2PB_CHECK_INPUT(scores);
    D2PB_CHECK_INPUT(tangent);
    TORCH_CHECK(scores.dim() == 3, "scores must be 3D");
    TORCH_CHECK(scores.sizes() == tangent.sizes(), "scores and tangent must have same shape");
    TORCH_CHECK(tangent.device() == scores.device(), "tangent must be on same device as scores, got ",
                tangent.device(), " vs ", scores.device());
    const Shape s = checked_affine_shape(scores);
    c10::cuda::CUDAGuard guard(scores.device());
    Tensor len = resolve_lengths(lengths, s, scores.device());
    return aff_hvp_raw(FAM, scores, tangent, (float)gap_open, (float)gap_ext, (float)temperature, len, s);
}

template <int FAM>
Tensor soft_aff_param_jacobian_cuda(Tensor scores, int64_t param_type, double gap_open,
                                          double gap_ext, double temperature,
                                          c10::optional<Tensor> lengths) {
    D2PB_CHECK_INPUT(scores);
    TORCH_CHECK(scores.dim() == 3, "scores must be 3D");
    TORCH_CHECK(param_type >= 0 && param_type <= 2, "param_type must be 0, 1, or 2");
    const Shape s = checked_affine_shape(scores);
    c10::cuda::CUDAGuard guard(scores.device());
    Tensor len = resolve_lengths(lengths, s, scores.device());
    return aff_jac_raw(FAM, scores, (int)param_type, (float)gap_open, (float)gap_ext, (float)temperature, len, s);
}

template <int FAM>
std::tuple<Tensor, Tensor, Tensor, Tensor> soft_aff_backward_full_cuda(
    Tensor scores, Tensor grad_alignment, double gap_open, double gap_ext, double temperature,
    c10::optional<Tensor> lengths) {
    D2PB_CHECK_INPUT(scores);
    TORCH_CHECK(scores.dim() == 3, "scores must be 3D (B, L1, L2)");
    TORCH_CHECK(grad_alignment.sizes() == scores.sizes(), "grad_alignment must have same shape as scores");
    TORCH_CHECK(grad_alignment.is_cuda(), "grad_alignment must be a CUDA tensor");
    TORCH_CHECK(grad_alignment.device() == scores.device(),
                "grad_alignment must be on same device as scores, got ", grad_alignment.device(), " vs ",
                scores.device());
    const Shape s = checked_affine_shape(scores);
    c10::cuda::CUDAGuard guard(scores.device());
    Tensor len = resolve_lengths(lengths, s, scores.device());
    Tensor G = grad_alignment.contiguous();
    if (G.scalar_type() != torch::kFloat32) G = G.to(torch::kFloat32);
    return aff_backward_full_raw(FAM, scores, G, (float)gap_open, (float)gap_ext, (float)temperature, len, s);
}

// namespaced aliases (src/sw_affine/torch_cuda.cpp:820-911; src/nw_affine/torch_cuda.cpp:700-785)
template <int FAM>
std::vector<Tensor> aff_forward_alias(Tensor scores, double go, double ge, double temp,
                                      c10::optional<Tensor> lengths) {
    return soft_aff_float_cuda<FAM>(scores, go, ge, temp, lengths);
}
template <int FAM>
std::vector<Tensor> aff_forward_t_alias(Tensor scores, Tensor go, Tensor ge, Tensor temp, Tensor lengths) {
    return soft_aff_cuda<FAM>(scores, go, ge, temp, lengths);
}
template <int FAM>
std::tuple<Tensor, Tensor, Tensor> aff_value_grad_params_alias(Tensor scores, double go, double ge, double temp,
                                                               c10::optional<Tensor> lengths) {
    auto r = soft_aff_with_grads_cuda<FAM>(scores, go, ge, temp, lengths);
    return {std::get<2>(r), std::get<3>(r), std::get<4>(r)};
}
template <int FAM>
std::tuple<Tensor, Tensor, Tensor, Tensor> aff_marginals_backward_alias(Tensor scores, Tensor g, double go, double ge,
                                                                        double temp,
                                                                        c10::optional<Tensor> lengths) {
    return soft_aff_backward_full_cuda<FAM>(scores, g, go, ge, temp, lengths);
}
template <int FAM>
Tensor aff_marginals_hvp_alias(Tensor scores, Tensor v, double go, double ge, double temp,
                               c10::optional<Tensor> lengths) {
    return soft_aff_hvp_cuda<FAM>(scores, v, go, ge, temp, lengths);
}
template <int FAM, int PT>
Tensor aff_marginals_grad_alias(Tensor scores, double go, double ge, double temp, c10::optional<Tensor> lengths) {
    return soft_aff_param_jacobian_cuda<FAM>(scores, PT, go, ge, temp, lengths);
}

constexpr int kAff = D2P_FAMILY_AFFINE;
constexpr int kNWAff = D2P_FAMILY_NW_AFFINE;

// =============================================================================
// soft DTW (reference SoftDTWCUDAFunction and bindings, src/dtw/torch_cuda.cpp:140-600)
// =============================================================================
// the reference's bandwidth range check (src/dtw/torch_cuda.cpp:73-80)
int checked_dtw_bandwidth(int64_t bandwidth) {
    TORCH_CHECK(bandwidth >= std::numeric_limits<int>::min() && bandwidth <= std::numeric_limits<int>::max(),
                "DTW bandwidth is out of CUDA int range: ", bandwidth);
    return static_cast<int>(bandwidth);
}

Shape checked_dtw_shape(const Tensor& costs) {
    TORCH_CHECK(costs.dim() == 3, "costs must be 3D (B, L1, L2)");
    return checked_shape(costs);
}

struct DtwFwd {
    Tensor value, marginals, dT;   // dT [B]: dS/dT (undefined if not requested)
};

DtwFwd dtw_forward(const Tensor& costs, const Param& T, const Tensor& lengths, const Shape& s, int bw,
                   bool want_T) {
    auto opt = costs.options();
    DtwFwd r;
    r.value = torch::empty({s.B}, opt);
    r.marginals = torch::empty({s.B, s.L1, s.L2}, opt);
    if (want_T) r.dT = torch::empty({s.B}, opt);
    size_t wb = 0;
    Tensor ws = workspace(D2P_FAMILY_DTW, D2P_OP_FORWARD_BACKWARD, s, costs.device(), &wb);
    check_rc(d2p_dtw_forward_backward(costs.data_ptr<float>(), len_ptr(lengths), s.B, s.L1, s.L2, T.host, T.dev, bw,
                                      r.value.data_ptr<float>(), r.marginals.data_ptr<float>(),
                                      want_T ? r.dT.data_ptr<float>() : nullptr, ws.data_ptr(), wb, cur_stream()),
             "d2p_dtw_forward_backward");
    return r;
}

Tensor dtw_hvp_raw(const Tensor& costs, const Tensor& tangent, float T, const Tensor& lengths, const Shape& s,
                   int bw) {
    Tensor H = torch::empty({s.B, s.L1, s.L2}, costs.options());
    size_t wb = 0;
    Tensor ws = workspace(D2P_FAMILY_DTW, D2P_OP_HVP, s, costs.device(), &wb);
    check_rc(d2p_dtw_hvp(costs.data_ptr<float>(), tangent.data_ptr<float>(), len_ptr(lengths), s.B, s.L1, s.L2, T,
                         bw, H.data_ptr<float>(), ws.data_ptr(), wb, cur_stream()),
             "d2p_dtw_hvp");
    return H;
}

Tensor dtw_jac_raw(const Tensor& costs, float T, const Tensor& lengths, const Shape& s, int bw) {
    Tensor J = torch::empty({s.B, s.L1, s.L2}, costs.options());
    size_t wb = 0;
    Tensor ws = workspace(D2P_FAMILY_DTW, D2P_OP_PARAM_JACOBIAN, s, costs.device(), &wb);
    check_rc(d2p_dtw_param_jacobian(costs.data_ptr<float>(), len_ptr(lengths), s.B, s.L1, s.L2, T, bw,
                                    J.data_ptr<float>(), ws.data_ptr(), wb, cur_stream()),
             "d2p_dtw_param_jacobian");
    return J;
}

std::tuple<Tensor, Tensor> dtw_backward_full_raw(const Tensor& costs, const Tensor& G, float T,
                                                 const Tensor& lengths, const Shape& s, int bw) {
    auto opt = costs.options();
    Tensor gc = torch::empty({s.B, s.L1, s.L2}, opt);
    Tensor gT = torch::empty({1}, opt);
    size_t wb = 0;
    Tensor ws = workspace(D2P_FAMILY_DTW, D2P_OP_BACKWARD_FULL, s, costs.device(), &wb);
    check_rc(d2p_dtw_backward_full(costs.data_ptr<float>(), G.data_ptr<float>(), len_ptr(lengths), s.B, s.L1, s.L2,
                                   T, bw, gc.data_ptr<float>(), gT.data_ptr<float>(), ws.data_ptr(), wb,
                                   cur_stream()),
             "d2p_dtw_backward_full");
    return {gc, gT};
}

// outputs (cost [B], alignment [B,L1,L2]); backward: (grad costs, grad T [1],
// none for lengths and bandwidth)
class SoftDTWFunction : public torch::autograd::Function<SoftDTWFunction> {
   public:
    static tensor_list forward(AutogradContext* ctx, Tensor costs, Tensor temperature,
                               c10::optional<Tensor> lengths_opt, int64_t bandwidth) {
        Tensor lengths = lengths_opt.has_value() ? *lengths_opt : Tensor();
        ctx->set_materialize_grads(false);
        D2PB_CHECK_INPUT(costs);
        const Shape s = checked_dtw_shape(costs);
        c10::cuda::CUDAGuard guard(costs.device());
        const int bw = checked_dtw_bandwidth(bandwidth);
        Param pT = read_param(temperature, costs, "temperature");
        if (lengths.defined()) validate_lengths(lengths, s, costs.device());
        DtwFwd r = dtw_forward(costs, pT, lengths, s, bw, temperature.requires_grad());
        ctx->save_for_backward({costs, r.marginals, r.dT, temperature});
        ctx->saved_data["lengths"] = lengths.defined() ? c10::IValue(lengths) : c10::IValue();
        ctx->saved_data["bandwidth"] = static_cast<int64_t>(bw);
        return {r.value, r.marginals};
    }

    static tensor_list backward(AutogradContext* ctx, tensor_list grad_outputs) {
        auto saved = ctx->get_saved_variables();
        Tensor costs = saved[0], marginals = saved[1], dT = saved[2], temperature = saved[3];
        Tensor lengths;
        if (!ctx->saved_data["lengths"].isNone()) lengths = ctx->saved_data["lengths"].toTensor();
        const int bw = static_cast<int>(ctx->saved_data["bandwidth"].toInt());
        const Shape s = checked_dtw_shape(costs);
        c10::cuda::CUDAGuard guard(costs.device());
        auto opt = costs.options();
        Tensor gv = grad_outputs[0], gm = grad_outputs[1];
        Tensor grad_costs;
        Tensor grad_T = ctx->needs_input_grad(1) ? torch::zeros({1}, opt) : Tensor();
        bool have = false;
        if (gv.defined() && gv.numel() > 0) {
            Tensor g = gv.to(torch::kFloat32).contiguous();
            if (g.device() != costs.device()) g = g.to(costs.device());
            grad_costs = torch::empty({s.B, s.L1, s.L2}, opt);
            const bool param = dT.defined();
            Tensor gp = param ? torch::empty({1}, opt) : Tensor();
            check_rc(d2p_sw_value_backward_lengths(g.data_ptr<float>(), marginals.data_ptr<float>(),
                                                   lengths.defined() ? lengths.data_ptr<int>() : nullptr,
                                                   param ? dT.data_ptr<float>() : nullptr, param ? 1 : 0, s.B,
                                                   s.L1, s.L2, grad_costs.data_ptr<float>(),
                                                   param ? gp.data_ptr<float>() : nullptr, cur_stream()),
                     "d2p_sw_value_backward_lengths");
            if (param) grad_T = gp;
            have = true;
        }
        if (gm.defined() && gm.numel() > 0) {
            Tensor G = prep_grad(gm, costs, "grad_posteriors");
            auto r = dtw_backward_full_raw(costs, G, host_value(temperature), lengths, s, bw);
            grad_costs = have ? grad_costs + std::get<0>(r) : std::get<0>(r);
            if (ctx->needs_input_grad(1)) grad_T = grad_T + std::get<1>(r);
            have = true;
        }
        if (!have) grad_costs = torch::zeros({s.B, s.L1, s.L2}, opt);
        if (!ctx->needs_input_grad(1)) grad_T = Tensor();
        return {grad_costs, grad_T, Tensor(), Tensor()};
    }
};

std::vector<Tensor> soft_dtw_cuda(Tensor costs, Tensor temperature, Tensor lengths, int64_t bandwidth) {
    return SoftDTWFunction::apply(costs, temperature, c10::optional<Tensor>(lengths), bandwidth);
}

std::vector<Tensor> soft_dtw_float_cuda(Tensor costs, double temperature, c10::optional<Tensor> lengths,
                                        c10::optional<int64_t> bandwidth) {
    D2PB_CHECK_INPUT(costs);
    const Shape s = checked_dtw_shape(costs);
    c10::cuda::CUDAGuard guard(costs.device());
    Tensor len = resolve_lengths(lengths, s, costs.device());
    auto cpu = torch::TensorOptions().dtype(torch::kFloat32);
    return SoftDTWFunction::apply(costs, torch::full({1}, (float)temperature, cpu),
                                  len.defined() ? c10::optional<Tensor>(len) : c10::nullopt,
                                  bandwidth.has_value() ? *bandwidth : -1);
}

std::tuple<Tensor, Tensor, Tensor> soft_dtw_with_grads_cuda(Tensor costs, double temperature,
                                                            c10::optional<Tensor> lengths,
                                                            c10::optional<int64_t> bandwidth) {
    D2PB_CHECK_INPUT(costs);
    const Shape s = checked_dtw_shape(costs);
    c10::cuda::CUDAGuard guard(costs.device());
    Tensor len = resolve_lengths(lengths, s, costs.device());
    Param pT;
    pT.host = (float)temperature;
    DtwFwd r = dtw_forward(costs, pT, len, s, checked_dtw_bandwidth(bandwidth.has_value() ? *bandwidth : -1), true);
    return {r.value, r.marginals, r.dT};
}

Tensor soft_dtw_hvp_cuda(Tensor costs, Tensor tangent, double temperature, c10::optional<Tensor> lengths,
                         c10::optional<int64_t> bandwidth) {
    D2PB_CHECK_INPUT(costs);
    D2PB_CHECK_INPUT(tangent);
    TORCH_CHECK(costs.dim() == 3, "costs must be 3D");
    TORCH_CHECK(tangent.sizes() == costs.sizes(), "tangent must have same shape as costs");
    TORCH_CHECK(tangent.device() == costs.device(), "tangent must be on same device as costs, got ",
                tangent.device(), " vs ", costs.device());
    const Shape s = checked_dtw_shape(costs);
    c10::cuda::CUDAGuard guard(costs.device());
    Tensor len = resolve_lengths(lengths, s, costs.device());
    return dtw_hvp_raw(costs, tangent, (float)temperature, len, s,
                       checked_dtw_bandwidth(bandwidth.has_value() ? *bandwidth : -1));
}

Tensor soft_dtw_param_jacobian_cuda(Tensor costs, double temperature, c10::optional<Tensor> lengths,
                                    c10::optional<int64_t> bandwidth) {
    D2PB_CHECK_INPUT(costs);
    TORCH_CHECK(costs.dim() == 3, "costs must be 3D");
    const Shape s = checked_dtw_shape(costs);
    c10::cuda::CUDAGuard guard(costs.device());
    Tensor len = resolve_lengths(lengths, s, costs.device());
    return dtw_jac_raw(costs, (float)temperature, len, s,
                       checked_dtw_bandwidth(bandwidth.has_value() ? *bandwidth : -1));
}

std::tuple<Tensor, Tensor> soft_dtw_backward_full_cuda(Tensor costs, Tensor grad_alignment, double temperature,
                                                       c10::optional<Tensor> lengths,
                                                       c10::optional<int64_t> bandwidth) {
    D2PB_CHECK_INPUT(costs);
    TORCH_CHECK(costs.dim() == 3, "costs must be 3D (B, L1, L2)");
    TORCH_CHECK(grad_alignment.sizes() == costs.sizes(), "grad_alignment must have same shape as costs");
    TORCH_CHECK(grad_alignment.is_cuda(), "grad_alignment must be a CUDA tensor");
    TORCH_CHECK(grad_alignment.device() == costs.device(), "grad_alignment must be on same device as costs, got ",
                grad_alignment.device(), " vs ", costs.device());
    const Shape s = checked_dtw_shape(costs);
    c10::cuda::CUDAGuard guard(costs.device());
    Tensor len = resolve_lengths(lengths, s, costs.device());
    Tensor G = grad_alignment.contiguous();
    if (G.scalar_type() != torch::kFloat32) G = G.to(torch::kFloat32);
    return dtw_backward_full_raw(costs, G, (float)temperature, len, s,
                                 checked_dtw_bandwidth(bandwidth.has_value() ? *bandwidth : -1));
}

}  // namespace

// =============================================================================
// schemas (verbatim from the reference registries) and implementations
// =============================================================================
// =============================================================================
// score producer (no reference operator: its examples build the score plane
// with an einsum, docs/examples.md:9-23): scores = scale * x y^T on tcgen05
// =============================================================================
Tensor embed_scores_cuda(const Tensor& x, const Tensor& y, double scale) {
    TORCH_CHECK(x.is_cuda() && y.is_cuda(), "embed_scores: x and y must be CUDA tensors");
    TORCH_CHECK(x.scalar_type() == at::kBFloat16 && y.scalar_type() == at::kBFloat16,
                "embed_scores: x and y must be bfloat16");
    TORCH_CHECK(x.dim() == 3 && y.dim() == 3, "embed_scores: x must be [B, L1, D] and y [B, L2, D]");
    TORCH_CHECK(x.size(0) == y.size(0) && x.size(2) == y.size(2), "embed_scores: x and y must share B and D");
    TORCH_CHECK(x.device() == y.device(), "embed_scores: x and y must be on the same device");
    const c10::cuda::CUDAGuard guard(x.device());
    const Tensor xc = x.contiguous(), yc = y.contiguous();
    const int64_t B = x.size(0), L1 = x.size(1), L2 = y.size(1), D = x.size(2);
    TORCH_CHECK(B <= 65535 && L1 <= std::numeric_limits<int>::max() && L2 <= std::numeric_limits<int>::max(),
                "embed_scores: sizes out of range");
    Tensor out = torch::empty({B, L1, L2}, x.options().dtype(at::kFloat));
    check_rc(d2p_embed_scores(xc.data_ptr(), yc.data_ptr(), (int)B, (int)L1, (int)L2, (int)D, (float)scale,
                              out.data_ptr<float>(), nullptr, cur_stream()),
             "d2p_embed_scores");
    return out;
}

// bf16(scale * grad_value[b] * marginals[b]): the scores' gradient of a loss of the values
Tensor embed_grad_scores_cuda(const Tensor& marginals, const Tensor& grad_value, double scale) {
    TORCH_CHECK(marginals.is_cuda() && marginals.scalar_type() == at::kFloat && marginals.dim() == 3,
                "embed_grad_scores: marginals must be a [B, L1, L2] fp32 CUDA tensor");
    TORCH_CHECK(grad_value.is_cuda() && grad_value.scalar_type() == at::kFloat && grad_value.numel() == marginals.size(0),
                "embed_grad_scores: grad_value must be a [B] fp32 CUDA tensor");
    const c10::cuda::CUDAGuard guard(marginals.device());
    const Tensor P = marginals.contiguous(), g = grad_value.contiguous();
    Tensor out = torch::empty(P.sizes(), P.options().dtype(at::kBFloat16));
    check_rc(d2p_embed_grad_scores(P.data_ptr<float>(), g.data_ptr<float>(), (int)P.size(0), (int)P.size(1),
                                   (int)P.size(2), (float)scale, out.data_ptr(), cur_stream()),
             "d2p_embed_grad_scores");
    return out;
}

TORCH_LIBRARY_FRAGMENT(d2p_b200, m) {
    m.def("embed_scores(Tensor x, Tensor y, float scale) -> Tensor");
    m.def("embed_grad_scores(Tensor marginals, Tensor grad_value, float scale) -> Tensor");
}
TORCH_LIBRARY_IMPL(d2p_b200, CUDA, m) {
    m.impl("embed_scores", embed_scores_cuda);
    m.impl("embed_grad_scores", embed_grad_scores_cuda);
}

TORCH_LIBRARY_FRAGMENT(d2p, m) {
    // src/sw/registry.cpp:30-44
    m.def("soft_sw(Tensor scores, Tensor gap, Tensor temperature, Tensor lengths) -> Tensor[]");
    m.def("soft_sw_float(Tensor scores, float gap, float temperature, Tensor? lengths) -> Tensor[]");
    m.def("soft_sw_with_grads(Tensor scores, float gap, float temperature, Tensor? lengths) -> (Tensor, Tensor, Tensor, Tensor)");
    m.def("soft_sw_hvp(Tensor scores, Tensor tangent, float gap, float temperature, Tensor? lengths) -> Tensor");
    m.def("soft_sw_param_jacobian(Tensor scores, int param_type, float gap, float temperature, Tensor? lengths) -> Tensor");
    m.def("soft_sw_backward_full(Tensor scores, Tensor grad_alignment, float gap, float temperature, Tensor? lengths) -> (Tensor, Tensor, Tensor)");
    m.def("sw_forward(Tensor scores, float gap, float temp, Tensor? lengths) -> Tensor[]");
    m.def("sw_forward_t(Tensor scores, Tensor gap, Tensor temp, Tensor lengths) -> Tensor[]");
    m.def("sw_value_grad_params(Tensor scores, float gap, float temp, Tensor? lengths) -> (Tensor, Tensor)");
    m.def("sw_marginals_backward(Tensor scores, Tensor grad_marginals, float gap, float temp, Tensor? lengths) -> (Tensor, Tensor, Tensor)");
    m.def("sw_marginals_hvp(Tensor scores, Tensor v, float gap, float temp, Tensor? lengths) -> Tensor");
    m.def("sw_marginals_grad_gap(Tensor scores, float gap, float temp, Tensor? lengths) -> Tensor");
    m.def("sw_marginals_grad_temp(Tensor scores, float gap, float temp, Tensor? lengths) -> Tensor");
    // soft Needleman-Wunsch, linear gap (src/nw/registry.cpp:35-49)
    m.def("soft_nw(Tensor scores, Tensor gap, Tensor temperature, Tensor lengths) -> Tensor[]");
    m.def("soft_nw_float(Tensor scores, float gap, float temperature, Tensor? lengths) -> Tensor[]");
    m.def("soft_nw_with_grads(Tensor scores, float gap, float temperature, Tensor? lengths) -> (Tensor, Tensor, Tensor, Tensor)");
    m.def("soft_nw_hvp(Tensor scores, Tensor tangent, float gap, float temperature, Tensor? lengths) -> Tensor");
    m.def("soft_nw_param_jacobian(Tensor scores, int param_type, float gap, float temperature, Tensor? lengths) -> Tensor");
    m.def("soft_nw_backward_full(Tensor scores, Tensor grad_alignment, float gap, float temperature, Tensor? lengths) -> (Tensor, Tensor, Tensor)");
    m.def("nw_forward(Tensor scores, float gap, float temp, Tensor? lengths) -> Tensor[]");
    m.def("nw_forward_t(Tensor scores, Tensor gap, Tensor temp, Tensor lengths) -> Tensor[]");
    m.def("nw_value_grad_params(Tensor scores, float gap, float temp, Tensor? lengths) -> (Tensor, Tensor)");
    m.def("nw_marginals_backward(Tensor scores, Tensor grad_marginals, float gap, float temp, Tensor? lengths) -> (Tensor, Tensor, Tensor)");
    m.def("nw_marginals_hvp(Tensor scores, Tensor v, float gap, float temp, Tensor? lengths) -> Tensor");
    m.def("nw_marginals_grad_gap(Tensor scores, float gap, float temp, Tensor? lengths) -> Tensor");
    m.def("nw_marginals_grad_temp(Tensor scores, float gap, float temp, Tensor? lengths) -> Tensor");
    // src/sw_affine/registry.cpp:27-42
    m.def("soft_sw_affine(Tensor scores, Tensor gap_open, Tensor gap_ext, Tensor temperature, Tensor lengths) -> Tensor[]");
    m.def("soft_sw_affine_float(Tensor scores, float gap_open, float gap_ext, float temperature, Tensor? lengths) -> Tensor[]");
    m.def("soft_sw_affine_with_grads(Tensor scores, float gap_open, float gap_ext, float temperature, Tensor? lengths) -> (Tensor, Tensor, Tensor, Tensor, Tensor)");
    m.def("soft_sw_affine_hvp(Tensor scores, Tensor tangent, float gap_open, float gap_ext, float temperature, Tensor? lengths) -> Tensor");
    m.def("soft_sw_affine_param_jacobian(Tensor scores, int param_type, float gap_open, float gap_ext, float temperature, Tensor? lengths) -> Tensor");
    m.def("soft_sw_affine_backward_full(Tensor scores, Tensor grad_alignment, float gap_open, float gap_ext, float temperature, Tensor? lengths) -> (Tensor, Tensor, Tensor, Tensor)");
    m.def("sw_affine_forward(Tensor scores, float gap_open, float gap_ext, float temp, Tensor? lengths) -> Tensor[]");
    m.def("sw_affine_forward_t(Tensor scores, Tensor gap_open, Tensor gap_ext, Tensor temp, Tensor lengths) -> Tensor[]");
    m.def("sw_affine_value_grad_params(Tensor scores, float gap_open, float gap_ext, float temp, Tensor? lengths) -> (Tensor, Tensor, Tensor)");
    m.def("sw_affine_marginals_backward(Tensor scores, Tensor grad_marginals, float gap_open, float gap_ext, float temp, Tensor? lengths) -> (Tensor, Tensor, Tensor, Tensor)");
    m.def("sw_affine_marginals_hvp(Tensor scores, Tensor v, float gap_open, float gap_ext, float temp, Tensor? lengths) -> Tensor");
    m.def("sw_affine_marginals_grad_gap_open(Tensor scores, float gap_open, float gap_ext, float temp, Tensor? lengths) -> Tensor");
    m.def("sw_affine_marginals_grad_gap_ext(Tensor scores, float gap_open, float gap_ext, float temp, Tensor? lengths) -> Tensor");
    m.def("sw_affine_marginals_grad_temp(Tensor scores, float gap_open, float gap_ext, float temp, Tensor? lengths) -> Tensor");
    // soft Needleman-Wunsch, affine gaps (src/nw_affine/registry.cpp:35-50)
    m.def("soft_nw_affine(Tensor scores, Tensor gap_open, Tensor gap_ext, Tensor temperature, Tensor lengths) -> Tensor[]");
    m.def("soft_nw_affine_float(Tensor scores, float gap_open, float gap_ext, float temperature, Tensor? lengths) -> Tensor[]");
    m.def("soft_nw_affine_with_grads(Tensor scores, float gap_open, float gap_ext, float temperature, Tensor? lengths) -> (Tensor, Tensor, Tensor, Tensor, Tensor)");
    m.def("soft_nw_affine_hvp(Tensor scores, Tensor tangent, float gap_open, float gap_ext, float temperature, Tensor? lengths) -> Tensor");
    m.def("soft_nw_affine_param_jacobian(Tensor scores, int param_type, float gap_open, float gap_ext, float temperature, Tensor? lengths) -> Tensor");
    m.def("soft_nw_affine_backward_full(Tensor scores, Tensor grad_alignment, float gap_open, float gap_ext, float temperature, Tensor? lengths) -> (Tensor, Tensor, Tensor, Tensor)");
    m.def("nw_affine_forward(Tensor scores, float gap_open, float gap_ext, float temp, Tensor? lengths) -> Tensor[]");
    m.def("nw_affine_forward_t(Tensor scores, Tensor gap_open, Tensor gap_ext, Tensor temp, Tensor lengths) -> Tensor[]");
    m.def("nw_affine_value_grad_params(Tensor scores, float gap_open, float gap_ext, float temp, Tensor? lengths) -> (Tensor, Tensor, Tensor)");
    m.def("nw_affine_marginals_backward(Tensor scores, Tensor grad_marginals, float gap_open, float gap_ext, float temp, Tensor? lengths) -> (Tensor, Tensor, Tensor, Tensor)");
    m.def("nw_affine_marginals_hvp(Tensor scores, Tensor v, float gap_open, float gap_ext, float temp, Tensor? lengths) -> Tensor");
    m.def("nw_affine_marginals_grad_gap_open(Tensor scores, float gap_open, float gap_ext, float temp, Tensor? lengths) -> Tensor");
    m.def("nw_affine_marginals_grad_gap_ext(Tensor scores, float gap_open, float gap_ext, float temp, Tensor? lengths) -> Tensor");
    m.def("nw_affine_marginals_grad_temp(Tensor scores, float gap_open, float gap_ext, float temp, Tensor? lengths) -> Tensor");
    // soft DTW (src/dtw/registry.cpp:35-40)
    m.def("soft_dtw(Tensor costs, Tensor temperature, Tensor lengths, int bandwidth) -> Tensor[]");
    m.def("soft_dtw_float(Tensor costs, float temperature, Tensor? lengths, int? bandwidth) -> Tensor[]");
    m.def("soft_dtw_with_grads(Tensor costs, float temperature, Tensor? lengths, int? bandwidth) -> (Tensor, Tensor, Tensor)");
    m.def("soft_dtw_hvp(Tensor costs, Tensor tangent, float temperature, Tensor? lengths, int? bandwidth) -> Tensor");
    m.def("soft_dtw_param_jacobian(Tensor costs, float temperature, Tensor? lengths, int? bandwidth) -> Tensor");
    m.def("soft_dtw_backward_full(Tensor costs, Tensor grad_alignment, float temperature, Tensor? lengths, int? bandwidth) -> (Tensor, Tensor)");
}

TORCH_LIBRARY_IMPL(d2p, CUDA, m) {
    m.impl("soft_sw", soft_lin_cuda<kSW>);
    m.impl("soft_sw_float", soft_lin_float_cuda<kSW>);
    m.impl("soft_sw_with_grads", soft_lin_with_grads_cuda<kSW>);
    m.impl("soft_sw_hvp", soft_lin_hvp_cuda<kSW>);
    m.impl("soft_sw_param_jacobian", soft_lin_param_jacobian_cuda<kSW>);
    m.impl("soft_sw_backward_full", soft_lin_backward_full_cuda<kSW>);
    m.impl("sw_forward", lin_forward_alias<kSW>);
    m.impl("sw_forward_t", lin_forward_t_alias<kSW>);
    m.impl("sw_value_grad_params", lin_value_grad_params_alias<kSW>);
    m.impl("sw_marginals_backward", lin_marginals_backward_alias<kSW>);
    m.impl("sw_marginals_hvp", lin_marginals_hvp_alias<kSW>);
    m.impl("sw_marginals_grad_gap", lin_marginals_grad_gap_alias<kSW>);
    m.impl("sw_marginals_grad_temp", lin_marginals_grad_temp_alias<kSW>);
    m.impl("soft_nw", soft_lin_cuda<kNW>);
    m.impl("soft_nw_float", soft_lin_float_cuda<kNW>);
    m.impl("soft_nw_with_grads", soft_lin_with_grads_cuda<kNW>);
    m.impl("soft_nw_hvp", soft_lin_hvp_cuda<kNW>);
    m.impl("soft_nw_param_jacobian", soft_lin_param_jacobian_cuda<kNW>);
    m.impl("soft_nw_backward_full", soft_lin_backward_full_cuda<kNW>);
    m.impl("nw_forward", lin_forward_alias<kNW>);
    m.impl("nw_forward_t", lin_forward_t_alias<kNW>);
    m.impl("nw_value_grad_params", lin_value_grad_params_alias<kNW>);
    m.impl("nw_marginals_backward", lin_marginals_backward_alias<kNW>);
    m.impl("nw_marginals_hvp", lin_marginals_hvp_alias<kNW>);
    m.impl("nw_marginals_grad_gap", lin_marginals_grad_gap_alias<kNW>);
    m.impl("nw_marginals_grad_temp", lin_marginals_grad_temp_alias<kNW>);
    m.impl("soft_sw_affine", soft_aff_cuda<kAff>);
    m.impl("soft_sw_affine_float", soft_aff_float_cuda<kAff>);
    m.impl("soft_sw_affine_with_grads", soft_aff_with_grads_cuda<kAff>);
    m.impl("soft_sw_affine_hvp", soft_aff_hvp_cuda<kAff>);
    m.impl("soft_sw_affine_param_jacobian", soft_aff_param_jacobian_cuda<kAff>);
    m.impl("soft_sw_affine_backward_full", soft_aff_backward_full_cuda<kAff>);
    m.impl("sw_affine_forward", aff_forward_alias<kAff>);
    m.impl("sw_affine_forward_t", aff_forward_t_alias<kAff>);
    m.impl("sw_affine_value_grad_params", aff_value_grad_params_alias<kAff>);
    m.impl("sw_affine_marginals_backward", aff_marginals_backward_alias<kAff>);
    m.impl("sw_affine_marginals_hvp", aff_marginals_hvp_alias<kAff>);
    m.impl("sw_affine_marginals_grad_gap_open", aff_marginals_grad_alias<kAff, 0>);
    m.impl("sw_affine_marginals_grad_gap_ext", aff_marginals_grad_alias<kAff, 1>);
    m.impl("sw_affine_marginals_grad_temp", aff_marginals_grad_alias<kAff, 2>);
    m.impl("soft_nw_affine", soft_aff_cuda<kNWAff>);
    m.impl("soft_nw_affine_float", soft_aff_float_cuda<kNWAff>);
    m.impl("soft_nw_affine_with_grads", soft_aff_with_grads_cuda<kNWAff>);
    m.impl("soft_nw_affine_hvp", soft_aff_hvp_cuda<kNWAff>);
    m.impl("soft_nw_affine_param_jacobian", soft_aff_param_jacobian_cuda<kNWAff>);
    m.impl("soft_nw_affine_backward_full", soft_aff_backward_full_cuda<kNWAff>);
    m.impl("nw_affine_forward", aff_forward_alias<kNWAff>);
    m.impl("nw_affine_forward_t", aff_forward_t_alias<kNWAff>);
    m.impl("nw_affine_value_grad_params", aff_value_grad_params_alias<kNWAff>);
    m.impl("nw_affine_marginals_backward", aff_marginals_backward_alias<kNWAff>);
    m.impl("nw_affine_marginals_hvp", aff_marginals_hvp_alias<kNWAff>);
    m.impl("nw_affine_marginals_grad_gap_open", aff_marginals_grad_alias<kNWAff, 0>);
    m.impl("nw_affine_marginals_grad_gap_ext", aff_marginals_grad_alias<kNWAff, 1>);
    m.impl("nw_affine_marginals_grad_temp", aff_marginals_grad_alias<kNWAff, 2>);
    m.impl("soft_dtw", soft_dtw_cuda);
    m.impl("soft_dtw_float", soft_dtw_float_cuda);
    m.impl("soft_dtw_with_grads", soft_dtw_with_grads_cuda);
    m.impl("soft_dtw_hvp", soft_dtw_hvp_cuda);
    m.impl("soft_dtw_param_jacobian", soft_dtw_param_jacobian_cuda);
    m.impl("soft_dtw_backward_full", soft_dtw_backward_full_cuda);
}

// No CPU kernels by design: CPU tensors get a clear error instead of a silent
// fallback (the reference's CPU path is used only as the test oracle).
void reject_cpu(const c10::OperatorHandle& op, torch::jit::Stack*) {
    TORCH_CHECK(false, op.schema().name(),
                ": scores must be a CUDA tensor (d2p_b200 implements the soft Smith-Waterman "
                "and Needleman-Wunsch operators for CUDA devices only)");
}

TORCH_LIBRARY_IMPL(d2p, CPU, m) {
    static const char* kOps[] = {
        "soft_sw", "soft_sw_float", "soft_sw_with_grads", "soft_sw_hvp", "soft_sw_param_jacobian",
        "soft_sw_backward_full", "sw_forward", "sw_forward_t", "sw_value_grad_params",
        "sw_marginals_backward", "sw_marginals_hvp", "sw_marginals_grad_gap", "sw_marginals_grad_temp",
        "soft_sw_affine", "soft_sw_affine_float", "soft_sw_affine_with_grads", "soft_sw_affine_hvp",
        "soft_sw_affine_param_jacobian", "soft_sw_affine_backward_full", "sw_affine_forward",
        "sw_affine_forward_t", "sw_affine_value_grad_params", "sw_affine_marginals_backward",
        "sw_affine_marginals_hvp", "sw_affine_marginals_grad_gap_open", "sw_affine_marginals_grad_gap_ext",
        "sw_affine_marginals_grad_temp", "soft_nw", "soft_nw_float", "soft_nw_with_grads", "soft_nw_hvp",
        "soft_nw_param_jacobian", "soft_nw_backward_full", "nw_forward", "nw_forward_t", "nw_value_grad_params",
        "nw_marginals_backward", "nw_marginals_hvp", "nw_marginals_grad_gap", "nw_marginals_grad_temp",
        "soft_nw_affine", "soft_nw_affine_float", "soft_nw_affine_with_grads", "soft_nw_affine_hvp",
        "soft_nw_affine_param_jacobian", "soft_nw_affine_backward_full", "nw_affine_forward", "nw_affine_forward_t",
        "nw_affine_value_grad_params", "nw_affine_marginals_backward", "nw_affine_marginals_hvp",
        "nw_affine_marginals_grad_gap_open", "nw_affine_marginals_grad_gap_ext", "nw_affine_marginals_grad_temp",
        "soft_dtw", "soft_dtw_float", "soft_dtw_with_grads", "soft_dtw_hvp", "soft_dtw_param_jacobian",
        "soft_dtw_backward_full"};
    for (const char* name : kOps) m.impl(name, torch::CppFunction::makeFromBoxedFunction<&reject_cpu>());
}

// The autograd kernels.  Fake tensors (FakeTensorMode, meta tracing) carry
// the Python dispatch key and no storage: they are handed on below autograd,
// where the registered fake kernel describes the outputs (no autograd graph is
// recorded for them; torch.compile traces the d2p_py:: custom ops, which carry
// their own autograd formulas).  Real tensors run the autograd Functions.
bool is_python_tensor(const Tensor& t) { return t.defined() && t.key_set().has(c10::DispatchKey::Python); }

template <class Sig>
c10::TypedOperatorHandle<Sig> op_handle(const char* name) {
    return c10::Dispatcher::singleton().findSchemaOrThrow(name, "").typed<Sig>();
}

// the C++ signatures the kernels were registered with (arguments by value)
using ForwardT = std::vector<Tensor>(Tensor, Tensor, Tensor, Tensor);
using ForwardF = std::vector<Tensor>(Tensor, double, double, c10::optional<Tensor>);
using AffForwardT = std::vector<Tensor>(Tensor, Tensor, Tensor, Tensor, Tensor);
using AffForwardF = std::vector<Tensor>(Tensor, double, double, double, c10::optional<Tensor>);
using DtwForwardT = std::vector<Tensor>(Tensor, Tensor, Tensor, int64_t);
using DtwForwardF = std::vector<Tensor>(Tensor, double, c10::optional<Tensor>, c10::optional<int64_t>);

std::vector<Tensor> dtw_fwd_t_autograd(Tensor costs, Tensor temperature, Tensor lengths, int64_t bandwidth) {
    if (is_python_tensor(costs)) {
        static auto op = op_handle<DtwForwardT>("d2p::soft_dtw");
        at::AutoDispatchBelowADInplaceOrView below;
        return op.call(costs, temperature, lengths, bandwidth);
    }
    return soft_dtw_cuda(costs, temperature, lengths, bandwidth);
}
std::vector<Tensor> dtw_fwd_f_autograd(Tensor costs, double temperature, c10::optional<Tensor> lengths,
                                       c10::optional<int64_t> bandwidth) {
    if (is_python_tensor(costs)) {
        static auto op = op_handle<DtwForwardF>("d2p::soft_dtw_float");
        at::AutoDispatchBelowADInplaceOrView below;
        return op.call(costs, temperature, lengths, bandwidth);
    }
    return soft_dtw_float_cuda(costs, temperature, lengths, bandwidth);
}

template <const char* Name, int FAM>
std::vector<Tensor> fwd_t_autograd(Tensor scores, Tensor gap, Tensor temperature, Tensor lengths) {
    if (is_python_tensor(scores)) {
        static auto op = op_handle<ForwardT>(Name);
        at::AutoDispatchBelowADInplaceOrView below;
        return op.call(scores, gap, temperature, lengths);
    }
    return soft_lin_cuda<FAM>(scores, gap, temperature, lengths);
}
template <const char* Name, int FAM>
std::vector<Tensor> fwd_f_autograd(Tensor scores, double gap, double temperature, c10::optional<Tensor> lengths) {
    if (is_python_tensor(scores)) {
        static auto op = op_handle<ForwardF>(Name);
        at::AutoDispatchBelowADInplaceOrView below;
        return op.call(scores, gap, temperature, lengths);
    }
    return soft_lin_float_cuda<FAM>(scores, gap, temperature, lengths);
}
template <const char* Name, int FAM>
std::vector<Tensor> aff_fwd_t_autograd(Tensor scores, Tensor go, Tensor ge, Tensor temperature, Tensor lengths) {
    if (is_python_tensor(scores)) {
        static auto op = op_handle<AffForwardT>(Name);
        at::AutoDispatchBelowADInplaceOrView below;
        return op.call(scores, go, ge, temperature, lengths);
    }
    return soft_aff_cuda<FAM>(scores, go, ge, temperature, lengths);
}
template <const char* Name, int FAM>
std::vector<Tensor> aff_fwd_f_autograd(Tensor scores, double go, double ge, double temperature,
                                       c10::optional<Tensor> lengths) {
    if (is_python_tensor(scores)) {
        static auto op = op_handle<AffForwardF>(Name);
        at::AutoDispatchBelowADInplaceOrView below;
        return op.call(scores, go, ge, temperature, lengths);
    }
    return soft_aff_float_cuda<FAM>(scores, go, ge, temperature, lengths);
}

constexpr char kSoftSW[] = "d2p::soft_sw";
constexpr char kSoftSWFloat[] = "d2p::soft_sw_float";
constexpr char kSWForward[] = "d2p::sw_forward";
constexpr char kSWForwardT[] = "d2p::sw_forward_t";
constexpr char kSoftSWAffine[] = "d2p::soft_sw_affine";
constexpr char kSoftSWAffineFloat[] = "d2p::soft_sw_affine_float";
constexpr char kSWAffineForward[] = "d2p::sw_affine_forward";
constexpr char kSWAffineForwardT[] = "d2p::sw_affine_forward_t";
constexpr char kSoftNW[] = "d2p::soft_nw";
constexpr char kSoftNWFloat[] = "d2p::soft_nw_float";
constexpr char kNWForward[] = "d2p::nw_forward";
constexpr char kNWForwardT[] = "d2p::nw_forward_t";
constexpr char kSoftNWAffine[] = "d2p::soft_nw_affine";
constexpr char kSoftNWAffineFloat[] = "d2p::soft_nw_affine_float";
constexpr char kNWAffineForward[] = "d2p::nw_affine_forward";
constexpr char kNWAffineForwardT[] = "d2p::nw_affine_forward_t";

TORCH_LIBRARY_IMPL(d2p, AutogradCUDA, m) {
    m.impl("soft_sw", fwd_t_autograd<kSoftSW, kSW>);
    m.impl("soft_sw_float", fwd_f_autograd<kSoftSWFloat, kSW>);
    m.impl("sw_forward", fwd_f_autograd<kSWForward, kSW>);
    m.impl("sw_forward_t", fwd_t_autograd<kSWForwardT, kSW>);
    m.impl("soft_nw", fwd_t_autograd<kSoftNW, kNW>);
    m.impl("soft_nw_float", fwd_f_autograd<kSoftNWFloat, kNW>);
    m.impl("nw_forward", fwd_f_autograd<kNWForward, kNW>);
    m.impl("nw_forward_t", fwd_t_autograd<kNWForwardT, kNW>);
    m.impl("soft_sw_affine", aff_fwd_t_autograd<kSoftSWAffine, kAff>);
    m.impl("soft_sw_affine_float", aff_fwd_f_autograd<kSoftSWAffineFloat, kAff>);
    m.impl("sw_affine_forward", aff_fwd_f_autograd<kSWAffineForward, kAff>);
    m.impl("sw_affine_forward_t", aff_fwd_t_autograd<kSWAffineForwardT, kAff>);
    m.impl("soft_nw_affine", aff_fwd_t_autograd<kSoftNWAffine, kNWAff>);
    m.impl("soft_nw_affine_float", aff_fwd_f_autograd<kSoftNWAffineFloat, kNWAff>);
    m.impl("nw_affine_forward", aff_fwd_f_autograd<kNWAffineForward, kNWAff>);
    m.impl("nw_affine_forward_t", aff_fwd_t_autograd<kNWAffineForwardT, kNWAff>);
    m.impl("soft_dtw", dtw_fwd_t_autograd);
    m.impl("soft_dtw_float", dtw_fwd_f_autograd);
}
