"""Low-level operator access (d2p/ops/__init__.py): ``ops.sw``, ``ops.sw_affine`` and
the flat op wrappers of the soft Smith-Waterman family and of the linear soft
Needleman-Wunsch operators."""
from . import sw, sw_affine
from .._ops import (  # noqa: F401
    d2p,
    soft_sw, soft_sw_float, soft_sw_with_grads, soft_sw_hvp, soft_sw_param_jacobian, soft_sw_backward_full,
    soft_sw_affine, soft_sw_affine_float, soft_sw_affine_with_grads, soft_sw_affine_hvp,
    soft_sw_affine_param_jacobian, soft_sw_affine_backward_full,
    sw_forward, sw_forward_t, sw_value_grad_params, sw_marginals_backward, sw_marginals_hvp,
    sw_marginals_grad_gap, sw_marginals_grad_temp,
    sw_affine_forward, sw_affine_forward_t, sw_affine_value_grad_params, sw_affine_marginals_backward,
    sw_affine_marginals_hvp, sw_affine_marginals_grad_gap_open, sw_affine_marginals_grad_gap_ext,
    sw_affine_marginals_grad_temp,
    soft_nw, soft_nw_float, soft_nw_with_grads, soft_nw_hvp, soft_nw_param_jacobian, soft_nw_backward_full,
    nw_forward, nw_forward_t, nw_value_grad_params, nw_marginals_backward, nw_marginals_hvp,
    nw_marginals_grad_gap, nw_marginals_grad_temp,
    soft_nw_affine, soft_nw_affine_float, soft_nw_affine_with_grads, soft_nw_affine_hvp,
    soft_nw_affine_param_jacobian, soft_nw_affine_backward_full, nw_affine_forward, nw_affine_forward_t,
    nw_affine_value_grad_params, nw_affine_marginals_backward, nw_affine_marginals_hvp,
    nw_affine_marginals_grad_gap_open, nw_affine_marginals_grad_gap_ext, nw_affine_marginals_grad_temp,
    soft_dtw, soft_dtw_float, soft_dtw_with_grads, soft_dtw_hvp, soft_dtw_param_jacobian, soft_dtw_backward_full,
)

__all__ = [
    "sw", "sw_affine", "d2p",
    "soft_sw", "soft_sw_float", "soft_sw_with_grads", "soft_sw_hvp", "soft_sw_param_jacobian",
    "soft_sw_backward_full",
    "soft_sw_affine", "soft_sw_affine_float", "soft_sw_affine_with_grads", "soft_sw_affine_hvp",
    "soft_sw_affine_param_jacobian", "soft_sw_affine_backward_full",
    "sw_forward", "sw_forward_t", "sw_value_grad_params", "sw_marginals_backward", "sw_marginals_hvp",
    "sw_marginals_grad_gap", "sw_marginals_grad_temp",
    "sw_affine_forward", "sw_affine_forward_t", "sw_affine_value_grad_params", "sw_affine_marginals_backward",
    "sw_affine_marginals_hvp", "sw_affine_marginals_grad_gap_open", "sw_affine_marginals_grad_gap_ext",
    "sw_affine_marginals_grad_temp",
    "soft_nw", "soft_nw_float", "soft_nw_with_grads", "soft_nw_hvp", "soft_nw_param_jacobian",
    "soft_nw_backward_full", "nw_forward", "nw_forward_t", "nw_value_grad_params", "nw_marginals_backward",
    "nw_marginals_hvp", "nw_marginals_grad_gap", "nw_marginals_grad_temp",
    "soft_nw_affine", "soft_nw_affine_float", "soft_nw_affine_with_grads", "soft_nw_affine_hvp",
    "soft_nw_affine_param_jacobian", "soft_nw_affine_backward_full", "nw_affine_forward", "nw_affine_forward_t",
    "nw_affine_value_grad_params", "nw_affine_marginals_backward", "nw_affine_marginals_hvp",
    "nw_affine_marginals_grad_gap_open", "nw_affine_marginals_grad_gap_ext", "nw_affine_marginals_grad_temp",
    "soft_dtw", "soft_dtw_float", "soft_dtw_with_grads", "soft_dtw_hvp", "soft_dtw_param_jacobian",
    "soft_dtw_backward_full",
]
