"""Low-level operator access: loads the native libraries and wraps torch.ops.d2p.*.

Mirrors d2p/_ops.py (loader :25-167, soft Smith-Waterman wrappers :170-210,
soft Needleman-Wunsch wrappers :241-254, soft DTW wrappers :217-222) for the
soft Smith-Waterman, soft Needleman-Wunsch (linear and affine gaps) and soft
DTW operators.  The extension is in-tree (``_C.so`` next to this
file, linked to ``libd2p_b200.so``); there is no CPU kernel and no fallback:
importing fails loudly when the extension is missing, and CPU tensors are
rejected by the ops themselves.
"""
from __future__ import annotations

import os

import torch

from ._pt2_utils import use_pt2_ops

_HERE = os.path.dirname(os.path.abspath(__file__))
_extension_loaded = False
_cuda_dispatch_available = False
_lib_path = None


def _has_cuda_dispatch() -> bool:
    try:
        return torch._C._dispatch_has_kernel_for_dispatch_key("d2p::soft_sw_float", "CUDA")
    except (AttributeError, RuntimeError):
        return False


def _load_extension() -> None:
    global _extension_loaded, _cuda_dispatch_available, _lib_path
    if _extension_loaded:
        return
    path = os.path.join(_HERE, "_C.so")
    if not os.path.exists(path) and os.environ.get("D2P_B200_AUTOBUILD", "1") == "1":
        from . import _build

        _build.build()
    if not os.path.exists(path):
        raise ImportError(
            f"d2p_b200 native extension not found at {path}. Build it with "
            "`python -m d2p_b200._build` (needs nvcc for sm_100a and g++)."
        )
    try:
        torch.ops.load_library(path)
    except OSError as exc:
        if "undefined symbol" in str(exc):
            raise ImportError(
                f"d2p_b200's extension was built against a different torch than the "
                f"installed {torch.__version__}; rebuild with `python -m d2p_b200._build -f`.\n{exc}"
            ) from exc
        raise
    _lib_path = path
    _extension_loaded = True
    _cuda_dispatch_available = _has_cuda_dispatch()


def _ensure_loaded() -> None:
    if not _extension_loaded:
        _load_extension()


def _contains_cuda_tensor(value) -> bool:
    if isinstance(value, torch.Tensor):
        return value.is_cuda
    if isinstance(value, (list, tuple)):
        return any(_contains_cuda_tensor(v) for v in value)
    if isinstance(value, dict):
        return any(_contains_cuda_tensor(v) for v in value.values())
    return False


def _ensure_cuda_supported(args, kwargs) -> None:
    _ensure_loaded()
    if _cuda_dispatch_available:
        return
    if _contains_cuda_tensor(args) or _contains_cuda_tensor(kwargs):
        raise RuntimeError("This d2p_b200 build has no CUDA kernels registered.")


_load_extension()

#: the full ``torch.ops.d2p`` namespace for advanced users
d2p = torch.ops.d2p

# The d2p_py:: custom ops (set by the package __init__ once both modules are
# loaded): no import may run inside a call that Dynamo traces.
_pt2_mod = None


def _get_pt2_ops():
    return _pt2_mod


def _should_use_pt2(args, kwargs) -> bool:
    if not kwargs:
        return use_pt2_ops(*args)
    return use_pt2_ops(*args, *kwargs.values())


def _wrap(name: str):
    raw = getattr(torch.ops.d2p, name)

    def wrapped(*args, **kwargs):
        _ensure_cuda_supported(args, kwargs)
        if _should_use_pt2(args, kwargs):
            pt2 = _get_pt2_ops()
            if hasattr(pt2, name):
                return getattr(pt2, name)(*args, **kwargs)
        return raw(*args, **kwargs)

    wrapped.__name__ = name
    wrapped.__qualname__ = name
    wrapped.__doc__ = f"torch.ops.d2p.{name} (CUDA, sm_100a)"
    return wrapped


# Smith-Waterman (linear gap)
soft_sw = _wrap("soft_sw")
soft_sw_float = _wrap("soft_sw_float")
soft_sw_with_grads = _wrap("soft_sw_with_grads")
soft_sw_hvp = _wrap("soft_sw_hvp")
soft_sw_param_jacobian = _wrap("soft_sw_param_jacobian")
soft_sw_backward_full = _wrap("soft_sw_backward_full")

# Smith-Waterman (affine gap)
soft_sw_affine = _wrap("soft_sw_affine")
soft_sw_affine_float = _wrap("soft_sw_affine_float")
soft_sw_affine_with_grads = _wrap("soft_sw_affine_with_grads")
soft_sw_affine_hvp = _wrap("soft_sw_affine_hvp")
soft_sw_affine_param_jacobian = _wrap("soft_sw_affine_param_jacobian")
soft_sw_affine_backward_full = _wrap("soft_sw_affine_backward_full")

# namespaced names (linear)
sw_forward = _wrap("sw_forward")
sw_forward_t = _wrap("sw_forward_t")
sw_value_grad_params = _wrap("sw_value_grad_params")
sw_marginals_backward = _wrap("sw_marginals_backward")
sw_marginals_hvp = _wrap("sw_marginals_hvp")
sw_marginals_grad_gap = _wrap("sw_marginals_grad_gap")
sw_marginals_grad_temp = _wrap("sw_marginals_grad_temp")

# namespaced names (affine)
sw_affine_forward = _wrap("sw_affine_forward")
sw_affine_forward_t = _wrap("sw_affine_forward_t")
sw_affine_value_grad_params = _wrap("sw_affine_value_grad_params")
sw_affine_marginals_backward = _wrap("sw_affine_marginals_backward")
sw_affine_marginals_hvp = _wrap("sw_affine_marginals_hvp")
sw_affine_marginals_grad_gap_open = _wrap("sw_affine_marginals_grad_gap_open")
sw_affine_marginals_grad_gap_ext = _wrap("sw_affine_marginals_grad_gap_ext")
sw_affine_marginals_grad_temp = _wrap("sw_affine_marginals_grad_temp")

# Needleman-Wunsch (linear gap)
soft_nw = _wrap("soft_nw")
soft_nw_float = _wrap("soft_nw_float")
soft_nw_with_grads = _wrap("soft_nw_with_grads")
soft_nw_hvp = _wrap("soft_nw_hvp")
soft_nw_param_jacobian = _wrap("soft_nw_param_jacobian")
soft_nw_backward_full = _wrap("soft_nw_backward_full")
nw_forward = _wrap("nw_forward")
nw_forward_t = _wrap("nw_forward_t")
nw_value_grad_params = _wrap("nw_value_grad_params")
nw_marginals_backward = _wrap("nw_marginals_backward")
nw_marginals_hvp = _wrap("nw_marginals_hvp")
nw_marginals_grad_gap = _wrap("nw_marginals_grad_gap")
nw_marginals_grad_temp = _wrap("nw_marginals_grad_temp")

# Needleman-Wunsch (affine gaps)
soft_nw_affine = _wrap("soft_nw_affine")
soft_nw_affine_float = _wrap("soft_nw_affine_float")
soft_nw_affine_with_grads = _wrap("soft_nw_affine_with_grads")
soft_nw_affine_hvp = _wrap("soft_nw_affine_hvp")
soft_nw_affine_param_jacobian = _wrap("soft_nw_affine_param_jacobian")
soft_nw_affine_backward_full = _wrap("soft_nw_affine_backward_full")
nw_affine_forward = _wrap("nw_affine_forward")
nw_affine_forward_t = _wrap("nw_affine_forward_t")
nw_affine_value_grad_params = _wrap("nw_affine_value_grad_params")
nw_affine_marginals_backward = _wrap("nw_affine_marginals_backward")
nw_affine_marginals_hvp = _wrap("nw_affine_marginals_hvp")
nw_affine_marginals_grad_gap_open = _wrap("nw_affine_marginals_grad_gap_open")
nw_affine_marginals_grad_gap_ext = _wrap("nw_affine_marginals_grad_gap_ext")
nw_affine_marginals_grad_temp = _wrap("nw_affine_marginals_grad_temp")

# soft DTW
soft_dtw = _wrap("soft_dtw")
soft_dtw_float = _wrap("soft_dtw_float")
soft_dtw_with_grads = _wrap("soft_dtw_with_grads")
soft_dtw_hvp = _wrap("soft_dtw_hvp")
soft_dtw_param_jacobian = _wrap("soft_dtw_param_jacobian")
soft_dtw_backward_full = _wrap("soft_dtw_backward_full")

OP_NAMES = (
    "soft_sw", "soft_sw_float", "soft_sw_with_grads", "soft_sw_hvp", "soft_sw_param_jacobian",
    "soft_sw_backward_full", "sw_forward", "sw_forward_t", "sw_value_grad_params",
    "sw_marginals_backward", "sw_marginals_hvp", "sw_marginals_grad_gap", "sw_marginals_grad_temp",
    "soft_sw_affine", "soft_sw_affine_float", "soft_sw_affine_with_grads", "soft_sw_affine_hvp",
    "soft_sw_affine_param_jacobian", "soft_sw_affine_backward_full", "sw_affine_forward",
    "sw_affine_forward_t", "sw_affine_value_grad_params", "sw_affine_marginals_backward",
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
)
