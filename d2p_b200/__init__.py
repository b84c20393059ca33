"""d2p_b200 -- B200-native (sm_100a) soft Smith-Waterman operators, a drop-in for
d2p's ``soft_sw`` / ``soft_sw_affine`` path, plus the soft Needleman-Wunsch
operators (``soft_nw``, ``soft_nw_affine``) and soft DTW (``soft_dtw``).

    import d2p_b200 as d2p
    result = d2p.soft_sw(scores, gap=-1.0, temperature=1.0)        # value [B], marginals [B,L1,L2]
    result = d2p.soft_sw_affine(scores, gap_open=-2.0, gap_ext=-0.5)

The dispatcher ops keep the reference schemas under ``torch.ops.d2p.*``; fake
tensors and autocast rules are registered for torch.compile (d2p/__init__.py).
"""
from . import _ops  # loads the native extension (fails loudly if missing)
from . import _compile  # noqa: F401  register_fake / register_autocast
from . import _pt2_ops  # the d2p_py:: custom ops torch.compile traces

_ops._pt2_mod = _pt2_ops
from .sw import SoftSW, SoftSWAffine, SWResult, soft_sw, soft_sw_affine
from .nw import NWResult, SoftNW, SoftNWAffine, soft_nw, soft_nw_affine
from .dtw import DTWResult, SoftDTW, soft_dtw
from .embed import embed_scores, soft_sw_embed
from . import ops
from .engine import engine_counts, set_engine, use_engine

# legacy flat aliases (d2p/__init__.py, soft Smith-Waterman lines)
soft_sw_float = _ops.soft_sw_float
soft_sw_with_grads = _ops.soft_sw_with_grads
soft_sw_hvp = _ops.soft_sw_hvp
soft_sw_param_jacobian = _ops.soft_sw_param_jacobian
soft_sw_backward_full = _ops.soft_sw_backward_full
soft_sw_affine_float = _ops.soft_sw_affine_float
soft_sw_affine_with_grads = _ops.soft_sw_affine_with_grads
soft_sw_affine_hvp = _ops.soft_sw_affine_hvp
soft_sw_affine_param_jacobian = _ops.soft_sw_affine_param_jacobian
soft_sw_affine_backward_full = _ops.soft_sw_affine_backward_full
soft_nw_float = _ops.soft_nw_float
soft_nw_with_grads = _ops.soft_nw_with_grads
soft_nw_hvp = _ops.soft_nw_hvp
soft_nw_param_jacobian = _ops.soft_nw_param_jacobian
soft_nw_backward_full = _ops.soft_nw_backward_full
soft_nw_affine_float = _ops.soft_nw_affine_float
soft_nw_affine_with_grads = _ops.soft_nw_affine_with_grads
soft_nw_affine_hvp = _ops.soft_nw_affine_hvp
soft_nw_affine_param_jacobian = _ops.soft_nw_affine_param_jacobian
soft_nw_affine_backward_full = _ops.soft_nw_affine_backward_full
soft_dtw_float = _ops.soft_dtw_float
soft_dtw_with_grads = _ops.soft_dtw_with_grads
soft_dtw_hvp = _ops.soft_dtw_hvp
soft_dtw_param_jacobian = _ops.soft_dtw_param_jacobian
soft_dtw_backward_full = _ops.soft_dtw_backward_full

__version__ = "0.1.0"

__all__ = [
    "soft_sw", "soft_sw_affine", "SWResult", "SoftSW", "SoftSWAffine", "ops", "embed_scores", "soft_sw_embed",
    "soft_sw_float", "soft_sw_with_grads", "soft_sw_hvp", "soft_sw_param_jacobian", "soft_sw_backward_full",
    "soft_sw_affine_float", "soft_sw_affine_with_grads", "soft_sw_affine_hvp", "soft_sw_affine_param_jacobian",
    "soft_sw_affine_backward_full", "engine_counts", "set_engine", "use_engine",
    "soft_nw", "NWResult", "SoftNW", "soft_nw_float", "soft_nw_with_grads", "soft_nw_hvp",
    "soft_nw_param_jacobian", "soft_nw_backward_full", "soft_nw_affine", "SoftNWAffine", "soft_nw_affine_float",
    "soft_nw_affine_with_grads", "soft_nw_affine_hvp", "soft_nw_affine_param_jacobian",
    "soft_nw_affine_backward_full", "soft_dtw", "DTWResult", "SoftDTW", "soft_dtw_float", "soft_dtw_with_grads",
    "soft_dtw_hvp", "soft_dtw_param_jacobian", "soft_dtw_backward_full",
]
