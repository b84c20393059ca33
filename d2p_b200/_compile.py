"""Fake-tensor (meta) shapes and autocast rules for the soft Smith-Waterman,
soft Needleman-Wunsch and soft DTW ops.

Mirrors d2p/_compile.py:18-250 (register_fake) and :857-901 (register_autocast)
for the sw / sw_affine families.  Output shapes per op:

* ``[B]`` values and per-problem parameter gradients,
* ``[B, L1, L2]`` marginals, HVPs and parameter Jacobians,
* ``[1]`` batch-summed parameter gradients of the ``*_backward_full`` /
  ``*_marginals_backward`` ops.

Deviation kept on purpose: the reference's fakes for ``soft_sw_backward_full`` /
``soft_sw_affine_backward_full`` declare ``[B]`` parameter gradients
(d2p/_compile.py:62-70, :118-127) while its real ops return ``[1]``
(src/sw/torch_cuda.cpp:756-768).  The fakes here follow the real ops, as the
reference's own PT2 layer does (d2p/_pt2_ops.py:143-149).
"""
from __future__ import annotations

import torch
from torch.library import register_fake

from . import _ops  # noqa: F401  (ensures the schemas are registered)

_B = "B"        # [B]
_P = "P"        # [B, L1, L2]
_ONE = "1"      # [1]

# op name -> output layout; a list means the schema returns Tensor[]
_OUTPUTS = {
    "soft_sw": [_B, _P],
    "soft_sw_float": [_B, _P],
    "soft_sw_with_grads": (_B, _P, _B, _B),
    "soft_sw_hvp": _P,
    "soft_sw_param_jacobian": _P,
    "soft_sw_backward_full": (_P, _ONE, _ONE),
    "sw_forward": [_B, _P],
    "sw_forward_t": [_B, _P],
    "sw_value_grad_params": (_B, _B),
    "sw_marginals_backward": (_P, _ONE, _ONE),
    "sw_marginals_hvp": _P,
    "sw_marginals_grad_gap": _P,
    "sw_marginals_grad_temp": _P,
    "soft_sw_affine": [_B, _P],
    "soft_sw_affine_float": [_B, _P],
    "soft_sw_affine_with_grads": (_B, _P, _B, _B, _B),
    "soft_sw_affine_hvp": _P,
    "soft_sw_affine_param_jacobian": _P,
    "soft_sw_affine_backward_full": (_P, _ONE, _ONE, _ONE),
    "sw_affine_forward": [_B, _P],
    "sw_affine_forward_t": [_B, _P],
    "sw_affine_value_grad_params": (_B, _B, _B),
    "sw_affine_marginals_backward": (_P, _ONE, _ONE, _ONE),
    "sw_affine_marginals_hvp": _P,
    "sw_affine_marginals_grad_gap_open": _P,
    "sw_affine_marginals_grad_gap_ext": _P,
    "sw_affine_marginals_grad_temp": _P,
    # soft Needleman-Wunsch, linear gap (d2p/_compile.py:257-308)
    "soft_nw": [_B, _P],
    "soft_nw_float": [_B, _P],
    "soft_nw_with_grads": (_B, _P, _B, _B),
    "soft_nw_hvp": _P,
    "soft_nw_param_jacobian": _P,
    "soft_nw_backward_full": (_P, _ONE, _ONE),
    "nw_forward": [_B, _P],
    "nw_forward_t": [_B, _P],
    "nw_value_grad_params": (_B, _B),
    "nw_marginals_backward": (_P, _ONE, _ONE),
    "nw_marginals_hvp": _P,
    "nw_marginals_grad_gap": _P,
    "nw_marginals_grad_temp": _P,
    # soft Needleman-Wunsch, affine gaps (d2p/_compile.py:311-370)
    "soft_nw_affine": [_B, _P],
    "soft_nw_affine_float": [_B, _P],
    "soft_nw_affine_with_grads": (_B, _P, _B, _B, _B),
    "soft_nw_affine_hvp": _P,
    "soft_nw_affine_param_jacobian": _P,
    "soft_nw_affine_backward_full": (_P, _ONE, _ONE, _ONE),
    "nw_affine_forward": [_B, _P],
    "nw_affine_forward_t": [_B, _P],
    "nw_affine_value_grad_params": (_B, _B, _B),
    "nw_affine_marginals_backward": (_P, _ONE, _ONE, _ONE),
    "nw_affine_marginals_hvp": _P,
    "nw_affine_marginals_grad_gap_open": _P,
    "nw_affine_marginals_grad_gap_ext": _P,
    "nw_affine_marginals_grad_temp": _P,
    # soft DTW (d2p/_compile.py:371-415)
    "soft_dtw": [_B, _P],
    "soft_dtw_float": [_B, _P],
    "soft_dtw_with_grads": (_B, _P, _B),
    "soft_dtw_hvp": _P,
    "soft_dtw_param_jacobian": _P,
    "soft_dtw_backward_full": (_P, _ONE),
}


def _alloc(scores: torch.Tensor, kind: str) -> torch.Tensor:
    B, L1, L2 = scores.shape
    shape = {_B: [B], _P: [B, L1, L2], _ONE: [1]}[kind]
    return scores.new_empty(shape, dtype=torch.float32)


def _make_fake(spec):
    def fake(scores, *args, **kwargs):
        if isinstance(spec, list):
            return [_alloc(scores, k) for k in spec]
        if isinstance(spec, tuple):
            return tuple(_alloc(scores, k) for k in spec)
        return _alloc(scores, spec)

    return fake


for _name, _spec in _OUTPUTS.items():
    register_fake("d2p::" + _name)(_make_fake(_spec))

# DP recurrences need fp32 (long dependent logsumexp chains): under
# torch.autocast every op runs on fp32 inputs (reference d2p/_compile.py:857-901).
try:
    from torch.library import register_autocast

    for _name in _OUTPUTS:
        register_autocast("d2p::" + _name, "cuda", torch.float32)
except ImportError:  # pragma: no cover - older torch
    pass
