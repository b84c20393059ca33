"""Differentiable soft Smith-Waterman (local alignment), B200 CUDA implementation.

Drop-in for d2p/sw.py:1-620: same functions, classes, argument names, defaults,
validation and error types.

    result = soft_sw(scores, gap=-1.0, temperature=1.0)
    result = soft_sw_affine(scores, gap_open=-2.0, gap_ext=-0.5, temperature=1.0)
    result.value [B], result.marginals [B, L1, L2]   (aliases .score / .alignment / .posteriors)
"""
from __future__ import annotations

import warnings
from typing import NamedTuple, Optional, Union

import torch
import torch.nn as nn

from . import _ops
from ._pt2_utils import use_pt2_ops


class SWResult(NamedTuple):
    """(value [B], marginals [B, L1, L2]) -- d2p/sw.py:44-72."""

    value: torch.Tensor
    marginals: torch.Tensor

    @property
    def score(self) -> torch.Tensor:
        return self.value

    @property
    def alignment(self) -> torch.Tensor:
        return self.marginals

    @property
    def posteriors(self) -> torch.Tensor:
        return self.marginals


# ----------------------------------------------------------------------------
# validation (d2p/sw.py:80-239)
# ----------------------------------------------------------------------------

def _validate_temperature(temperature, name: str = "temperature") -> None:
    """ValueError for a non-positive Python scalar or fixed scalar tensor."""
    if isinstance(temperature, (int, float)):
        if temperature <= 0:
            raise ValueError(f"{name} must be positive, got {temperature}")
    elif isinstance(temperature, torch.Tensor):
        if use_pt2_ops(temperature):
            return
        if not temperature.requires_grad and temperature.numel() == 1:
            val = temperature.item()
            if val <= 0:
                raise ValueError(f"{name} must be positive, got {val}")


def _validate_gap(gap, name: str = "gap") -> None:
    """UserWarning for a positive Python-scalar gap (almost always a sign error)."""
    if isinstance(gap, (int, float)) and gap > 0:
        warnings.warn(
            f"{name}={gap} is positive. Gap penalties are typically negative. "
            "If this is intentional, pass as tensor to suppress this warning.",
            UserWarning,
            stacklevel=3,
        )


def _normalize_param_tensor(param: torch.Tensor, scores: torch.Tensor) -> torch.Tensor:
    """0-D -> [1]; moved to the scores' device, cast to fp32 (the op computes in fp32)."""
    if param.dim() == 0:
        param = param.view(1)
    want = torch.float32
    if param.device != scores.device or param.dtype != want:
        param = param.to(device=scores.device, dtype=want)
    return param


def _make_lengths(scores: torch.Tensor) -> torch.Tensor:
    B, L1, L2 = scores.shape
    return torch.tensor([L1, L2], dtype=torch.int32, device=scores.device).repeat(B, 1)


def _validate_prefix_mask(mask: torch.Tensor, name: str) -> torch.Tensor:
    """Lengths of a prefix-only boolean mask [B, L]; ValueError if it has holes."""
    m = mask.to(torch.int32)
    if m.shape[1] > 1:
        holes = (m[:, 1:] - m[:, :-1] > 0).any(dim=1)
        if holes.any():
            bad = holes.nonzero(as_tuple=True)[0].tolist()
            raise ValueError(
                f"{name} is not prefix-only (has holes) at batch indices: {bad}. "
                "Masks must have all True values at the beginning, followed by all False values."
            )
    return m.sum(dim=1).to(torch.int32)


def _masks_to_lengths(mask1, mask2, B: int, L1: int, L2: int, device) -> torch.Tensor:
    lengths = torch.empty((B, 2), dtype=torch.int32, device=device)
    lengths[:, 0] = _validate_prefix_mask(mask1, "mask1") if mask1 is not None else L1
    lengths[:, 1] = _validate_prefix_mask(mask2, "mask2") if mask2 is not None else L2
    return lengths


def _resolve_lengths(scores, lengths, mask1, mask2, need_tensor: bool):
    if lengths is not None and (mask1 is not None or mask2 is not None):
        raise ValueError("Cannot specify both 'lengths' and 'mask1'/'mask2'")
    B, L1, L2 = scores.shape
    if mask1 is not None or mask2 is not None:
        return _masks_to_lengths(mask1, mask2, B, L1, L2, scores.device)
    if lengths is None and need_tensor:
        return _make_lengths(scores)
    # lengths=None on the float path means "full lengths" to the op: no [B,2]
    # tensor is built and no host->device copy is made.
    return lengths


def _as_param(value, scores: torch.Tensor) -> torch.Tensor:
    if isinstance(value, torch.Tensor):
        return _normalize_param_tensor(value, scores)
    return torch.tensor([float(value)], device=scores.device, dtype=torch.float32)


# ----------------------------------------------------------------------------
# high-level API (d2p/sw.py:247-421)
# ----------------------------------------------------------------------------

def soft_sw(
    scores: torch.Tensor,
    gap: Union[float, torch.Tensor] = -1.0,
    temperature: Union[float, torch.Tensor] = 1.0,
    lengths: Optional[torch.Tensor] = None,
    *,
    mask1: Optional[torch.Tensor] = None,
    mask2: Optional[torch.Tensor] = None,
) -> SWResult:
    """Soft Smith-Waterman with a linear gap penalty.

    Args:
        scores: similarity matrix [B, L1, L2] (fp32; CUDA).
        gap: gap penalty (float, or scalar tensor for a learnable gap).
        temperature: soft-max temperature (> 0; float or scalar tensor).
        lengths: optional [B, 2] int32 actual lengths.
        mask1, mask2: optional prefix boolean masks [B, L1] / [B, L2]
            (mutually exclusive with ``lengths``).

    Returns:
        SWResult(value [B], marginals [B, L1, L2]).
    """
    _validate_temperature(temperature)
    _validate_gap(gap)
    tensor_params = isinstance(gap, torch.Tensor) or isinstance(temperature, torch.Tensor)
    lengths = _resolve_lengths(scores, lengths, mask1, mask2, need_tensor=tensor_params)
    if tensor_params:
        result = _ops.soft_sw(scores, _as_param(gap, scores), _as_param(temperature, scores), lengths)
    else:
        result = _ops.soft_sw_float(scores, gap, temperature, lengths)
    return SWResult(result[0], result[1])


def soft_sw_affine(
    scores: torch.Tensor,
    gap_open: Union[float, torch.Tensor] = -2.0,
    gap_ext: Union[float, torch.Tensor] = -0.5,
    temperature: Union[float, torch.Tensor] = 1.0,
    lengths: Optional[torch.Tensor] = None,
    *,
    mask1: Optional[torch.Tensor] = None,
    mask2: Optional[torch.Tensor] = None,
) -> SWResult:
    """Soft Smith-Waterman with affine gaps (gap of length k costs gap_open + k*gap_ext,
    3-state M/I/D model).  ``scores`` may be fp32 or bf16 (bf16 is read directly and
    accumulated in fp32)."""
    _validate_temperature(temperature)
    _validate_gap(gap_open, "gap_open")
    _validate_gap(gap_ext, "gap_ext")
    tensor_params = any(isinstance(p, torch.Tensor) for p in (gap_open, gap_ext, temperature))
    lengths = _resolve_lengths(scores, lengths, mask1, mask2, need_tensor=tensor_params)
    if tensor_params:
        result = _ops.soft_sw_affine(scores, _as_param(gap_open, scores), _as_param(gap_ext, scores),
                                     _as_param(temperature, scores), lengths)
    else:
        result = _ops.soft_sw_affine_float(scores, gap_open, gap_ext, temperature, lengths)
    return SWResult(result[0], result[1])


# ----------------------------------------------------------------------------
# nn.Module API (d2p/sw.py:429-604)
# ----------------------------------------------------------------------------

class SoftSW(nn.Module):
    """Soft Smith-Waterman module with optionally learnable gap / temperature."""

    def __init__(self, gap: float = -1.0, temperature: float = 1.0, learnable: Optional[bool] = None,
                 learn_gap: bool = False, learn_temperature: bool = False):
        super().__init__()
        if temperature <= 0:
            raise ValueError(f"temperature must be positive, got {temperature}")
        if learnable is not None:
            warnings.warn(
                "The 'learnable' parameter is deprecated. "
                "Use 'learn_gap' and/or 'learn_temperature' instead.",
                DeprecationWarning,
                stacklevel=2,
            )
            if learnable:
                learn_gap = learn_temperature = True
        for name, val, learn in (("gap", gap, learn_gap), ("temperature", temperature, learn_temperature)):
            t = torch.tensor([val])
            if learn:
                setattr(self, name, nn.Parameter(t))
            else:
                self.register_buffer(name, t)

    def forward(self, scores, lengths=None, *, mask1=None, mask2=None) -> SWResult:
        return soft_sw(scores, gap=self.gap, temperature=self.temperature, lengths=lengths,
                       mask1=mask1, mask2=mask2)


class SoftSWAffine(nn.Module):
    """Affine-gap soft Smith-Waterman module with optionally learnable parameters."""

    def __init__(self, gap_open: float = -2.0, gap_ext: float = -0.5, temperature: float = 1.0,
                 learnable: Optional[bool] = None, learn_gap_open: bool = False,
                 learn_gap_ext: bool = False, learn_temperature: bool = False):
        super().__init__()
        if temperature <= 0:
            raise ValueError(f"temperature must be positive, got {temperature}")
        if learnable is not None:
            warnings.warn(
                "The 'learnable' parameter is deprecated. "
                "Use 'learn_gap_open', 'learn_gap_ext', and/or 'learn_temperature' instead.",
                DeprecationWarning,
                stacklevel=2,
            )
            if learnable:
                learn_gap_open = learn_gap_ext = learn_temperature = True
        for name, val, learn in (("gap_open", gap_open, learn_gap_open), ("gap_ext", gap_ext, learn_gap_ext),
                                 ("temperature", temperature, learn_temperature)):
            t = torch.tensor([val])
            if learn:
                setattr(self, name, nn.Parameter(t))
            else:
                self.register_buffer(name, t)

    def forward(self, scores, lengths=None, *, mask1=None, mask2=None) -> SWResult:
        return soft_sw_affine(scores, gap_open=self.gap_open, gap_ext=self.gap_ext,
                              temperature=self.temperature, lengths=lengths, mask1=mask1, mask2=mask2)


# low-level re-exports (d2p/sw.py:612-620)
soft_sw_forward = _ops.soft_sw_float
soft_sw_with_grads = _ops.soft_sw_with_grads
soft_sw_hvp = _ops.soft_sw_hvp
soft_sw_backward_full = _ops.soft_sw_backward_full

soft_sw_affine_forward = _ops.soft_sw_affine_float
soft_sw_affine_with_grads = _ops.soft_sw_affine_with_grads
soft_sw_affine_hvp = _ops.soft_sw_affine_hvp
soft_sw_affine_backward_full = _ops.soft_sw_affine_backward_full
