"""Differentiable soft Needleman-Wunsch (global alignment), B200 CUDA
implementation.

Drop-in for d2p/nw.py:1-250: ``soft_nw``, ``soft_nw_affine``, ``NWResult``,
``SoftNW`` and ``SoftNWAffine`` with the same argument names, defaults,
validation and error types.  Both sequences are aligned end to end.  Linear
gap: alpha[0,0] = 0, alpha[i,0] = i*gap, alpha[0,j] = j*gap, and the value is
alpha[L1, L2].  Affine gaps (states M, I, D): a gap of length k costs
gap_open + (k-1)*gap_ext, and the value is the logsumexp of the three states
at (L1, L2).

    result = soft_nw(scores, gap=-1.0, temperature=1.0)
    result = soft_nw_affine(scores, gap_open=-2.0, gap_ext=-0.5, temperature=1.0)
    result.score [B], result.alignment [B, L1, L2]
"""
from __future__ import annotations

from typing import NamedTuple, Optional, Union

import torch
import torch.nn as nn

from . import _ops
from .sw import _as_param, _make_lengths, _validate_gap, _validate_temperature


class NWResult(NamedTuple):
    """(score [B], alignment [B, L1, L2]) -- d2p/nw.py:32-40."""

    score: torch.Tensor
    alignment: torch.Tensor


def soft_nw(
    scores: torch.Tensor,
    gap: Union[float, torch.Tensor] = -1.0,
    temperature: Union[float, torch.Tensor] = 1.0,
    lengths: Optional[torch.Tensor] = None,
) -> NWResult:
    """Soft Needleman-Wunsch with a linear gap penalty.

    Args:
        scores: similarity matrix [B, L1, L2] (fp32; CUDA).
        gap: gap penalty (float, or scalar tensor for a learnable gap).
        temperature: soft-max temperature (> 0; float or scalar tensor).
        lengths: optional [B, 2] int32 actual lengths; the alignment of problem
            b runs from (0, 0) to (lengths[b,0], lengths[b,1]).

    Returns:
        NWResult(score [B], alignment [B, L1, L2]); the alignment is zero
        outside each problem's lengths.
    """
    _validate_temperature(temperature)
    _validate_gap(gap)
    tensor_params = isinstance(gap, torch.Tensor) or isinstance(temperature, torch.Tensor)
    if tensor_params:
        if lengths is None:
            lengths = _make_lengths(scores)
        result = _ops.soft_nw(scores, _as_param(gap, scores), _as_param(temperature, scores), lengths)
    else:
        # lengths=None means full lengths to the op: no [B, 2] tensor is built
        result = _ops.soft_nw_float(scores, gap, temperature, lengths)
    return NWResult(result[0], result[1])


class SoftNW(nn.Module):
    """Soft Needleman-Wunsch module (d2p/nw.py:159-196): gap and temperature
    are parameters when ``learnable``, buffers otherwise."""

    def __init__(self, gap: float = -1.0, temperature: float = 1.0, learnable: bool = False):
        super().__init__()
        if temperature <= 0:
            raise ValueError(f"temperature must be positive, got {temperature}")
        for name, val in (("gap", gap), ("temperature", temperature)):
            t = torch.tensor([val])
            if learnable:
                setattr(self, name, nn.Parameter(t))
            else:
                self.register_buffer(name, t)

    def forward(self, scores: torch.Tensor, lengths: Optional[torch.Tensor] = None) -> NWResult:
        if lengths is None:
            lengths = _make_lengths(scores)
        result = _ops.soft_nw(scores, _as_param(self.gap, scores), _as_param(self.temperature, scores), lengths)
        return NWResult(result[0], result[1])


def soft_nw_affine(
    scores: torch.Tensor,
    gap_open: Union[float, torch.Tensor] = -2.0,
    gap_ext: Union[float, torch.Tensor] = -0.5,
    temperature: Union[float, torch.Tensor] = 1.0,
    lengths: Optional[torch.Tensor] = None,
) -> NWResult:
    """Soft Needleman-Wunsch with affine gap penalties (d2p/nw.py:115-156).

    Args:
        scores: similarity matrix [B, L1, L2] (fp32; CUDA).
        gap_open: cost of a gap's first position (float or scalar tensor).
        gap_ext: cost of each further position of a gap.
        temperature: soft-max temperature (> 0; float or scalar tensor).
        lengths: optional [B, 2] int32 actual lengths.

    Returns:
        NWResult(score [B], alignment [B, L1, L2]): the alignment is the
        probability that the path matches (i, j), zero outside each problem.
    """
    _validate_temperature(temperature)
    _validate_gap(gap_open, "gap_open")
    _validate_gap(gap_ext, "gap_ext")
    tensor_params = any(isinstance(p, torch.Tensor) for p in (gap_open, gap_ext, temperature))
    if tensor_params:
        if lengths is None:
            lengths = _make_lengths(scores)
        result = _ops.soft_nw_affine(scores, _as_param(gap_open, scores), _as_param(gap_ext, scores),
                                     _as_param(temperature, scores), lengths)
    else:
        result = _ops.soft_nw_affine_float(scores, gap_open, gap_ext, temperature, lengths)
    return NWResult(result[0], result[1])


class SoftNWAffine(nn.Module):
    """Soft Needleman-Wunsch module with affine gaps (d2p/nw.py:198-250):
    gap_open, gap_ext and temperature are parameters when ``learnable``,
    buffers otherwise."""

    def __init__(self, gap_open: float = -2.0, gap_ext: float = -0.5, temperature: float = 1.0,
                 learnable: bool = False):
        super().__init__()
        if temperature <= 0:
            raise ValueError(f"temperature must be positive, got {temperature}")
        for name, val in (("gap_open", gap_open), ("gap_ext", gap_ext), ("temperature", temperature)):
            t = torch.tensor([val])
            if learnable:
                setattr(self, name, nn.Parameter(t))
            else:
                self.register_buffer(name, t)

    def forward(self, scores: torch.Tensor, lengths: Optional[torch.Tensor] = None) -> NWResult:
        if lengths is None:
            lengths = _make_lengths(scores)
        result = _ops.soft_nw_affine(scores, _as_param(self.gap_open, scores), _as_param(self.gap_ext, scores),
                                     _as_param(self.temperature, scores), lengths)
        return NWResult(result[0], result[1])
