"""Differentiable soft dynamic time warping, B200 CUDA implementation.

Drop-in for d2p/dtw.py:1-157: ``soft_dtw``, ``DTWResult`` and ``SoftDTW`` with
the same argument names, defaults, validation and error types.  The warping
path runs from (1, 1) to (L1, L2) by diagonal, down and right moves and pays
the cost of every cell it visits; the value is the soft minimum of the paths'
costs (softmin with temperature T), and the alignment is each cell's visit
probability.  ``bandwidth`` > 0 restricts the path to the Sakoe-Chiba band
|j - i L2 / L1| <= bandwidth; 0 means no band.

    result = soft_dtw(costs, temperature=1.0, bandwidth=0)
    result.cost [B], result.alignment [B, L1, L2]
"""
from __future__ import annotations

from typing import NamedTuple, Optional, Union

import torch
import torch.nn as nn

from . import _ops
from .sw import _as_param, _make_lengths, _validate_temperature


class DTWResult(NamedTuple):
    """(cost [B], alignment [B, L1, L2]) -- d2p/dtw.py:30-38."""

    cost: torch.Tensor
    alignment: torch.Tensor


def _band(bandwidth: int) -> int:
    # 0 means no band; the operators take any negative value for that
    return bandwidth if bandwidth > 0 else -1


def soft_dtw(
    costs: torch.Tensor,
    temperature: Union[float, torch.Tensor] = 1.0,
    bandwidth: int = 0,
    lengths: Optional[torch.Tensor] = None,
) -> DTWResult:
    """Soft dynamic time warping (d2p/dtw.py:57-105).

    Args:
        costs: cost matrix [B, L1, L2] (lower = better match; fp32; CUDA).
        temperature: softmin temperature (> 0; float or scalar tensor); lower
            values approach hard DTW.
        bandwidth: Sakoe-Chiba band width (0 = no constraint).
        lengths: optional [B, 2] int32 actual lengths.

    Returns:
        DTWResult(cost [B], alignment [B, L1, L2]).
    """
    _validate_temperature(temperature)
    bw = _band(bandwidth)
    if isinstance(temperature, torch.Tensor):
        if lengths is None:
            lengths = _make_lengths(costs)
        result = _ops.soft_dtw(costs, _as_param(temperature, costs), lengths, bw)
    else:
        # lengths=None means full lengths to the op: no [B, 2] tensor is built
        result = _ops.soft_dtw_float(costs, temperature, lengths, bw)
    return DTWResult(result[0], result[1])


class SoftDTW(nn.Module):
    """Soft DTW module (d2p/dtw.py:108-150): the temperature is a parameter
    when ``learnable``, a buffer otherwise."""

    def __init__(self, temperature: float = 1.0, bandwidth: int = 0, learnable: bool = False):
        super().__init__()
        if temperature <= 0:
            raise ValueError(f"temperature must be positive, got {temperature}")
        self.bandwidth = bandwidth
        t = torch.tensor([temperature])
        if learnable:
            self.temperature = nn.Parameter(t)
        else:
            self.register_buffer("temperature", t)

    def forward(self, costs: torch.Tensor, lengths: Optional[torch.Tensor] = None) -> DTWResult:
        if lengths is None:
            lengths = _make_lengths(costs)
        result = _ops.soft_dtw(costs, _as_param(self.temperature, costs), lengths, _band(self.bandwidth))
        return DTWResult(result[0], result[1])


# low-level re-exports (d2p/dtw.py:153-157)
soft_dtw_forward = _ops.soft_dtw_float
soft_dtw_with_grads = _ops.soft_dtw_with_grads
soft_dtw_hvp = _ops.soft_dtw_hvp
soft_dtw_backward_full = _ops.soft_dtw_backward_full
