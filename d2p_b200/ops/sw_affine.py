"""ops.sw_affine -- structured low-level API for the affine-gap family (d2p/ops/sw_affine.py)."""
from typing import Optional, Tuple

from torch import Tensor

from .. import _ops


def forward(scores: Tensor, gap_open: float, gap_ext: float, temp: float,
            lengths: Optional[Tensor] = None) -> Tuple[Tensor, Tensor]:
    return _ops.sw_affine_forward(scores, gap_open, gap_ext, temp, lengths)


def forward_t(scores: Tensor, gap_open: Tensor, gap_ext: Tensor, temp: Tensor,
              lengths: Optional[Tensor] = None) -> Tuple[Tensor, Tensor]:
    return _ops.sw_affine_forward_t(scores, gap_open, gap_ext, temp, lengths)


def value_grad_params(scores: Tensor, gap_open: float, gap_ext: float, temp: float,
                      lengths: Optional[Tensor] = None) -> Tuple[Tensor, Tensor, Tensor]:
    return _ops.sw_affine_value_grad_params(scores, gap_open, gap_ext, temp, lengths)


def marginals_backward(scores: Tensor, grad_marginals: Tensor, gap_open: float, gap_ext: float, temp: float,
                       lengths: Optional[Tensor] = None) -> Tuple[Tensor, Tensor, Tensor, Tensor]:
    return _ops.sw_affine_marginals_backward(scores, grad_marginals, gap_open, gap_ext, temp, lengths)


def marginals_hvp(scores: Tensor, v: Tensor, gap_open: float, gap_ext: float, temp: float,
                  lengths: Optional[Tensor] = None) -> Tensor:
    return _ops.sw_affine_marginals_hvp(scores, v, gap_open, gap_ext, temp, lengths)


def marginals_grad_gap_open(scores: Tensor, gap_open: float, gap_ext: float, temp: float,
                            lengths: Optional[Tensor] = None) -> Tensor:
    return _ops.sw_affine_marginals_grad_gap_open(scores, gap_open, gap_ext, temp, lengths)


def marginals_grad_gap_ext(scores: Tensor, gap_open: float, gap_ext: float, temp: float,
                           lengths: Optional[Tensor] = None) -> Tensor:
    return _ops.sw_affine_marginals_grad_gap_ext(scores, gap_open, gap_ext, temp, lengths)


def marginals_grad_temp(scores: Tensor, gap_open: float, gap_ext: float, temp: float,
                        lengths: Optional[Tensor] = None) -> Tensor:
    return _ops.sw_affine_marginals_grad_temp(scores, gap_open, gap_ext, temp, lengths)
