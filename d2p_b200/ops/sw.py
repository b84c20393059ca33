"""ops.sw -- structured low-level API for the linear-gap family (d2p/ops/sw.py)."""
from typing import Optional, Tuple

from torch import Tensor

from .. import _ops


def forward(scores: Tensor, gap: float, temp: float, lengths: Optional[Tensor] = None) -> Tuple[Tensor, Tensor]:
    """(value [B], marginals [B,L1,L2]) with scalar parameters."""
    return _ops.sw_forward(scores, gap, temp, lengths)


def forward_t(scores: Tensor, gap: Tensor, temp: Tensor, lengths: Optional[Tensor] = None) -> Tuple[Tensor, Tensor]:
    """(value, marginals) with tensor (learnable) parameters."""
    return _ops.sw_forward_t(scores, gap, temp, lengths)


def value_grad_params(scores: Tensor, gap: float, temp: float, lengths: Optional[Tensor] = None) -> Tuple[Tensor, Tensor]:
    """Per-problem (dvalue/dgap [B], dvalue/dtemp [B])."""
    return _ops.sw_value_grad_params(scores, gap, temp, lengths)


def marginals_backward(scores: Tensor, grad_marginals: Tensor, gap: float, temp: float,
                       lengths: Optional[Tensor] = None) -> Tuple[Tensor, Tensor, Tensor]:
    """Gradients of <grad_marginals, marginals>: (scores [B,L1,L2], gap [1], temp [1])."""
    return _ops.sw_marginals_backward(scores, grad_marginals, gap, temp, lengths)


def marginals_hvp(scores: Tensor, v: Tensor, gap: float, temp: float, lengths: Optional[Tensor] = None) -> Tensor:
    """Hessian-vector product d(marginals)/d(scores) . v  [B,L1,L2]."""
    return _ops.sw_marginals_hvp(scores, v, gap, temp, lengths)


def marginals_grad_gap(scores: Tensor, gap: float, temp: float, lengths: Optional[Tensor] = None) -> Tensor:
    """d(marginals)/d(gap)  [B,L1,L2]."""
    return _ops.sw_marginals_grad_gap(scores, gap, temp, lengths)


def marginals_grad_temp(scores: Tensor, gap: float, temp: float, lengths: Optional[Tensor] = None) -> Tensor:
    """d(marginals)/d(temperature)  [B,L1,L2]."""
    return _ops.sw_marginals_grad_temp(scores, gap, temp, lengths)
