"""PT2-safe custom ops (``d2p_py::*``) used while compiling or on fake tensors.

Mirrors the soft Smith-Waterman, soft Needleman-Wunsch and soft DTW parts of
d2p/_pt2_ops.py:72-1010: each op wraps
the dispatcher op, carries a fake implementation, and the differentiable ones
(``soft_sw``, ``soft_sw_float``, affine analogues) register an autograd formula
built from the saved marginals (value branch) and ``*_backward_full`` (marginal
branch).
"""
from __future__ import annotations

from typing import Optional

import torch
from torch.library import custom_op


def _add(a, b):
    if a is None:
        return b
    if b is None:
        return a
    return a + b


def _expand_batch(g: Optional[torch.Tensor], marg: torch.Tensor):
    if g is None:
        return None
    return g.view([marg.size(0)] + [1] * (marg.dim() - 1)) * marg


def _batch_dot(g: Optional[torch.Tensor], per_batch: torch.Tensor):
    if g is None:
        return None
    return (g * per_batch).sum().reshape([1])


def _like(scores, *kinds):
    B, L1, L2 = scores.shape
    out = []
    for k in kinds:
        shape = {"B": [B], "P": [B, L1, L2], "1": [1]}[k]
        out.append(scores.new_empty(shape, dtype=torch.float32))
    return tuple(out) if len(out) > 1 else out[0]


# --------------------------------------------------------------------------- linear
# The linear-gap Smith-Waterman ops (prefix "soft_sw") and the Needleman-Wunsch
# ops (prefix "soft_nw", d2p/_pt2_ops.py:495-570) have the same schemas and
# autograd formulas; one factory builds both sets.
def _make_linear_family(prefix: str):
    raw = torch.ops.d2p

    @custom_op(f"d2p_py::{prefix}_with_grads", mutates_args=())
    def with_grads(scores: torch.Tensor, gap: float, temperature: float,
                   lengths: Optional[torch.Tensor]) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor]:
        v, m, gg, gt = getattr(raw, f"{prefix}_with_grads")(scores, gap, temperature, lengths)
        return v, m, gg, gt

    @with_grads.register_fake
    def _(scores, gap, temperature, lengths):
        return _like(scores, "B", "P", "B", "B")

    @custom_op(f"d2p_py::{prefix}_hvp", mutates_args=())
    def hvp(scores: torch.Tensor, tangent: torch.Tensor, gap: float, temperature: float,
            lengths: Optional[torch.Tensor]) -> torch.Tensor:
        return getattr(raw, f"{prefix}_hvp")(scores, tangent, gap, temperature, lengths)

    @hvp.register_fake
    def _(scores, tangent, gap, temperature, lengths):
        return _like(scores, "P")

    @custom_op(f"d2p_py::{prefix}_param_jacobian", mutates_args=())
    def param_jacobian(scores: torch.Tensor, param_type: int, gap: float, temperature: float,
                       lengths: Optional[torch.Tensor]) -> torch.Tensor:
        return getattr(raw, f"{prefix}_param_jacobian")(scores, param_type, gap, temperature, lengths)

    @param_jacobian.register_fake
    def _(scores, param_type, gap, temperature, lengths):
        return _like(scores, "P")

    @custom_op(f"d2p_py::{prefix}_backward_full", mutates_args=())
    def backward_full(scores: torch.Tensor, grad_alignment: torch.Tensor, gap: float, temperature: float,
                      lengths: Optional[torch.Tensor]) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
        a, b, c = getattr(raw, f"{prefix}_backward_full")(scores, grad_alignment, gap, temperature, lengths)
        return a, b, c

    @backward_full.register_fake
    def _(scores, grad_alignment, gap, temperature, lengths):
        return _like(scores, "P", "1", "1")

    @custom_op(f"d2p_py::{prefix}", mutates_args=())
    def tensor_op(scores: torch.Tensor, gap: torch.Tensor, temperature: torch.Tensor,
                  lengths: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
        v, m = getattr(raw, prefix)(scores, gap, temperature, lengths)
        return v, m

    @tensor_op.register_fake
    def _(scores, gap, temperature, lengths):
        return _like(scores, "B", "P")

    # The backward of the tensor-parameter op needs the parameters' values as
    # scalars.  Read while tracing, they would be frozen into the compiled
    # graph (or be data-dependent), so the backward formula calls these ops,
    # which take the parameters as tensors and read them only when they run.
    @custom_op(f"d2p_py::{prefix}_param_grads_t", mutates_args=())
    def param_grads_t(scores: torch.Tensor, gap: torch.Tensor, temperature: torch.Tensor,
                      lengths: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
        _, _, dgap, dt = getattr(raw, f"{prefix}_with_grads")(scores, float(gap), float(temperature), lengths)
        return dgap, dt

    @param_grads_t.register_fake
    def _(scores, gap, temperature, lengths):
        return _like(scores, "B", "B")

    @custom_op(f"d2p_py::{prefix}_backward_full_t", mutates_args=())
    def backward_full_t(scores: torch.Tensor, grad_alignment: torch.Tensor, gap: torch.Tensor,
                        temperature: torch.Tensor,
                        lengths: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
        a, b, c = getattr(raw, f"{prefix}_backward_full")(scores, grad_alignment, float(gap), float(temperature),
                                                           lengths)
        return a, b, c

    @backward_full_t.register_fake
    def _(scores, grad_alignment, gap, temperature, lengths):
        return _like(scores, "P", "1", "1")

    def tensor_setup(ctx, inputs, output):
        scores, gap, temperature, lengths = inputs
        ctx.save_for_backward(scores, output[1], gap.detach(), temperature.detach())
        ctx.lengths = lengths

    def tensor_backward(ctx, grad_value, grad_marg):
        scores, marg, gap, temperature = ctx.saved_tensors
        grad_scores = _expand_batch(grad_value, marg)
        need_gap, need_t = ctx.needs_input_grad[1], ctx.needs_input_grad[2]
        g_gap = g_t = None
        if grad_value is not None and (need_gap or need_t):
            dgap, dt = param_grads_t(scores, gap, temperature, ctx.lengths)
            g_gap = _batch_dot(grad_value, dgap) if need_gap else None
            g_t = _batch_dot(grad_value, dt) if need_t else None
        if grad_marg is not None:
            gs, gg, gt = backward_full_t(scores, grad_marg, gap, temperature, ctx.lengths)
            grad_scores = _add(grad_scores, gs)
            g_gap = _add(g_gap, gg) if need_gap else None
            g_t = _add(g_t, gt) if need_t else None
        return grad_scores, g_gap, g_t, None

    tensor_op.register_autograd(tensor_backward, setup_context=tensor_setup)

    @custom_op(f"d2p_py::{prefix}_float", mutates_args=())
    def float_op(scores: torch.Tensor, gap: float, temperature: float,
                 lengths: Optional[torch.Tensor]) -> tuple[torch.Tensor, torch.Tensor]:
        v, m = getattr(raw, f"{prefix}_float")(scores, gap, temperature, lengths)
        return v, m

    @float_op.register_fake
    def _(scores, gap, temperature, lengths):
        return _like(scores, "B", "P")

    def float_setup(ctx, inputs, output):
        scores, gap, temperature, lengths = inputs
        ctx.save_for_backward(scores, output[1])
        ctx.gap, ctx.temperature, ctx.lengths = gap, temperature, lengths

    def float_backward(ctx, grad_value, grad_marg):
        scores, marg = ctx.saved_tensors
        grad_scores = _expand_batch(grad_value, marg)
        if grad_marg is not None:
            gs, _, _ = backward_full(scores, grad_marg, ctx.gap, ctx.temperature, ctx.lengths)
            grad_scores = _add(grad_scores, gs)
        return grad_scores, None, None, None

    float_op.register_autograd(float_backward, setup_context=float_setup)
    return {
        prefix: tensor_op, f"{prefix}_float": float_op, f"{prefix}_with_grads": with_grads,
        f"{prefix}_hvp": hvp, f"{prefix}_param_jacobian": param_jacobian, f"{prefix}_backward_full": backward_full,
        f"{prefix}_param_grads_t": param_grads_t, f"{prefix}_backward_full_t": backward_full_t,
    }


globals().update(_make_linear_family("soft_sw"))
globals().update(_make_linear_family("soft_nw"))


# --------------------------------------------------------------------------- affine
# The affine-gap Smith-Waterman ops (prefix "soft_sw_affine") and the affine
# Needleman-Wunsch ops (prefix "soft_nw_affine", d2p/_pt2_ops.py:575-660)
# have the same schemas and autograd formulas; one factory builds both sets.
def _make_affine_family(prefix: str):
    raw = torch.ops.d2p

    @custom_op(f"d2p_py::{prefix}_with_grads", mutates_args=())
    def with_grads(scores: torch.Tensor, gap_open: float, gap_ext: float, temperature: float,
                   lengths: Optional[torch.Tensor]
                   ) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor]:
        v, m, a, b, c = getattr(raw, f"{prefix}_with_grads")(scores, gap_open, gap_ext, temperature, lengths)
        return v, m, a, b, c

    @with_grads.register_fake
    def _(scores, gap_open, gap_ext, temperature, lengths):
        return _like(scores, "B", "P", "B", "B", "B")

    @custom_op(f"d2p_py::{prefix}_hvp", mutates_args=())
    def hvp(scores: torch.Tensor, tangent: torch.Tensor, gap_open: float, gap_ext: float,
            temperature: float, lengths: Optional[torch.Tensor]) -> torch.Tensor:
        return getattr(raw, f"{prefix}_hvp")(scores, tangent, gap_open, gap_ext, temperature, lengths)

    @hvp.register_fake
    def _(scores, tangent, gap_open, gap_ext, temperature, lengths):
        return _like(scores, "P")

    @custom_op(f"d2p_py::{prefix}_param_jacobian", mutates_args=())
    def param_jacobian(scores: torch.Tensor, param_type: int, gap_open: float, gap_ext: float,
                       temperature: float, lengths: Optional[torch.Tensor]) -> torch.Tensor:
        return getattr(raw, f"{prefix}_param_jacobian")(scores, param_type, gap_open, gap_ext, temperature, lengths)

    @param_jacobian.register_fake
    def _(scores, param_type, gap_open, gap_ext, temperature, lengths):
        return _like(scores, "P")

    @custom_op(f"d2p_py::{prefix}_backward_full", mutates_args=())
    def backward_full(scores: torch.Tensor, grad_alignment: torch.Tensor, gap_open: float, gap_ext: float,
                      temperature: float, lengths: Optional[torch.Tensor]
                      ) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor]:
        a, b, c, d = getattr(raw, f"{prefix}_backward_full")(scores, grad_alignment, gap_open, gap_ext,
                                                              temperature, lengths)
        return a, b, c, d

    @backward_full.register_fake
    def _(scores, grad_alignment, gap_open, gap_ext, temperature, lengths):
        return _like(scores, "P", "1", "1", "1")

    @custom_op(f"d2p_py::{prefix}", mutates_args=())
    def tensor_op(scores: torch.Tensor, gap_open: torch.Tensor, gap_ext: torch.Tensor,
                  temperature: torch.Tensor, lengths: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
        v, m = getattr(raw, prefix)(scores, gap_open, gap_ext, temperature, lengths)
        return v, m

    @tensor_op.register_fake
    def _(scores, gap_open, gap_ext, temperature, lengths):
        return _like(scores, "B", "P")

    # parameters as tensors, read only when the op runs (see the linear family)
    @custom_op(f"d2p_py::{prefix}_param_grads_t", mutates_args=())
    def param_grads_t(scores: torch.Tensor, gap_open: torch.Tensor, gap_ext: torch.Tensor,
                      temperature: torch.Tensor,
                      lengths: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
        r = getattr(raw, f"{prefix}_with_grads")(scores, float(gap_open), float(gap_ext), float(temperature),
                                                  lengths)
        return r[2], r[3], r[4]

    @param_grads_t.register_fake
    def _(scores, gap_open, gap_ext, temperature, lengths):
        return _like(scores, "B", "B", "B")

    @custom_op(f"d2p_py::{prefix}_backward_full_t", mutates_args=())
    def backward_full_t(scores: torch.Tensor, grad_alignment: torch.Tensor, gap_open: torch.Tensor,
                        gap_ext: torch.Tensor, temperature: torch.Tensor, lengths: torch.Tensor
                        ) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor]:
        a, b, c, d = getattr(raw, f"{prefix}_backward_full")(scores, grad_alignment, float(gap_open),
                                                              float(gap_ext), float(temperature), lengths)
        return a, b, c, d

    @backward_full_t.register_fake
    def _(scores, grad_alignment, gap_open, gap_ext, temperature, lengths):
        return _like(scores, "P", "1", "1", "1")

    def tensor_setup(ctx, inputs, output):
        scores, go, ge, temperature, lengths = inputs
        ctx.save_for_backward(scores, output[1], go.detach(), ge.detach(), temperature.detach())
        ctx.lengths = lengths

    def tensor_backward(ctx, grad_value, grad_marg):
        scores, marg, go, ge, temperature = ctx.saved_tensors
        grad_scores = _expand_batch(grad_value, marg)
        need = ctx.needs_input_grad[1:4]
        grads = [None, None, None]
        if grad_value is not None and any(need):
            pg = param_grads_t(scores, go, ge, temperature, ctx.lengths)
            for k in range(3):
                if need[k]:
                    grads[k] = _batch_dot(grad_value, pg[k])
        if grad_marg is not None:
            r = backward_full_t(scores, grad_marg, go, ge, temperature, ctx.lengths)
            grad_scores = _add(grad_scores, r[0])
            for k in range(3):
                if need[k]:
                    grads[k] = _add(grads[k], r[1 + k])
        return grad_scores, grads[0], grads[1], grads[2], None

    tensor_op.register_autograd(tensor_backward, setup_context=tensor_setup)

    @custom_op(f"d2p_py::{prefix}_float", mutates_args=())
    def float_op(scores: torch.Tensor, gap_open: float, gap_ext: float, temperature: float,
                 lengths: Optional[torch.Tensor]) -> tuple[torch.Tensor, torch.Tensor]:
        v, m = getattr(raw, f"{prefix}_float")(scores, gap_open, gap_ext, temperature, lengths)
        return v, m

    @float_op.register_fake
    def _(scores, gap_open, gap_ext, temperature, lengths):
        return _like(scores, "B", "P")

    def float_setup(ctx, inputs, output):
        scores, go, ge, temperature, lengths = inputs
        ctx.save_for_backward(scores, output[1])
        ctx.go, ctx.ge, ctx.temperature, ctx.lengths = go, ge, temperature, lengths

    def float_backward(ctx, grad_value, grad_marg):
        scores, marg = ctx.saved_tensors
        grad_scores = _expand_batch(grad_value, marg)
        if grad_marg is not None:
            r = backward_full(scores, grad_marg, ctx.go, ctx.ge, ctx.temperature, ctx.lengths)
            grad_scores = _add(grad_scores, r[0])
        return grad_scores, None, None, None, None

    float_op.register_autograd(float_backward, setup_context=float_setup)
    return {
        prefix: tensor_op, f"{prefix}_float": float_op, f"{prefix}_with_grads": with_grads, f"{prefix}_hvp": hvp,
        f"{prefix}_param_jacobian": param_jacobian, f"{prefix}_backward_full": backward_full,
        f"{prefix}_param_grads_t": param_grads_t, f"{prefix}_backward_full_t": backward_full_t,
    }


globals().update(_make_affine_family("soft_sw_affine"))
globals().update(_make_affine_family("soft_nw_affine"))


# --------------------------------------------------------------------------- soft DTW
# (d2p/_pt2_ops.py:905-1010): the temperature is the one parameter; bandwidth
# is an int (< 0: no band)
@custom_op("d2p_py::soft_dtw_with_grads", mutates_args=())
def soft_dtw_with_grads(costs: torch.Tensor, temperature: float, lengths: Optional[torch.Tensor],
                        bandwidth: Optional[int]) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    v, m, gt = torch.ops.d2p.soft_dtw_with_grads(costs, temperature, lengths, bandwidth)
    return v, m, gt


@soft_dtw_with_grads.register_fake
def _(costs, temperature, lengths, bandwidth):
    return _like(costs, "B", "P", "B")


@custom_op("d2p_py::soft_dtw_hvp", mutates_args=())
def soft_dtw_hvp(costs: torch.Tensor, tangent: torch.Tensor, temperature: float, lengths: Optional[torch.Tensor],
                 bandwidth: Optional[int]) -> torch.Tensor:
    return torch.ops.d2p.soft_dtw_hvp(costs, tangent, temperature, lengths, bandwidth)


@soft_dtw_hvp.register_fake
def _(costs, tangent, temperature, lengths, bandwidth):
    return _like(costs, "P")


@custom_op("d2p_py::soft_dtw_param_jacobian", mutates_args=())
def soft_dtw_param_jacobian(costs: torch.Tensor, temperature: float, lengths: Optional[torch.Tensor],
                            bandwidth: Optional[int]) -> torch.Tensor:
    return torch.ops.d2p.soft_dtw_param_jacobian(costs, temperature, lengths, bandwidth)


@soft_dtw_param_jacobian.register_fake
def _(costs, temperature, lengths, bandwidth):
    return _like(costs, "P")


@custom_op("d2p_py::soft_dtw_backward_full", mutates_args=())
def soft_dtw_backward_full(costs: torch.Tensor, grad_alignment: torch.Tensor, temperature: float,
                           lengths: Optional[torch.Tensor],
                           bandwidth: Optional[int]) -> tuple[torch.Tensor, torch.Tensor]:
    a, b = torch.ops.d2p.soft_dtw_backward_full(costs, grad_alignment, temperature, lengths, bandwidth)
    return a, b


@soft_dtw_backward_full.register_fake
def _(costs, grad_alignment, temperature, lengths, bandwidth):
    return _like(costs, "P", "1")


@custom_op("d2p_py::soft_dtw", mutates_args=())
def soft_dtw(costs: torch.Tensor, temperature: torch.Tensor, lengths: torch.Tensor,
             bandwidth: int) -> tuple[torch.Tensor, torch.Tensor]:
    v, m = torch.ops.d2p.soft_dtw(costs, temperature, lengths, bandwidth)
    return v, m


@soft_dtw.register_fake
def _(costs, temperature, lengths, bandwidth):
    return _like(costs, "B", "P")


@custom_op("d2p_py::soft_dtw_grad_t", mutates_args=())
def soft_dtw_grad_t(costs: torch.Tensor, temperature: torch.Tensor, lengths: torch.Tensor,
                    bandwidth: int) -> torch.Tensor:
    return torch.ops.d2p.soft_dtw_with_grads(costs, float(temperature), lengths, bandwidth)[2]


@soft_dtw_grad_t.register_fake
def _(costs, temperature, lengths, bandwidth):
    return _like(costs, "B")


@custom_op("d2p_py::soft_dtw_backward_full_t", mutates_args=())
def soft_dtw_backward_full_t(costs: torch.Tensor, grad_alignment: torch.Tensor, temperature: torch.Tensor,
                             lengths: torch.Tensor, bandwidth: int) -> tuple[torch.Tensor, torch.Tensor]:
    a, b = torch.ops.d2p.soft_dtw_backward_full(costs, grad_alignment, float(temperature), lengths, bandwidth)
    return a, b


@soft_dtw_backward_full_t.register_fake
def _(costs, grad_alignment, temperature, lengths, bandwidth):
    return _like(costs, "P", "1")


def _soft_dtw_setup(ctx, inputs, output):
    costs, temperature, lengths, bandwidth = inputs
    ctx.save_for_backward(costs, output[1], temperature.detach())
    ctx.lengths, ctx.bandwidth = lengths, bandwidth


def _soft_dtw_backward(ctx, grad_value, grad_marg):
    costs, marg, temperature = ctx.saved_tensors
    grad_costs = _expand_batch(grad_value, marg)
    need_t = ctx.needs_input_grad[1]
    g_t = None
    if grad_value is not None and need_t:
        g_t = _batch_dot(grad_value, soft_dtw_grad_t(costs, temperature, ctx.lengths, ctx.bandwidth))
    if grad_marg is not None:
        gc, gt = soft_dtw_backward_full_t(costs, grad_marg, temperature, ctx.lengths, ctx.bandwidth)
        grad_costs = _add(grad_costs, gc)
        g_t = _add(g_t, gt) if need_t else None
    return grad_costs, g_t, None, None


soft_dtw.register_autograd(_soft_dtw_backward, setup_context=_soft_dtw_setup)


@custom_op("d2p_py::soft_dtw_float", mutates_args=())
def soft_dtw_float(costs: torch.Tensor, temperature: float, lengths: Optional[torch.Tensor],
                   bandwidth: Optional[int]) -> tuple[torch.Tensor, torch.Tensor]:
    v, m = torch.ops.d2p.soft_dtw_float(costs, temperature, lengths, bandwidth)
    return v, m


@soft_dtw_float.register_fake
def _(costs, temperature, lengths, bandwidth):
    return _like(costs, "B", "P")


def _soft_dtw_float_setup(ctx, inputs, output):
    costs, temperature, lengths, bandwidth = inputs
    ctx.save_for_backward(costs, output[1])
    ctx.temperature, ctx.lengths, ctx.bandwidth = temperature, lengths, bandwidth


def _soft_dtw_float_backward(ctx, grad_value, grad_marg):
    costs, marg = ctx.saved_tensors
    grad_costs = _expand_batch(grad_value, marg)
    if grad_marg is not None:
        gc, _ = soft_dtw_backward_full(costs, grad_marg, ctx.temperature, ctx.lengths, ctx.bandwidth)
        grad_costs = _add(grad_costs, gc)
    return grad_costs, None, None, None


soft_dtw_float.register_autograd(_soft_dtw_float_backward, setup_context=_soft_dtw_float_setup)
