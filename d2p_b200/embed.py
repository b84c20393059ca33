"""Score producer: soft Smith-Waterman from embeddings.

The reference's operators take the score plane ([B, L1, L2], d2p/sw.py:247);
its examples build that plane from per-position embeddings with an einsum
(docs/examples.md:9-23).  ``embed_scores`` builds it on the tcgen05 tensor
cores (``torch.ops.d2p_b200.embed_scores``, d2p_b200/csrc/sw_embed.cu: bf16
inputs, fp32 accumulation and output) and ``soft_sw_embed`` feeds it to the
soft SW value + marginals pass as one autograd node.  Gradients flow back to the embeddings: with G = dL/dscores
(the marginals times the value's gradient for ``value.sum()``),
dL/dx = scale G y and dL/dy = scale G^T x, two plain batched bf16 GEMMs
(cuBLAS, fp32 accumulation).
"""
from __future__ import annotations

from typing import Optional, Union

import torch
import torch.nn.functional as F

from . import _ops  # noqa: F401  the native extension (fails loudly if missing)
from .sw import SWResult, _validate_gap, _validate_temperature, soft_sw

_K = 64       # the producer reads the embedding dimension in chunks of 64
_MAX_D = 256


def _padded(t: torch.Tensor) -> torch.Tensor:
    d = t.shape[-1]
    pad = (-d) % _K
    return F.pad(t, (0, pad)) if pad else t


class _EmbedScores(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, y, scale):
        ctx.save_for_backward(x, y)
        ctx.scale = scale
        return torch.ops.d2p_b200.embed_scores(_padded(x), _padded(y), float(scale))

    @staticmethod
    def backward(ctx, g):
        # bf16 GEMMs with fp32 accumulation (cuBLAS): the gradients are bf16
        # like the embeddings, and rounding G to bf16 stays inside that
        x, y = ctx.saved_tensors
        gx = gy = None
        gb = (g.float() * ctx.scale).to(torch.bfloat16)
        if ctx.needs_input_grad[0]:
            gx = torch.bmm(gb, y)
        if ctx.needs_input_grad[1]:
            gy = torch.bmm(gb.transpose(1, 2), x)
        return gx, gy, None


def embed_scores(x: torch.Tensor, y: torch.Tensor, scale: float = 1.0) -> torch.Tensor:
    """scores[b] = scale * x[b] @ y[b]^T in fp32, for bfloat16 CUDA embeddings
    x [B, L1, D] and y [B, L2, D] (D <= 256; other D are zero-padded to a
    multiple of 64, which leaves every dot product unchanged)."""
    embed_scores_checks(x, y)
    return _EmbedScores.apply(x, y, scale)


def embed_scores_checks(x: torch.Tensor, y: torch.Tensor) -> None:
    if x.dtype != torch.bfloat16 or y.dtype != torch.bfloat16:
        raise TypeError("embed_scores: x and y must be bfloat16 (cast the embeddings first)")
    if x.dim() != 3 or y.dim() != 3 or x.shape[0] != y.shape[0] or x.shape[2] != y.shape[2]:
        raise ValueError("embed_scores: x must be [B, L1, D] and y [B, L2, D] with the same B and D")
    if x.shape[2] > _MAX_D:
        raise ValueError(f"embed_scores: embedding dimension {x.shape[2]} exceeds {_MAX_D}")


class _SoftSWEmbed(torch.autograd.Function):
    """Producer + soft SW as one autograd node (float gap and temperature).
    Backward: G = dL/dscores = g_value P (+ the marginals' term H g_P when the
    loss reaches the marginals, from backward_full), formed in bf16 in one pass
    over the marginals, then dL/dx = scale G y and dL/dy = scale G^T x."""

    @staticmethod
    def forward(ctx, x, y, gap, temperature, lengths, scale):
        S = torch.ops.d2p_b200.embed_scores(_padded(x), _padded(y), float(scale))
        v, P = torch.ops.d2p.soft_sw_float(S, gap, temperature, lengths)
        ctx.set_materialize_grads(False)
        ctx.save_for_backward(x, y, S, P, lengths)
        ctx.gap, ctx.temperature, ctx.scale = gap, temperature, float(scale)
        return v, P

    @staticmethod
    def backward(ctx, g_value, g_marginals):
        x, y, S, P, lengths = ctx.saved_tensors
        G = None
        if g_value is not None:
            G = torch.ops.d2p_b200.embed_grad_scores(P, g_value.float().contiguous(), ctx.scale)
        if g_marginals is not None:
            gS, _, _ = torch.ops.d2p.soft_sw_backward_full(S, g_marginals.float().contiguous(), ctx.gap,
                                                            ctx.temperature, lengths)
            gS = gS * ctx.scale
            G = (gS if G is None else G.float() + gS).to(torch.bfloat16)
        if G is None:
            return None, None, None, None, None, None
        gx = torch.bmm(G, y) if ctx.needs_input_grad[0] else None
        gy = torch.bmm(G.transpose(1, 2), x) if ctx.needs_input_grad[1] else None
        return gx, gy, None, None, None, None


def soft_sw_embed(
    x: torch.Tensor,
    y: torch.Tensor,
    gap: Union[float, torch.Tensor] = -1.0,
    temperature: Union[float, torch.Tensor] = 1.0,
    lengths: Optional[torch.Tensor] = None,
    scale: float = 1.0,
) -> SWResult:
    """Soft Smith-Waterman (linear gap) of the scores scale * x y^T, with
    gradients to x and y (and to gap / temperature when they are tensors)."""
    if isinstance(gap, torch.Tensor) or isinstance(temperature, torch.Tensor):
        return soft_sw(embed_scores(x, y, scale), gap=gap, temperature=temperature, lengths=lengths)
    _validate_temperature(temperature)
    _validate_gap(gap)
    embed_scores_checks(x, y)
    v, P = _SoftSWEmbed.apply(x, y, float(gap), float(temperature), lengths, scale)
    return SWResult(v, P)


def _embed_scores_fake(x, y, scale):
    return x.new_empty((x.shape[0], x.shape[1], y.shape[1]), dtype=torch.float32)


def _has_op() -> bool:
    try:
        torch.ops.d2p_b200.embed_scores
        return True
    except (AttributeError, RuntimeError):
        return False


# (a library built before the producer existed has no such op; calls then fail loudly)
if _has_op():
    torch.library.register_fake("d2p_b200::embed_scores")(_embed_scores_fake)
