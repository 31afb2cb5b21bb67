"""Result types and gold-segmentation scoring.

``Segment`` / ``ViterbiResult`` mirror helpers.py:10-78 of the reference.
``score_gold_vectorized`` keeps the signature and semantics of
helpers.py:365-544 but runs as one CUDA kernel per call (one thread walks one
sequence's label runs) with a CUDA backward, instead of a per-batch Python
loop with host synchronisations.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch
from torch import Tensor

from . import _lib


@dataclass
class Segment:
    """A labelled segment [start, end] (inclusive) with its score contribution."""

    start: int
    end: int
    label: int
    score: float = 0.0

    @property
    def duration(self) -> int:
        return self.end - self.start + 1


@dataclass
class ViterbiResult:
    """Best scores (batch,) and the per-sequence optimal segment lists."""

    scores: Tensor
    segments: list[list[Segment]]


class _GoldScore(torch.autograd.Function):
    @staticmethod
    def forward(ctx, cum_scores, transition, duration_bias, labels, lengths, K):
        out = _lib.score_gold(cum_scores, labels, lengths, transition, duration_bias, K)
        ctx.save_for_backward(labels, lengths)
        ctx.shape = (cum_scores.shape[0], cum_scores.shape[1] - 1, int(K), cum_scores.shape[2])
        ctx.dtypes = (cum_scores.dtype, transition.dtype, duration_bias.dtype)
        ctx.device = cum_scores.device
        return out.to(cum_scores.dtype)

    @staticmethod
    def backward(ctx, grad_out):
        labels, lengths = ctx.saved_tensors
        B, T, K, C = ctx.shape
        gc, gt, gd = _lib.score_gold_backward(labels, lengths, grad_out, B, T, K, C, ctx.device)
        return gc.to(ctx.dtypes[0]), gt.to(ctx.dtypes[1]), gd.to(ctx.dtypes[2]), None, None, None


def score_gold_vectorized(
    cum_scores: torch.Tensor,
    labels: torch.Tensor,
    lengths: torch.Tensor,
    transition: torch.Tensor,
    duration_bias: torch.Tensor,
    max_duration: int,
) -> torch.Tensor:
    """Score of the gold segmentation implied by per-position ``labels``.

    Segments are maximal runs of equal labels inside [0, length); a segment
    [st, en] with label c contributes cum[en+1,c] - cum[st,c] +
    duration_bias[clamp(en-st+1, 1, K-1), c] + transition[prev, c] (no
    transition for the first segment).  Differentiable in cum_scores,
    transition and duration_bias.
    """
    if transition.dim() != 2:
        raise NotImplementedError("gold scoring supports (C, C) transitions")
    B, T1, C = cum_scores.shape
    if T1 - 1 == 0:
        return torch.zeros(B, device=cum_scores.device, dtype=cum_scores.dtype)
    return _GoldScore.apply(cum_scores, transition, duration_bias, labels, lengths,
                            int(max_duration))
