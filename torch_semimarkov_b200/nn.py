"""SemiMarkovCRFHead: the reference's CRF head (nn.py:55-565) on the CUDA path.

Same constructor, parameters, methods and return types.  ``forward`` /
``compute_loss`` / ``decode`` call the streaming kernels; ``decode_with_traceback``
runs the max-semiring chain with compact backpointers and a GPU backtrace in
one call (the reference re-runs a per-sequence PyTorch loop and a host
backtrace).  ``use_triton`` is accepted and ignored.
"""

from __future__ import annotations

from typing import Optional, Union

import torch
import torch.nn as nn
from torch import Tensor

from . import _lib
from .duration import DurationDistribution, LearnedDuration, create_duration_distribution
from .helpers import Segment, ViterbiResult, score_gold_vectorized
from .streaming import semi_crf_streaming_forward


class SemiMarkovCRFHead(nn.Module):
    """CRF head for semi-Markov sequence labelling.

    Args:
        num_classes: number of labels C.
        max_duration: maximum segment duration K (durations 1..max(1, K-1)).
        hidden_dim: if given, a Linear(hidden_dim -> C) projection is applied.
        init_scale: std of the N(0, init_scale^2) transition / duration init.
        duration_distribution: None / "learned" or a DurationDistribution.
    """

    def __init__(
        self,
        num_classes: int,
        max_duration: int,
        hidden_dim: Optional[int] = None,
        init_scale: float = 0.1,
        duration_distribution: Optional[Union[str, DurationDistribution]] = None,
    ):
        super().__init__()
        self.num_classes = num_classes
        self.max_duration = max_duration
        self.transition = nn.Parameter(torch.randn(num_classes, num_classes) * init_scale)
        if duration_distribution is None or duration_distribution == "learned":
            self.duration_dist = LearnedDuration(max_duration, num_classes, init_std=init_scale)
        else:
            self.duration_dist = create_duration_distribution(
                duration_distribution, max_duration, num_classes)
        self.projection = nn.Linear(hidden_dim, num_classes) if hidden_dim is not None else None

    @property
    def duration_bias(self) -> Tensor:
        return self.duration_dist()

    def _cum_scores(self, hidden_states: Tensor) -> Tensor:
        batch, T, _ = hidden_states.shape
        scores = self.projection(hidden_states) if self.projection is not None else hidden_states
        cum = torch.zeros(batch, T + 1, self.num_classes, dtype=torch.float32,
                          device=scores.device)
        cum[:, 1:] = torch.cumsum(scores.float(), dim=1)
        return cum

    def forward(self, hidden_states: Tensor, lengths: Tensor, use_triton: bool = True) -> dict:
        """Returns {"partition": (batch,), "cum_scores": (batch, T+1, C)}."""
        cum_scores = self._cum_scores(hidden_states)
        partition = semi_crf_streaming_forward(
            cum_scores, self.transition, self.duration_bias, lengths, self.max_duration,
            semiring="log")
        return {"partition": partition, "cum_scores": cum_scores}

    def compute_loss(self, hidden_states: Tensor, lengths: Tensor, labels: Tensor,
                     use_triton: bool = True, reduction: str = "mean") -> Tensor:
        """NLL = log Z - score(gold segmentation); reduction "mean" | "sum" | "none"."""
        result = self.forward(hidden_states, lengths, use_triton)
        gold = self._score_gold(result["cum_scores"], labels, lengths)
        nll = result["partition"] - gold
        if reduction == "mean":
            return nll.mean()
        if reduction == "sum":
            return nll.sum()
        return nll

    def _score_gold(self, cum_scores: Tensor, labels: Tensor, lengths: Tensor) -> Tensor:
        return score_gold_vectorized(cum_scores=cum_scores, labels=labels, lengths=lengths,
                                     transition=self.transition,
                                     duration_bias=self.duration_bias,
                                     max_duration=self.max_duration)

    def decode(self, hidden_states: Tensor, lengths: Tensor, use_triton: bool = True) -> Tensor:
        """Best (max-semiring) segmentation score, shape (batch,)."""
        cum_scores = self._cum_scores(hidden_states)
        return semi_crf_streaming_forward(
            cum_scores, self.transition, self.duration_bias, lengths, self.max_duration,
            semiring="max")

    @torch.no_grad()
    def decode_with_traceback(self, hidden_states: Tensor, lengths: Tensor,
                              max_traceback_length: int = 10000) -> ViterbiResult:
        """Best scores and segmentations.  Sequences longer than
        ``max_traceback_length`` (or empty) get an empty segment list."""
        cum_scores = self._cum_scores(hidden_states)
        prob = _lib.Problem(cum_scores, self.transition, self.duration_bias, lengths,
                            self.max_duration, "max")
        scores, ss, se, sl, sv, ns = _lib.viterbi(prob, max_traceback_length)
        ns_h = ns.cpu().tolist()
        nmax = max(ns_h) if ns_h else 0
        segments: list[list[Segment]] = []
        if nmax > 0:
            ss_h = ss[:, :nmax].cpu().tolist()
            se_h = se[:, :nmax].cpu().tolist()
            sl_h = sl[:, :nmax].cpu().tolist()
            sv_h = sv[:, :nmax].cpu().tolist()
        for b, n in enumerate(ns_h):
            if n == 0:
                segments.append([])
                continue
            segments.append([Segment(start=ss_h[b][i], end=se_h[b][i], label=sl_h[b][i],
                                     score=sv_h[b][i]) for i in range(n)])
        return ViterbiResult(scores=scores, segments=segments)

    def extra_repr(self) -> str:
        parts = [f"num_classes={self.num_classes}", f"max_duration={self.max_duration}"]
        if self.projection is not None:
            parts.append(f"hidden_dim={self.projection.in_features}")
        parts.append(f"duration_dist={self.duration_dist.__class__.__name__}")
        return ", ".join(parts)
