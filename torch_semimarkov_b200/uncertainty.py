"""Uncertainty quantification on the streaming path (reference uncertainty.py:36-498).

``UncertaintyMixin`` and ``UncertaintySemiMarkovCRFHead`` keep the reference's
method names, arguments and return shapes.  Every streaming method runs one
forward and one backward of the CUDA scan: the marginal signals are gradients
of log Z with respect to the cumulative scores (boundary marginals,
uncertainty.py:92-163) or the projected scores (position marginals,
uncertainty.py:263-328), so they work at chromosome-scale T without an edge
tensor.

The reference's exact variants (``compute_boundary_marginals(use_streaming=False)``
and ``compute_entropy_exact``, uncertainty.py:165-219 and :370-416) run its
separate edge-tensor library (``SemiMarkov`` over a (batch, T-1, K, C, C)
tensor with Log / Entropy semirings).  That library is not part of this
package, so they raise ``NotImplementedError``.
"""

from __future__ import annotations

from typing import Optional, Union

import torch
from torch import Tensor

from .duration import DurationDistribution
from .nn import SemiMarkovCRFHead
from .streaming import semi_crf_streaming_forward

_EXACT_MSG = ("exact edge-tensor marginals and entropy need the reference's O(T*K*C^2) "
              "SemiMarkov library, which torch_semimarkov_b200 does not include; use the "
              "streaming methods (use_streaming=True, compute_entropy_streaming)")


class UncertaintyMixin:
    """Boundary / position marginals, streaming entropy and uncertainty-weighted loss.

    Classes using the mixin need ``projection``, ``transition``,
    ``duration_bias``, ``num_classes`` and ``max_duration`` attributes.
    """

    def _label_scores(self, hidden_states: Tensor) -> Tensor:
        if self.projection is not None:
            with torch.no_grad():
                return self.projection(hidden_states)
        return hidden_states

    def _log_z(self, cum_scores: Tensor, lengths: Tensor) -> Tensor:
        return semi_crf_streaming_forward(
            cum_scores, self.transition.detach(), self.duration_bias.detach(), lengths,
            self.max_duration, semiring="log", use_triton=False)

    def compute_boundary_marginals(self, hidden_states: Tensor, lengths: Tensor,
                                   use_streaming: bool = True, normalize: bool = True) -> Tensor:
        """Boundary signal per position, shape (batch, T) (uncertainty.py:56-90)."""
        if not use_streaming:
            raise NotImplementedError(_EXACT_MSG)
        return self._compute_boundary_marginals_streaming(hidden_states, lengths, normalize)

    def _compute_boundary_marginals_streaming(self, hidden_states: Tensor, lengths: Tensor,
                                              normalize: bool = True) -> Tensor:
        """sum_c |d log Z / d cum_scores[:, t, c]| for t = 1..T (uncertainty.py:92-163)."""
        batch, T, _ = hidden_states.shape
        scores = self._label_scores(hidden_states)
        with torch.enable_grad():
            cum_scores = torch.zeros(batch, T + 1, self.num_classes, dtype=torch.float32,
                                     device=scores.device)
            cum_scores[:, 1:] = torch.cumsum(scores.float().detach(), dim=1)
            cum_scores = cum_scores.requires_grad_(True)
            self._log_z(cum_scores, lengths).sum().backward()
        signal = cum_scores.grad[:, 1:].abs().sum(dim=-1)
        if normalize:
            signal = signal / (signal.max(dim=-1, keepdim=True)[0] + 1e-8)
        return signal

    def _compute_boundary_marginals_exact(self, hidden_states: Tensor, lengths: Tensor,
                                          normalize: bool = True) -> Tensor:
        raise NotImplementedError(_EXACT_MSG)

    def compute_position_marginals(self, hidden_states: Tensor, lengths: Tensor) -> Tensor:
        """softmax_c |d log Z / d scores[:, t, c]|, shape (batch, T, C) (uncertainty.py:263-328)."""
        batch, T, _ = hidden_states.shape
        scores = self._label_scores(hidden_states)
        with torch.enable_grad():
            scores_for_grad = scores.detach().requires_grad_(True)
            cum_scores = torch.zeros(batch, T + 1, self.num_classes, dtype=torch.float32,
                                     device=scores_for_grad.device)
            cum_scores[:, 1:] = torch.cumsum(scores_for_grad.float(), dim=1)
            self._log_z(cum_scores, lengths).sum().backward()
        return torch.softmax(scores_for_grad.grad.abs(), dim=-1)

    def compute_entropy_streaming(self, hidden_states: Tensor, lengths: Tensor) -> Tensor:
        """Entropy of the normalised boundary signal, shape (batch,) (uncertainty.py:330-368)."""
        p = self.compute_boundary_marginals(hidden_states, lengths, use_streaming=True,
                                            normalize=False)
        p = p / (p.sum(dim=-1, keepdim=True) + 1e-8)
        return -(p * torch.log(p.clamp(min=1e-10))).sum(dim=-1)

    def compute_entropy_exact(self, hidden_states: Tensor, lengths: Tensor) -> Tensor:
        raise NotImplementedError(_EXACT_MSG)

    def compute_loss_uncertainty_weighted(self, hidden_states: Tensor, lengths: Tensor,
                                          labels: Tensor, uncertainty_weight: float = 1.0,
                                          focus_mode: str = "high_uncertainty",
                                          use_triton: bool = False,
                                          reduction: str = "mean") -> Tensor:
        """(1 + lambda * u) * NLL with u from the streaming entropy or the mean boundary
        signal (uncertainty.py:418-497)."""
        with torch.no_grad():
            if focus_mode == "high_uncertainty":
                u = self.compute_entropy_streaming(hidden_states.detach(), lengths)
                u = u / (u.max() + 1e-8)
            elif focus_mode == "boundary_regions":
                u = self.compute_boundary_marginals(hidden_states.detach(), lengths,
                                                    use_streaming=True).mean(dim=-1)
            else:
                raise ValueError(f"Unknown focus_mode: {focus_mode}")
        result = self.forward(hidden_states, lengths, use_triton)
        nll = result["partition"] - self._score_gold(result["cum_scores"], labels, lengths)
        weighted = nll * (1.0 + uncertainty_weight * u)
        if reduction == "mean":
            return weighted.mean()
        if reduction == "sum":
            return weighted.sum()
        return weighted


class UncertaintySemiMarkovCRFHead(UncertaintyMixin, SemiMarkovCRFHead):
    """SemiMarkovCRFHead with the uncertainty methods (uncertainty.py:500-933).

    Same constructor, parameters and forward / compute_loss / decode /
    decode_with_traceback as ``SemiMarkovCRFHead``.
    """

    def __init__(self, num_classes: int, max_duration: int, hidden_dim: Optional[int] = None,
                 init_scale: float = 0.1,
                 duration_distribution: Optional[Union[str, DurationDistribution]] = None):
        SemiMarkovCRFHead.__init__(self, num_classes, max_duration, hidden_dim, init_scale,
                                   duration_distribution)
