"""Duration parameterisations producing the (K, C) duration bias.

``LearnedDuration`` (duration.py:91-126 of the reference) is the default of
``SemiMarkovCRFHead``.  Any ``DurationDistribution`` subclass -- an
``nn.Module`` whose forward returns a (K, C) tensor -- can be passed to the
head instead.
"""

from __future__ import annotations

import torch
import torch.nn as nn
from torch import Tensor


class DurationDistribution(nn.Module):
    """Base class: forward() returns the (max_duration, num_classes) log-space bias."""

    def __init__(self, max_duration: int, num_classes: int):
        super().__init__()
        self.max_duration = max_duration
        self.num_classes = num_classes

    def forward(self) -> Tensor:  # pragma: no cover - abstract
        raise NotImplementedError


class LearnedDuration(DurationDistribution):
    """Independent learned bias per (duration, class), initialised N(0, init_std^2)."""

    def __init__(self, max_duration: int, num_classes: int, init_std: float = 0.1):
        super().__init__(max_duration, num_classes)
        self.duration_bias = nn.Parameter(torch.randn(max_duration, num_classes) * init_std)

    def forward(self) -> Tensor:
        return self.duration_bias


def create_duration_distribution(distribution, max_duration: int, num_classes: int):
    """Factory for the head's ``duration_distribution`` argument."""
    if distribution is None or distribution == "learned":
        return LearnedDuration(max_duration, num_classes)
    if isinstance(distribution, DurationDistribution):
        return distribution
    raise NotImplementedError(
        f"duration distribution {distribution!r}: only 'learned' and DurationDistribution "
        "instances are provided")
