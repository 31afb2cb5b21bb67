"""Duration parameterisations producing the (K, C) duration bias.

Each is an ``nn.Module`` whose forward returns the (max_duration, num_classes)
log-space bias that the scan adds to a segment of duration k (row k).  They
carry the reference's class names, constructor arguments, parameter names
and formulas (duration.py:54-558), so state dicts and the head's
``duration_distribution`` argument carry over:

- ``LearnedDuration``: a free (K, C) parameter, N(0, init_std^2) at start;
- ``GeometricDuration``: log p + (k-1) log(1-p), p = sigmoid(logit_p) per class;
- ``NegativeBinomialDuration``: log C(k+r-2, k-1) + r log p + (k-1) log(1-p);
- ``PoissonDuration``: k log(lambda) - log k! - lambda (a shifted Poisson);
- ``UniformDuration``: zeros;
- ``CallableDuration``: whatever ``func(K, C, device)`` returns.

The probabilities enter their logs with the reference's 1e-8 guard, and r
with its 1e-8 floor, so the biases agree value for value.
"""

from __future__ import annotations

import warnings
from typing import Callable, Optional, Union

import torch
import torch.nn as nn
from torch import Tensor

_EPS = 1e-8


class DurationDistribution(nn.Module):
    """Base class: forward() returns the (max_duration, num_classes) log-space bias."""

    def __init__(self, max_duration: int, num_classes: int):
        super().__init__()
        self.max_duration = max_duration
        self.num_classes = num_classes

    def forward(self) -> Tensor:  # pragma: no cover - abstract
        raise NotImplementedError

    def _per_class(self, name: str, value: float, learn: bool) -> None:
        """A (C,) tensor named ``name``: a parameter if learned, else a buffer."""
        t = torch.full((self.num_classes,), float(value))
        if learn:
            setattr(self, name, nn.Parameter(t))
        else:
            self.register_buffer(name, t)

    def _durations(self, like: Tensor) -> Tensor:
        """k = 1 .. K as a (K, 1) column in the dtype and device of ``like``."""
        return torch.arange(1, self.max_duration + 1, device=like.device,
                            dtype=like.dtype).unsqueeze(1)


class LearnedDuration(DurationDistribution):
    """Independent learned bias per (duration, class), initialised N(0, init_std^2)."""

    def __init__(self, max_duration: int, num_classes: int, init_std: float = 0.1):
        super().__init__(max_duration, num_classes)
        self.duration_bias = nn.Parameter(torch.randn(max_duration, num_classes) * init_std)

    def forward(self) -> Tensor:
        return self.duration_bias


class GeometricDuration(DurationDistribution):
    """P(k) proportional to p (1-p)^(k-1), one learned rate per class."""

    def __init__(self, max_duration: int, num_classes: int, init_logit: float = 0.0,
                 learn_rate: bool = True):
        super().__init__(max_duration, num_classes)
        self._per_class("logit_p", init_logit, learn_rate)

    def forward(self) -> Tensor:
        p = torch.sigmoid(self.logit_p)
        k = self._durations(p)
        return torch.log(p + _EPS).unsqueeze(0) + (k - 1) * torch.log(1 - p + _EPS).unsqueeze(0)


class NegativeBinomialDuration(DurationDistribution):
    """P(k) proportional to C(k+r-2, k-1) p^r (1-p)^(k-1); r = 1 is geometric.

    Very small r (log_r below about -10) overflows lgamma; the bias then holds
    non-finite entries and a UserWarning says so.
    """

    def __init__(self, max_duration: int, num_classes: int, init_logit: float = 0.0,
                 init_log_r: float = 0.0, learn_rate: bool = True, learn_shape: bool = True):
        super().__init__(max_duration, num_classes)
        self._per_class("logit_p", init_logit, learn_rate)
        self._per_class("log_r", init_log_r, learn_shape)

    def forward(self) -> Tensor:
        p = torch.sigmoid(self.logit_p)
        r = (torch.exp(self.log_r) + _EPS).unsqueeze(0)  # (1, C)
        k = self._durations(p)                           # (K, 1)
        log_choose = torch.lgamma(k + r - 1) - torch.lgamma(r) - torch.lgamma(k)
        out = (log_choose + r * torch.log(p + _EPS).unsqueeze(0)
               + (k - 1) * torch.log(1 - p + _EPS).unsqueeze(0))
        if not torch.jit.is_scripting() and not torch.compiler.is_compiling():
            bad = int((~torch.isfinite(out)).sum())
            if bad:
                warnings.warn(
                    f"NegativeBinomialDuration produced {bad} non-finite values; r is very "
                    f"small (min r={float(r.detach().min()):.2e}). Use a larger init_log_r or "
                    "GeometricDuration.", stacklevel=2)
        return out


class PoissonDuration(DurationDistribution):
    """Shifted Poisson: log P(k) = k log(lambda) - log(k!) - lambda, k >= 1."""

    def __init__(self, max_duration: int, num_classes: int, init_log_lambda: float = 1.0,
                 learn_rate: bool = True):
        super().__init__(max_duration, num_classes)
        self._per_class("log_lambda", init_log_lambda, learn_rate)

    def forward(self) -> Tensor:
        lam = torch.exp(self.log_lambda).unsqueeze(0)  # (1, C)
        k = self._durations(lam)
        return k * torch.log(lam + _EPS) - torch.lgamma(k + 1) - lam


class CallableDuration(DurationDistribution):
    """The bias ``func(max_duration, num_classes, device)`` of a user function.

    A one-element parameter without gradient moves with the module across
    devices, so that ``func`` is told where to build its tensor.
    """

    def __init__(self, max_duration: int, num_classes: int,
                 func: Callable[[int, int, torch.device], Tensor]):
        super().__init__(max_duration, num_classes)
        self._func = func
        self._device_tracker = nn.Parameter(torch.zeros(1), requires_grad=False)

    def forward(self) -> Tensor:
        return self._func(self.max_duration, self.num_classes, self._device_tracker.device)


class UniformDuration(DurationDistribution):
    """No duration preference: a zero bias."""

    def __init__(self, max_duration: int, num_classes: int):
        super().__init__(max_duration, num_classes)
        self.register_buffer("_zeros", torch.zeros(max_duration, num_classes))

    def forward(self) -> Tensor:
        return self._zeros


_BY_NAME = {
    "geometric": GeometricDuration,
    "negative_binomial": NegativeBinomialDuration,
    "negbin": NegativeBinomialDuration,
    "poisson": PoissonDuration,
}


def create_duration_distribution(distribution: Optional[Union[str, DurationDistribution]],
                                 max_duration: int, num_classes: int,
                                 **kwargs) -> DurationDistribution:
    """Factory for the head's ``duration_distribution`` argument (duration.py:493-558).

    None / "learned", "geometric", "negative_binomial" / "negbin", "poisson",
    "uniform", or a DurationDistribution instance (returned as is); extra
    keyword arguments go to the constructor.  Any other string raises ValueError.
    """
    if distribution is None or distribution == "learned":
        return LearnedDuration(max_duration, num_classes, **kwargs)
    if isinstance(distribution, DurationDistribution):
        return distribution
    if distribution == "uniform":
        return UniformDuration(max_duration, num_classes)
    cls = _BY_NAME.get(distribution) if isinstance(distribution, str) else None
    if cls is None:
        raise ValueError(f"Unknown duration distribution: {distribution}. "
                         "Options: learned, geometric, negative_binomial, poisson, uniform")
    return cls(max_duration, num_classes, **kwargs)
