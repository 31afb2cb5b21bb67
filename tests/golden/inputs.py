"""Seeded synthetic inputs for the streaming semi-CRF scan.

These generators restate the synthetic workloads of the benchmark
configurations and the reference test suite's
``create_streaming_inputs`` helper (tests/test_streaming_triton.py:23-46 of
torch-semimarkov).  Everything is drawn from a seeded ``torch.Generator`` on
the CPU, in float64, then cast to float32 -- so the same seed gives the same
tensors here and on the GPU box.

Used by tests/golden/make_golden.py (fixture generation), tests/ and bench.py.
"""

from __future__ import annotations

import math

import torch

NEG_MASK = -1e4  # grammar-mask value of configuration 4


def checksum(t: torch.Tensor):
    t = t.detach().double()
    return torch.tensor([float(t.sum()), float(t.abs().sum())], dtype=torch.float64).numpy()


def _prefix(emissions: torch.Tensor) -> torch.Tensor:
    """cum[:, 0] = 0; cum[:, 1:] = cumsum(emissions) -- accumulated in float64."""
    B, T, C = emissions.shape
    cum = torch.zeros(B, T + 1, C, dtype=torch.float64)
    cum[:, 1:] = torch.cumsum(emissions.double(), dim=1)
    return cum.float()


def lognormal_duration_prior(K: int, C: int, g: torch.Generator, mu=4.5, sigma=1.0,
                             noise=0.05) -> torch.Tensor:
    """Configuration 3's duration bias: a log-normal-shaped prior over k plus noise."""
    k = torch.arange(K, dtype=torch.float64).clamp(min=1.0)
    base = -torch.log(k * sigma * math.sqrt(2 * math.pi)) - (torch.log(k) - mu) ** 2 / (2 * sigma ** 2)
    db = base[:, None].expand(K, C) + torch.randn(K, C, generator=g, dtype=torch.float64) * noise
    db = db.clone()
    db[0, :] = 0.0
    return db.float()


def make_streaming_inputs(B, T, K, C, seed, gen="default", proj=None, kcc=False):
    """Inputs of ``semi_crf_streaming_forward`` for one configuration.

    gen: "default" (reference test helper: zero-centred N(0,1) emissions,
    N(0, 0.1^2) parameters) or "cfg2"/"cfg3"/"cfg4"/"cfg5".
    """
    g = torch.Generator().manual_seed(int(seed))
    f64 = torch.float64
    if gen == "default":
        projected = torch.randn(B, T, C, generator=g, dtype=f64)
        projected = projected - projected.mean(dim=1, keepdim=True)
        cum = _prefix(projected)
        tr = torch.randn(C, C, generator=g, dtype=f64) * 0.1
        db = torch.randn(K, C, generator=g, dtype=f64) * 0.1
    elif gen == "cfg2":
        cum = _prefix(torch.randn(B, T, C, generator=g, dtype=f64) / math.sqrt(C))
        tr = torch.randn(C, C, generator=g, dtype=f64) * 0.1
        db = torch.randn(K, C, generator=g, dtype=f64) * 0.1
    elif gen == "cfg3":
        cum = _prefix(torch.randn(B, T, C, generator=g, dtype=f64))
        tr = torch.randn(C, C, generator=g, dtype=f64) * 0.1
        db = lognormal_duration_prior(K, C, g).double()
    elif gen == "cfg4":
        cum = _prefix(torch.randn(B, T, C, generator=g, dtype=f64) / math.sqrt(C))
        tr = torch.randn(C, C, generator=g, dtype=f64) * 0.1
        mask = torch.rand(C, C, generator=g, dtype=f64) < 0.5
        tr = torch.where(mask, torch.full_like(tr, NEG_MASK), tr)
        db = torch.randn(K, C, generator=g, dtype=f64) * 0.1
    elif gen == "cfg5":
        cum = _prefix(torch.randn(B, T, C, generator=g, dtype=f64))
        tr = torch.randn(C, C, generator=g, dtype=f64) * 0.2
        db = torch.randn(K, C, generator=g, dtype=f64) * 0.2
    else:
        raise ValueError(gen)
    if kcc:
        tr = torch.randn(K, C, C, generator=g, dtype=f64) * 0.1
    ps = pe = None
    if proj in ("both", "start"):
        ps = (torch.randn(B, T, C, generator=g, dtype=f64) * 0.1).float()
    if proj in ("both", "end"):
        pe = (torch.randn(B, T, C, generator=g, dtype=f64) * 0.1).float()
    return {
        "cum_scores": cum.float(),
        "transition": tr.float(),
        "duration_bias": db.float(),
        "proj_start": ps,
        "proj_end": pe,
    }


def config_lengths(gen, B, T, seed):
    """Per-configuration lengths: cfg2 uniform in [0.8T, T], cfg5 in [T/2, T]."""
    g = torch.Generator().manual_seed(int(seed) + 1000)
    if gen == "cfg2":
        return torch.randint(int(0.8 * T), T + 1, (B,), generator=g)
    if gen == "cfg5":
        return torch.randint(T // 2, T + 1, (B,), generator=g)
    return torch.full((B,), T, dtype=torch.long)


def make_hidden(B, T, C, K, seed, gen="default", hidden_dim=None):
    """Inputs of ``SemiMarkovCRFHead`` (hidden states, parameters, labels)."""
    g = torch.Generator().manual_seed(int(seed) + 7)
    f64 = torch.float64
    out = {}
    if gen == "cfg1":
        out["transition"] = (torch.randn(C, C, generator=g, dtype=f64) * 0.1).float()
        out["duration_bias"] = (torch.randn(K, C, generator=g, dtype=f64) * 0.1).float()
        bound = math.sqrt(6.0 / (hidden_dim + C))  # xavier_uniform_ on (C, hidden)
        out["proj_weight"] = ((torch.rand(C, hidden_dim, generator=g, dtype=f64) * 2 - 1)
                              * bound).float()
        out["proj_bias"] = torch.zeros(C)
        out["hidden"] = torch.randn(B, T, hidden_dim, generator=g, dtype=f64).float()
    elif gen == "cfg5":
        out["transition"] = (torch.randn(C, C, generator=g, dtype=f64) * 0.2).float()
        out["duration_bias"] = (torch.randn(K, C, generator=g, dtype=f64) * 0.2).float()
        out["hidden"] = torch.randn(B, T, C, generator=g, dtype=f64).float()
    else:
        out["transition"] = (torch.randn(C, C, generator=g, dtype=f64) * 0.1).float()
        out["duration_bias"] = (torch.randn(K, C, generator=g, dtype=f64) * 0.1).float()
        if hidden_dim is not None:
            bound = math.sqrt(6.0 / (hidden_dim + C))
            out["proj_weight"] = ((torch.rand(C, hidden_dim, generator=g, dtype=f64) * 2 - 1)
                                  * bound).float()
            out["proj_bias"] = torch.zeros(C)
            out["hidden"] = torch.randn(B, T, hidden_dim, generator=g, dtype=f64).float()
        else:
            out["hidden"] = torch.randn(B, T, C, generator=g, dtype=f64).float()
    out["labels"] = torch.randint(0, C, (B, T), generator=g)
    return out
