"""Edge-potential and checkpoint-interval helpers of the streaming API.

These mirror two public helpers of the reference
(streaming/pytorch_reference.py:25-45 and :48-113).  They are small tensor
expressions used for inspection and tests; the CUDA kernels never build an
edge block -- they use the factorised recurrence instead.
"""

from __future__ import annotations

import math
from typing import Optional

import torch


def _compute_checkpoint_interval(T: int, K: int) -> int:
    """Checkpoint interval S = max(K, floor(sqrt(T*K))), which minimises
    (T/S)*K*C + S*C + K*C memory (pytorch_reference.py:25-45)."""
    return max(K, int(math.sqrt(T * K)))


def compute_edge_block_streaming(
    cum_scores: torch.Tensor,
    transition: torch.Tensor,
    duration_bias: torch.Tensor,
    t: int,
    k: int,
    proj_start: Optional[torch.Tensor] = None,
    proj_end: Optional[torch.Tensor] = None,
) -> torch.Tensor:
    """Edge block (batch, C_dst, C_src) for segments starting at ``t`` with
    duration ``k`` (pytorch_reference.py:48-113):

        edge[c_dst, c_src] = cum[t+k, c_dst] - cum[t, c_dst]
                             + duration_bias[min(k, K-1), c_dst]
                             (+ proj_start[t, c_dst] + proj_end[t+k-1, c_dst])
                             + transition[c_src, c_dst]      (or transition[k])
    """
    seg = cum_scores[:, t + k, :] - cum_scores[:, t, :]
    K = duration_bias.shape[0]
    seg = seg + duration_bias[min(k, K - 1)]
    if proj_start is not None:
        seg = seg + proj_start[:, t, :]
    if proj_end is not None:
        seg = seg + proj_end[:, t + k - 1, :]
    trans_k = transition if transition.ndim == 2 else transition[k]
    return seg.unsqueeze(-1) + trans_k.T.unsqueeze(0)
