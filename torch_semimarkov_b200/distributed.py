"""Batch sharding over ranks and the one collective of a training step.

The sequences of a streaming semi-CRF batch are independent: the reference
runs one program per sequence (streaming/triton_forward.py:665,
streaming/triton_backward.py:703) and its only cross-sequence coupling is the
sum of the shared-parameter gradients, sum_b grad_output[b] * d log Z_b /
d(transition, duration_bias) (streaming/autograd.py:134-150).  So a batch
shards over GPUs (one process per GPU) with no exchange on the data path:

  * ``shard_sequences`` assigns whole sequences to ranks, longest first to
    the least-loaded rank (the scan's cost is proportional to the length);
  * ``SharedGradReducer`` sums [grad_transition | grad_duration_bias | loss]
    over the ranks with one all-reduce per step (C*C + K*C + 1 float32
    values: 31 KB at C=24, K=300).  grad_cum and the projection gradients
    stay on the rank that owns the sequence.

The collective goes through ``torch.distributed`` (NCCL on GPUs, gloo on
CPU); a rank that fails or never arrives surfaces as an error on the others
once the process group's timeout expires.
"""

from __future__ import annotations

import heapq
from typing import Optional, Sequence, Tuple

import torch
import torch.distributed as dist


def shard_sequences(lengths: Sequence[int], world_size: int, rank: int) -> torch.Tensor:
    """Indices (ascending) of the sequences that ``rank`` owns.

    Longest-processing-time assignment: sequences in descending length (ties
    by index) each go to the rank with the least total length so far (ties
    by rank).  Deterministic, so every rank computes the same partition
    without communicating.  Every index is owned by exactly one rank.
    """
    if world_size < 1 or not 0 <= rank < world_size:
        raise ValueError(f"rank {rank} is outside a world of size {world_size}")
    lens = [int(v) for v in (lengths.tolist() if isinstance(lengths, torch.Tensor) else lengths)]
    order = sorted(range(len(lens)), key=lambda i: (-lens[i], i))
    heap = [(0, r) for r in range(world_size)]
    mine = []
    for i in order:
        load, r = heapq.heappop(heap)
        if r == rank:
            mine.append(i)
        heapq.heappush(heap, (load + max(lens[i], 1), r))
    return torch.tensor(sorted(mine), dtype=torch.int64)


class SharedGradReducer:
    """Sums the shared-parameter gradients and the loss over all ranks.

    One flat float32 buffer [grad_transition | grad_duration_bias | loss] is
    all-reduced (sum) per call, so a step issues exactly one collective.
    """

    def __init__(self, C: int, K: int, device, group: Optional[dist.ProcessGroup] = None,
                 transition_shape: Optional[Tuple[int, ...]] = None):
        self.tr_shape = tuple(transition_shape) if transition_shape else (C, C)
        self.ntr = 1
        for d in self.tr_shape:
            self.ntr *= int(d)
        self.ndb = K * C
        self.db_shape = (K, C)
        self.group = group
        self.buf = torch.empty(self.ntr + self.ndb + 1, dtype=torch.float32, device=device)

    def __call__(self, grad_transition: torch.Tensor, grad_duration_bias: torch.Tensor,
                 loss: torch.Tensor):
        n0, n1 = self.ntr, self.ntr + self.ndb
        self.buf[:n0].copy_(grad_transition.reshape(-1))
        self.buf[n0:n1].copy_(grad_duration_bias.reshape(-1))
        self.buf[n1:].copy_(loss.detach().reshape(1))
        if dist.is_available() and dist.is_initialized():
            dist.all_reduce(self.buf, op=dist.ReduceOp.SUM, group=self.group)
        return (self.buf[:n0].view(self.tr_shape), self.buf[n0:n1].view(self.db_shape),
                self.buf[n1:].view(()))
