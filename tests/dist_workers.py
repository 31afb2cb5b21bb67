"""Rank bodies for the two-rank gloo tests (spawned processes import this).

The CPU oracle stands in for the CUDA kernels: each rank computes its
shard's partitions and gradients with it, then the package's host logic
(torch_semimarkov_b200.distributed) shards the batch and reduces the shared
gradients exactly as a GPU rank does.
"""

import datetime
import json
import os
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
for p in (ROOT, os.path.join(ROOT, "tests", "golden")):
    if p not in sys.path:
        sys.path.insert(0, p)


def _init(rank, world, port, timeout_s):
    import torch.distributed as dist

    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank,
                            world_size=world, timeout=datetime.timedelta(seconds=timeout_s))


def step_worker(rank, world, port, case, out_path):
    """One data-parallel training step: shard, compute, all-reduce."""
    import numpy as np
    import torch
    import torch.distributed as dist

    from inputs import make_streaming_inputs
    from oracle import oracle
    from torch_semimarkov_b200.distributed import SharedGradReducer, shard_sequences

    B, T, K, C, seed = case
    _init(rank, world, port, 60)
    inp = make_streaming_inputs(B, T, K, C, seed=seed)
    lengths = np.array([T, T - 3, T // 2, T - 1, 5, T - 7][:B])
    mine = shard_sequences(lengths, world, rank).numpy()
    part, grads = oracle.forward_backward(
        inp["cum_scores"].numpy()[mine], inp["transition"].numpy(),
        inp["duration_bias"].numpy(), lengths[mine], K)
    red = SharedGradReducer(C, K, torch.device("cpu"))
    gt, gd, loss = red(torch.as_tensor(grads["transition"], dtype=torch.float32),
                       torch.as_tensor(grads["duration_bias"], dtype=torch.float32),
                       torch.tensor(float(part.sum())))
    res = {"rank": rank, "mine": mine.tolist(), "gt": gt.tolist(), "gd": gd.tolist(),
           "loss": float(loss)}
    with open(out_path, "w") as f:
        json.dump(res, f)
    dist.barrier()
    dist.destroy_process_group()


def failing_worker(rank, world, port, out_path):
    """Rank 1 fails before the step's collective; rank 0 must get an error,
    not hang (the process group's timeout bounds the wait)."""
    import torch
    import torch.distributed as dist

    from torch_semimarkov_b200.distributed import SharedGradReducer

    _init(rank, world, port, 5)
    if rank == 1:
        os._exit(3)  # dies between steps: nothing of its own is in flight
    red = SharedGradReducer(2, 3, torch.device("cpu"))
    status = "no error"
    try:
        red(torch.zeros(2, 2), torch.zeros(3, 2), torch.tensor(0.0))
    except Exception as e:  # noqa: BLE001 -- any collective error is the expected outcome
        status = "error: " + type(e).__name__
    with open(out_path, "w") as f:
        f.write(status)
    os._exit(0)
