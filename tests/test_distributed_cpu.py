"""Multi-rank host logic on CPU (gloo, world size 2): batch sharding and the
one all-reduce of the shared gradients, against the single-process result."""

import json
import multiprocessing as mp
import os
import socket

import numpy as np
import pytest

import dist_workers
from torch_semimarkov_b200.distributed import shard_sequences


def _port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_shard_sequences_partition_and_balance():
    lengths = [10000, 9000, 8000, 8000, 100, 5000, 7000, 6000, 0]
    for world in (1, 2, 3, 4):
        shards = [shard_sequences(lengths, world, r).tolist() for r in range(world)]
        flat = sorted(i for s in shards for i in s)
        assert flat == list(range(len(lengths)))
        loads = [sum(lengths[i] for i in s) for s in shards]
        # LPT: no rank exceeds the lightest by more than the longest sequence
        assert max(loads) - min(loads) <= max(lengths)
    assert shard_sequences(lengths, 2, 0).tolist() == shard_sequences(lengths, 2, 0).tolist()
    with pytest.raises(ValueError):
        shard_sequences(lengths, 2, 2)


def _run(target, args_of_rank, world=2, timeout=120):
    ctx = mp.get_context("spawn")
    procs = [ctx.Process(target=target, args=args_of_rank(r)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout)
    for p in procs:
        if p.is_alive():
            p.kill()
            p.join()
    return [p.exitcode for p in procs]


def test_two_rank_step_matches_single_process(tmp_path, oracle):
    from inputs import make_streaming_inputs

    case = (6, 40, 7, 5, 11)
    port = _port()
    outs = [str(tmp_path / f"r{r}.json") for r in range(2)]
    codes = _run(dist_workers.step_worker, lambda r: (r, 2, port, case, outs[r]))
    assert codes == [0, 0]
    res = [json.load(open(o)) for o in outs]
    B, T, K, C, seed = case
    inp = make_streaming_inputs(B, T, K, C, seed=seed)
    lengths = np.array([T, T - 3, T // 2, T - 1, 5, T - 7][:B])
    part, grads = oracle.forward_backward(inp["cum_scores"].numpy(), inp["transition"].numpy(),
                                          inp["duration_bias"].numpy(), lengths, K)
    assert sorted(res[0]["mine"] + res[1]["mine"]) == list(range(B))
    for r in res:  # every rank holds the same reduced values
        np.testing.assert_allclose(r["gt"], grads["transition"], rtol=1e-5, atol=1e-6)
        np.testing.assert_allclose(r["gd"], grads["duration_bias"], rtol=1e-5, atol=1e-6)
        assert abs(r["loss"] - float(part.sum())) <= 1e-5 * abs(float(part.sum()))


def test_failed_rank_surfaces_as_error_not_hang(tmp_path):
    port = _port()
    out = str(tmp_path / "r0.txt")
    codes = _run(dist_workers.failing_worker, lambda r: (r, 2, port, out), timeout=90)
    assert codes[1] == 3
    assert codes[0] == 0, "rank 0 hung or crashed instead of reporting the failure"
    assert open(out).read().startswith("error"), open(out).read()
