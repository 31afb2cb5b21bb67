"""Pin the CPU oracle against golden vectors produced by the reference itself.

tests/golden/*.npz were written by tests/golden/make_golden.py, which runs the
reference package (torch-semimarkov 0.2.0, CPU PyTorch path) on seeded inputs.
These tests run the oracle (oracle/semicrf_oracle.c, float64) on the same
inputs and require agreement to float64 round-off.
"""

import numpy as np
import pytest

from conftest import golden_names, load_golden, streaming_inputs_from_golden

STREAM = golden_names("stream_") + golden_names("cfg")
HEAD = golden_names("head_")
GOLD = golden_names("gold_")


def _np(t):
    return None if t is None else t.numpy()


@pytest.mark.parametrize("name", STREAM)
def test_oracle_streaming_matches_reference(name, oracle):
    g = load_golden(name)
    inp = streaming_inputs_from_golden(g)
    K = int(g["K"])
    semiring = str(g["semiring"])
    ckpt = int(g["ckpt_arg"])
    cum, tr, db = _np(inp["cum_scores"]), _np(inp["transition"]), _np(inp["duration_bias"])
    ps, pe = _np(inp["proj_start"]), _np(inp["proj_end"])
    part, ck, S = oracle.forward(cum, tr, db, g["lengths"], K, semiring, ps, pe,
                                 checkpoint_interval_=None if ckpt < 0 else ckpt, threads=4)
    assert S == int(g["checkpoint_interval"])
    np.testing.assert_allclose(part, g["partition_lowlevel"], rtol=1e-12, atol=1e-9)
    if "ring_checkpoints" in g:
        np.testing.assert_allclose(ck, g["ring_checkpoints"], rtol=1e-12, atol=1e-9)
    else:
        np.testing.assert_allclose(ck.sum(), g["ring_checkpoints_checksum"], rtol=1e-12)
    # Public entry point (default interval) forward + backward with grad_output.
    part2, grads = oracle.forward_backward(cum, tr, db, g["lengths"], K, g["grad_output"],
                                           semiring, ps, pe, threads=4)
    np.testing.assert_allclose(part2, g["partition"], rtol=1e-12, atol=1e-9)
    if "grad_cum_scores" in g:
        np.testing.assert_allclose(grads["cum_scores"], g["grad_cum_scores"], rtol=1e-9, atol=1e-11)
    else:
        gc = grads["cum_scores"]
        np.testing.assert_allclose(gc[:, :64], g["grad_cum_head"], rtol=1e-9, atol=1e-11)
        np.testing.assert_allclose([gc.sum(), np.abs(gc).sum()], g["grad_cum_checksum"],
                                   rtol=1e-9, atol=1e-9)
    np.testing.assert_allclose(grads["transition"], g["grad_transition"], rtol=1e-9, atol=1e-11)
    np.testing.assert_allclose(grads["duration_bias"], g["grad_duration_bias"], rtol=1e-9,
                               atol=1e-11)
    for key in ("proj_start", "proj_end"):
        if "grad_" + key in g:
            np.testing.assert_allclose(grads[key], g["grad_" + key], rtol=1e-9, atol=1e-11)


@pytest.mark.parametrize("name", HEAD)
def test_oracle_viterbi_matches_reference(name, oracle):
    import torch

    from inputs import checksum, make_hidden

    g = load_golden(name)
    B, T, K, C = int(g["B"]), int(g["T"]), int(g["K"]), int(g["C"])
    hd = int(g["hidden_dim"])
    p = make_hidden(B, T, C, K, int(g["seed"]), str(g["gen"]), None if hd < 0 else hd)
    np.testing.assert_allclose(checksum(p["hidden"]), g["hidden_checksum"], rtol=0, atol=0)
    hidden = p["hidden"]
    if hd > 0:
        scores = hidden @ p["proj_weight"].T + p["proj_bias"]
    else:
        scores = hidden
    cum = torch.zeros(B, T + 1, C)
    cum[:, 1:] = torch.cumsum(scores.float(), dim=1)
    # The reference traceback keeps alpha in float32 (nn.py:464); the float32
    # oracle replays the same additions in the same order and must match it
    # exactly.
    lengths = g["lengths"]
    sc32, segs32 = oracle.viterbi(cum.numpy(), g["transition"], g["duration_bias"], lengths, K,
                                  int(g["max_traceback_length"]), dtype=np.float32)
    np.testing.assert_allclose(sc32[lengths > 0], g["viterbi_scores"][lengths > 0],
                               rtol=2e-6, atol=2e-4)
    for b in range(B):
        n = int(g["nseg"][b])
        assert len(segs32[b]) == n, (b, len(segs32[b]), n)
        got = np.array([s[:3] for s in segs32[b]], dtype=np.int64).reshape(n, 3)
        np.testing.assert_array_equal(got, g["segments"][b, :n])
        gsc = np.array([s[3] for s in segs32[b]])
        np.testing.assert_allclose(gsc, g["segment_scores"][b, :n], rtol=1e-6, atol=1e-5)
    # The float64 oracle may break rounding-level near-ties differently; the
    # reference's segmentation must then still be optimal to 1e-6 relative.
    sc64, segs64 = oracle.viterbi(cum.numpy(), g["transition"], g["duration_bias"], lengths, K,
                                  int(g["max_traceback_length"]))
    np.testing.assert_allclose(sc64[lengths > 0], g["viterbi_scores"][lengths > 0],
                               rtol=2e-6, atol=2e-4)
    cum64 = cum.numpy().astype(np.float64)
    tr64 = g["transition"].astype(np.float64)
    db64 = g["duration_bias"].astype(np.float64)
    for b in range(B):
        n = int(g["nseg"][b])
        ref = [tuple(x) for x in g["segments"][b, :n]]
        if [s[:3] for s in segs64[b]] == ref or n == 0:
            continue
        tot, prev = 0.0, None
        for (st, en, c) in ref:
            d = min(en - st + 1, K - 1)
            tot += cum64[b, en + 1, c] - cum64[b, st, c] + db64[d, c]
            # first segment: transition from the best virtual start label
            tot += tr64[prev, c] if prev is not None else tr64[:, c].max()
            prev = c
        assert abs(tot - sc64[b]) <= 1e-6 * abs(sc64[b]) + 1e-6, (b, tot, sc64[b])


@pytest.mark.parametrize("name", GOLD)
def test_oracle_gold_score_matches_reference(name, oracle):
    g = load_golden(name)
    out = oracle.score_gold(g["cum_scores"], g["labels"], g["lengths"], g["transition"],
                            g["duration_bias"], int(g["K"]))
    np.testing.assert_allclose(out, g["gold_score"], rtol=1e-12, atol=1e-12)


def test_oracle_checkpoint_interval(oracle):
    assert oracle.checkpoint_interval(10000, 300) == 1732
    assert oracle.checkpoint_interval(1000000, 1000) == 31622
    assert oracle.checkpoint_interval(4096, 64) == 512
    assert oracle.checkpoint_interval(2048, 32) == 256
    assert oracle.checkpoint_interval(10, 50) == 50
