"""Parity at the benchmark's full shapes against float64 oracle fixtures.

bench.py times configuration 2 (B=64, T=10,000, K=300, C=24), configuration 3
(B=1, T=10^6, K=1000, C=8), configuration 4 (B=32, T=4096, K=64, C=256) and
configuration 5's Viterbi batch (B=512, T=2048, K=32, C=16).  These tests run
the CUDA path on exactly those inputs (regenerated from their seeds; a stored
checksum proves they are the same tensors) and compare with the float64 oracle
fixtures of tests/golden/make_fullsize.py:

  * log Z / Viterbi score: |d| <= 1e-5 * |ref| + 1e-5
  * gradients, norm-wise: ||d||_inf <= 1e-5 * ||ref||_inf + 1e-6, applied to
    the stored grad_cum samples and row maxima, and 32x that to the stored
    sums (plain and absolute) over blocks of 32 positions
  * segmentations identical, or (at rounding-level near-ties) a decoded path
    whose float64 score equals the oracle optimum to 1e-6 relative.
"""

import numpy as np
import pytest
import torch

from conftest import load_golden
from inputs import checksum, config_lengths, make_streaming_inputs

pytestmark = pytest.mark.gpu

RTOL = 1e-5
BLK = 32


def _dev():
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    return torch.device("cuda:0")


def _inputs(g, gen):
    B, T, K, C = (int(g[k]) for k in ("B", "T", "K", "C"))
    inp = make_streaming_inputs(B, T, K, C, seed=int(g["seed"]), gen=gen)
    # the checksums are float64 sums over up to 10^7 elements, whose
    # parallel summation order differs between host CPUs by an ulp or two
    for key, name in (("cum_scores", "cum_checksum"), ("transition", "tr_checksum"),
                      ("duration_bias", "db_checksum")):
        if name in g:
            np.testing.assert_allclose(checksum(inp[key]), g[name], rtol=1e-12, atol=0)
    return inp, config_lengths(gen, B, T, seed=int(g["seed"]))


def assert_close_rel(got, ref, what):
    got = np.asarray(got, dtype=np.float64)
    ref = np.asarray(ref, dtype=np.float64)
    err = np.abs(got - ref)
    assert (err <= RTOL * np.abs(ref) + 1e-5).all(), f"{what}: max err {err.max():.3e}"


def assert_grad_close(got, ref, what):
    got = np.asarray(got, dtype=np.float64)
    ref = np.asarray(ref, dtype=np.float64)
    err = np.abs(got - ref).max()
    scale = np.abs(ref).max()
    assert err <= RTOL * scale + 1e-6, f"{what}: ||d||inf={err:.3e} ||ref||inf={scale:.3e}"


def assert_gc_signature(gc, g, what):
    """grad_cum (rows in fixture order) against the stored signature."""
    gc = np.asarray(gc, dtype=np.float64)
    B, T1, C = gc.shape
    scale = float(np.max(g["gc_inf"]))
    tol = RTOL * scale + 1e-6
    samp = gc.reshape(-1)[g["gc_samp_idx"]]
    err = np.abs(samp - g["gc_samp"]).max()
    assert err <= tol, f"{what} samples: {err:.3e} > {tol:.3e}"
    inf = np.abs(gc).reshape(B, -1).max(axis=1)
    assert np.abs(inf - g["gc_inf"]).max() <= tol, f"{what} row maxima"
    nb = (T1 + BLK - 1) // BLK
    pad = np.zeros((B, nb * BLK, C))
    pad[:, :T1] = gc
    blk = pad.reshape(B, nb, BLK, C)
    for name, got in (("gc_blk", blk.sum(axis=2)), ("gc_abs_blk", np.abs(blk).sum(axis=2))):
        err = np.abs(got - g[name]).max()
        assert err <= BLK * tol, f"{what} {name}: {err:.3e} > {BLK * tol:.3e}"


def _fwd_bwd(cum, tr, db, lengths, K):
    from torch_semimarkov_b200 import semi_crf_streaming_forward

    dev = _dev()
    c = cum.to(dev).requires_grad_(True)
    t = tr.to(dev).requires_grad_(True)
    d = db.to(dev).requires_grad_(True)
    part = semi_crf_streaming_forward(c, t, d, torch.as_tensor(lengths).to(dev), K)
    part.sum().backward()
    torch.cuda.synchronize()
    return (part.detach().cpu().numpy(), c.grad.cpu().numpy(), t.grad.cpu().numpy(),
            d.grad.cpu().numpy())


def _rows_case(name, gen, monkeypatch, mode):
    """Selected rows as their own batch: log Z and every gradient."""
    monkeypatch.setenv("TORCH_SEMIMARKOV_B200_BACKWARD", mode)
    g = load_golden(name)
    inp, _ = _inputs(g, gen)
    sel = torch.as_tensor(g["sel"])
    Tu = int(g["T_used"])
    part, gc, gt, gd = _fwd_bwd(inp["cum_scores"][sel, : Tu + 1].contiguous(),
                                inp["transition"], inp["duration_bias"], g["lengths"],
                                int(g["K"]))
    assert_close_rel(part, g["log_Z"], f"{name} log Z")
    assert_grad_close(gt, g["grad_transition"], f"{name} grad_transition")
    assert_grad_close(gd, g["grad_duration_bias"], f"{name} grad_duration_bias")
    assert_gc_signature(gc, g, f"{name} grad_cum")


@pytest.mark.parametrize("mode", ["keep", "recompute"])
def test_cfg2_full_rows_vs_oracle(mode, monkeypatch):
    """Four rows of the configuration-2 batch at full T = 10,000 (the longest,
    the shortest, rows 0 and 1) as a batch of their own: with the kept tables
    this runs the time-chunked chains (few sequences leave SMs idle); the
    recompute mode runs the checkpointed backward."""
    _rows_case("full_cfg2", "cfg2", monkeypatch, mode)


def test_cfg2_full_batch_vs_oracle(monkeypatch):
    """The whole configuration-2 batch that bench.py times (64 whole chains
    per direction): log Z and grad_cum of the fixture's rows."""
    monkeypatch.setenv("TORCH_SEMIMARKOV_B200_BACKWARD", "keep")
    g = load_golden("full_cfg2")
    inp, lengths = _inputs(g, "cfg2")
    np.testing.assert_array_equal(lengths.numpy()[g["sel"]], g["lengths"])
    part, gc, _, _ = _fwd_bwd(inp["cum_scores"], inp["transition"], inp["duration_bias"],
                              lengths, int(g["K"]))
    sel = g["sel"]
    assert_close_rel(part[sel], g["log_Z"], "cfg2 batch log Z")
    assert_gc_signature(gc[sel], g, "cfg2 batch grad_cum")


def test_cfg3_full_logz_vs_oracle():
    """Configuration 3's single sequence of 10^6 positions (time-chunked
    chains on one GPU): log Z against the oracle's full-length forward."""
    from torch_semimarkov_b200 import semi_crf_streaming_forward

    g = load_golden("full_cfg3")
    inp, _ = _inputs(g, "cfg3")
    dev = _dev()
    with torch.no_grad():
        part = semi_crf_streaming_forward(inp["cum_scores"].to(dev), inp["transition"].to(dev),
                                          inp["duration_bias"].to(dev),
                                          torch.as_tensor(g["lengths"]).to(dev), int(g["K"]))
    assert_close_rel(part.cpu().numpy(), g["log_Z"], "cfg3 log Z (T=1e6)")


def test_cfg3_grad_1e5_vs_oracle(monkeypatch):
    """Configuration 3's sequence cut to its first 10^5 positions: log Z and
    every gradient."""
    _rows_case("full_cfg3_grad", "cfg3", monkeypatch, "keep")


def test_cfg4_full_rows_vs_oracle(monkeypatch):
    """Two rows of configuration 4 (C=256, half the transitions masked to
    -1e4) at full T = 4096 as their own batch."""
    _rows_case("full_cfg4", "cfg4", monkeypatch, "keep")


def test_cfg4_full_batch_vs_oracle(monkeypatch):
    """The whole configuration-4 batch that bench.py times (32 sequences, two
    chains per cluster): log Z and grad_cum of the fixture's rows."""
    monkeypatch.setenv("TORCH_SEMIMARKOV_B200_BACKWARD", "keep")
    g = load_golden("full_cfg4")
    inp, lengths = _inputs(g, "cfg4")
    part, gc, _, _ = _fwd_bwd(inp["cum_scores"], inp["transition"], inp["duration_bias"],
                              lengths, int(g["K"]))
    sel = g["sel"]
    assert_close_rel(part[sel], g["log_Z"], "cfg4 batch log Z")
    assert_gc_signature(gc[sel], g, "cfg4 batch grad_cum")


def _unpack_segments(g):
    B, T = int(g["B"]), int(g["T"])
    ends = np.unpackbits(g["ends"], axis=1)[:, :T].astype(bool)
    lab = np.empty(2 * len(g["labels"]), dtype=np.int64)
    lab[0::2] = g["labels"] & 15
    lab[1::2] = g["labels"] >> 4
    out, pos = [], 0
    for b in range(B):
        e = np.nonzero(ends[b])[0]
        n = int(g["nseg"][b])
        assert len(e) == n
        s = np.concatenate([[0], e[:-1] + 1]) if n else np.zeros(0, dtype=np.int64)
        out.append(list(zip(s.tolist(), e.tolist(), lab[pos: pos + n].tolist())))
        pos += n
    return out


def _path_score64(cum, tr, db, K, segs):
    """float64 score of a segmentation under the Viterbi objective: content +
    duration bias + transition from the previous label (the first segment
    from the best virtual start label, max over c' of tr[c', c])."""
    total, prev = 0.0, None
    for (s, e, c) in segs:
        dur = e - s + 1
        total += float(cum[e + 1, c]) - float(cum[s, c]) + float(db[min(dur, K - 1), c])
        total += float(tr[:, c].max()) if prev is None else float(tr[prev, c])
        prev = c
    return total


def test_cfg5_full_viterbi_vs_oracle():
    """Configuration 5's whole Viterbi batch (B=512, lengths in [1024, 2048]):
    every score, and every segmentation identical to the oracle's except at
    rounding-level ties."""
    from torch_semimarkov_b200 import _lib

    g = load_golden("full_cfg5")
    inp, lengths = _inputs(g, "cfg5")
    np.testing.assert_array_equal(lengths.numpy(), g["lengths"])
    K = int(g["K"])
    dev = _dev()
    prob = _lib.Problem(inp["cum_scores"].to(dev), inp["transition"].to(dev),
                        inp["duration_bias"].to(dev), lengths.to(dev), K, "max")
    scores, ss, se, sl, sv, ns = _lib.viterbi(prob, 10000)
    torch.cuda.synchronize()
    assert_close_rel(scores.cpu().numpy(), g["scores"], "cfg5 Viterbi scores")
    ref = _unpack_segments(g)
    ss, se, sl, sv, ns = (x.cpu().numpy() for x in (ss, se, sl, sv, ns))
    cum = inp["cum_scores"].numpy().astype(np.float64)
    tr = inp["transition"].numpy().astype(np.float64)
    db = inp["duration_bias"].numpy().astype(np.float64)
    ties = 0
    for b in range(int(g["B"])):
        n = int(ns[b])
        got = list(zip(ss[b, :n].tolist(), se[b, :n].tolist(), sl[b, :n].tolist()))
        assert got[0][0] == 0 and got[-1][1] == int(lengths[b]) - 1, b
        assert all(got[i][0] == got[i - 1][1] + 1 for i in range(1, n)), b
        assert abs(float(sv[b, :n].sum()) - float(g["seg_score_sum"][b])) <= \
            1e-5 * abs(float(g["seg_score_sum"][b])) + 1e-3, b
        if got != ref[b]:
            ties += 1
            best = float(g["scores"][b])
            mine = _path_score64(cum[b], tr, db, K, got)
            assert abs(mine - best) <= 1e-6 * abs(best), \
                f"sequence {b}: decoded path scores {mine!r}, optimum {best!r}"
    assert ties <= 8, f"{ties} of 512 segmentations differ (all at near-ties)"
