"""CUDA path vs the reference (golden fixtures) and the CPU oracle.

Tolerances (north star: 1e-5 relative against a float64 reference run):
  * partition / Viterbi score: |d| <= 1e-5 * |ref| + 1e-5
  * gradients: norm-wise, ||d||_inf <= 1e-5 * ||ref||_inf + 1e-6 (per-element
    relative error is ill-posed for near-zero marginals)
  * segmentations: identical, or -- at rounding-level near-ties -- a path whose
    float64 score equals the float64 optimum to 1e-6 relative.
"""

import numpy as np
import pytest
import torch

from conftest import golden_names, load_golden, streaming_inputs_from_golden

pytestmark = pytest.mark.gpu

RTOL = 1e-5


def _dev():
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    return torch.device("cuda:0")


def assert_close_rel(got, ref, rtol=RTOL, atol=1e-5, what=""):
    got = np.asarray(got, dtype=np.float64)
    ref = np.asarray(ref, dtype=np.float64)
    err = np.abs(got - ref)
    bound = rtol * np.abs(ref) + atol
    bad = err > bound
    assert not bad.any(), f"{what}: max err {err.max():.3e} at {np.argwhere(bad)[:3].tolist()}"


def assert_grad_close(got, ref, rtol=RTOL, floor=1e-6, what=""):
    got = np.asarray(got, dtype=np.float64)
    ref = np.asarray(ref, dtype=np.float64)
    scale = max(np.abs(ref).max(), 0.0)
    err = np.abs(got - ref).max() if got.size else 0.0
    assert err <= rtol * scale + floor, f"{what}: ||d||inf={err:.3e} ||ref||inf={scale:.3e}"


STREAM = golden_names("stream_") + golden_names("cfg")


@pytest.mark.parametrize("name", STREAM)
def test_streaming_forward_backward_vs_reference(name):
    from torch_semimarkov_b200 import semi_crf_streaming_forward

    dev = _dev()
    g = load_golden(name)
    inp = streaming_inputs_from_golden(g)
    K = int(g["K"])
    semiring = str(g["semiring"])
    leaves = {k: (None if v is None else v.to(dev).requires_grad_(True)) for k, v in inp.items()}
    lengths = torch.as_tensor(g["lengths"]).to(dev)
    part = semi_crf_streaming_forward(leaves["cum_scores"], leaves["transition"],
                                      leaves["duration_bias"], lengths, K, semiring=semiring,
                                      proj_start=leaves["proj_start"],
                                      proj_end=leaves["proj_end"])
    part.backward(torch.as_tensor(g["grad_output"], dtype=torch.float32, device=dev))
    torch.cuda.synchronize()
    assert_close_rel(part.detach().cpu().numpy(), g["partition"], what="partition")
    gc = leaves["cum_scores"].grad.cpu().numpy()
    if "grad_cum_scores" in g:
        assert_grad_close(gc, g["grad_cum_scores"], what="grad_cum")
    else:
        assert_grad_close(gc[:, :64], g["grad_cum_head"], what="grad_cum head")
        np.testing.assert_allclose([gc.sum(), np.abs(gc).sum()], g["grad_cum_checksum"],
                                   rtol=1e-4, atol=1e-3)
    assert_grad_close(leaves["transition"].grad.cpu().numpy(), g["grad_transition"],
                      what="grad_transition")
    assert_grad_close(leaves["duration_bias"].grad.cpu().numpy(), g["grad_duration_bias"],
                      what="grad_duration_bias")
    for key in ("proj_start", "proj_end"):
        if "grad_" + key in g:
            assert_grad_close(leaves[key].grad.cpu().numpy(), g["grad_" + key], what=key)


@pytest.mark.parametrize("name", ["stream_basic", "stream_ckpt_div", "stream_zero_len",
                                  "stream_k1", "stream_c24", "stream_basic_max", "stream_kcc",
                                  "stream_kcc_max"])
def test_ring_checkpoints_layout_and_values(name):
    from torch_semimarkov_b200 import launch_streaming_triton_kernel

    dev = _dev()
    g = load_golden(name)
    inp = streaming_inputs_from_golden(g)
    K, T = int(g["K"]), int(g["T"])
    part, ck, S = launch_streaming_triton_kernel(
        inp["cum_scores"].to(dev), inp["transition"].to(dev), inp["duration_bias"].to(dev),
        torch.as_tensor(g["lengths"]).to(dev), K, semiring=str(g["semiring"]))
    assert S == int(g["checkpoint_interval"])
    assert ck.shape == ((g["B"]), (T + S - 1) // S + 1, K, int(g["C"]))
    ref = g["ring_checkpoints"]  # reference PyTorch layout: ceil(T/S) checkpoints
    got = ck[:, : ref.shape[1]].cpu().numpy()
    unset = ref <= -1e8
    np.testing.assert_array_equal(got[unset], np.float32(-1e9))
    assert_close_rel(got[~unset], ref[~unset], what="checkpoints")
    assert torch.all(ck[:, 0, 0] == 0)


@pytest.mark.parametrize("C", [6, 96])
def test_ring_checkpoints_large_scale_vs_oracle(C, oracle):
    """The reference launcher's ring checkpoints come from the generic chain;
    with emissions N(0, 60^2) its factors clip and the rerun in the log domain
    rewrites log Z and the checkpoint rows, which must match the float64 oracle."""
    from torch_semimarkov_b200 import launch_streaming_triton_kernel

    dev = _dev()
    B, T, K = 2, 160, 20
    g = torch.Generator().manual_seed(13)
    em = torch.randn(B, T, C, generator=g, dtype=torch.float64) * 60.0
    cum = torch.cat([torch.zeros(B, 1, C, dtype=torch.float64), em.cumsum(1)], 1).float()
    tr = (torch.randn(C, C, generator=g, dtype=torch.float64) * 0.1).float()
    db = (torch.randn(K, C, generator=g, dtype=torch.float64) * 0.1).float()
    lengths = np.array([T, T - 37])
    part_ref, ck_ref, S_ref = oracle.forward(cum.numpy(), tr.numpy(), db.numpy(), lengths, K)
    part, ck, S = launch_streaming_triton_kernel(cum.to(dev), tr.to(dev), db.to(dev),
                                                 torch.as_tensor(lengths).to(dev), K)
    assert S == S_ref
    assert_close_rel(part.cpu().numpy(), part_ref, what="partition")
    got = ck[:, : ck_ref.shape[1]].cpu().numpy()
    unset = ck_ref <= -1e8
    np.testing.assert_array_equal(got[unset], np.float32(-1e9))
    assert_close_rel(got[~unset], ck_ref[~unset], what="checkpoints")


HEAD = golden_names("head_")


@pytest.mark.parametrize("name", HEAD)
def test_head_decode_and_loss_vs_reference(name, oracle):
    from inputs import make_hidden

    from torch_semimarkov_b200 import SemiMarkovCRFHead

    dev = _dev()
    g = load_golden(name)
    B, T, K, C = int(g["B"]), int(g["T"]), int(g["K"]), int(g["C"])
    hd = int(g["hidden_dim"])
    p = make_hidden(B, T, C, K, int(g["seed"]), str(g["gen"]), None if hd < 0 else hd)
    crf = SemiMarkovCRFHead(num_classes=C, max_duration=K, hidden_dim=None if hd < 0 else hd)
    with torch.no_grad():
        crf.transition.copy_(p["transition"])
        crf.duration_dist.duration_bias.copy_(p["duration_bias"])
        if hd > 0:
            crf.projection.weight.copy_(p["proj_weight"])
            crf.projection.bias.copy_(p["proj_bias"])
    crf = crf.to(dev)
    hidden = p["hidden"].to(dev)
    lengths = torch.as_tensor(g["lengths"]).to(dev)
    labels = p["labels"].to(dev)

    res = crf(hidden, lengths)
    # float64 oracle on the same float32 cum_scores: the tight (1e-5) check
    cum_np = res["cum_scores"].detach().cpu().numpy()
    part_ref, gr = oracle.forward_backward(cum_np, g["transition"], g["duration_bias"],
                                           g["lengths"], K, threads=8)
    assert_close_rel(res["partition"].detach().cpu().numpy(), part_ref, what="partition")
    # the fixture was produced by the reference module in float32: compare loosely
    assert_close_rel(res["partition"].detach().cpu().numpy(), g["partition"], rtol=2e-4,
                     atol=1e-2, what="partition vs float32 reference")
    loss = crf.compute_loss(hidden, lengths, labels, reduction="sum")
    loss.backward()
    gold = oracle.score_gold(cum_np, g["labels"], g["lengths"], g["transition"],
                             g["duration_bias"], K)
    lv = float(loss.detach())
    assert abs(lv - float((part_ref - gold).sum())) <= 1e-5 * abs(lv) + 1e-3
    assert abs(lv - float(g["loss_sum"])) <= 2e-4 * abs(float(g["loss_sum"])) + 1e-2
    # d loss / d transition = d partition / d transition - gold transition counts
    lab, Ls = g["labels"], g["lengths"]
    gt_gold = np.zeros((C, C))
    gd_gold = np.zeros((K, C))
    for b in range(B):
        st, prev = 0, None
        for pos in range(Ls[b]):
            if pos == Ls[b] - 1 or lab[b, pos] != lab[b, pos + 1]:
                cl = lab[b, st]
                gd_gold[min(max(pos - st + 1, 1), K - 1), cl] += 1
                if prev is not None:
                    gt_gold[prev, cl] += 1
                prev, st = cl, pos + 1
    assert_grad_close(crf.transition.grad.cpu().numpy(), gr["transition"] - gt_gold,
                      what="grad_transition")
    assert_grad_close(crf.duration_dist.duration_bias.grad.cpu().numpy(),
                      gr["duration_bias"] - gd_gold, what="grad_duration_bias")
    assert_grad_close(crf.transition.grad.cpu().numpy(), g["grad_transition"], rtol=2e-3,
                      floor=1e-3, what="grad_transition vs float32 reference")
    if hd > 0:
        assert_grad_close(crf.projection.weight.grad.cpu().numpy(), g["grad_proj_weight"],
                          rtol=2e-3, floor=1e-3, what="grad_proj_weight vs float32 reference")

    with torch.no_grad():
        sc = crf.decode(hidden, lengths)
        vr = crf.decode_with_traceback(hidden, lengths,
                                       max_traceback_length=int(g["max_traceback_length"]))
    L = g["lengths"]
    assert_close_rel(sc.cpu().numpy()[L > 0], g["decode_scores"][L > 0], what="decode")
    assert_close_rel(vr.scores.cpu().numpy()[L > 0], g["viterbi_scores"][L > 0], what="viterbi")
    # float64 optimum of the same float32 cum_scores for near-tie arbitration
    cum = crf._cum_scores(hidden).detach().cpu().numpy()
    sc64, _ = oracle.viterbi(cum, g["transition"], g["duration_bias"], L, K, 0)
    cum64 = cum.astype(np.float64)
    tr64 = g["transition"].astype(np.float64)
    db64 = g["duration_bias"].astype(np.float64)
    for b in range(B):
        n = int(g["nseg"][b])
        got = [(s.start, s.end, s.label) for s in vr.segments[b]]
        ref = [tuple(int(v) for v in x) for x in g["segments"][b, :n]]
        if got == ref:
            np.testing.assert_allclose([s.score for s in vr.segments[b]],
                                       g["segment_scores"][b, :n], rtol=1e-6, atol=1e-5)
            continue
        assert len(got) > 0 and got[0][0] == 0 and got[-1][1] == L[b] - 1
        tot, prev = 0.0, None
        for (st, en, c) in got:
            assert en >= st
            d = min(en - st + 1, K - 1)
            tot += cum64[b, en + 1, c] - cum64[b, st, c] + db64[d, c]
            tot += tr64[prev, c] if prev is not None else tr64[:, c].max()
            prev = c
        assert abs(tot - sc64[b]) <= 1e-6 * abs(sc64[b]) + 1e-5, (name, b, tot, sc64[b])


@pytest.mark.parametrize("name", golden_names("gold_"))
def test_gold_score_vs_reference(name):
    from torch_semimarkov_b200 import score_gold_vectorized

    dev = _dev()
    g = load_golden(name)
    cum = torch.as_tensor(g["cum_scores"]).float().to(dev).requires_grad_(True)
    tr = torch.as_tensor(g["transition"]).float().to(dev).requires_grad_(True)
    db = torch.as_tensor(g["duration_bias"]).float().to(dev).requires_grad_(True)
    labels = torch.as_tensor(g["labels"]).to(dev)
    lengths = torch.as_tensor(g["lengths"]).to(dev)
    K = int(g["K"])
    out = score_gold_vectorized(cum, labels, lengths, tr, db, K)
    assert_close_rel(out.detach().cpu().numpy(), g["gold_score"], rtol=1e-5, atol=1e-4,
                     what="gold")
    w = torch.linspace(0.5, 1.5, out.shape[0], device=dev)
    (out * w).sum().backward()
    # expected gradients: +-w at segment boundaries, transition / duration counts
    lab, L, T = g["labels"], g["lengths"], int(g["T"])
    C = int(g["C"])
    gc = np.zeros((len(L), T + 1, C))
    gt = np.zeros((C, C))
    gd = np.zeros((K, C))
    for b in range(len(L)):
        wb = float(w[b])
        if T == 1:
            if L[b] > 0:
                gc[b, 1, lab[b, 0]] += wb
                gc[b, 0, lab[b, 0]] -= wb
                gd[1, lab[b, 0]] += wb
            continue
        st, prev = 0, None
        for p in range(L[b]):
            if p == L[b] - 1 or lab[b, p] != lab[b, p + 1]:
                c = lab[b, st]
                gc[b, p + 1, c] += wb
                gc[b, st, c] -= wb
                gd[min(max(p - st + 1, 1), K - 1), c] += wb
                if prev is not None:
                    gt[prev, c] += wb
                prev, st = c, p + 1
    np.testing.assert_allclose(cum.grad.cpu().numpy(), gc, atol=1e-6)
    np.testing.assert_allclose(tr.grad.cpu().numpy(), gt, atol=1e-5)
    np.testing.assert_allclose(db.grad.cpu().numpy(), gd, atol=1e-5)


# ---------------------------------------------------------------------------
# seeded random cases against the float64 oracle (sizes it finishes in seconds)
# ---------------------------------------------------------------------------

ORACLE_CASES = [
    # B, T, K, C, gen, proj, semiring
    (4, 257, 17, 5, "default", None, "log"),
    (3, 300, 40, 24, "cfg2", None, "log"),
    (2, 400, 64, 8, "cfg3", "both", "log"),
    (2, 97, 13, 33, "default", "start", "log"),
    (2, 150, 10, 64, "default", None, "log"),
    (2, 60, 9, 130, "default", "end", "log"),
    (3, 180, 25, 16, "cfg5", None, "max"),
    (2, 120, 1, 6, "default", None, "log"),
    (2, 90, 2, 7, "default", None, "max"),
    # large label sets (the cluster chain), odd batches, and enough chains for
    # two per cluster
    (2, 100, 20, 200, "default", "both", "log"),
    (3, 70, 5, 65, "cfg2", None, "log"),
    (20, 48, 6, 70, "default", "both", "log"),
    (21, 40, 9, 96, "cfg2", None, "log"),
]


@pytest.mark.parametrize("case", ORACLE_CASES)
def test_random_vs_oracle(case, oracle):
    _random_vs_oracle(case, oracle)


@pytest.mark.parametrize("case", [ORACLE_CASES[1], ORACLE_CASES[2], ORACLE_CASES[5],
                                  ORACLE_CASES[6], ORACLE_CASES[7]])
def test_random_vs_oracle_recompute(case, oracle, monkeypatch):
    """The memory-light layout: ring checkpoints saved, alpha recomputed."""
    monkeypatch.setenv("TORCH_SEMIMARKOV_B200_BACKWARD", "recompute")
    _random_vs_oracle(case, oracle)


# (K, C, C) transitions (kcc.cu): both semirings, projections, K > T, C = 1,
# C > 32 (several row tiles of the transition marginals), factors resident in
# shared memory, streamed through it in chunks (K*C*C large), and read
# directly from L2 (C = 130)
KCC_CASES = [
    (3, 60, 6, 5, "default", None, "log"),
    (2, 80, 12, 24, "cfg2", "both", "log"),
    (2, 50, 5, 40, "default", "start", "log"),
    (2, 40, 4, 100, "default", None, "log"),
    (3, 70, 9, 7, "cfg5", "end", "max"),
    (2, 30, 40, 3, "default", None, "log"),
    (2, 50, 2, 1, "default", None, "log"),
    (2, 300, 64, 16, "default", None, "log"),
    (2, 64, 33, 9, "default", "both", "max"),
    (2, 30, 3, 130, "default", None, "log"),
    (2, 150, 120, 20, "cfg2", None, "log"),
    (2, 90, 70, 24, "default", None, "max"),
    # many 16-position blocks with ragged lengths, and N(0,1) emissions that
    # move the per-label frames between blocks
    (3, 400, 40, 6, "cfg2", "both", "log"),
    (2, 500, 50, 8, "cfg5", None, "log"),
    (2, 200, 17, 33, "cfg5", "end", "log"),
    # batches whose forward (two chains per sequence) runs the blocked chain on
    # clusters of 4, 2 and 1 CTAs per chain (small batches use 8)
    (12, 120, 30, 6, "cfg2", None, "log"),
    (20, 80, 20, 4, "default", "both", "log"),
    (40, 50, 6, 5, "default", None, "log"),
    # the max-plus chain with one CTA per chain, and with C > 32 (weights not in registers)
    (40, 50, 6, 5, "default", "both", "max"),
    (2, 60, 9, 40, "cfg5", None, "max"),
    # more labels than the blocked kernels take: the per-position gather chain
    (2, 30, 3, 130, "default", "both", "max"),
]


@pytest.mark.parametrize("case", KCC_CASES)
def test_kcc_transitions_vs_oracle(case, oracle):
    _random_vs_oracle(case, oracle, kcc=True)


def _random_vs_oracle(case, oracle, kcc=False):
    from inputs import make_streaming_inputs

    from torch_semimarkov_b200 import semi_crf_streaming_forward

    B, T, K, C, gen, proj, semiring = case
    inp = make_streaming_inputs(B, T, K, C, seed=100 + T + K + C, gen=gen, proj=proj, kcc=kcc)
    rng = np.random.default_rng(T)
    lengths = np.concatenate([[T], rng.integers(max(1, T // 3), T + 1, size=B - 1)])
    gout = rng.uniform(0.5, 1.5, size=B)
    _check_vs_oracle(inp, lengths, gout, K, semiring, oracle)


def _check_vs_oracle(inp, lengths, gout, K, semiring, oracle):
    """Forward + backward through semi_crf_streaming_forward vs the float64 oracle."""
    from torch_semimarkov_b200 import semi_crf_streaming_forward

    dev = _dev()
    np_in = {k: (None if v is None else v.numpy()) for k, v in inp.items()}
    part_ref, grads_ref = oracle.forward_backward(
        np_in["cum_scores"], np_in["transition"], np_in["duration_bias"], lengths, K, gout,
        semiring, np_in["proj_start"], np_in["proj_end"], threads=8)
    leaves = {k: (None if v is None else v.to(dev).requires_grad_(True)) for k, v in inp.items()}
    part = semi_crf_streaming_forward(leaves["cum_scores"], leaves["transition"],
                                      leaves["duration_bias"], torch.as_tensor(lengths).to(dev),
                                      K, semiring=semiring, proj_start=leaves["proj_start"],
                                      proj_end=leaves["proj_end"])
    part.backward(torch.as_tensor(gout, dtype=torch.float32, device=dev))
    assert_close_rel(part.detach().cpu().numpy(), part_ref, what="partition")
    assert_grad_close(leaves["cum_scores"].grad.cpu().numpy(), grads_ref["cum_scores"],
                      what="grad_cum")
    assert_grad_close(leaves["transition"].grad.cpu().numpy(), grads_ref["transition"],
                      what="grad_tr")
    assert_grad_close(leaves["duration_bias"].grad.cpu().numpy(), grads_ref["duration_bias"],
                      what="grad_db")
    for key in ("proj_start", "proj_end"):
        if leaves[key] is not None:
            assert_grad_close(leaves[key].grad.cpu().numpy(), grads_ref[key], what=key)


def test_decode_batch_vs_oracle(oracle):
    """Config-5-shaped Viterbi batch (ragged lengths) against the float64 oracle."""
    from inputs import make_streaming_inputs

    from torch_semimarkov_b200 import _lib

    dev = _dev()
    B, T, K, C = 16, 512, 32, 16
    inp = make_streaming_inputs(B, T, K, C, seed=55, gen="cfg5")
    lengths = np.random.default_rng(5).integers(T // 2, T + 1, size=B)
    prob = _lib.Problem(inp["cum_scores"].to(dev), inp["transition"].to(dev),
                        inp["duration_bias"].to(dev), torch.as_tensor(lengths).to(dev), K, "max")
    scores, ss, se, sl, sv, ns = _lib.viterbi(prob, 10000)
    sc64, segs64 = oracle.viterbi(inp["cum_scores"].numpy(), inp["transition"].numpy(),
                                  inp["duration_bias"].numpy(), lengths, K, 10000, threads=8)
    assert_close_rel(scores.cpu().numpy(), sc64, what="viterbi score")
    ns = ns.cpu().numpy()
    same = 0
    for b in range(B):
        got = list(zip(ss[b, : ns[b]].tolist(), se[b, : ns[b]].tolist(), sl[b, : ns[b]].tolist()))
        ref = [s[:3] for s in segs64[b]]
        same += got == ref
        # coverage and score of the decoded path
        assert got[0][0] == 0 and got[-1][1] == lengths[b] - 1
        assert all(got[i][0] == got[i - 1][1] + 1 for i in range(1, len(got)))
        seg_sum = float(sv[b, : ns[b]].sum())
        assert abs(seg_sum - sc64[b]) <= 1e-5 * abs(sc64[b]) + 1e-3
    assert same >= B - 1, f"only {same}/{B} segmentations identical"


# score-only max-semiring forward (no autograd): the warp chain for C <= 32 and
# K-1 <= 64, the block chain otherwise
MAX_FWD_CASES = [
    # B, T, K, C, gen, proj
    (4, 300, 33, 16, "cfg5", None),
    (3, 200, 9, 5, "default", "both"),
    (2, 100, 1, 3, "default", None),
    (2, 150, 65, 32, "default", None),
    (3, 120, 100, 24, "default", None),
    (2, 90, 12, 40, "default", None),
]


@pytest.mark.parametrize("case", MAX_FWD_CASES)
def test_max_forward_no_grad_vs_oracle(case, oracle):
    from inputs import make_streaming_inputs

    from torch_semimarkov_b200 import semi_crf_streaming_forward

    B, T, K, C, gen, proj = case
    dev = _dev()
    inp = make_streaming_inputs(B, T, K, C, seed=7 + T + K + C, gen=gen, proj=proj)
    rng = np.random.default_rng(K)
    lengths = np.concatenate([[T], rng.integers(0, T + 1, size=B - 1)])
    np_in = {k: (None if v is None else v.numpy()) for k, v in inp.items()}
    ref, _, _ = oracle.forward(np_in["cum_scores"], np_in["transition"], np_in["duration_bias"],
                               lengths, K, "max", np_in["proj_start"], np_in["proj_end"],
                               threads=4)
    with torch.no_grad():
        got = semi_crf_streaming_forward(
            inp["cum_scores"].to(dev), inp["transition"].to(dev), inp["duration_bias"].to(dev),
            torch.as_tensor(lengths).to(dev), K, semiring="max",
            proj_start=None if inp["proj_start"] is None else inp["proj_start"].to(dev),
            proj_end=None if inp["proj_end"] is None else inp["proj_end"].to(dev))
    assert_close_rel(got.cpu().numpy(), ref, what="max score")


# time-chunked chains (keep mode, batches that leave SMs idle): chunks start
# early from a guessed state and are joined after a projective check; a short
# forced warm-up exercises the serial rerun of sequences that do not join, and
# a short one with a longer second warm-up the rerun of their chunks
CHUNK_CASES = [
    # B, T, K, C, gen, proj, env
    (1, 5000, 20, 8, "cfg3", None, "auto"),
    (2, 4000, 33, 24, "cfg2", "both", "auto"),
    (1, 3000, 20, 8, "default", None, "8"),
    (2, 3000, 20, 8, "default", None, "8,64"),
    (1, 12000, 1000, 8, "cfg3", None, "auto"),
]


@pytest.mark.parametrize("case", CHUNK_CASES)
def test_chunked_chains_vs_oracle(case, oracle, monkeypatch):
    B, T, K, C, gen, proj, env = case
    monkeypatch.setenv("TORCH_SEMIMARKOV_B200_CHUNKS", env)
    monkeypatch.setenv("TORCH_SEMIMARKOV_B200_BACKWARD", "keep")
    from torch_semimarkov_b200 import _lib

    lib = _lib.load()
    dev = _dev()
    from inputs import make_streaming_inputs

    inp = make_streaming_inputs(B, T, K, C, seed=31 + T, gen=gen, proj=proj)
    prob = _lib.Problem(inp["cum_scores"].to(dev), inp["transition"].to(dev),
                        inp["duration_bias"].to(dev), torch.full((B,), T).to(dev), K, "log",
                        None if inp["proj_start"] is None else inp["proj_start"].to(dev),
                        None if inp["proj_end"] is None else inp["proj_end"].to(dev))
    # the plan really chunks (the saved state then carries the hand-off buffers)
    prob_off = _lib.SemicrfProblem.from_buffer_copy(prob.c)
    prob_off.chunk_warmup = -1
    import ctypes

    assert lib.semicrf_saved_size(prob.cref) > lib.semicrf_saved_size(ctypes.byref(prob_off))
    gout = np.random.default_rng(T).uniform(0.5, 1.5, size=B)
    _check_vs_oracle(inp, np.full(B, T), gout, K, "log", oracle)


@pytest.mark.parametrize("scale,kcc,semiring", [(12.0, False, "log"), (20.0, False, "log"),
                                                (60.0, False, "log"),
                                                (12.0, True, "log"), (20.0, True, "log"),
                                                (60.0, True, "max")])
def test_large_emission_scale_vs_oracle(scale, kcc, semiring, oracle):
    """Emissions N(0, scale^2) per position: scores spread over hundreds of
    log-units inside one block.  The (C, C) duration gradient then takes its
    term-by-term fallback (and from about N(0, 30^2) the chain its log-domain
    rerun), the (K, C, C) chain and gradients their per-position log-domain
    fallback; everything must still match the float64 oracle."""
    B, T, K, C = 2, 160, 20, 6
    g = torch.Generator().manual_seed(7)
    em = torch.randn(B, T, C, generator=g, dtype=torch.float64) * scale
    cum = torch.cat([torch.zeros(B, 1, C, dtype=torch.float64), em.cumsum(1)], 1).float()
    shape = (K, C, C) if kcc else (C, C)
    tr = (torch.randn(*shape, generator=g, dtype=torch.float64) * 0.1).float()
    db = (torch.randn(K, C, generator=g, dtype=torch.float64) * 0.1).float()
    inp = {"cum_scores": cum, "transition": tr, "duration_bias": db, "proj_start": None,
           "proj_end": None}
    _check_vs_oracle(inp, np.array([T, T - 37]), np.array([1.0, 0.7]), K, semiring, oracle)


@pytest.mark.parametrize("scale", [5.0, 60.0])
@pytest.mark.parametrize("C", [6, 40])
def test_recompute_mode_large_scale_vs_oracle(scale, C, oracle, monkeypatch):
    """The memory-light backward (restart records every S' positions, tables
    rebuilt in the backward) at emission scales whose float64 frames clip
    (N(0, 60^2)): the forward flags it in the saved state, corrects log Z in
    the log domain, and the backward rebuilds both chains' tables in the log
    domain; at N(0, 5^2) nothing clips."""
    monkeypatch.setenv("TORCH_SEMIMARKOV_B200_BACKWARD", "recompute")
    B, T, K = 2, 160, 20
    g = torch.Generator().manual_seed(13)
    em = torch.randn(B, T, C, generator=g, dtype=torch.float64) * scale
    cum = torch.cat([torch.zeros(B, 1, C, dtype=torch.float64), em.cumsum(1)], 1).float()
    tr = (torch.randn(C, C, generator=g, dtype=torch.float64) * 0.1).float()
    db = (torch.randn(K, C, generator=g, dtype=torch.float64) * 0.1).float()
    inp = {"cum_scores": cum, "transition": tr, "duration_bias": db, "proj_start": None,
           "proj_end": None}
    _check_vs_oracle(inp, np.array([T, T - 37]), np.array([1.0, 0.7]), K, "log", oracle)


@pytest.mark.parametrize("chains", ["1", "2", "3"])
def test_cluster_chain_counts_vs_oracle(chains, oracle, monkeypatch):
    """64 < C <= 256 on clusters of four CTAs with 1, 2 or 3 chains per cluster
    (the library picks the fewest with which all clusters are resident at once;
    SEMICRF_CLUSTER_CHAINS forces one), odd batch and ragged lengths so that a
    cluster's chains end at different positions and the last cluster is partial."""
    monkeypatch.setenv("SEMICRF_CLUSTER_CHAINS", chains)
    monkeypatch.setenv("TORCH_SEMIMARKOV_B200_BACKWARD", "keep")
    from inputs import make_streaming_inputs

    B, T, K, C = 5, 120, 12, 96
    inp = make_streaming_inputs(B, T, K, C, seed=71)
    lengths = np.array([T, 97, 64, 120, 33])
    _check_vs_oracle(inp, lengths, np.linspace(0.5, 1.5, B), K, "log", oracle)


@pytest.mark.parametrize("C", [96, 256])
def test_cluster_chain_large_scale_vs_oracle(C, oracle):
    """64 < C <= 256 runs the cluster chain; with emissions N(0, 60^2) its factors
    clip and the chains are rerun in the log domain (at C = 96 with the
    transition staged in shared memory, at C = 256 read from global memory)."""
    B, T, K = 2, 96, 12
    g = torch.Generator().manual_seed(11)
    em = torch.randn(B, T, C, generator=g, dtype=torch.float64) * 60.0
    cum = torch.cat([torch.zeros(B, 1, C, dtype=torch.float64), em.cumsum(1)], 1).float()
    tr = (torch.randn(C, C, generator=g, dtype=torch.float64) * 0.1).float()
    db = (torch.randn(K, C, generator=g, dtype=torch.float64) * 0.1).float()
    inp = {"cum_scores": cum, "transition": tr, "duration_bias": db, "proj_start": None,
           "proj_end": None}
    _check_vs_oracle(inp, np.array([T, T - 29]), np.array([1.0, 0.7]), K, "log", oracle)


def test_chunked_chains_large_scale_vs_oracle(oracle, monkeypatch):
    """Time-chunked chains with emissions N(0, 60^2): the chunks' frames clip and
    the whole chains are rerun in the log domain."""
    monkeypatch.setenv("TORCH_SEMIMARKOV_B200_CHUNKS", "8")
    monkeypatch.setenv("TORCH_SEMIMARKOV_B200_BACKWARD", "keep")
    B, T, K, C = 1, 3000, 20, 8
    g = torch.Generator().manual_seed(9)
    em = torch.randn(B, T, C, generator=g, dtype=torch.float64) * 60.0
    cum = torch.cat([torch.zeros(B, 1, C, dtype=torch.float64), em.cumsum(1)], 1).float()
    tr = (torch.randn(C, C, generator=g, dtype=torch.float64) * 0.1).float()
    db = (torch.randn(K, C, generator=g, dtype=torch.float64) * 0.1).float()
    inp = {"cum_scores": cum, "transition": tr, "duration_bias": db, "proj_start": None,
           "proj_end": None}
    _check_vs_oracle(inp, np.array([T]), np.array([1.0]), K, "log", oracle)


@pytest.mark.parametrize("proj", [None, "both"])
def test_backward_launcher_raw(proj, oracle):
    """launch_streaming_triton_kernel -> launch_streaming_triton_backward called
    as the reference's raw-launcher tests call them
    (tests/test_streaming_triton.py:322-356 and :522-560 of torch-semimarkov):
    shapes and finiteness, then the gradients against the float64 oracle, and
    mismatched checkpoints / log Z rejected with ValueError."""
    from inputs import make_streaming_inputs

    from torch_semimarkov_b200 import (launch_streaming_triton_backward,
                                       launch_streaming_triton_kernel)

    dev = _dev()
    B, T, K, C = 2, 30, 5, 4
    inp = make_streaming_inputs(B, T, K, C, seed=61, proj=proj)
    cum, tr, db = (inp[k].to(dev) for k in ("cum_scores", "transition", "duration_bias"))
    ps = None if inp["proj_start"] is None else inp["proj_start"].to(dev)
    pe = None if inp["proj_end"] is None else inp["proj_end"].to(dev)
    lengths = torch.tensor([T, 21], device=dev)
    part, ck, S = launch_streaming_triton_kernel(cum, tr, db, lengths, K, proj_start=ps,
                                                 proj_end=pe)
    gout = torch.tensor([1.0, 0.5], device=dev)
    gc, gt, gd, gps, gpe = launch_streaming_triton_backward(
        cum, tr, db, lengths, part, ck, S, gout, proj_start=ps, proj_end=pe)
    assert gc.shape == cum.shape and gt.shape == tr.shape and gd.shape == db.shape
    for g in (gc, gt, gd, gps, gpe):
        assert g is None or torch.isfinite(g).all()
    np_in = {k: (None if v is None else v.numpy()) for k, v in inp.items()}
    _, ref = oracle.forward_backward(np_in["cum_scores"], np_in["transition"],
                                     np_in["duration_bias"], lengths.cpu().numpy(), K,
                                     grad_output=gout.cpu().numpy(),
                                     proj_start=np_in["proj_start"], proj_end=np_in["proj_end"])
    assert_grad_close(gc.cpu().numpy(), ref["cum_scores"], what="grad_cum")
    assert_grad_close(gt.cpu().numpy(), ref["transition"], what="grad_transition")
    assert_grad_close(gd.cpu().numpy(), ref["duration_bias"], what="grad_duration_bias")
    if proj:
        assert_grad_close(gps.cpu().numpy(), ref["proj_start"], what="grad_proj_start")
        assert_grad_close(gpe.cpu().numpy(), ref["proj_end"], what="grad_proj_end")
    with pytest.raises(ValueError):  # checkpoints of another layout
        launch_streaming_triton_backward(cum, tr, db, lengths, part, ck[:, :-1], S, gout,
                                         proj_start=ps, proj_end=pe)
    with pytest.raises(ValueError):  # log Z of other inputs
        launch_streaming_triton_backward(cum, tr, db, lengths, part + 1.0, ck, S, gout,
                                         proj_start=ps, proj_end=pe)


def test_backward_launcher_reuses_forward_state(monkeypatch, oracle):
    """launch_streaming_triton_backward given the ring checkpoints that
    launch_streaming_triton_kernel returned runs no forward: it uses the float64
    state kept beside them.  After an in-place change of an input it recomputes
    (and then rejects the stale log Z)."""
    from inputs import make_streaming_inputs

    from torch_semimarkov_b200 import (_lib, launch_streaming_triton_backward,
                                       launch_streaming_triton_kernel)

    dev = _dev()
    B, T, K, C = 3, 200, 12, 6
    inp = make_streaming_inputs(B, T, K, C, seed=62)
    cum, tr, db = (inp[k].to(dev) for k in ("cum_scores", "transition", "duration_bias"))
    lengths = torch.tensor([T, 150, 77], device=dev)
    part, ck, S = launch_streaming_triton_kernel(cum, tr, db, lengths, K)
    gout = torch.tensor([1.0, -0.5, 2.0], device=dev)
    calls = []
    real_forward = _lib.forward
    monkeypatch.setattr(_lib, "forward", lambda *a, **k: calls.append(1) or real_forward(*a, **k))
    gc, gt, gd, _, _ = launch_streaming_triton_backward(cum, tr, db, lengths, part, ck, S, gout)
    assert not calls, "the backward launcher reran the forward"
    np_in = {k: (None if v is None else v.numpy()) for k, v in inp.items()}
    z_ref, ref = oracle.forward_backward(np_in["cum_scores"], np_in["transition"],
                                         np_in["duration_bias"], lengths.cpu().numpy(), K,
                                         grad_output=gout.cpu().numpy())
    np.testing.assert_allclose(part.cpu().numpy(), z_ref, rtol=1e-5, atol=1e-5)
    assert_grad_close(gc.cpu().numpy(), ref["cum_scores"], what="grad_cum")
    assert_grad_close(gt.cpu().numpy(), ref["transition"], what="grad_transition")
    assert_grad_close(gd.cpu().numpy(), ref["duration_bias"], what="grad_duration_bias")
    # the inputs changed after the forward: state is recomputed, and the old
    # log Z no longer belongs to them
    cum.add_(0.5 * torch.arange(T + 1, device=dev, dtype=cum.dtype).view(1, -1, 1) / T)
    with pytest.raises(ValueError):
        launch_streaming_triton_backward(cum, tr, db, lengths, part, ck, S, gout)
    assert calls, "changed inputs must be recomputed"
