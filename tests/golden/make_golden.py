"""Generate golden fixtures for the streaming semi-CRF scan from the reference.

Run once, in the container where the reference is mounted:

    TORCH_SEMIMARKOV_REF_SRC=/path/to/torch-semimarkov/src \
        python tests/golden/make_golden.py [case ...]

It imports the reference package (torch-semimarkov 0.2.0) and runs its CPU
PyTorch path -- ``semi_crf_streaming_forward(..., use_triton=False)`` with
autograd, ``semi_crf_streaming_forward_pytorch`` for checkpoints,
``SemiMarkovCRFHead`` (forward / compute_loss / decode /
decode_with_traceback) and ``score_gold_vectorized`` -- on seeded synthetic
inputs, and writes inputs + outputs to ``tests/golden/<case>.npz``.  Large
inputs are not stored: they are regenerated from the stored seed with
torch's CPU generator by ``tests/golden/inputs.py`` and pinned by a stored
checksum.

The fixtures pin the CPU oracle (oracle/) and the CUDA path (tests/).  The
reference is never needed at test time.
"""

from __future__ import annotations

import math
import os
import sys
import time

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, HERE)
from inputs import (  # noqa: E402
    checksum,
    make_hidden,
    make_streaming_inputs,
)

# the reference's source tree (its src/ directory) must be named explicitly
REF_SRC = os.environ.get("TORCH_SEMIMARKOV_REF_SRC")
if not REF_SRC:
    sys.exit("set TORCH_SEMIMARKOV_REF_SRC to the reference's src/ directory "
             "(the one holding the torch_semimarkov package)")
if REF_SRC not in sys.path:
    sys.path.insert(0, REF_SRC)

from torch_semimarkov import SemiMarkovCRFHead, UncertaintySemiMarkovCRFHead  # noqa: E402
from torch_semimarkov.helpers import score_gold_vectorized  # noqa: E402
from torch_semimarkov.streaming import (  # noqa: E402
    semi_crf_streaming_forward,
    semi_crf_streaming_forward_pytorch,
)

torch.set_num_threads(max(1, os.cpu_count() or 1))


def _np(t):
    return None if t is None else t.detach().cpu().numpy()


def save(name, **arrays):
    path = os.path.join(HERE, name + ".npz")
    clean = {k: v for k, v in arrays.items() if v is not None}
    np.savez_compressed(path, **clean)
    print(f"wrote {path} ({os.path.getsize(path) / 1024:.1f} KiB)")


# ---------------------------------------------------------------------------
# Streaming forward/backward cases (float64 reference CPU path)
# ---------------------------------------------------------------------------

STREAMING_CASES = {
    # name: dict(B, T, K, C, lengths, seed, semiring, proj, kcc, grad_output, ckpt)
    "stream_basic": dict(B=3, T=37, K=6, C=4, lengths=[37, 20, 1], seed=11),
    "stream_basic_max": dict(B=3, T=37, K=6, C=4, lengths=[37, 20, 1], seed=11, semiring="max"),
    "stream_k1": dict(B=2, T=12, K=1, C=3, lengths=[12, 7], seed=12),
    "stream_k2": dict(B=2, T=15, K=2, C=3, lengths=[15, 9], seed=13),
    "stream_k_gt_t": dict(B=2, T=9, K=12, C=3, lengths=[9, 4], seed=14),
    "stream_c1": dict(B=2, T=20, K=5, C=1, lengths=[20, 13], seed=15),
    "stream_t1": dict(B=2, T=1, K=4, C=3, lengths=[1, 1], seed=16),
    "stream_t2": dict(B=1, T=2, K=3, C=2, lengths=[2], seed=17),
    "stream_zero_len": dict(B=3, T=10, K=4, C=3, lengths=[10, 0, 5], seed=18),
    "stream_proj_both": dict(B=2, T=25, K=5, C=4, lengths=[25, 17], seed=19, proj="both"),
    "stream_proj_start": dict(B=2, T=25, K=5, C=4, lengths=[25, 17], seed=20, proj="start"),
    "stream_proj_end": dict(B=2, T=25, K=5, C=4, lengths=[25, 17], seed=21, proj="end"),
    "stream_kcc": dict(B=2, T=20, K=5, C=3, lengths=[20, 11], seed=22, kcc=True),
    "stream_kcc_max": dict(B=2, T=20, K=5, C=3, lengths=[20, 11], seed=22, kcc=True,
                           semiring="max"),
    "stream_grad_out": dict(B=3, T=30, K=5, C=4, lengths=[30, 22, 9], seed=23,
                            grad_output=[0.5, 2.0, -1.0]),
    "stream_ckpt_small": dict(B=2, T=40, K=5, C=3, lengths=[40, 33], seed=24, ckpt=3),
    "stream_ckpt_div": dict(B=2, T=100, K=8, C=4, lengths=[100, 64], seed=25),
    "stream_c24": dict(B=2, T=120, K=30, C=24, lengths=[120, 97], seed=26),
    "stream_c24_max": dict(B=2, T=120, K=30, C=24, lengths=[120, 97], seed=26, semiring="max"),
    "stream_c33": dict(B=2, T=60, K=9, C=33, lengths=[60, 41], seed=27),
    # BASELINE-config-shaped cases at truncated sizes (same generators).
    "cfg2_trunc": dict(B=2, T=600, K=300, C=24, lengths=[600, 555], seed=2, gen="cfg2"),
    "cfg3_trunc": dict(B=1, T=1100, K=1000, C=8, lengths=[1100], seed=3, gen="cfg3"),
    "cfg4_trunc": dict(B=2, T=72, K=64, C=256, lengths=[72, 70], seed=4, gen="cfg4"),
}


def run_streaming_case(name, spec):
    t0 = time.time()
    B, T, K, C = spec["B"], spec["T"], spec["K"], spec["C"]
    semiring = spec.get("semiring", "log")
    inp = make_streaming_inputs(B, T, K, C, spec["seed"], spec.get("gen", "default"),
                                proj=spec.get("proj"), kcc=spec.get("kcc", False))
    lengths = torch.tensor(spec["lengths"], dtype=torch.long)
    cum = inp["cum_scores"].double()
    tr = inp["transition"].double()
    db = inp["duration_bias"].double()
    ps = None if inp["proj_start"] is None else inp["proj_start"].double()
    pe = None if inp["proj_end"] is None else inp["proj_end"].double()

    # Checkpoints / interval from the low-level reference forward.
    part_lo, ckpts, S = semi_crf_streaming_forward_pytorch(
        cum, tr, db, lengths, K, semiring=semiring, proj_start=ps, proj_end=pe,
        checkpoint_interval=spec.get("ckpt"))

    # Public entry point with autograd (SemiCRFStreaming path on CPU).
    leaves = [cum.clone().requires_grad_(True), tr.clone().requires_grad_(True),
              db.clone().requires_grad_(True)]
    psl = None if ps is None else ps.clone().requires_grad_(True)
    pel = None if pe is None else pe.clone().requires_grad_(True)
    part = semi_crf_streaming_forward(leaves[0], leaves[1], leaves[2], lengths, K,
                                      semiring=semiring, proj_start=psl, proj_end=pel,
                                      use_triton=False)
    go = spec.get("grad_output")
    go = torch.ones(B, dtype=torch.float64) if go is None else torch.tensor(go, dtype=torch.float64)
    part.backward(go)
    big = cum.numel() > 200_000
    save(name,
         B=B, T=T, K=K, C=C, seed=spec["seed"], semiring=np.array(semiring),
         gen=np.array(spec.get("gen", "default")), proj=np.array(spec.get("proj") or ""),
         kcc=int(spec.get("kcc", False)), ckpt_arg=-1 if spec.get("ckpt") is None else spec["ckpt"],
         lengths=lengths.numpy(),
         cum_scores=None if big else _np(inp["cum_scores"]),
         cum_checksum=checksum(inp["cum_scores"]),
         transition=_np(inp["transition"]), duration_bias=_np(inp["duration_bias"]),
         proj_start=_np(inp["proj_start"]), proj_end=_np(inp["proj_end"]),
         grad_output=go.numpy(),
         partition=_np(part), partition_lowlevel=_np(part_lo),
         ring_checkpoints=None if big else _np(ckpts), checkpoint_interval=S,
         ring_checkpoints_checksum=float(ckpts.sum()) if big else 0.0,
         grad_cum_scores=None if big else _np(leaves[0].grad),
         grad_cum_checksum=np.array([float(leaves[0].grad.sum()), float(leaves[0].grad.abs().sum())]),
         grad_cum_head=_np(leaves[0].grad[:, :64]),
         grad_transition=_np(leaves[1].grad), grad_duration_bias=_np(leaves[2].grad),
         grad_proj_start=None if psl is None else _np(psl.grad),
         grad_proj_end=None if pel is None else _np(pel.grad))
    print(f"  {name}: {time.time() - t0:.1f}s")


# ---------------------------------------------------------------------------
# CRF head cases (float32, as the module computes)
# ---------------------------------------------------------------------------

HEAD_CASES = {
    "head_viterbi_basic": dict(B=3, T=40, K=8, C=4, lengths=[40, 25, 1], seed=31),
    "head_viterbi_k1": dict(B=2, T=10, K=1, C=3, lengths=[10, 6], seed=32),
    "head_viterbi_c1": dict(B=1, T=50, K=10, C=1, lengths=[50], seed=33),
    "head_viterbi_maxlen": dict(B=3, T=30, K=6, C=3, lengths=[30, 12, 20], seed=34,
                                max_traceback_length=15),
    "head_viterbi_cfg5": dict(B=4, T=300, K=32, C=16, lengths=[300, 211, 160, 299], seed=5,
                              gen="cfg5"),
    "head_quickstart_cfg1": dict(B=4, T=1000, K=100, C=24, hidden=512,
                                 lengths=[1000, 1000, 1000, 1000], seed=1, gen="cfg1"),
}


def run_head_case(name, spec):
    t0 = time.time()
    B, T, K, C = spec["B"], spec["T"], spec["K"], spec["C"]
    hidden_dim = spec.get("hidden")
    torch.manual_seed(spec["seed"])
    crf = SemiMarkovCRFHead(num_classes=C, max_duration=K, hidden_dim=hidden_dim)
    gen = spec.get("gen", "default")
    params = make_hidden(B, T, C, K, spec["seed"], gen, hidden_dim)
    with torch.no_grad():
        crf.transition.copy_(params["transition"])
        crf.duration_dist.duration_bias.copy_(params["duration_bias"])
        if hidden_dim is not None:
            crf.projection.weight.copy_(params["proj_weight"])
            crf.projection.bias.copy_(params["proj_bias"])
    hidden = params["hidden"]
    lengths = torch.tensor(spec["lengths"], dtype=torch.long)
    labels = params["labels"]
    out = {}
    res = crf(hidden, lengths, use_triton=False)
    out["partition"] = _np(res["partition"])
    loss = crf.compute_loss(hidden, lengths, labels, use_triton=False, reduction="sum")
    loss.backward()
    out["loss_sum"] = float(loss)
    out["grad_transition"] = _np(crf.transition.grad)
    out["grad_duration_bias"] = _np(crf.duration_dist.duration_bias.grad)
    if hidden_dim is not None:
        out["grad_proj_weight"] = _np(crf.projection.weight.grad)
        out["grad_proj_bias"] = _np(crf.projection.bias.grad)
    with torch.no_grad():
        out["decode_scores"] = _np(crf.decode(hidden, lengths, use_triton=False))
        mtl = spec.get("max_traceback_length", 10000)
        vr = crf.decode_with_traceback(hidden, lengths, max_traceback_length=mtl)
    nseg = np.array([len(s) for s in vr.segments], dtype=np.int64)
    segs = np.zeros((B, max(1, int(nseg.max())), 3), dtype=np.int64)
    segsc = np.zeros((B, max(1, int(nseg.max()))), dtype=np.float64)
    for b, sl in enumerate(vr.segments):
        for i, s in enumerate(sl):
            segs[b, i] = (s.start, s.end, s.label)
            segsc[b, i] = s.score
    out["viterbi_scores"] = _np(vr.scores)
    out["nseg"] = nseg
    out["segments"] = segs
    out["segment_scores"] = segsc
    out["max_traceback_length"] = spec.get("max_traceback_length", 10000)
    big = hidden.numel() > 200_000
    save(name, B=B, T=T, K=K, C=C, seed=spec["seed"], gen=np.array(gen),
         hidden_dim=-1 if hidden_dim is None else hidden_dim,
         lengths=lengths.numpy(), labels=labels.numpy(),
         hidden=None if big else _np(hidden), hidden_checksum=checksum(hidden),
         transition=_np(params["transition"]), duration_bias=_np(params["duration_bias"]),
         proj_weight=_np(params.get("proj_weight")), proj_bias=_np(params.get("proj_bias")),
         **out)
    print(f"  {name}: {time.time() - t0:.1f}s")


# ---------------------------------------------------------------------------
# Uncertainty cases (reference uncertainty.py, float32 CPU path)
# ---------------------------------------------------------------------------

UNCERT_CASES = {
    "uncert_basic": dict(B=3, T=40, K=6, C=4, lengths=[40, 25, 9], seed=51),
    "uncert_proj": dict(B=2, T=60, K=8, C=5, lengths=[60, 33], seed=52, hidden=16),
}


def run_uncert_case(name, spec):
    t0 = time.time()
    B, T, K, C = spec["B"], spec["T"], spec["K"], spec["C"]
    hidden_dim = spec.get("hidden")
    torch.manual_seed(spec["seed"])
    crf = UncertaintySemiMarkovCRFHead(num_classes=C, max_duration=K, hidden_dim=hidden_dim)
    params = make_hidden(B, T, C, K, spec["seed"], "default", hidden_dim)
    with torch.no_grad():
        crf.transition.copy_(params["transition"])
        crf.duration_dist.duration_bias.copy_(params["duration_bias"])
        if hidden_dim is not None:
            crf.projection.weight.copy_(params["proj_weight"])
            crf.projection.bias.copy_(params["proj_bias"])
    hidden = params["hidden"]
    lengths = torch.tensor(spec["lengths"], dtype=torch.long)
    labels = params["labels"]
    out = {
        "boundary": _np(crf.compute_boundary_marginals(hidden, lengths)),
        "boundary_raw": _np(crf.compute_boundary_marginals(hidden, lengths, normalize=False)),
        "position": _np(crf.compute_position_marginals(hidden, lengths)),
        "entropy": _np(crf.compute_entropy_streaming(hidden, lengths)),
        "loss_boundary": _np(crf.compute_loss_uncertainty_weighted(
            hidden, lengths, labels, uncertainty_weight=0.5, focus_mode="boundary_regions",
            reduction="none")),
    }
    loss = crf.compute_loss_uncertainty_weighted(hidden, lengths, labels, reduction="sum")
    loss.backward()
    out["loss_high_sum"] = float(loss.detach())
    out["grad_transition"] = _np(crf.transition.grad)
    out["grad_duration_bias"] = _np(crf.duration_dist.duration_bias.grad)
    if hidden_dim is not None:
        out["grad_proj_weight"] = _np(crf.projection.weight.grad)
    save(name, B=B, T=T, K=K, C=C, seed=spec["seed"],
         hidden_dim=-1 if hidden_dim is None else hidden_dim, lengths=lengths.numpy(),
         labels=labels.numpy(), hidden=_np(hidden), transition=_np(params["transition"]),
         duration_bias=_np(params["duration_bias"]), proj_weight=_np(params.get("proj_weight")),
         proj_bias=_np(params.get("proj_bias")), **out)
    print(f"  {name}: {time.time() - t0:.1f}s")


# ---------------------------------------------------------------------------
# Duration distributions (reference duration.py) and heads that use them
# ---------------------------------------------------------------------------


def run_duration_dists(name="duration_dists"):
    from torch_semimarkov.duration import (
        GeometricDuration,
        NegativeBinomialDuration,
        PoissonDuration,
    )

    K, C = 12, 4
    g = torch.Generator().manual_seed(61)
    w = torch.randn(K, C, generator=g)
    out = {"K": K, "C": C, "weights": _np(w)}
    specs = {
        "geometric": (GeometricDuration, {"logit_p": torch.randn(C, generator=g)}),
        "negbin": (NegativeBinomialDuration, {"logit_p": torch.randn(C, generator=g),
                                               "log_r": torch.randn(C, generator=g)}),
        "poisson": (PoissonDuration, {"log_lambda": torch.randn(C, generator=g) + 1.0}),
    }
    for kind, (cls, params) in specs.items():
        d = cls(K, C)
        with torch.no_grad():
            for pname, v in params.items():
                getattr(d, pname).copy_(v)
        bias = d()
        (bias * w).sum().backward()
        out[kind + "_bias"] = _np(bias)
        for pname, v in params.items():
            out[kind + "_" + pname] = _np(v)
            out[kind + "_grad_" + pname] = _np(getattr(d, pname).grad)
    save(name, **out)


HEAD_DIST_CASES = {
    "dhead_geometric": dict(B=2, T=50, K=8, C=4, lengths=[50, 31], seed=71, dist="geometric",
                           params={"logit_p": [-0.5, 0.2, 1.0, -1.5]}),
    "dhead_negbin": dict(B=2, T=50, K=8, C=4, lengths=[50, 40], seed=72, dist="negbin",
                        params={"logit_p": [0.3, -0.4, 0.1, 0.8],
                                "log_r": [0.5, -0.2, 1.1, 0.0]}),
}


def run_head_dist_case(name, spec):
    B, T, K, C = spec["B"], spec["T"], spec["K"], spec["C"]
    torch.manual_seed(spec["seed"])
    crf = SemiMarkovCRFHead(num_classes=C, max_duration=K, duration_distribution=spec["dist"])
    p = make_hidden(B, T, C, K, spec["seed"], "default", None)
    with torch.no_grad():
        crf.transition.copy_(p["transition"])
        for pname, v in spec["params"].items():
            getattr(crf.duration_dist, pname).copy_(torch.tensor(v))
    lengths = torch.tensor(spec["lengths"], dtype=torch.long)
    res = crf(p["hidden"], lengths, use_triton=False)
    loss = crf.compute_loss(p["hidden"], lengths, p["labels"], use_triton=False, reduction="sum")
    loss.backward()
    out = {"partition": _np(res["partition"]), "loss_sum": float(loss.detach()),
           "grad_transition": _np(crf.transition.grad)}
    for pname in spec["params"]:
        out["param_" + pname] = _np(getattr(crf.duration_dist, pname).detach())
        out["grad_" + pname] = _np(getattr(crf.duration_dist, pname).grad)
    save(name, B=B, T=T, K=K, C=C, seed=spec["seed"], dist=np.array(spec["dist"]),
         lengths=lengths.numpy(), labels=p["labels"].numpy(), hidden=_np(p["hidden"]),
         transition=_np(p["transition"]), **out)


# ---------------------------------------------------------------------------
# Edge-tensor scan (reference triton_scan.py, float64 PyTorch scan)
# ---------------------------------------------------------------------------

ESCAN_CASES = {
    "escan_basic": dict(B=4, N=30, K=5, C=4, lengths=[30, 17, 1, 2], seed=81),
    "escan_k1": dict(B=2, N=12, K=1, C=3, lengths=[12, 7], seed=82),
    "escan_wide": dict(B=2, N=24, K=8, C=6, lengths=[24, 15], seed=83),
    "escan_oob": dict(B=3, N=10, K=4, C=3, lengths=[0, 10, 11], seed=84),
}


def run_escan_case(name, spec):
    from torch_semimarkov.triton_scan import semi_crf_forward_pytorch

    B, N, K, C = spec["B"], spec["N"], spec["K"], spec["C"]
    g = torch.Generator().manual_seed(spec["seed"])
    edge = torch.randn(B, N - 1, K, C, C, generator=g).float()
    lengths = torch.tensor(spec["lengths"], dtype=torch.long)
    gout = torch.rand(B, generator=g, dtype=torch.float64) + 0.5
    out = {}
    for semi in ("log", "max"):
        e = edge.double().requires_grad_(True)
        part = semi_crf_forward_pytorch(e, lengths, semiring=semi)
        part.backward(gout)
        out[semi + "_partition"] = _np(part)
        out[semi + "_grad_edge"] = _np(e.grad).astype(np.float32)
    save(name, B=B, N=N, K=K, C=C, edge=_np(edge), lengths=lengths.numpy(),
         grad_output=_np(gout), **out)


# ---------------------------------------------------------------------------
# Gold scoring cases (float64)
# ---------------------------------------------------------------------------

GOLD_CASES = {
    "gold_basic": dict(B=4, T=30, K=6, C=4, lengths=[30, 17, 1, 0], seed=41),
    "gold_t1": dict(B=3, T=1, K=4, C=3, lengths=[1, 0, 1], seed=42),
    "gold_k1": dict(B=2, T=12, K=1, C=3, lengths=[12, 5], seed=43),
    "gold_long_segs": dict(B=2, T=60, K=5, C=2, lengths=[60, 44], seed=44, runs=True),
}


def run_gold_case(name, spec):
    B, T, K, C = spec["B"], spec["T"], spec["K"], spec["C"]
    g = torch.Generator().manual_seed(spec["seed"])
    cum = torch.zeros(B, T + 1, C, dtype=torch.float64)
    cum[:, 1:] = torch.cumsum(torch.randn(B, T, C, generator=g, dtype=torch.float64), dim=1)
    tr = torch.randn(C, C, generator=g, dtype=torch.float64) * 0.3
    db = torch.randn(K, C, generator=g, dtype=torch.float64) * 0.3
    if spec.get("runs"):
        # piecewise-constant labels with runs longer than K (exercises the clamp)
        labels = torch.zeros(B, T, dtype=torch.long)
        for b in range(B):
            pos, lab = 0, 0
            while pos < T:
                run = int(torch.randint(1, 3 * K, (1,), generator=g))
                labels[b, pos:pos + run] = lab
                lab = (lab + 1) % C
                pos += run
    else:
        labels = torch.randint(0, C, (B, T), generator=g)
    lengths = torch.tensor(spec["lengths"], dtype=torch.long)
    score = score_gold_vectorized(cum, labels, lengths, tr, db, K)
    save(name, B=B, T=T, K=K, C=C, cum_scores=_np(cum), labels=labels.numpy(),
         lengths=lengths.numpy(), transition=_np(tr), duration_bias=_np(db),
         gold_score=_np(score))


def main(argv):
    want = set(argv)
    for name, spec in STREAMING_CASES.items():
        if not want or name in want:
            run_streaming_case(name, spec)
    for name, spec in HEAD_CASES.items():
        if not want or name in want:
            run_head_case(name, spec)
    for name, spec in GOLD_CASES.items():
        if not want or name in want:
            run_gold_case(name, spec)
    for name, spec in UNCERT_CASES.items():
        if not want or name in want:
            run_uncert_case(name, spec)
    for name, spec in ESCAN_CASES.items():
        if not want or name in want:
            run_escan_case(name, spec)
    if not want or "duration_dists" in want:
        run_duration_dists()
    for name, spec in HEAD_DIST_CASES.items():
        if not want or name in want:
            run_head_dist_case(name, spec)


if __name__ == "__main__":
    main(sys.argv[1:])
