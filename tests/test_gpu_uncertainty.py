"""Uncertainty methods (reference uncertainty.py) on the CUDA path.

The fixtures come from the reference's UncertaintySemiMarkovCRFHead on its
float32 CPU path, so they are compared at 1e-4; the boundary signal is also
checked at 1e-5 against the float64 oracle's gradients on the same float32
cumulative scores.
"""

import numpy as np
import pytest
import torch

from conftest import load_golden

CASES = ["uncert_basic", "uncert_proj"]


def _head(g, dev):
    from torch_semimarkov_b200 import UncertaintySemiMarkovCRFHead

    hd = int(g["hidden_dim"])
    crf = UncertaintySemiMarkovCRFHead(num_classes=int(g["C"]), max_duration=int(g["K"]),
                                       hidden_dim=None if hd < 0 else hd)
    with torch.no_grad():
        crf.transition.copy_(torch.as_tensor(g["transition"]))
        crf.duration_dist.duration_bias.copy_(torch.as_tensor(g["duration_bias"]))
        if hd > 0:
            crf.projection.weight.copy_(torch.as_tensor(g["proj_weight"]))
            crf.projection.bias.copy_(torch.as_tensor(g["proj_bias"]))
    return crf.to(dev)


def _close(got, ref, rtol, atol, what):
    got = np.asarray(got, dtype=np.float64)
    ref = np.asarray(ref, dtype=np.float64)
    err = np.abs(got - ref)
    assert (err <= rtol * np.abs(ref) + atol).all(), f"{what}: max err {err.max():.3e}"


@pytest.mark.gpu
@pytest.mark.parametrize("name", CASES)
def test_uncertainty_vs_reference(name, oracle):
    dev = torch.device("cuda:0")
    g = load_golden(name)
    crf = _head(g, dev)
    hidden = torch.as_tensor(g["hidden"]).to(dev)
    lengths = torch.as_tensor(g["lengths"]).to(dev)
    labels = torch.as_tensor(g["labels"]).to(dev)

    b = crf.compute_boundary_marginals(hidden, lengths)
    _close(b.cpu(), g["boundary"], 1e-4, 1e-6, "boundary")
    raw = crf.compute_boundary_marginals(hidden, lengths, normalize=False)
    _close(raw.cpu(), g["boundary_raw"], 1e-4, 1e-6, "boundary_raw")
    # tight: the float64 oracle's d logZ / d cum on the same float32 cum_scores
    with torch.no_grad():
        scores = crf.projection(hidden) if crf.projection is not None else hidden
        cum = torch.zeros(hidden.shape[0], hidden.shape[1] + 1, crf.num_classes,
                          device=dev)
        cum[:, 1:] = torch.cumsum(scores.float(), dim=1)
    _, gr = oracle.forward_backward(cum.cpu().numpy(), g["transition"], g["duration_bias"],
                                    g["lengths"], int(g["K"]), threads=4)
    want = np.abs(gr["cum_scores"][:, 1:]).sum(-1)
    err = np.abs(raw.cpu().numpy() - want).max()
    assert err <= 1e-5 * np.abs(want).max() + 1e-6, f"boundary vs oracle: {err:.3e}"

    pm = crf.compute_position_marginals(hidden, lengths)
    _close(pm.cpu(), g["position"], 1e-4, 1e-6, "position marginals")
    np.testing.assert_allclose(pm.sum(-1).cpu().numpy(), 1.0, rtol=1e-5)
    ent = crf.compute_entropy_streaming(hidden, lengths)
    _close(ent.cpu(), g["entropy"], 1e-4, 1e-5, "entropy")
    lb = crf.compute_loss_uncertainty_weighted(hidden, lengths, labels, uncertainty_weight=0.5,
                                               focus_mode="boundary_regions", reduction="none")
    _close(lb.detach().cpu(), g["loss_boundary"], 1e-4, 1e-3, "loss (boundary_regions)")
    loss = crf.compute_loss_uncertainty_weighted(hidden, lengths, labels, reduction="sum")
    loss.backward()
    _close([float(loss.detach())], [float(g["loss_high_sum"])], 1e-4, 1e-3, "loss (high)")
    for key, t in (("grad_transition", crf.transition.grad),
                   ("grad_duration_bias", crf.duration_dist.duration_bias.grad)):
        ref = g[key]
        err = np.abs(t.cpu().numpy() - ref).max()
        assert err <= 1e-4 * np.abs(ref).max() + 1e-5, f"{key}: {err:.3e}"
    if "grad_proj_weight" in g:
        ref = g["grad_proj_weight"]
        err = np.abs(crf.projection.weight.grad.cpu().numpy() - ref).max()
        assert err <= 1e-4 * np.abs(ref).max() + 1e-5, f"grad_proj_weight: {err:.3e}"


def test_exact_variants_are_refused():
    """The edge-tensor exact methods are not part of this package: they say so."""
    from torch_semimarkov_b200 import UncertaintySemiMarkovCRFHead

    crf = UncertaintySemiMarkovCRFHead(4, 6)
    h = torch.zeros(1, 5, 4)
    with pytest.raises(NotImplementedError, match="SemiMarkov"):
        crf.compute_boundary_marginals(h, torch.tensor([5]), use_streaming=False)
    with pytest.raises(NotImplementedError, match="SemiMarkov"):
        crf.compute_entropy_exact(h, torch.tensor([5]))
    with pytest.raises(ValueError):
        crf.compute_loss_uncertainty_weighted(h, torch.tensor([5]), torch.zeros(1, 5).long(),
                                              focus_mode="nope")
