"""Duration parameterisations against the reference (duration.py).

CPU: every distribution's bias and parameter gradients match fixtures made
by the reference's own classes.  GPU: heads built with a geometric or
negative-binomial duration prior match the reference head's partition, loss
and gradients (the duration parameters' gradients flow through the scan's
grad_duration_bias).
"""

import numpy as np
import pytest
import torch

from conftest import load_golden


@pytest.mark.parametrize("kind,params", [("geometric", ["logit_p"]),
                                         ("negbin", ["logit_p", "log_r"]),
                                         ("poisson", ["log_lambda"])])
def test_distribution_bias_and_grads(kind, params):
    from torch_semimarkov_b200 import create_duration_distribution

    g = load_golden("duration_dists")
    K, C = int(g["K"]), int(g["C"])
    d = create_duration_distribution(kind, K, C)
    with torch.no_grad():
        for p in params:
            getattr(d, p).copy_(torch.as_tensor(g[f"{kind}_{p}"]))
    bias = d()
    (bias * torch.as_tensor(g["weights"])).sum().backward()
    np.testing.assert_allclose(bias.detach().numpy(), g[f"{kind}_bias"], rtol=1e-6, atol=1e-6)
    for p in params:
        np.testing.assert_allclose(getattr(d, p).grad.numpy(), g[f"{kind}_grad_{p}"],
                                   rtol=1e-5, atol=1e-6)


def test_factory_and_fixed_parameters():
    from torch_semimarkov_b200 import (CallableDuration, GeometricDuration, LearnedDuration,
                                       NegativeBinomialDuration, PoissonDuration, UniformDuration,
                                       create_duration_distribution)

    assert isinstance(create_duration_distribution(None, 5, 3), LearnedDuration)
    assert isinstance(create_duration_distribution("negative_binomial", 5, 3),
                      NegativeBinomialDuration)
    u = create_duration_distribution("uniform", 5, 3)
    assert isinstance(u, UniformDuration) and torch.equal(u(), torch.zeros(5, 3))
    mine = PoissonDuration(5, 3)
    assert create_duration_distribution(mine, 5, 3) is mine
    d = create_duration_distribution("geometric", 5, 3, init_logit=-1.0, learn_rate=False)
    assert "logit_p" in dict(d.named_buffers()) and not list(d.parameters())
    torch.testing.assert_close(d()[0], torch.log(torch.sigmoid(torch.tensor(-1.0)) + 1e-8)
                               .expand(3))
    cd = CallableDuration(4, 2, lambda K, C, dev: torch.ones(K, C, device=dev))
    assert torch.equal(cd(), torch.ones(4, 2))
    with pytest.raises(ValueError, match="Unknown duration distribution"):
        create_duration_distribution("lognormal", 5, 3)
    with pytest.warns(UserWarning, match="non-finite"):
        NegativeBinomialDuration(5, 3, init_log_r=-200.0)()
    assert isinstance(GeometricDuration(5, 3)(), torch.Tensor)


@pytest.mark.gpu
@pytest.mark.parametrize("name", ["dhead_geometric", "dhead_negbin"])
def test_head_with_duration_prior_vs_reference(name):
    from torch_semimarkov_b200 import SemiMarkovCRFHead

    g = load_golden(name)
    dev = torch.device("cuda:0")
    C, K = int(g["C"]), int(g["K"])
    crf = SemiMarkovCRFHead(num_classes=C, max_duration=K, duration_distribution=str(g["dist"]))
    params = [k[len("param_"):] for k in g if k.startswith("param_")]
    with torch.no_grad():
        crf.transition.copy_(torch.as_tensor(g["transition"]))
        for p in params:
            getattr(crf.duration_dist, p).copy_(torch.as_tensor(g["param_" + p]))
    crf = crf.to(dev)
    hidden = torch.as_tensor(g["hidden"]).to(dev)
    lengths = torch.as_tensor(g["lengths"]).to(dev)
    labels = torch.as_tensor(g["labels"]).to(dev)
    res = crf(hidden, lengths)
    # the fixture is the reference's float32 CPU run: compare at its accuracy
    np.testing.assert_allclose(res["partition"].detach().cpu().numpy(), g["partition"],
                               rtol=2e-4, atol=1e-3)
    loss = crf.compute_loss(hidden, lengths, labels, reduction="sum")
    loss.backward()
    assert abs(float(loss.detach()) - float(g["loss_sum"])) <= 2e-4 * abs(float(g["loss_sum"])) + 1e-3
    for key, t in [("grad_transition", crf.transition.grad)] + [
            ("grad_" + p, getattr(crf.duration_dist, p).grad) for p in params]:
        ref = g[key]
        err = np.abs(t.cpu().numpy() - ref).max()
        assert err <= 2e-4 * np.abs(ref).max() + 1e-4, f"{key}: {err:.3e}"
