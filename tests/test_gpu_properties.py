"""Size-independent properties of the CUDA path (the reference's regression tests).

- grad_output scaling: the shared gradients are sum_b g_b * marginals_b, so
  they are linear in grad_output, and a sequence with g_b = 0 contributes
  nothing (test_streaming_triton.py:901-1087 of the reference), for (C, C) and
  (K, C, C) transitions;
- central finite differences of log Z agree with the analytic gradients
  (an oracle-free check, like the reference's gradcheck tests);
- non-contiguous inputs give the same results as contiguous ones;
- Viterbi tracebacks tile [0, L) with inclusive segment ends, use durations
  1..max(1, K-1), and their segment scores add up to the Viterbi score
  (test_edge_cases.py:209-250 of the reference).
"""

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _dev():
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    return torch.device("cuda:0")


def _inputs(B, T, K, C, seed, kcc=False, proj=None):
    from inputs import make_streaming_inputs

    inp = make_streaming_inputs(B, T, K, C, seed=seed, gen="default", proj=proj, kcc=kcc)
    return {k: (None if v is None else v.to(_dev())) for k, v in inp.items()}


def _grads(inp, lengths, K, gout, semiring="log"):
    from torch_semimarkov_b200 import semi_crf_streaming_forward

    leaves = {k: (None if v is None else v.detach().clone().requires_grad_(True))
              for k, v in inp.items()}
    part = semi_crf_streaming_forward(leaves["cum_scores"], leaves["transition"],
                                      leaves["duration_bias"], lengths, K, semiring=semiring,
                                      proj_start=leaves["proj_start"], proj_end=leaves["proj_end"])
    part.backward(gout)
    return part.detach(), {k: v.grad.detach().double() for k, v in leaves.items() if v is not None}


@pytest.mark.parametrize("kcc", [False, True])
def test_grad_output_linearity_and_zero_mask(kcc):
    dev = _dev()
    B, T, K, C = 4, 90, 7, 5
    inp = _inputs(B, T, K, C, seed=301, kcc=kcc, proj="both")
    lengths = torch.tensor([90, 71, 55, 90], device=dev)
    g1 = torch.tensor([1.0, -0.5, 2.0, 0.25], device=dev)
    g2 = torch.tensor([0.3, 1.5, -1.0, 0.0], device=dev)
    a, b = 0.7, -1.3
    _, r1 = _grads(inp, lengths, K, g1)
    _, r2 = _grads(inp, lengths, K, g2)
    _, r3 = _grads(inp, lengths, K, a * g1 + b * g2)
    for key in r1:
        want = a * r1[key] + b * r2[key]
        err = (r3[key] - want).abs().max().item()
        scale = want.abs().max().item()
        assert err <= 1e-5 * scale + 1e-6, f"{key}: linearity error {err:.3e}"
    # g_b = 0: nothing of sequence 3 reaches any gradient
    gz = torch.tensor([1.0, -0.5, 2.0, 0.0], device=dev)
    _, rz = _grads(inp, lengths, K, gz)
    for key in ("cum_scores", "proj_start", "proj_end"):
        assert torch.count_nonzero(rz[key][3]) == 0, key
    sub = {k: (None if v is None else (v if k in ("transition", "duration_bias") else v[:3]))
           for k, v in inp.items()}
    _, rs = _grads(sub, lengths[:3], K, gz[:3])
    for key in ("transition", "duration_bias"):
        err = (rz[key] - rs[key]).abs().max().item()
        assert err <= 1e-5 * rs[key].abs().max().item() + 1e-6, f"{key}: zero-mask error {err:.3e}"


@pytest.mark.parametrize("kcc", [False, True])
def test_finite_differences(kcc):
    """Central differences of sum(log Z) in float64 arithmetic on float32 inputs."""
    dev = _dev()
    B, T, K, C = 2, 24, 5, 3
    inp = _inputs(B, T, K, C, seed=302, kcc=kcc)
    lengths = torch.tensor([24, 17], device=dev)
    ones = torch.ones(B, device=dev)
    part, grads = _grads(inp, lengths, K, ones)
    rng = np.random.default_rng(3)
    eps = 1e-2
    for key in ("cum_scores", "transition", "duration_bias"):
        base = inp[key]
        for _ in range(6):
            idx = tuple(int(rng.integers(0, n)) for n in base.shape)
            if key == "duration_bias" and idx[0] == 0:
                idx = (1,) + idx[1:]  # row 0 is never used
            plus = {k: (None if v is None else v.clone()) for k, v in inp.items()}
            minus = {k: (None if v is None else v.clone()) for k, v in inp.items()}
            plus[key][idx] += eps
            minus[key][idx] -= eps
            fp, _ = _grads(plus, lengths, K, ones)
            fm, _ = _grads(minus, lengths, K, ones)
            fd = (fp.double().sum() - fm.double().sum()).item() / (2 * eps)
            an = grads[key][idx].item()
            assert abs(fd - an) <= 2e-3 * max(1.0, abs(an)), f"{key}{idx}: fd {fd} vs {an}"


def test_noncontiguous_inputs():
    from torch_semimarkov_b200 import semi_crf_streaming_forward

    dev = _dev()
    B, T, K, C = 3, 40, 6, 4
    inp = _inputs(B, T, K, C, seed=303)
    lengths = torch.tensor([40, 33, 12], device=dev)
    cum_t = inp["cum_scores"].transpose(0, 1).contiguous().transpose(0, 1)  # strided view
    tr_t = inp["transition"].t().contiguous().t()
    assert not cum_t.is_contiguous() and not tr_t.is_contiguous()
    a = semi_crf_streaming_forward(inp["cum_scores"], inp["transition"], inp["duration_bias"],
                                   lengths, K)
    b = semi_crf_streaming_forward(cum_t, tr_t, inp["duration_bias"], lengths, K)
    assert torch.equal(a, b)


@pytest.mark.parametrize("B,T,K,C", [(6, 300, 12, 5), (4, 120, 40, 3), (3, 60, 1, 4)])
def test_traceback_invariants(B, T, K, C):
    from torch_semimarkov_b200 import SemiMarkovCRFHead

    dev = _dev()
    torch.manual_seed(304 + T)
    crf = SemiMarkovCRFHead(num_classes=C, max_duration=K).to(dev)
    hidden = torch.randn(B, T, C, device=dev)
    lengths = torch.randint(T // 2, T + 1, (B,), device=dev)
    lengths[0] = T
    res = crf.decode_with_traceback(hidden, lengths)
    kmax = max(1, K - 1)
    for b in range(B):
        L = int(lengths[b])
        segs = res.segments[b]
        assert segs[0].start == 0 and segs[-1].end == L - 1
        for i, s in enumerate(segs):
            assert 0 <= s.label < C and 1 <= s.end - s.start + 1 <= kmax
            if i:
                assert s.start == segs[i - 1].end + 1
        total = sum(s.score for s in segs)
        score = float(res.scores[b])
        assert abs(total - score) <= 1e-5 * abs(score) + 1e-4, f"{b}: {total} vs {score}"


@pytest.mark.parametrize("kcc", [False, True])
def test_float64_inputs(kcc):
    """float64 inputs (the dtype of the reference's gradcheck tests) give the
    float32 results up to input rounding, with gradients in the inputs' dtype."""
    from torch_semimarkov_b200 import semi_crf_streaming_forward

    dev = _dev()
    B, T, K, C = 3, 50, 6, 4
    inp = _inputs(B, T, K, C, seed=305, kcc=kcc)
    lengths = torch.tensor([50, 37, 21], device=dev)
    p32, g32 = _grads(inp, lengths, K, torch.ones(B, device=dev))
    leaves = {k: v.detach().double().requires_grad_(True) for k, v in inp.items() if v is not None}
    p64 = semi_crf_streaming_forward(leaves["cum_scores"], leaves["transition"],
                                     leaves["duration_bias"], lengths, K)
    assert p64.dtype == torch.float64
    p64.sum().backward()
    torch.testing.assert_close(p64, p32.double(), rtol=1e-6, atol=1e-5)
    for key in ("cum_scores", "transition", "duration_bias"):
        g = leaves[key].grad
        assert g.dtype == torch.float64, key
        torch.testing.assert_close(g, g32[key], rtol=1e-5, atol=1e-6)
