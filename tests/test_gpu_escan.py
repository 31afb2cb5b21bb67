"""Edge-tensor scan (reference triton_scan.py) on the CUDA path.

Fixtures: the reference's float64 PyTorch scan and its autograd gradients on
seeded float32 edge tensors (both semirings, K = 1, lengths 0, 1, full and
beyond N).  The CUDA scan computes in float64, so partitions are compared at
1e-5 relative and gradients norm-wise at 1e-5.
"""

import numpy as np
import pytest
import torch

from conftest import load_golden

CASES = ["escan_basic", "escan_k1", "escan_wide", "escan_oob"]


@pytest.mark.gpu
@pytest.mark.parametrize("semiring", ["log", "max"])
@pytest.mark.parametrize("name", CASES)
def test_edge_scan_vs_reference(name, semiring):
    from torch_semimarkov_b200.triton_scan import (launch_triton_kernel, semi_crf_forward_pytorch,
                                                   semi_crf_triton_forward)

    dev = torch.device("cuda:0")
    g = load_golden(name)
    edge = torch.as_tensor(g["edge"]).to(dev).requires_grad_(True)
    lengths = torch.as_tensor(g["lengths"]).to(dev)
    part = semi_crf_triton_forward(edge, lengths, semiring=semiring)
    part.backward(torch.as_tensor(g["grad_output"], dtype=torch.float32, device=dev))
    ref = g[semiring + "_partition"]
    got = part.detach().cpu().numpy().astype(np.float64)
    assert np.all(np.abs(got - ref) <= 1e-5 * np.abs(ref) + 1e-5), (got, ref)
    gref = g[semiring + "_grad_edge"].astype(np.float64)
    err = np.abs(edge.grad.cpu().numpy() - gref).max()
    assert err <= 1e-5 * np.abs(gref).max() + 1e-6, f"grad_edge: {err:.3e}"
    # the other names run the same forward
    with torch.no_grad():
        for fn in (launch_triton_kernel, semi_crf_forward_pytorch):
            assert torch.equal(fn(edge.detach(), lengths, semiring=semiring), part.detach())


def test_edge_scan_rejects_cpu_and_bad_input():
    from torch_semimarkov_b200 import _lib
    from torch_semimarkov_b200.triton_scan import semi_crf_triton_forward

    with pytest.raises(RuntimeError, match="CUDA"):
        semi_crf_triton_forward(torch.zeros(1, 3, 2, 2, 2), torch.tensor([4]))
    with pytest.raises(ValueError, match="semiring"):
        semi_crf_triton_forward(torch.zeros(1, 3, 2, 2, 2), torch.tensor([4]), semiring="sum")
    lib = _lib.load()
    assert lib.semicrf_edge_scan_saved_size(2, 10, 3, 4, 0) >= 8 * (2 + 2 * 10 * 4)
    assert lib.semicrf_edge_scan_saved_size(2, 10, 3, 4, 1) > lib.semicrf_edge_scan_saved_size(
        2, 10, 3, 4, 0)  # the max semiring keeps backpointers
    assert lib.semicrf_edge_scan_saved_size(2, 0, 3, 4, 0) == 0  # N >= 1
    assert lib.semicrf_edge_scan_forward(2, 10, 3, 4, None, None, 7, None, None, None) == 5
    assert lib.semicrf_edge_scan_forward(2, 10, 3, 4, None, None, 0, None, None, None) == 1
    assert lib.semicrf_edge_scan_forward(0, 10, 3, 4, None, None, 0, None, None, None) == 0
