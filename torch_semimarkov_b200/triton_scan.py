"""The edge-tensor scan (reference triton_scan.py) on the CUDA path.

The reference's older API takes a materialised edge tensor (batch, N-1, K, C, C)
of segment log potentials and scans it (triton_scan.py:163-273); it routes
inference to a Triton kernel and training to ``torch.compile`` of its PyTorch
scan (:773-860).  Here every entry point runs the float64 CUDA scan of
``csrc/escan.cu`` through ``semicrf_edge_scan_forward`` / ``_backward``:

- ``semi_crf_triton_forward(edge, lengths, use_triton, validate, semiring,
  use_compile)``: the public entry; ``use_triton`` and ``use_compile`` are
  accepted and ignored, ``validate`` (the reference's float64 check) is what
  the kernel always computes;
- ``SemiCRFTritonForward``: the autograd Function, whose backward gives the
  segment marginals (log) or the first-maximum path (max) directly instead of
  re-running the scan under autograd;
- ``launch_triton_kernel`` and ``semi_crf_forward_pytorch``: the same forward
  under the reference's other two names.

The edge tensor holds O(T K C^2) values, so this path suits short sequences;
the streaming scan (``semi_crf_streaming_forward``) is the one for long ones.
CPU tensors raise: there is no CPU fallback.
"""

from __future__ import annotations

import torch
from torch import Tensor

from . import _lib


class SemiCRFTritonForward(torch.autograd.Function):
    """Edge-tensor scan with its gradient (triton_scan.py:715-770)."""

    @staticmethod
    def forward(ctx, edge: Tensor, lengths: Tensor, use_triton: bool = True,
                semiring: str = "log") -> Tensor:
        part, saved = _lib.edge_scan_forward(edge, lengths, semiring,
                                             want_saved=ctx.needs_input_grad[0])
        ctx.semiring = semiring
        ctx.saved = saved
        ctx.save_for_backward(edge, lengths)
        return part.to(edge.dtype)

    @staticmethod
    def backward(ctx, grad_output: Tensor):
        edge, lengths = ctx.saved_tensors
        grad = _lib.edge_scan_backward(edge, lengths, ctx.semiring, ctx.saved, grad_output)
        ctx.saved = None
        return grad.to(edge.dtype), None, None, None


def semi_crf_triton_forward(edge: Tensor, lengths: Tensor, use_triton: bool = True,
                            validate: bool = False, semiring: str = "log",
                            use_compile: bool = True) -> Tensor:
    """Log partition (or Viterbi score) of the edge tensor, shape (batch,).

    Same arguments as the reference (triton_scan.py:773); the scan always runs
    in float64 and returns the edge's dtype, so ``validate`` changes nothing.
    """
    if semiring not in ("log", "max"):
        raise ValueError(f"semiring must be 'log' or 'max', got {semiring!r}")
    return SemiCRFTritonForward.apply(edge, lengths, use_triton, semiring)


def launch_triton_kernel(edge: Tensor, lengths: Tensor, semiring: str = "log") -> Tensor:
    """Forward only (triton_scan.py:594-656)."""
    part, _ = _lib.edge_scan_forward(edge, lengths, semiring, want_saved=False)
    return part.to(edge.dtype)


def semi_crf_forward_pytorch(edge: Tensor, lengths: Tensor, semiring: str = "log") -> Tensor:
    """The reference's PyTorch scan (triton_scan.py:163), here the CUDA scan with gradients."""
    return semi_crf_triton_forward(edge, lengths, semiring=semiring)
