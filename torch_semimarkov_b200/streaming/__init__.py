"""Streaming semi-CRF on B200: the public surface of the reference's
``torch_semimarkov.streaming`` package (streaming/__init__.py:136-177)."""

from .autograd import (
    HAS_TRITON,
    SemiCRFStreaming,
    SemiCRFStreamingTriton,
    launch_streaming_triton_backward,
    launch_streaming_triton_kernel,
    semi_crf_streaming_forward,
)
from .constants import NEG_INF
from .edge import _compute_checkpoint_interval, compute_edge_block_streaming

__all__ = [
    "semi_crf_streaming_forward",
    "SemiCRFStreaming",
    "SemiCRFStreamingTriton",
    "compute_edge_block_streaming",
    "_compute_checkpoint_interval",
    "NEG_INF",
    "HAS_TRITON",
    "launch_streaming_triton_backward",
    "launch_streaming_triton_kernel",
]
