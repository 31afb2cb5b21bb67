"""torch_semimarkov_b200 -- the streaming semi-CRF scan of torch-semimarkov on B200.

A drop-in for the reference's streaming hot path
(``torch_semimarkov.streaming.semi_crf_streaming_forward`` and
``SemiMarkovCRFHead.forward / compute_loss / decode / decode_with_traceback``)
backed by hand-written sm_100a CUDA kernels in libsemicrf.so (C ABI:
include/semicrf.h).  There is no Triton, no backend dispatch and no CPU
fallback.
"""

from .duration import (
    CallableDuration,
    DurationDistribution,
    GeometricDuration,
    LearnedDuration,
    NegativeBinomialDuration,
    PoissonDuration,
    UniformDuration,
    create_duration_distribution,
)
from .helpers import Segment, ViterbiResult, score_gold_vectorized
from .nn import SemiMarkovCRFHead
from .streaming import (
    NEG_INF,
    SemiCRFStreaming,
    SemiCRFStreamingTriton,
    compute_edge_block_streaming,
    launch_streaming_triton_backward,
    launch_streaming_triton_kernel,
    semi_crf_streaming_forward,
)
from .uncertainty import UncertaintyMixin, UncertaintySemiMarkovCRFHead

__version__ = "0.2.0+b200"

__all__ = [
    "SemiMarkovCRFHead",
    "Segment",
    "ViterbiResult",
    "score_gold_vectorized",
    "DurationDistribution",
    "LearnedDuration",
    "GeometricDuration",
    "NegativeBinomialDuration",
    "PoissonDuration",
    "UniformDuration",
    "CallableDuration",
    "create_duration_distribution",
    "semi_crf_streaming_forward",
    "SemiCRFStreaming",
    "SemiCRFStreamingTriton",
    "compute_edge_block_streaming",
    "launch_streaming_triton_kernel",
    "launch_streaming_triton_backward",
    "NEG_INF",
    "UncertaintyMixin",
    "UncertaintySemiMarkovCRFHead",
]
