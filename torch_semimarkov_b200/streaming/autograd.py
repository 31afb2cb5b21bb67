"""Autograd functions and the public entry point of the streaming semi-CRF.

Mirrors streaming/autograd.py of torch-semimarkov 0.2.0 (the drop-in
boundary): ``semi_crf_streaming_forward`` keeps its signature and semantics
(:270-431); ``use_triton`` / ``use_compile`` are accepted and ignored because
there is exactly one backend -- the sm_100a kernels of libsemicrf.so.
``SemiCRFStreaming`` and ``SemiCRFStreamingTriton`` are the same
autograd.Function (the reference has a PyTorch one and a Triton one,
:33-267).  The launcher names of the reference's Triton path
(``launch_streaming_triton_kernel`` / ``launch_streaming_triton_backward``,
triton_forward.py:554 / triton_backward.py:556) are kept with their return
conventions so callers and tests written against them run unchanged.
"""

from __future__ import annotations

import weakref
from typing import Optional

import torch

from .. import _lib

HAS_TRITON = True  # kept for API compatibility: the launcher names below exist


class SemiCRFStreaming(torch.autograd.Function):
    """Streaming semi-CRF log-partition (or max score) with a checkpointed backward.

    Forward (log semiring): the alpha chain and the beta chain of every
    sequence run side by side in one launch (one CTA per chain, the O(K*C)
    ring on chip) and keep their float64 tables; when those tables would be
    too large, the forward keeps normalised ring checkpoints every S' >= S =
    max(K, sqrt(T*K)) instead and the backward recomputes alpha between them
    and runs the beta chains.  Backward: every gradient is a parallel map or
    reduction over the tables.  Shared-parameter gradients are
    sum_b grad_output[b] * marginals_b (reference autograd.py:134-145).
    """

    @staticmethod
    def forward(ctx, cum_scores, transition, duration_bias, lengths, K, semiring="log",
                proj_start=None, proj_end=None):
        prob = _lib.Problem(cum_scores, transition, duration_bias, lengths, K, semiring,
                            proj_start, proj_end)
        partition, _, saved = _lib.forward(prob, want_saved=True)
        ctx.prob = prob
        ctx.saved_state = saved
        ctx.in_dtypes = (cum_scores.dtype, transition.dtype, duration_bias.dtype,
                         None if proj_start is None else proj_start.dtype,
                         None if proj_end is None else proj_end.dtype)
        return partition.to(cum_scores.dtype)

    @staticmethod
    def backward(ctx, grad_output):
        prob = ctx.prob
        gc, gt, gd, gps, gpe = _lib.backward(prob, ctx.saved_state, grad_output)
        dts = ctx.in_dtypes
        gc = gc.to(dts[0])
        gt = gt.to(dts[1])
        gd = gd.to(dts[2])
        if gps is not None:
            gps = gps.to(dts[3])
        if gpe is not None:
            gpe = gpe.to(dts[4])
        ctx.prob = None
        ctx.saved_state = None
        return gc, gt, gd, None, None, None, gps, gpe


SemiCRFStreamingTriton = SemiCRFStreaming


def semi_crf_streaming_forward(
    cum_scores: torch.Tensor,
    transition: torch.Tensor,
    duration_bias: torch.Tensor,
    lengths: torch.Tensor,
    K: int,
    semiring: str = "log",
    proj_start: Optional[torch.Tensor] = None,
    proj_end: Optional[torch.Tensor] = None,
    use_triton: bool = True,
    use_compile: bool = False,
) -> torch.Tensor:
    """Semi-CRF partition function (log) or best score (max) with streaming
    edges, shape (batch,).  Same arguments as the reference
    (streaming/autograd.py:270-431):

    cum_scores (batch, T+1, C) float32 prefix sums of the projected scores;
    transition (C, C) [src, dst] or (K, C, C); duration_bias (K, C);
    lengths (batch,); K max duration (durations 1..max(1, K-1));
    semiring "log" | "max"; proj_start / proj_end (batch, T, C) optional.
    ``use_triton`` and ``use_compile`` are ignored (one backend).
    """
    if semiring not in ("log", "max"):
        raise ValueError(f"semiring must be 'log' or 'max', got {semiring!r}")
    needs_grad = (
        cum_scores.requires_grad
        or transition.requires_grad
        or duration_bias.requires_grad
        or (proj_start is not None and proj_start.requires_grad)
        or (proj_end is not None and proj_end.requires_grad)
    )
    if needs_grad and torch.is_grad_enabled():
        return SemiCRFStreaming.apply(cum_scores, transition, duration_bias, lengths, K,
                                      semiring, proj_start, proj_end)
    prob = _lib.Problem(cum_scores, transition, duration_bias, lengths, K, semiring,
                        proj_start, proj_end)
    partition, _, _ = _lib.forward(prob, want_saved=False)
    return partition.to(cum_scores.dtype)


# Forward state of launch_streaming_triton_kernel calls, keyed by the ring
# checkpoint tensor each returned: launch_streaming_triton_backward called with
# that tensor (and unchanged inputs) uses it instead of recomputing the chains.
# An entry lives as long as its ring checkpoint tensor (keyed by identity:
# tensors compare elementwise, so they cannot be dictionary keys themselves).
_LAUNCHER_STATE: dict = {}


def _input_key(*ts):
    """Identity and version of the tensors a forward read: equal keys mean the
    same storage, not written since."""
    return tuple(None if t is None else (t.data_ptr(), tuple(t.shape), t.dtype, t._version)
                 for t in ts)


def launch_streaming_triton_kernel(cum_scores, transition, duration_bias, lengths, K,
                                   semiring="log", checkpoint_interval=None, proj_start=None,
                                   proj_end=None):
    """Forward launcher with the reference Triton launcher's contract
    (triton_forward.py:554-714): returns (partition (B,), ring_checkpoints
    (B, ceil(T/S)+1, K, C), S).  Checkpoint i holds the ring of alpha after
    position i*S (slot p % K holds alpha[p]); unset entries are NEG_INF.

    In the log semiring the launch also keeps this library's float64 backward
    state (the chain tables, or restart records when those would not fit in
    memory), tied to the returned ring checkpoint tensor, so that
    launch_streaming_triton_backward given that tensor runs no forward again."""
    prob = _lib.Problem(cum_scores, transition, duration_bias, lengths, K, semiring,
                        proj_start, proj_end, checkpoint_interval)
    n = (prob.T + prob.S - 1) // prob.S + 1
    log = semiring == "log"
    partition, ck, saved = _lib.forward(prob, want_saved=log, num_ring_checkpoints=n)
    if log and ck is not None:
        _LAUNCHER_STATE[id(ck)] = (weakref.ref(ck), _input_key(cum_scores, transition,
                                                               duration_bias, lengths,
                                                               proj_start, proj_end),
                                   prob, saved)
        weakref.finalize(ck, _LAUNCHER_STATE.pop, id(ck), None)
    return partition, ck, prob.S


def launch_streaming_triton_backward(cum_scores, transition, duration_bias, lengths, log_Z,
                                     ring_checkpoints, checkpoint_interval, grad_output,
                                     proj_start=None, proj_end=None):
    """Backward launcher with the reference contract (triton_backward.py:556-790):
    returns (grad_cum, grad_transition, grad_duration_bias, grad_proj_start,
    grad_proj_end), shared-parameter gradients already reduced with
    grad_output.  K is taken from duration_bias.shape[0].

    The caller's forward outputs are checked, not trusted:
      * ``ring_checkpoints`` must have the launcher's layout (batch,
        ceil(T/S) + 1, K, C) for S = ``checkpoint_interval`` (S >= K), else
        ValueError;
      * ``log_Z`` (batch,) must agree with this call's float64 log partition to
        float32 rounding (1e-4 relative), else ValueError: the checkpoints and
        log Z then belong to other inputs.
    The gradients come from this library's float64 state: the state that
    launch_streaming_triton_kernel kept beside these ring checkpoints when they
    come from it and the inputs are unchanged (no forward runs), else state
    recomputed from the inputs.  The float32 checkpoint values themselves are
    not used: absolute log-alpha values in float32 carry rounding of
    |log alpha| * 6e-8 (about 2e-3 at T = 10^4), which the 1e-5 gradient
    contract cannot absorb -- the reference's own tests compare its Triton
    gradients at 1e-2."""
    K = duration_bias.shape[0]
    prob = _lib.Problem(cum_scores, transition, duration_bias, lengths, K, "log",
                        proj_start, proj_end, checkpoint_interval)
    n_ck = (prob.T + prob.S - 1) // prob.S + 1
    want = (prob.B, n_ck, K, prob.C)
    if not isinstance(ring_checkpoints, torch.Tensor) or tuple(ring_checkpoints.shape) != want:
        got = tuple(ring_checkpoints.shape) if isinstance(ring_checkpoints, torch.Tensor) else None
        raise ValueError(f"ring_checkpoints must have shape {want} (batch, ceil(T/S)+1, K, C) "
                         f"for checkpoint_interval S={prob.S}, got {got}")
    if not isinstance(log_Z, torch.Tensor) or tuple(log_Z.shape) != (prob.B,):
        raise ValueError(f"log_Z must have shape ({prob.B},)")
    kept = _LAUNCHER_STATE.get(id(ring_checkpoints))
    key = _input_key(cum_scores, transition, duration_bias, lengths, proj_start, proj_end)
    if (kept is not None and kept[0]() is ring_checkpoints and kept[1] == key
            and kept[2].S == prob.S):
        _, _, prob, saved = kept
        partition = _lib.saved_log_partition(prob, saved)
    else:
        partition, _, saved = _lib.forward(prob, want_saved=True)
    lz = log_Z.detach().to(device=partition.device, dtype=torch.float64)
    ours = partition.double()
    bad = (lz - ours).abs() > 1e-4 * ours.abs() + 1e-3
    if bool(bad.any()):
        i = int(bad.nonzero()[0])
        raise ValueError(f"log_Z[{i}] = {float(lz[i])!r} does not match the log partition of "
                         f"these inputs ({float(ours[i])!r}): the checkpoints and log Z come "
                         "from other inputs")
    return _lib.backward(prob, saved, grad_output)
