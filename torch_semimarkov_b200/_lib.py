"""ctypes binding of libsemicrf.so (include/semicrf.h).

This is the only place that touches the C ABI.  Tensors are validated here,
made contiguous, and passed as raw device pointers together with the current
CUDA stream; every buffer (outputs and scratch) is allocated by PyTorch's
caching allocator.  There is no CPU fallback: CPU tensors and a missing
shared library raise.
"""

from __future__ import annotations

import ctypes
import math
import os
from typing import Optional

import torch

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libsemicrf.so")

SEMICRF_OK = 0
SEMICRF_ERR_INVALID_ARGUMENT = 1
SEMICRF_ERR_UNSUPPORTED = 2
SEMICRF_ERR_WORKSPACE = 3
SEMICRF_ERR_CUDA = 4
SEMICRF_ERR_SEMIRING = 5
SEMIRINGS = {"log": 0, "max": 1}
KEEP_ALPHA, RECOMPUTE = 0, 1
# Keep the float64 tables of both chains (alpha, and beta computed beside it
# in the forward launch) for the backward when they fit comfortably in the
# memory this process can still get: below KEEP_ALPHA_ALWAYS_BYTES always;
# above it while they take at most KEEP_ALPHA_FREE_FRACTION of the device's
# free memory plus the caching allocator's unused reserve.  Otherwise the
# forward keeps sqrt(T)-spaced ring checkpoints and the backward recomputes
# alpha between them and runs the beta chain itself.  The environment
# variable TORCH_SEMIMARKOV_B200_BACKWARD=keep|recompute forces one or the
# other.
KEEP_ALPHA_ALWAYS_BYTES = 1 << 30
KEEP_ALPHA_FREE_FRACTION = 0.5


def chunk_warmup_from_env() -> int:
    """Time chunking of the log-semiring chains (semicrf_problem.chunk_warmup):
    TORCH_SEMIMARKOV_B200_CHUNKS=off disables it, =<n> forces it with an
    n-position warm-up, =<n>,<m> with an n-position warm-up and an m-position
    second pass for sequences that do not join; unset or auto lets the
    library decide."""
    env = os.environ.get("TORCH_SEMIMARKOV_B200_CHUNKS", "").lower()
    if env in ("", "auto"):
        return 0
    if env == "off":
        return -1
    first, _, second = env.partition(",")
    n = min(max(1, int(first)), 0xFFFF)
    m = min(max(0, int(second)), 0x7FFF) if second else 0
    return n | (m << 16)


def keep_table_bytes(B: int, T: int, C: int) -> int:
    """Bytes of the float64 tables the keep mode saves: a, A and n per chain."""
    return 16 * B * (T + 1) * (2 * C + 1)


def backward_mode_for(B: int, T: int, C: int, device=None) -> int:
    env = os.environ.get("TORCH_SEMIMARKOV_B200_BACKWARD", "").lower()
    if env == "recompute":
        return RECOMPUTE
    if env == "keep":
        return KEEP_ALPHA
    need = keep_table_bytes(B, T, C)
    if need <= KEEP_ALPHA_ALWAYS_BYTES:
        return KEEP_ALPHA
    if device is None or not torch.cuda.is_available():
        return RECOMPUTE
    free, _ = torch.cuda.mem_get_info(device)
    spare = torch.cuda.memory_reserved(device) - torch.cuda.memory_allocated(device)
    return KEEP_ALPHA if need <= KEEP_ALPHA_FREE_FRACTION * (free + spare) else RECOMPUTE


# every symbol include/semicrf.h declares
EXPORTED_SYMBOLS = (
    "semicrf_checkpoint_interval",
    "semicrf_saved_size",
    "semicrf_forward_workspace_size",
    "semicrf_forward",
    "semicrf_backward_workspace_size",
    "semicrf_backward",
    "semicrf_viterbi_workspace_size",
    "semicrf_viterbi",
    "semicrf_score_gold",
    "semicrf_score_gold_backward",
    "semicrf_score_gold_workspace_size",
    "semicrf_strerror",
    "semicrf_abi_version",
    "semicrf_forward_noalloc",
    "semicrf_edge_scan_saved_size",
    "semicrf_edge_scan_forward",
    "semicrf_edge_scan_backward_workspace_size",
    "semicrf_edge_scan_backward",
)


class SemicrfProblem(ctypes.Structure):
    """Mirror of ``struct semicrf_problem``."""

    _fields_ = [
        ("batch", ctypes.c_int64),
        ("T", ctypes.c_int64),
        ("K", ctypes.c_int64),
        ("C", ctypes.c_int64),
        ("cum_scores", ctypes.c_void_p),
        ("transition", ctypes.c_void_p),
        ("transition_ndim", ctypes.c_int32),
        ("semiring", ctypes.c_int32),
        ("duration_bias", ctypes.c_void_p),
        ("lengths", ctypes.c_void_p),
        ("proj_start", ctypes.c_void_p),
        ("proj_end", ctypes.c_void_p),
        ("checkpoint_interval", ctypes.c_int64),
        ("backward_mode", ctypes.c_int32),
        ("chunk_warmup", ctypes.c_int32),
    ]


_lib = None


def load():
    """Load libsemicrf.so; raise if it has not been built."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        raise RuntimeError(
            f"{LIB_PATH} is missing: build it with `python -m torch_semimarkov_b200.build_ext` "
            "(torch_semimarkov_b200 has no CPU or Triton fallback)")
    lib = ctypes.CDLL(LIB_PATH)
    P = ctypes.POINTER(SemicrfProblem)
    vp, i64, sz, ci = ctypes.c_void_p, ctypes.c_int64, ctypes.c_size_t, ctypes.c_int
    lib.semicrf_checkpoint_interval.restype = i64
    lib.semicrf_checkpoint_interval.argtypes = [i64, i64]
    for name in ("semicrf_saved_size", "semicrf_forward_workspace_size",
                 "semicrf_backward_workspace_size", "semicrf_viterbi_workspace_size"):
        f = getattr(lib, name)
        f.restype = sz
        f.argtypes = [P]
    lib.semicrf_forward.restype = ci
    lib.semicrf_forward.argtypes = [P, vp, vp, i64, vp, vp, sz, vp]
    lib.semicrf_backward.restype = ci
    lib.semicrf_backward.argtypes = [P, vp, vp, vp, vp, vp, vp, vp, vp, sz, vp]
    lib.semicrf_viterbi.restype = ci
    lib.semicrf_viterbi.argtypes = [P, i64, vp, vp, vp, vp, vp, vp, vp, sz, vp]
    lib.semicrf_score_gold.restype = ci
    lib.semicrf_score_gold.argtypes = [i64, i64, i64, i64, vp, vp, vp, vp, vp, vp, vp]
    lib.semicrf_score_gold_backward.restype = ci
    lib.semicrf_score_gold_backward.argtypes = [i64, i64, i64, i64, vp, vp, vp, vp, vp, vp, vp,
                                                sz, vp]
    lib.semicrf_score_gold_workspace_size.restype = sz
    lib.semicrf_score_gold_workspace_size.argtypes = [i64, i64, i64, i64]
    lib.semicrf_strerror.restype = ctypes.c_char_p
    lib.semicrf_strerror.argtypes = [ci]
    lib.semicrf_abi_version.restype = ci
    lib.semicrf_forward_noalloc.restype = ci
    lib.semicrf_forward_noalloc.argtypes = [P, vp, vp]
    for name in ("semicrf_edge_scan_saved_size", "semicrf_edge_scan_backward_workspace_size"):
        f = getattr(lib, name)
        f.restype = sz
        f.argtypes = [i64, i64, i64, i64, ci]
    lib.semicrf_edge_scan_forward.restype = ci
    lib.semicrf_edge_scan_forward.argtypes = [i64, i64, i64, i64, vp, vp, ci, vp, vp, vp]
    lib.semicrf_edge_scan_backward.restype = ci
    lib.semicrf_edge_scan_backward.argtypes = [i64, i64, i64, i64, vp, vp, ci, vp, vp, vp, vp,
                                               sz, vp]
    _lib = lib
    return lib


def check(status: int, what: str):
    if status == SEMICRF_OK:
        return
    msg = f"{what}: {load().semicrf_strerror(status).decode()} (status {status})"
    if status in (SEMICRF_ERR_INVALID_ARGUMENT, SEMICRF_ERR_SEMIRING):
        raise ValueError(msg)
    if status == SEMICRF_ERR_UNSUPPORTED:
        raise NotImplementedError(msg)
    raise RuntimeError(msg)


def checkpoint_interval(T: int, K: int) -> int:
    """_compute_checkpoint_interval (pytorch_reference.py:25-45)."""
    return max(K, int(math.sqrt(T * K)))


def _ptr(t: Optional[torch.Tensor]):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def _stream(device) -> ctypes.c_void_p:
    return ctypes.c_void_p(torch.cuda.current_stream(device).cuda_stream)


def _scratch(nbytes: int, device) -> torch.Tensor:
    return torch.empty(max(int(nbytes), 1), dtype=torch.uint8, device=device)


class Problem:
    """Validated, contiguous inputs of one streaming call plus its C struct."""

    def __init__(self, cum_scores, transition, duration_bias, lengths, K, semiring="log",
                 proj_start=None, proj_end=None, checkpoint_interval_: Optional[int] = None,
                 backward_mode: Optional[int] = None):
        if semiring not in SEMIRINGS:
            raise ValueError(f"semiring must be 'log' or 'max', got {semiring!r}")
        if not isinstance(cum_scores, torch.Tensor) or cum_scores.dim() != 3:
            raise ValueError("cum_scores must be a (batch, T+1, C) tensor")
        if not cum_scores.is_cuda:
            raise RuntimeError("torch_semimarkov_b200 runs on CUDA devices only "
                               "(cum_scores is on the CPU; there is no CPU fallback)")
        dev = cum_scores.device
        B, T1, C = cum_scores.shape
        T = T1 - 1
        K = int(K)
        if T < 0:
            raise ValueError("cum_scores must have at least one row (T+1 >= 1)")
        if K < 1:
            raise ValueError(f"K must be >= 1, got {K}")

        def f32(t, name, shape=None):
            if t is None:
                return None
            if not isinstance(t, torch.Tensor):
                raise ValueError(f"{name} must be a tensor")
            if t.device != dev:
                raise ValueError(f"{name} is on {t.device}, expected {dev}")
            if shape is not None and tuple(t.shape) != tuple(shape):
                raise ValueError(f"{name} has shape {tuple(t.shape)}, expected {tuple(shape)}")
            return t.detach().to(torch.float32).contiguous()

        self.cum = f32(cum_scores, "cum_scores")
        if transition.dim() == 2:
            self.tr = f32(transition, "transition", (C, C))
        elif transition.dim() == 3:
            self.tr = f32(transition, "transition", (K, C, C))
        else:
            raise ValueError("transition must be (C, C) or (K, C, C)")
        self.db = f32(duration_bias, "duration_bias", (K, C))
        self.ps = f32(proj_start, "proj_start", (B, T, C))
        self.pe = f32(proj_end, "proj_end", (B, T, C))
        if not isinstance(lengths, torch.Tensor):
            lengths = torch.as_tensor(lengths)
        if lengths.shape != (B,):
            raise ValueError(f"lengths must have shape ({B},)")
        if lengths.device.type == "cpu" and B > 0:
            lo, hi = int(lengths.min()), int(lengths.max())
            if lo < 0 or hi > T:
                raise ValueError(f"lengths must lie in [0, {T}], got [{lo}, {hi}]")
        self.lengths = lengths.to(device=dev, dtype=torch.int64).contiguous()
        self.B, self.T, self.K, self.C = B, T, K, C
        self.semiring = semiring
        if checkpoint_interval_ is None:
            S = checkpoint_interval(T, K)
        else:
            S = max(int(checkpoint_interval_), K)
        self.S = S
        self.device = dev
        self.backward_mode = (backward_mode_for(B, T, C, dev) if backward_mode is None
                              else int(backward_mode))
        self.c = SemicrfProblem(
            batch=B, T=T, K=K, C=C, cum_scores=self.cum.data_ptr(),
            transition=self.tr.data_ptr(), transition_ndim=self.tr.dim(),
            semiring=SEMIRINGS[semiring], duration_bias=self.db.data_ptr(),
            lengths=self.lengths.data_ptr(),
            proj_start=None if self.ps is None else self.ps.data_ptr(),
            proj_end=None if self.pe is None else self.pe.data_ptr(),
            checkpoint_interval=S, backward_mode=self.backward_mode,
            chunk_warmup=chunk_warmup_from_env())

    @property
    def cref(self):
        return ctypes.byref(self.c)


def forward(prob: Problem, want_saved: bool, num_ring_checkpoints: int = 0):
    """Run semicrf_forward.  Returns (partition, ring_checkpoints or None, saved or None)."""
    lib = load()
    dev = prob.device
    with torch.cuda.device(dev):
        part = torch.empty(prob.B, dtype=torch.float32, device=dev)
        ck = None
        if num_ring_checkpoints > 0:
            ck = torch.empty((prob.B, num_ring_checkpoints, prob.K, prob.C), dtype=torch.float32,
                             device=dev)
        saved = None
        if want_saved:
            n = lib.semicrf_saved_size(prob.cref)
            if n == 0 and prob.B > 0:
                check(SEMICRF_ERR_UNSUPPORTED, "semicrf_saved_size")
            saved = _scratch(n, dev)
        nws = lib.semicrf_forward_workspace_size(prob.cref)
        if nws == 0 and prob.B > 0:
            # validation failed: let semicrf_forward report why
            pass
        ws = _scratch(nws, dev)
        st = lib.semicrf_forward(prob.cref, _ptr(part), _ptr(ck), num_ring_checkpoints,
                                 _ptr(saved), _ptr(ws), ws.numel(), _stream(dev))
        check(st, "semicrf_forward")
    return part, ck, saved


def saved_log_partition(prob: Problem, saved: torch.Tensor) -> torch.Tensor:
    """The float64 log partition (B,) a log-semiring forward stored at the
    start of its saved state (semicrf_saved_size: log Z comes first)."""
    return saved[: 8 * prob.B].view(torch.float64)


def backward(prob: Problem, saved: torch.Tensor, grad_output: torch.Tensor):
    """Run semicrf_backward.  Returns (grad_cum, grad_tr, grad_db, grad_ps, grad_pe)."""
    lib = load()
    dev = prob.device
    with torch.cuda.device(dev):
        g = grad_output.detach().to(device=dev, dtype=torch.float32).contiguous()
        gc = torch.empty_like(prob.cum)
        gt = torch.empty_like(prob.tr)
        gd = torch.empty_like(prob.db)
        gps = torch.empty_like(prob.ps) if prob.ps is not None else None
        gpe = torch.empty_like(prob.pe) if prob.pe is not None else None
        ws = _scratch(lib.semicrf_backward_workspace_size(prob.cref), dev)
        st = lib.semicrf_backward(prob.cref, _ptr(saved), _ptr(g), _ptr(gc), _ptr(gt), _ptr(gd),
                                  _ptr(gps), _ptr(gpe), _ptr(ws), ws.numel(), _stream(dev))
        check(st, "semicrf_backward")
    return gc, gt, gd, gps, gpe


def viterbi(prob: Problem, max_traceback_length: int):
    """Run semicrf_viterbi.  Returns device tensors (scores, starts, ends, labels, seg_scores, nseg)."""
    lib = load()
    dev = prob.device
    with torch.cuda.device(dev):
        B, T = prob.B, max(prob.T, 1)
        scores = torch.empty(B, dtype=torch.float32, device=dev)
        ss = torch.empty((B, T), dtype=torch.int32, device=dev)
        se = torch.empty((B, T), dtype=torch.int32, device=dev)
        sl = torch.empty((B, T), dtype=torch.int32, device=dev)
        sv = torch.empty((B, T), dtype=torch.float64, device=dev)
        ns = torch.empty(B, dtype=torch.int32, device=dev)
        ws = _scratch(lib.semicrf_viterbi_workspace_size(prob.cref), dev)
        st = lib.semicrf_viterbi(prob.cref, int(max_traceback_length), _ptr(scores), _ptr(ss),
                                 _ptr(se), _ptr(sl), _ptr(sv), _ptr(ns), _ptr(ws), ws.numel(),
                                 _stream(dev))
        check(st, "semicrf_viterbi")
    return scores, ss, se, sl, sv, ns


def score_gold(cum, labels, lengths, transition, duration_bias, K):
    lib = load()
    dev = cum.device
    if not cum.is_cuda:
        raise RuntimeError("torch_semimarkov_b200 runs on CUDA devices only")
    B, T1, C = cum.shape
    with torch.cuda.device(dev):
        cum = cum.detach().float().contiguous()
        lab = labels.to(device=dev, dtype=torch.int64).contiguous()
        ln = lengths.to(device=dev, dtype=torch.int64).contiguous()
        tr = transition.detach().float().contiguous()
        db = duration_bias.detach().float().contiguous()
        out = torch.empty(B, dtype=torch.float32, device=dev)
        st = lib.semicrf_score_gold(B, T1 - 1, int(K), C, _ptr(cum), _ptr(lab), _ptr(ln),
                                    _ptr(tr), _ptr(db), _ptr(out), _stream(dev))
        if st == SEMICRF_ERR_INVALID_ARGUMENT and T1 - 1 == 1 and K < 2:
            raise IndexError("index 1 is out of bounds for duration_bias with K < 2")
        check(st, "semicrf_score_gold")
    return out


def score_gold_backward(labels, lengths, grad_out, B, T, K, C, device):
    lib = load()
    with torch.cuda.device(device):
        lab = labels.to(device=device, dtype=torch.int64).contiguous()
        ln = lengths.to(device=device, dtype=torch.int64).contiguous()
        g = grad_out.detach().to(device=device, dtype=torch.float32).contiguous()
        gc = torch.empty((B, T + 1, C), dtype=torch.float32, device=device)
        gt = torch.empty((C, C), dtype=torch.float32, device=device)
        gd = torch.empty((K, C), dtype=torch.float32, device=device)
        ws = _scratch(lib.semicrf_score_gold_workspace_size(B, T, K, C), device)
        st = lib.semicrf_score_gold_backward(B, T, int(K), C, _ptr(lab), _ptr(ln), _ptr(g),
                                             _ptr(gc), _ptr(gt), _ptr(gd), _ptr(ws), ws.numel(),
                                             _stream(device))
        check(st, "semicrf_score_gold_backward")
    return gc, gt, gd


def _edge_inputs(edge, lengths):
    if not isinstance(edge, torch.Tensor) or edge.dim() != 5 or edge.shape[3] != edge.shape[4]:
        raise ValueError("edge must be a (batch, N-1, K, C, C) tensor")
    if not edge.is_cuda:
        raise RuntimeError("torch_semimarkov_b200 runs on CUDA devices only "
                           "(edge is on the CPU; there is no CPU fallback)")
    B, N1, K, C, _ = edge.shape
    if not isinstance(lengths, torch.Tensor):
        lengths = torch.as_tensor(lengths)
    if lengths.shape != (B,):
        raise ValueError(f"lengths must have shape ({B},)")
    e = edge.detach().to(torch.float32).contiguous()
    ln = lengths.to(device=edge.device, dtype=torch.int64).contiguous()
    return e, ln, B, N1 + 1, K, C


def edge_scan_forward(edge, lengths, semiring="log", want_saved=False):
    """semicrf_edge_scan_forward.  Returns (partition float32 (B,), saved or None)."""
    if semiring not in SEMIRINGS:
        raise ValueError(f"semiring must be 'log' or 'max', got {semiring!r}")
    lib = load()
    e, ln, B, N, K, C = _edge_inputs(edge, lengths)
    sr = SEMIRINGS[semiring]
    dev = e.device
    with torch.cuda.device(dev):
        part = torch.empty(B, dtype=torch.float32, device=dev)
        saved = None
        if want_saved:
            n = lib.semicrf_edge_scan_saved_size(B, N, K, C, sr)
            if n == 0 and B > 0:
                check(SEMICRF_ERR_UNSUPPORTED, "semicrf_edge_scan_saved_size")
            saved = _scratch(n, dev)
        st = lib.semicrf_edge_scan_forward(B, N, K, C, _ptr(e), _ptr(ln), sr, _ptr(part),
                                           _ptr(saved), _stream(dev))
        check(st, "semicrf_edge_scan_forward")
    return part, saved


def edge_scan_backward(edge, lengths, semiring, saved, grad_output):
    """semicrf_edge_scan_backward.  Returns grad_edge shaped like edge (float32)."""
    lib = load()
    e, ln, B, N, K, C = _edge_inputs(edge, lengths)
    sr = SEMIRINGS[semiring]
    dev = e.device
    with torch.cuda.device(dev):
        g = grad_output.detach().to(device=dev, dtype=torch.float32).contiguous()
        ge = torch.zeros_like(e)
        ws = _scratch(lib.semicrf_edge_scan_backward_workspace_size(B, N, K, C, sr), dev)
        st = lib.semicrf_edge_scan_backward(B, N, K, C, _ptr(e), _ptr(ln), sr, _ptr(saved),
                                            _ptr(g), _ptr(ge), _ptr(ws), ws.numel(), _stream(dev))
        check(st, "semicrf_edge_scan_backward")
    return ge
