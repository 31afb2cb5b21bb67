"""ctypes front end of the CPU oracle -- TEST INFRASTRUCTURE ONLY.

The oracle (oracle/semicrf_oracle.c) is a plain-C restatement of the
reference implementation of the streaming semi-CRF scan
(torch-semimarkov 0.2.0, src/torch_semimarkov/streaming/pytorch_reference.py,
nn.py:444-555, helpers.py:365-544).  Only tests/, bench.py's CPU legs and
__graft_entry__.smoke() import this module, and only to check or to time the
reference algorithm on the host.  The product package never imports it.

All functions take and return numpy arrays.  ``dtype`` selects the float64
parity oracle or the float32 CPU baseline.
"""

from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "_build", "libsemicrf_oracle.so")
_lib = None

NEG_INF = -1e9


def build() -> str:
    """Compile the oracle shared library (make -C oracle)."""
    subprocess.run(["make", "-s", "-C", _HERE], check=True)
    return _LIB_PATH


def _load():
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(_LIB_PATH):
        build()
    lib = ctypes.CDLL(_LIB_PATH)
    i64 = ctypes.c_int64
    vp = ctypes.c_void_p
    ci = ctypes.c_int
    lib.oracle_checkpoint_interval.restype = i64
    lib.oracle_checkpoint_interval.argtypes = [i64, i64]
    lib.oracle_num_threads_available.restype = ci
    for sfx in ("f64", "f32"):
        f = getattr(lib, "oracle_forward_" + sfx)
        f.restype = ci
        f.argtypes = [vp, vp, ci, vp, vp, vp, vp, i64, i64, i64, i64, ci, i64, vp, vp, ci]
        f = getattr(lib, "oracle_backward_" + sfx)
        f.restype = ci
        f.argtypes = [vp, vp, ci, vp, vp, vp, vp, i64, i64, i64, i64, ci, vp, vp, i64, i64,
                      vp, vp, vp, vp, vp, ci]
        f = getattr(lib, "oracle_viterbi_" + sfx)
        f.restype = ci
        f.argtypes = [vp, vp, vp, vp, i64, i64, i64, i64, i64, vp, vp, vp, vp, vp, vp, ci]
        f = getattr(lib, "oracle_score_gold_" + sfx)
        f.restype = ci
        f.argtypes = [vp, vp, vp, vp, vp, i64, i64, i64, i64, vp]
    _lib = lib
    return lib


def _ptr(a):
    return None if a is None else a.ctypes.data_as(ctypes.c_void_p)


def _arr(a, dtype):
    if a is None:
        return None
    return np.ascontiguousarray(np.asarray(a), dtype=dtype)


def _sfx(dtype):
    return "f64" if np.dtype(dtype) == np.float64 else "f32"


def max_threads() -> int:
    return int(_load().oracle_num_threads_available())


def checkpoint_interval(T: int, K: int) -> int:
    """_compute_checkpoint_interval (pytorch_reference.py:25-45)."""
    return int(_load().oracle_checkpoint_interval(T, K))


def forward(cum, tr, db, lengths, K, semiring="log", proj_start=None, proj_end=None,
            checkpoint_interval_=None, dtype=np.float64, threads=1):
    """semi_crf_streaming_forward_pytorch (pytorch_reference.py:116-273).

    Returns (partition (B,), ring_checkpoints (B, ceil(T/S), K, C), S).
    """
    lib = _load()
    cum = _arr(cum, dtype)
    B, T1, C = cum.shape
    T = T1 - 1
    tr = _arr(tr, dtype)
    db = _arr(db, dtype)
    lengths = _arr(lengths, np.int64)
    ps = _arr(proj_start, dtype)
    pe = _arr(proj_end, dtype)
    if checkpoint_interval_ is None:
        S = checkpoint_interval(T, K)
    else:
        S = max(int(checkpoint_interval_), K)
    N = (T + S - 1) // S
    part = np.empty(B, dtype=dtype)
    ck = np.empty((B, N, K, C), dtype=dtype)
    rc = getattr(lib, "oracle_forward_" + _sfx(dtype))(
        _ptr(cum), _ptr(tr), tr.ndim, _ptr(db), _ptr(lengths), _ptr(ps), _ptr(pe),
        B, T, K, C, 0 if semiring == "log" else 1, S, _ptr(part), _ptr(ck), threads)
    if rc != 0:
        raise ValueError(f"oracle_forward failed rc={rc}")
    return part, ck, S


def backward(cum, tr, db, lengths, K, log_Z, ring_ckpts, S, semiring="log",
             proj_start=None, proj_end=None, dtype=np.float64, threads=1):
    """semi_crf_streaming_backward_pytorch (pytorch_reference.py:276-525).

    Returns per-batch gradients (grad_cum, grad_tr, grad_db, grad_ps, grad_pe)
    exactly as the reference does (shared-parameter grads NOT yet reduced).
    """
    lib = _load()
    cum = _arr(cum, dtype)
    B, T1, C = cum.shape
    T = T1 - 1
    tr = _arr(tr, dtype)
    db = _arr(db, dtype)
    lengths = _arr(lengths, np.int64)
    ps = _arr(proj_start, dtype)
    pe = _arr(proj_end, dtype)
    lz = _arr(log_Z, dtype)
    ck = _arr(ring_ckpts, dtype)
    N = ck.shape[1]
    gc = np.empty((B, T + 1, C), dtype=dtype)
    gt = np.empty((B,) + tr.shape, dtype=dtype)
    gd = np.empty((B, K, C), dtype=dtype)
    gps = np.empty((B, T, C), dtype=dtype) if ps is not None else None
    gpe = np.empty((B, T, C), dtype=dtype) if pe is not None else None
    rc = getattr(lib, "oracle_backward_" + _sfx(dtype))(
        _ptr(cum), _ptr(tr), tr.ndim, _ptr(db), _ptr(lengths), _ptr(ps), _ptr(pe),
        B, T, K, C, 0 if semiring == "log" else 1, _ptr(lz), _ptr(ck), N, S,
        _ptr(gc), _ptr(gt), _ptr(gd), _ptr(gps), _ptr(gpe), threads)
    if rc != 0:
        raise ValueError(f"oracle_backward failed rc={rc}")
    return gc, gt, gd, gps, gpe


def forward_backward(cum, tr, db, lengths, K, grad_output=None, semiring="log",
                     proj_start=None, proj_end=None, dtype=np.float64, threads=1):
    """SemiCRFStreaming.forward + backward (streaming/autograd.py:55-161).

    Shared-parameter gradients are reduced with grad_output as in
    autograd.py:134-150.  Returns (partition, grads dict).
    """
    part, ck, S = forward(cum, tr, db, lengths, K, semiring, proj_start, proj_end,
                          dtype=dtype, threads=threads)
    gc, gt, gd, gps, gpe = backward(cum, tr, db, lengths, K, part, ck, S, semiring,
                                    proj_start, proj_end, dtype=dtype, threads=threads)
    B = part.shape[0]
    g = np.ones(B, dtype=dtype) if grad_output is None else np.asarray(grad_output, dtype)
    out = {
        "cum_scores": gc * g[:, None, None],
        "transition": np.tensordot(g, gt, axes=(0, 0)),
        "duration_bias": np.tensordot(g, gd, axes=(0, 0)),
        "proj_start": None if gps is None else gps * g[:, None, None],
        "proj_end": None if gpe is None else gpe * g[:, None, None],
    }
    return part, out


def viterbi(cum, tr, db, lengths, K, max_traceback_length=10000, dtype=np.float64, threads=1):
    """SemiMarkovCRFHead.decode_with_traceback core (nn.py:360-555).

    Returns (scores (B,), segments list[list[(start, end, label, score)]]).
    """
    lib = _load()
    cum = _arr(cum, dtype)
    B, T1, C = cum.shape
    T = T1 - 1
    tr = _arr(tr, dtype)
    db = _arr(db, dtype)
    lengths = _arr(lengths, np.int64)
    sc = np.empty(B, dtype=dtype)
    Tm = max(T, 1)
    ss = np.zeros((B, Tm), np.int64)
    se = np.zeros((B, Tm), np.int64)
    sl = np.zeros((B, Tm), np.int64)
    sv = np.zeros((B, Tm), np.float64)
    ns = np.zeros(B, np.int64)
    rc = getattr(lib, "oracle_viterbi_" + _sfx(dtype))(
        _ptr(cum), _ptr(tr), _ptr(db), _ptr(lengths), B, T, K, C, max_traceback_length,
        _ptr(sc), _ptr(ss), _ptr(se), _ptr(sl), _ptr(sv), _ptr(ns), threads)
    if rc != 0:
        raise ValueError(f"oracle_viterbi failed rc={rc}")
    segs = []
    for b in range(B):
        n = int(ns[b])
        segs.append([(int(ss[b, i]), int(se[b, i]), int(sl[b, i]), float(sv[b, i]))
                     for i in range(n)])
    return sc, segs


def score_gold(cum, labels, lengths, tr, db, K, dtype=np.float64):
    """score_gold_vectorized (helpers.py:365-544)."""
    lib = _load()
    cum = _arr(cum, dtype)
    B, T1, C = cum.shape
    T = T1 - 1
    labels = _arr(labels, np.int64)
    lengths = _arr(lengths, np.int64)
    tr = _arr(tr, dtype)
    db = _arr(db, dtype)
    out = np.empty(B, dtype=dtype)
    rc = getattr(lib, "oracle_score_gold_" + _sfx(dtype))(
        _ptr(cum), _ptr(labels), _ptr(lengths), _ptr(tr), _ptr(db), B, T, K, C, _ptr(out))
    if rc != 0:
        raise IndexError("duration_bias[1] is out of range for K < 2 at T == 1")
    return out
