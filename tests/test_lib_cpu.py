"""CPU-only checks of the C ABI library and the host-side logic (no GPU calls)."""

import ctypes
import os
import re

import pytest
import torch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _declared_symbols():
    src = open(os.path.join(ROOT, "include", "semicrf.h")).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    names = re.findall(r"\b(semicrf_[a-z_]+)\s*\(", src)
    return sorted(set(names))


def test_library_exports_every_declared_symbol():
    from torch_semimarkov_b200 import _lib

    lib = _lib.load()
    declared = _declared_symbols()
    assert len(declared) >= 12
    for name in declared:
        assert hasattr(lib, name), name
    assert sorted(_lib.EXPORTED_SYMBOLS) == declared


def test_abi_helpers():
    from torch_semimarkov_b200 import _lib

    lib = _lib.load()
    assert lib.semicrf_abi_version() == 1
    assert lib.semicrf_checkpoint_interval(10000, 300) == 1732
    assert lib.semicrf_checkpoint_interval(1_000_000, 1000) == 31622
    assert lib.semicrf_checkpoint_interval(5, 50) == 50
    assert lib.semicrf_strerror(0) == b"ok"
    assert b"semiring" in lib.semicrf_strerror(5)
    for T, K in [(10000, 300), (4096, 64), (7, 3)]:
        assert _lib.checkpoint_interval(T, K) == lib.semicrf_checkpoint_interval(T, K)


def _problem(**kw):
    from torch_semimarkov_b200 import _lib

    base = dict(batch=0, T=10, K=4, C=3, transition_ndim=2, semiring=0, checkpoint_interval=6,
                backward_mode=0)
    base.update(kw)
    return _lib.SemicrfProblem(**base)


def test_validation_codes_without_gpu():
    """Argument validation happens before any CUDA call."""
    from torch_semimarkov_b200 import _lib

    lib = _lib.load()
    p = _problem()  # batch 0: nothing to do
    assert lib.semicrf_forward(ctypes.byref(p), None, None, 0, None, None, 0, None) == 0
    p = _problem(K=0)
    assert lib.semicrf_forward(ctypes.byref(p), None, None, 0, None, None, 0, None) == 1
    p = _problem(semiring=7)
    assert lib.semicrf_forward(ctypes.byref(p), None, None, 0, None, None, 0, None) == 5
    p = _problem(checkpoint_interval=2)  # S < K
    assert lib.semicrf_forward(ctypes.byref(p), None, None, 0, None, None, 0, None) == 1
    p = _problem(C=300)
    assert lib.semicrf_forward(ctypes.byref(p), None, None, 0, None, None, 0, None) == 2
    p = _problem(batch=2)  # null tensors
    assert lib.semicrf_forward(ctypes.byref(p), None, None, 0, None, None, 0, None) == 1
    assert lib.semicrf_saved_size(ctypes.byref(_problem(K=0))) == 0
    assert lib.semicrf_backward_workspace_size(ctypes.byref(_problem(batch=2))) > 0
    assert lib.semicrf_score_gold(2, 1, 1, 3, None, None, None, None, None, None, None) == 1
    p = _problem(backward_mode=5)
    assert lib.semicrf_forward(ctypes.byref(p), None, None, 0, None, None, 0, None) == 1


def test_workspace_sizes_scale():
    from torch_semimarkov_b200 import _lib

    lib = _lib.load()
    # recompute mode: the backward workspace holds the recomputed alpha tables
    small = lib.semicrf_backward_workspace_size(ctypes.byref(_problem(batch=2, T=100,
                                                                      backward_mode=1)))
    big = lib.semicrf_backward_workspace_size(ctypes.byref(_problem(batch=4, T=1000,
                                                                    backward_mode=1)))
    assert big > 10 * small
    # max semiring keeps its float32 tables in the workspace
    mbig = lib.semicrf_backward_workspace_size(ctypes.byref(_problem(batch=4, T=1000, semiring=1)))
    assert mbig > 4 * 1001 * 3 * 4 * 4
    keep = lib.semicrf_saved_size(ctypes.byref(_problem(batch=3, T=1000, K=30, C=24,
                                                       checkpoint_interval=173)))
    rec = lib.semicrf_saved_size(ctypes.byref(_problem(batch=3, T=1000, K=30, C=24,
                                                      checkpoint_interval=173, backward_mode=1)))
    # keep-alpha holds float64 tables (2*C+1 doubles per position); recompute
    # holds ~T/S' ring checkpoints of K*C doubles
    assert keep >= 8 * 3 * 1001 * 49
    assert rec < keep / 3


def test_cpu_tensors_raise_no_fallback():
    from torch_semimarkov_b200 import semi_crf_streaming_forward

    cum = torch.zeros(1, 5, 2)
    with pytest.raises(RuntimeError, match="CUDA"):
        semi_crf_streaming_forward(cum, torch.zeros(2, 2), torch.zeros(3, 2),
                                   torch.tensor([4]), 3)


def test_bad_semiring_raises():
    from torch_semimarkov_b200 import semi_crf_streaming_forward

    with pytest.raises(ValueError, match="semiring"):
        semi_crf_streaming_forward(torch.zeros(1, 5, 2), torch.zeros(2, 2), torch.zeros(3, 2),
                                   torch.tensor([4]), 3, semiring="sum")


def test_edge_block_helper_matches_oracle_formula():
    from torch_semimarkov_b200 import compute_edge_block_streaming
    from torch_semimarkov_b200.streaming import _compute_checkpoint_interval

    g = torch.Generator().manual_seed(0)
    cum = torch.randn(2, 9, 3, generator=g)
    tr = torch.randn(3, 3, generator=g)
    db = torch.randn(4, 3, generator=g)
    ps = torch.randn(2, 8, 3, generator=g)
    e = compute_edge_block_streaming(cum, tr, db, 2, 3, proj_start=ps)
    want = (cum[:, 5] - cum[:, 2] + db[3] + ps[:, 2]).unsqueeze(-1) + tr.T.unsqueeze(0)
    torch.testing.assert_close(e, want)
    # K=1 clamps the duration index to 0
    e1 = compute_edge_block_streaming(cum, tr, db[:1], 0, 1)
    torch.testing.assert_close(e1, (cum[:, 1] - cum[:, 0] + db[0]).unsqueeze(-1) + tr.T)
    assert _compute_checkpoint_interval(10000, 300) == 1732


def test_lib_has_no_oracle_dependency():
    """The product package must not import or link the oracle."""
    pkg = os.path.join(ROOT, "torch_semimarkov_b200")
    for dirpath, _, files in os.walk(pkg):
        for f in files:
            if f.endswith((".py", ".cu", ".cuh", ".h")):
                txt = open(os.path.join(dirpath, f)).read()
                assert "oracle" not in txt.lower().replace("oracles", ""), f


def test_kcc_shapes_and_sizes():
    """(K, C, C) transitions: accepted shapes, saved tables, rejections."""
    from torch_semimarkov_b200 import _lib

    lib = _lib.load()
    B, T, K, C = 2, 100, 6, 5
    p = _problem(batch=B, T=T, K=K, C=C, transition_ndim=3)
    # saved: log Z, log alpha, the row maxima of alpha and log beta (float64)
    n = B * (T + 1)
    assert lib.semicrf_saved_size(ctypes.byref(p)) >= 8 * (B + 2 * n * C + n)
    # forward workspace: exp(tr) factors in both directions plus three (K, C) tables
    assert lib.semicrf_forward_workspace_size(ctypes.byref(p)) >= 8 * (2 * K * C * C + 3 * K * C)
    assert lib.semicrf_backward_workspace_size(ctypes.byref(p)) >= 8 * 2 * n * C
    # transition[k] is read for k = 1 .. K-1, so K = 1 has no usable matrix
    p1 = _problem(batch=B, T=T, K=1, C=C, transition_ndim=3, checkpoint_interval=10)
    assert lib.semicrf_forward_workspace_size(ctypes.byref(p1)) == 0
    assert lib.semicrf_forward(ctypes.byref(p1), None, None, 0, None, None, 0, None) == 2
    # the Viterbi head takes (C, C) transitions only
    pv = _problem(batch=B, T=T, K=K, C=C, transition_ndim=3, semiring=1)
    assert lib.semicrf_viterbi_workspace_size(ctypes.byref(pv)) == 0
    # a ring window too large for one CTA's shared memory is refused up front
    big = _problem(batch=B, T=T, K=2000, C=64, transition_ndim=3, checkpoint_interval=2000)
    assert lib.semicrf_forward(ctypes.byref(big), None, None, 0, None, None, 0, None) == 2
