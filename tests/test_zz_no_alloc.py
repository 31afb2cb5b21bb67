"""semicrf_forward_noalloc (the allocation-free partition entry point).

Called through the C ABI (ctypes) and compared with semicrf_forward on the
same problem, on calls in a row with different inputs, so a second call cannot
pass on scratch left over from the first.  The file sorts last so the entry
point is also exercised after every other test has used the device.
"""

import ctypes

import numpy as np
import pytest
import torch

from golden.inputs import make_streaming_inputs

RTOL = 1e-5


def _lib():
    from torch_semimarkov_b200 import _lib

    return _lib


def _problem(B, T, K, C, seed, semiring, gen="default", proj=None, kcc=False):
    L = _lib()
    dev = torch.device("cuda:0")
    inp = make_streaming_inputs(B, T, K, C, seed, gen=gen, proj=proj, kcc=kcc)
    g = torch.Generator().manual_seed(seed + 7)
    lengths = torch.randint(max(1, T // 2), T + 1, (B,), generator=g)
    lengths[0] = T
    return L.Problem(inp["cum_scores"].to(dev), inp["transition"].to(dev),
                     inp["duration_bias"].to(dev), lengths.to(dev), K, semiring=semiring,
                     proj_start=None if inp.get("proj_start") is None
                     else inp["proj_start"].to(dev),
                     proj_end=None if inp.get("proj_end") is None else inp["proj_end"].to(dev))


def _noalloc(prob):
    L = _lib()
    lib = L.load()
    part = torch.full((prob.B,), float("nan"), dtype=torch.float32, device=prob.device)
    st = lib.semicrf_forward_noalloc(prob.cref, ctypes.c_void_p(part.data_ptr()),
                                     ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    L.check(st, "semicrf_forward_noalloc")
    return part


@pytest.mark.gpu
@pytest.mark.parametrize("semiring", ["log", "max"])
def test_noalloc_matches_forward_two_calls(semiring):
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    L = _lib()
    cases = [(_problem(4, 300, 40, 24, 11, semiring, gen="cfg2"), "cfg2"),
             (_problem(3, 200, 12, 7, 12, semiring, proj="both"), "proj"),
             (_problem(2, 150, 64, 256, 13, semiring, gen="cfg4"), "c256"),
             # duration-dependent (K, C, C) transitions: their per-duration
             # factor tables and the blocked chain's overflow flag live in the
             # same scratch
             (_problem(3, 90, 12, 8, 14, semiring, kcc=True), "kcc")]
    for prob, what in cases:
        got = _noalloc(prob)
        ref, _, _ = L.forward(prob, want_saved=False)
        torch.cuda.synchronize()
        got = got.cpu().double().numpy()
        ref = ref.cpu().double().numpy()
        assert np.isfinite(got).all(), what
        err = np.abs(got - ref)
        assert (err <= RTOL * np.abs(ref) + 1e-5).all(), f"{semiring}/{what}: {err.max():.3e}"


def _shape(**kw):
    L = _lib()
    base = dict(batch=0, T=1000, K=4, C=3, transition_ndim=2, semiring=0,
                checkpoint_interval=1000, backward_mode=0)
    base.update(kw)
    return L.SemicrfProblem(**base)


def test_noalloc_size_checks_without_gpu():
    """Needs no GPU: validation and the scratch-size check precede any CUDA call."""
    L = _lib()
    lib = L.load()
    # every shape the scan accepts fits the 2 MiB scratch: for each C the
    # largest accepted K (found by bisection) needs the most
    for C in (1, 8, 24, 64, 128, 256):
        lo, hi = 1, 32767
        while lo < hi:
            mid = (lo + hi + 1) // 2
            p = _shape(C=C, K=mid, checkpoint_interval=max(mid, 1000))
            if lib.semicrf_forward_workspace_size(ctypes.byref(p)) > 0:
                lo = mid
            else:
                hi = mid - 1
        p = _shape(C=C, K=lo, checkpoint_interval=max(lo, 1000))
        need = lib.semicrf_forward_workspace_size(ctypes.byref(p))
        assert 0 < need <= (2 << 20), (C, lo, need)
        assert lib.semicrf_forward_noalloc(ctypes.byref(p), None, None) == L.SEMICRF_OK
        big = _shape(C=C, K=lo + 1, checkpoint_interval=max(lo + 1, 1000))
        want = lib.semicrf_forward(ctypes.byref(big), None, None, 0, None, None, 0, None)
        assert want != L.SEMICRF_OK and lib.semicrf_forward_noalloc(ctypes.byref(big), None,
                                                                    None) == want
    # (K, C, C) transitions: the per-duration tables grow as K*C*C, so a shape
    # just past 2 MiB of forward workspace is refused with SEMICRF_ERR_WORKSPACE
    # (before any device work), and the one just below it is accepted
    for semiring in (0, 1):
        C = 16
        lo, hi = 2, 1024
        while lo < hi:
            mid = (lo + hi + 1) // 2
            p = _shape(C=C, K=mid, transition_ndim=3, semiring=semiring,
                       checkpoint_interval=max(mid, 1000))
            if 0 < lib.semicrf_forward_workspace_size(ctypes.byref(p)) <= (2 << 20):
                lo = mid
            else:
                hi = mid - 1
        ok = _shape(C=C, K=lo, transition_ndim=3, semiring=semiring,
                    checkpoint_interval=max(lo, 1000))
        assert 0 < lib.semicrf_forward_workspace_size(ctypes.byref(ok)) <= (2 << 20)
        assert lib.semicrf_forward_noalloc(ctypes.byref(ok), None, None) == L.SEMICRF_OK
        # a one-sequence problem, so that the calls get past the empty-batch
        # return; its pointers are host addresses that are never dereferenced,
        # because both calls stop at the workspace check, before any CUDA call
        host = (ctypes.c_double * 4)()
        addr = ctypes.addressof(host)
        big = _shape(C=C, K=lo + 1, transition_ndim=3, semiring=semiring,
                     checkpoint_interval=max(lo + 1, 1000), batch=1, cum_scores=addr,
                     transition=addr, duration_bias=addr, lengths=addr)
        assert lib.semicrf_forward_workspace_size(ctypes.byref(big)) > (2 << 20)
        # semicrf_forward itself accepts the shape (it only lacks a workspace)
        assert lib.semicrf_forward(ctypes.byref(big), ctypes.c_void_p(addr), None, 0, None,
                                   None, 0, None) == L.SEMICRF_ERR_WORKSPACE
        assert lib.semicrf_forward_noalloc(ctypes.byref(big), ctypes.c_void_p(addr),
                                           None) == L.SEMICRF_ERR_WORKSPACE, semiring
    # shapes the scan rejects get semicrf_forward's code, before any device work
    for kw in [dict(K=0), dict(semiring=7), dict(C=300), dict(batch=2)]:
        p = _shape(**kw)
        want = lib.semicrf_forward(ctypes.byref(p), None, None, 0, None, None, 0, None)
        assert want != L.SEMICRF_OK, kw
        assert lib.semicrf_forward_noalloc(ctypes.byref(p), None, None) == want, kw
