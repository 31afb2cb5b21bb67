"""Host-side choices of the Python layer, checked without a GPU: the backward
mode from the memory the process can still get, the time-chunk environment
switch, and the checkpoint interval of the reference
(pytorch_reference.py:25-45)."""

import pytest
import torch

from torch_semimarkov_b200 import _lib


@pytest.fixture
def fake_cuda(monkeypatch):
    """A fake device with `free` bytes free and `spare` bytes reserved but unused."""
    state = {"free": 0, "spare": 0}
    monkeypatch.delenv("TORCH_SEMIMARKOV_B200_BACKWARD", raising=False)
    monkeypatch.setattr(torch.cuda, "is_available", lambda: True)
    monkeypatch.setattr(torch.cuda, "mem_get_info", lambda dev=None: (state["free"], 1 << 40))
    monkeypatch.setattr(torch.cuda, "memory_reserved", lambda dev=None: state["spare"])
    monkeypatch.setattr(torch.cuda, "memory_allocated", lambda dev=None: 0)
    return state


def test_keep_table_bytes_formula():
    # a, A (float64, C each) and the normaliser n per row, both chains
    B, T, C = 64, 10_000, 24
    assert _lib.keep_table_bytes(B, T, C) == 16 * B * (T + 1) * (2 * C + 1)


def test_small_tables_are_always_kept(fake_cuda):
    fake_cuda["free"] = 0  # nothing free: still kept below the fixed size
    B, T, C = 2, 100, 8
    assert _lib.keep_table_bytes(B, T, C) <= _lib.KEEP_ALPHA_ALWAYS_BYTES
    assert _lib.backward_mode_for(B, T, C, device="cuda:0") == _lib.KEEP_ALPHA


def test_large_tables_follow_free_memory(fake_cuda):
    B, T, C = 64, 10_000, 256
    need = _lib.keep_table_bytes(B, T, C)
    assert need > _lib.KEEP_ALPHA_ALWAYS_BYTES
    fake_cuda["free"] = 2 * need  # exactly the fraction allowed
    assert _lib.backward_mode_for(B, T, C, device="cuda:0") == _lib.KEEP_ALPHA
    fake_cuda["free"] = 2 * need - 1024
    assert _lib.backward_mode_for(B, T, C, device="cuda:0") == _lib.RECOMPUTE
    # the caching allocator's unused reserve counts as available
    fake_cuda["spare"] = 4096
    assert _lib.backward_mode_for(B, T, C, device="cuda:0") == _lib.KEEP_ALPHA


def test_backward_mode_environment_override(fake_cuda, monkeypatch):
    B, T, C = 2, 100, 8
    monkeypatch.setenv("TORCH_SEMIMARKOV_B200_BACKWARD", "recompute")
    assert _lib.backward_mode_for(B, T, C, device="cuda:0") == _lib.RECOMPUTE
    monkeypatch.setenv("TORCH_SEMIMARKOV_B200_BACKWARD", "keep")
    fake_cuda["free"] = 0
    assert _lib.backward_mode_for(64, 10_000, 256, device="cuda:0") == _lib.KEEP_ALPHA


def test_no_device_means_recompute_for_large_tables(monkeypatch):
    monkeypatch.delenv("TORCH_SEMIMARKOV_B200_BACKWARD", raising=False)
    assert _lib.backward_mode_for(64, 10_000, 256, device=None) == _lib.RECOMPUTE


@pytest.mark.parametrize("value,expected", [
    ("", 0), ("auto", 0), ("AUTO", 0), ("off", -1),
    ("336", 336), ("0", 1), ("70000", 0xFFFF),
    ("336,664", 336 | (664 << 16)), ("8,64", 8 | (64 << 16)),
    ("8,40000", 8 | (0x7FFF << 16)),
])
def test_chunk_warmup_encoding(monkeypatch, value, expected):
    monkeypatch.setenv("TORCH_SEMIMARKOV_B200_CHUNKS", value)
    assert _lib.chunk_warmup_from_env() == expected


def test_chunk_warmup_unset(monkeypatch):
    monkeypatch.delenv("TORCH_SEMIMARKOV_B200_CHUNKS", raising=False)
    assert _lib.chunk_warmup_from_env() == 0


@pytest.mark.parametrize("T,K,S", [(10_000, 300, 1732), (1000, 100, 316), (50, 300, 300),
                                   (1, 1, 1), (1_000_000, 1000, 31622)])
def test_checkpoint_interval(T, K, S):
    # max(K, floor(sqrt(T K))), the reference's _compute_checkpoint_interval
    assert _lib.checkpoint_interval(T, K) == S


def test_launcher_input_key_tracks_storage_and_writes():
    # launch_streaming_triton_backward reuses a forward's state only while the
    # inputs are the same storage, unwritten since (autograd.py's _input_key)
    from torch_semimarkov_b200.streaming.autograd import _input_key

    a = torch.zeros(2, 5, 3)
    b = torch.zeros(3, 3)
    k0 = _input_key(a, b, None)
    assert _input_key(a, b, None) == k0
    assert _input_key(a.clone(), b, None) != k0  # other storage
    a.add_(1.0)  # an in-place write bumps the version
    assert _input_key(a, b, None) != k0
    assert _input_key(a, b, b) != _input_key(a, b, None)
