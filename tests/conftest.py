"""pytest configuration: markers, import paths and shared fixture loaders."""

from __future__ import annotations

import glob
import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
GOLDEN = os.path.join(ROOT, "tests", "golden")
for p in (ROOT, GOLDEN):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")
    config.addinivalue_line("markers", "slow: long-running test")


def golden_names(prefix):
    return sorted(os.path.basename(p)[:-4] for p in glob.glob(os.path.join(GOLDEN, prefix + "*.npz")))


def load_golden(name):
    with np.load(os.path.join(GOLDEN, name + ".npz"), allow_pickle=False) as z:
        return {k: z[k] for k in z.files}


def streaming_inputs_from_golden(g):
    """Rebuild the float32 inputs of a streaming fixture (regenerating big ones)."""
    from inputs import checksum, make_streaming_inputs

    B, T, K, C = int(g["B"]), int(g["T"]), int(g["K"]), int(g["C"])
    proj = str(g["proj"]) or None
    inp = make_streaming_inputs(B, T, K, C, int(g["seed"]), str(g["gen"]), proj=proj,
                                kcc=bool(int(g["kcc"])))
    if "cum_scores" in g:
        np.testing.assert_array_equal(inp["cum_scores"].numpy(), g["cum_scores"])
    np.testing.assert_allclose(checksum(inp["cum_scores"]), g["cum_checksum"], rtol=0, atol=0)
    np.testing.assert_array_equal(inp["transition"].numpy(), g["transition"])
    np.testing.assert_array_equal(inp["duration_bias"].numpy(), g["duration_bias"])
    return inp


@pytest.fixture(scope="session")
def oracle():
    from oracle import oracle as orc

    orc.build()
    return orc
