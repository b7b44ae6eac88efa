"""Shared fixtures.  GPU tests carry @pytest.mark.gpu; everything else runs on CPU."""
from __future__ import annotations

import os
import sys

import numpy as np
import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if REPO not in sys.path:
    sys.path.insert(0, REPO)

GOLDEN = os.path.join(REPO, "tests", "golden")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA (B200, sm_100a) device")


@pytest.fixture(scope="session")
def oracle():
    from oracle import oracle as O
    O.build()
    return O


@pytest.fixture(scope="session")
def golden():
    def load(name):
        return np.load(os.path.join(GOLDEN, name), allow_pickle=False)
    return load


@pytest.fixture(scope="session")
def lib():
    from pollux_b200 import build
    build.build()
    from pollux_b200 import _native
    return _native.load()


def tie_ok(oracle, x, ours, ref, rel=1e-5):
    """Parity rule: same index, or our squared distance is within `rel` of the
    reference choice's squared distance (fp64).  Returns the failing mask."""
    ours = np.asarray(ours, dtype=np.int64)
    ref = np.asarray(ref, dtype=np.int64)
    diff = ours != ref
    if not diff.any():
        return diff
    d_o = oracle.dist2_fp64(x[diff], ours[diff])
    d_r = oracle.dist2_fp64(x[diff], ref[diff])
    bad = np.zeros_like(diff)
    bad[np.nonzero(diff)[0]] = d_o > d_r * (1 + rel) + 1e-30
    return bad
