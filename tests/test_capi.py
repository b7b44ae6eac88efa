"""libh24.so loads on a machine without a GPU and exports every symbol that
include/h24.h declares; argument checks that need no device work here."""
from __future__ import annotations

import ctypes
import os
import re

import numpy as np
import pytest

from conftest import REPO


def _declared():
    src = open(os.path.join(REPO, "include", "h24.h")).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(h24_[a-z0-9_]+)\s*\(", src)))


def test_every_declared_symbol_is_exported(lib):
    names = _declared()
    assert len(names) >= 18
    for n in names:
        assert hasattr(lib, n), n


def test_binding_table_covers_header(lib):
    from pollux_b200 import _native
    assert sorted(_native.SIGNATURES) == _declared()


def test_struct_layout_matches_header():
    from pollux_b200 import _native
    assert ctypes.sizeof(_native.DequantLayer) == 40


def test_version_and_error_strings(lib):
    assert b"sm_100a" in lib.h24_version()
    assert isinstance(lib.h24_last_error(), bytes)


def test_host_codebook_equals_oracle(lib, oracle):
    raw = np.empty((196560, 24), dtype=np.int8)
    assert lib.h24_codebook_raw(raw.ctypes.data) == 0
    assert np.array_equal(raw, oracle.raw_kissing_points())


def test_validation_without_device(lib):
    from pollux_b200 import _native as N
    assert lib.h24_pack(None, -1, None, None) == N.H24_ERR_INVALID
    assert b"negative" in lib.h24_last_error()
    assert lib.h24_pack(None, 0, None, None) == N.H24_OK
    assert lib.h24_unpack(None, -2, 4, None, None) == N.H24_ERR_INVALID
    assert lib.h24_codebook_raw(None) == N.H24_ERR_INVALID
    with pytest.raises(ValueError):
        N.check(N.H24_ERR_INVALID, "x")
    with pytest.raises(IndexError):
        N.check(N.H24_ERR_RANGE, "x")
    with pytest.raises(N.H24Error):
        N.check(N.H24_ERR_TIMEOUT, "x")


def test_python_mirror_codebook(oracle):
    from pollux_b200 import castor
    import torch
    cb = castor.get_h24_codebook("cpu", torch.float32).numpy()
    assert np.array_equal(cb.view(np.uint32), oracle.codebook_f32().view(np.uint32))
    assert castor.codebook_fingerprint() == oracle.fingerprint()


def test_hot_path_refuses_to_run_without_cuda():
    import torch
    from pollux_b200 import castor
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    with pytest.raises(RuntimeError, match="CUDA"):
        castor.pack_indices(torch.arange(8))
    with pytest.raises(RuntimeError, match="CUDA"):
        castor.castor_quantize_leech(torch.zeros(4, 24), castor.get_h24_codebook("cpu", torch.float32))
