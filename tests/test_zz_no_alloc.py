"""The allocation-free entry point h24_quantize_noalloc, called through the C ABI.

Some callers cannot allocate device memory while they run (an external memory
manager owns every allocation, or the loop is latency-critical), so this entry
point keeps its scratch in a fixed array inside the library.  Its indices must
equal those of h24_quantize on the same atoms, call after call: the shared
array keeps the previous call's contents and the entry point must not depend
on them.  This file is collected last so that a failure here does not stop the
other tests of a run that stops at the first failure.
"""
from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def h24(lib):
    from pollux_b200 import _native as N
    torch.cuda.init()
    assert lib.h24_init(torch.cuda.current_device()) == N.H24_OK
    return lib


def _both(h24, x, rule):
    from pollux_b200 import _native as N
    x = x.contiguous()
    stream = torch.cuda.current_stream().cuda_stream
    ref = torch.empty(x.shape[0], dtype=torch.int32, device="cuda")
    got = torch.full((x.shape[0],), -7, dtype=torch.int32, device="cuda")
    N.check(h24.h24_quantize(x.data_ptr(), x.shape[0], rule, ref.data_ptr(), stream), "quantize")
    N.check(h24.h24_quantize_noalloc(x.data_ptr(), x.shape[0], rule, got.data_ptr(), stream),
            "quantize_noalloc")
    N.check(h24.h24_check(stream), "check")
    return ref.cpu().numpy(), got.cpu().numpy()


def test_matches_h24_quantize_on_two_calls_in_a_row(h24):
    from pollux_b200 import synth, castor
    gen = torch.Generator(device="cuda").manual_seed(101)
    first = torch.randn(20000, 24, generator=gen, device="cuda") * 1.4
    # The second call is larger and full of exact ties (many flagged chunks and
    # exhaustive scans), so any state left by the first call would show.
    second = synth.stress_atoms(32768, castor.get_h24_codebook("cuda", torch.float32), seed=9,
                                device="cuda")
    for x, rule in ((first, 0), (second, 1)):
        ref, got = _both(h24, x, rule)
        assert np.array_equal(ref, got)


def test_limits_and_errors(h24):
    from pollux_b200 import _native as N
    stream = torch.cuda.current_stream().cuda_stream
    x = torch.zeros(32769, 24, device="cuda")
    out = torch.empty(32769, dtype=torch.int32, device="cuda")
    assert h24.h24_quantize_noalloc(x.data_ptr(), 32769, 0, out.data_ptr(), stream) == N.H24_ERR_INVALID
    assert b"32768" in h24.h24_last_error()
    assert h24.h24_quantize_noalloc(x.data_ptr(), 0, 0, out.data_ptr(), stream) == N.H24_OK
    assert h24.h24_quantize_noalloc(x.data_ptr(), 8, 5, out.data_ptr(), stream) == N.H24_ERR_INVALID
