"""The failure path of the screening kernel, exercised without a GPU fault.

Every wait of the screen is bounded.  The test hook h24_debug_stall_screen
makes the next screening launch leave one Golay tile unloaded (a barrier that
nothing signals) and shortens the limit to 50 ms: the wait runs out, the kernel
drains its copies and MMAs, frees its TMEM and returns, and the host reads
H24_ERR_TIMEOUT -- through h24_check (castor.device_check) after an
asynchronous call, and as the return code of the synchronous host-memory
layer call (pack._quantize_h24_layer on a CPU weight).  The context stays
usable: the next call is exact again."""
from __future__ import annotations

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

LIMIT_NS = 50_000_000


@pytest.fixture
def stall(lib):
    from pollux_b200 import _native as N
    yield lambda launches: N.call("h24_debug_stall_screen", launches, LIMIT_NS)
    N.call("h24_debug_stall_screen", 0, 0)


def test_timeout_reported_by_check(stall, oracle):
    from pollux_b200 import castor, _native as N
    x = torch.randn(512, 24, device="cuda")
    castor.device_check()
    stall(1)
    castor.quantize_indices(x, 0)
    with pytest.raises(N.H24Error, match="bounded wait"):
        castor.device_check()
    castor.device_check()  # the error word was cleared
    idx = castor.quantize_indices(x, 0).cpu().numpy()
    castor.device_check()
    assert np.array_equal(idx, oracle.nearest_exact(x.cpu().numpy(), 0))


def test_timeout_returned_by_synchronous_host_call(stall):
    from pollux_b200 import castor, pack, _native as N
    w = torch.randn(64, 1920) * 0.02
    cb = castor.get_h24_codebook("cpu", torch.float32)
    good = pack._quantize_h24_layer(w, cb)
    stall(1)
    with pytest.raises(N.H24Error, match="bounded wait"):
        pack._quantize_h24_layer(w, cb)
    castor.device_check()
    again = pack._quantize_h24_layer(w, cb)
    assert torch.equal(again[0], good[0]) and torch.equal(again[1], good[1])
