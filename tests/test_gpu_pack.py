"""18-bit pack / unpack on the GPU through the C-ABI: bit-exact against the
reference's golden vectors and the oracle (castor.py:226-260)."""
from __future__ import annotations

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def C(lib):
    from pollux_b200 import castor
    return castor


def test_golden_vectors(C, golden):
    g = golden("pack_vectors.npz")
    for k in g.files:
        if not k.startswith("idx_"):
            continue
        tag = k[4:]
        v = torch.from_numpy(g[k]).cuda()
        p = C.pack_indices(v)
        assert p.device.type == "cuda"
        assert np.array_equal(p.cpu().numpy(), g["packed_" + tag]), tag
        p32 = C.pack_indices(v.to(torch.int32))
        assert np.array_equal(p32.cpu().numpy(), g["packed_" + tag]), tag
        if tag != "odd":
            u = C.unpack_indices(torch.from_numpy(g["packed_" + tag]).cuda(), len(v))
            assert u.dtype == torch.int64
            assert np.array_equal(u.cpu().numpy(), g["unpacked_" + tag]), tag
    rb = torch.from_numpy(g["rand_bytes"]).cuda()
    for n in (0, 1, 100, 148, 200):
        assert np.array_equal(C.unpack_indices(rb, n).cpu().numpy(), g[f"rand_unpacked_{n}"])


def test_host_tensors_are_staged_through_the_gpu(C, golden):
    g = golden("pack_vectors.npz")
    v = torch.from_numpy(g["idx_1000"])
    p = C.pack_indices(v)
    assert p.device.type == "cpu"
    assert np.array_equal(p.numpy(), g["packed_1000"])
    assert np.array_equal(C.unpack_indices(p, 1000).numpy(), g["unpacked_1000"])


@pytest.mark.parametrize("n", [4 * 4096 * 64 + 3, 33_177_600])
def test_large_round_trip_and_oracle(C, oracle, n):
    gen = torch.Generator(device="cuda").manual_seed(n)
    idx = torch.randint(0, 196561, (n,), generator=gen, device="cuda", dtype=torch.int32)
    p = C.pack_indices(idx)
    assert p.numel() == ((n + 3) // 4) * 9
    back = C.unpack_indices(p, n)
    assert torch.equal(back.to(torch.int32), idx)
    # Bit-exact against the oracle on a window that crosses kernel tiles.
    lo = (n // 2) // 4 * 4
    win = idx[lo:lo + 40000].cpu().numpy()
    assert np.array_equal(p[lo // 4 * 9: lo // 4 * 9 + 90000].cpu().numpy(), oracle.pack_indices(win))


def test_unaligned_views(C, oracle):
    base = torch.randint(0, 196561, (10001,), device="cuda", dtype=torch.int64)
    v = base[1:]  # 8-byte offset: not 16-byte aligned
    p = C.pack_indices(v)
    assert np.array_equal(p.cpu().numpy(), oracle.pack_indices(v.cpu().numpy()))
    pb = torch.zeros(p.numel() + 1, dtype=torch.uint8, device="cuda")
    pb[1:] = p
    u = C.unpack_indices(pb[1:], 10000)
    assert torch.equal(u, v)


def test_unpack_errors(C):
    with pytest.raises(RuntimeError):
        C.unpack_indices(torch.zeros(10, dtype=torch.uint8, device="cuda"), 4)
    with pytest.raises(TypeError):
        C.unpack_indices(torch.zeros(9, dtype=torch.int8, device="cuda"), 4)
    # Negative num_indices follows Python slicing like indices[:num_indices].
    p = C.pack_indices(torch.arange(8, device="cuda"))
    assert C.unpack_indices(p, -3).tolist() == [0, 1, 2, 3, 4]


@pytest.mark.parametrize("n", [511, 512, 513, 2048 + 5, 3 * 4096 + 1])
@pytest.mark.parametrize("dtype", [torch.int32, torch.int64])
def test_warp_tile_boundaries(C, oracle, n, dtype):
    gen = torch.Generator(device="cuda").manual_seed(n)
    idx = torch.randint(0, 196561, (n,), generator=gen, device="cuda").to(dtype)
    p = C.pack_indices(idx)
    assert np.array_equal(p.cpu().numpy(), oracle.pack_indices(idx.cpu().numpy().astype(np.int64)))
    back = C.unpack_indices(p, n)
    assert torch.equal(back, idx.to(torch.int64))


def test_unpack_capacity_below_count(C, oracle):
    # num_indices beyond the packed capacity: only the decodable prefix comes back.
    idx = torch.randint(0, 196561, (4 * 1000,), device="cuda")
    p = C.pack_indices(idx)
    for n in (4 * 1000 + 600, 4 * 1000 + 1, 8000):
        u = C.unpack_indices(p, n)
        ref = oracle.unpack_indices(p.cpu().numpy(), n)
        assert np.array_equal(u.cpu().numpy(), ref)


@pytest.mark.parametrize("rows,in_f", [(4608, 1152), (5461, 72), (3, 96), (60012, 40), (7, 24)])
@pytest.mark.parametrize("pinned", [True, False])
def test_host_layer_pipelined_equals_device_path(C, rows, in_f, pinned):
    # fp32 host weights go through h24_quantize_layer_host: row chunks of whole
    # 4-atom pack groups (atoms straddle rows when in_f is not a multiple of
    # 24) copied on a side stream while earlier chunks are searched; bytes and
    # sigma must equal the device-resident path.
    from pollux_b200 import pack
    gen = torch.Generator().manual_seed(rows)
    w = torch.randn(rows, in_f, generator=gen) * 0.02
    cb = C.get_h24_codebook("cuda", torch.float32)
    p_host, s_host = pack._quantize_h24_layer(w.pin_memory() if pinned else w, cb)
    p_dev, s_dev = pack._quantize_h24_layer(w.cuda(), cb)
    assert p_host.device.type == "cpu" and s_host.device.type == "cpu"
    assert p_host.is_pinned() == pinned
    assert torch.equal(p_host, p_dev) and torch.equal(s_host.view(torch.int16), s_dev.view(torch.int16))
