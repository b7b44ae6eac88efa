"""INT8 token embedding / output head on the GPU through the C-ABI
(pack._quantize_int8, pack.py:124-136; PackedInt8Embedding/Linear.materialize,
pollux.py:510-563): bit-exact against the reference's golden outputs and the
oracle."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from test_oracle_golden import _same_f16

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def mods(lib):
    from pollux_b200 import pack, packed_linear
    return pack, packed_linear


def test_golden_quantize_and_materialize(mods, golden):
    pack, pl = mods
    g = golden("int8.npz")
    for k in ("normal", "odd", "ties", "edge"):
        w = torch.from_numpy(g[k + "_w"])
        q, mu = pack._quantize_int8(w)              # host in, host out, like the reference
        assert q.device.type == "cpu" and q.dtype == torch.int8 and mu.dtype == torch.float16
        assert np.array_equal(q.numpy(), g[k + "_q"]), k
        assert _same_f16(mu.numpy(), g[k + "_mu"]), k
        rows, cols = w.shape
        emb = pl.PackedInt8Embedding(rows, cols).cuda()
        emb.weight_int8.copy_(torch.from_numpy(g[k + "_q"]))
        emb.mu_rows.copy_(torch.from_numpy(g[k + "_mu"]))
        emb.materialize()
        assert emb._materialized and not hasattr(emb, "weight_int8")
        assert _same_f16(emb.weight.detach().cpu().numpy(), g[k + "_emb"]), k
        head = pl.PackedInt8Linear(cols, rows).cuda()
        head.weight_int8.copy_(torch.from_numpy(g[k + "_q"]))
        head.mu_rows.copy_(torch.from_numpy(g[k + "_mu"]))
        head.materialize()
        assert _same_f16(head.weight.detach().cpu().numpy(), g[k + "_head"]), k


@pytest.mark.parametrize("shape", [(50304, 1152), (1000, 1920), (33, 100), (7, 3, 48)])
def test_large_and_odd_shapes_against_oracle(mods, oracle, shape):
    pack, pl = mods
    gen = torch.Generator(device="cuda").manual_seed(shape[0])
    w = torch.randn(*shape, generator=gen, device="cuda") * 0.02
    q, mu = pack.quantize_int8_device(w)
    assert q.shape == w.shape and mu.shape == w.shape[:-1]
    qo, muo = oracle.int8_quantize(w.cpu().numpy())
    assert np.array_equal(q.cpu().numpy(), qo)
    assert np.array_equal(mu.cpu().numpy().view(np.uint16), muo.view(np.uint16))
    w16 = pl.int8_dequant(q, mu)
    assert w16.shape == w.shape
    assert np.array_equal(w16.cpu().numpy().view(np.uint16), oracle.int8_dequant(qo, muo).view(np.uint16))


@pytest.mark.parametrize("cols", [1920, 4608])
def test_near_ties(mods, oracle, cols):
    """Elements at and around every rounding boundary of w / mu * 127: the
    kernel's product with fp32(127 / mu) must round like the reference's
    quotient-then-product on both sides of each half-integer (1920: the
    register path; 4608: the two-pass path)."""
    pack, _ = mods
    rows = 512
    g = np.random.default_rng(cols)
    mu = g.uniform(1e-3, 1.0, rows).astype(np.float32)
    k = g.integers(-127, 127, (rows, cols)).astype(np.float64)
    delta = g.choice([0.0, 1e-7, -1e-7, 3e-6, -3e-6, 3e-5, -3e-5, 1e-4, -1e-4, 0.25], (rows, cols))
    w = ((k + 0.5 + delta) * mu[:, None].astype(np.float64) / 127.0).astype(np.float32)
    # fp32 neighbours of the boundaries, and the row maximum itself.
    w[:, ::7] = np.nextafter(w[:, ::7], np.float32(np.inf))
    w[:, 1::7] = np.nextafter(w[:, 1::7], np.float32(-np.inf))
    w[:, 3] = mu
    w[:, 5] = -mu
    q, m = pack.quantize_int8_device(torch.from_numpy(w).cuda())
    qo, mo = oracle.int8_quantize(w)
    assert np.array_equal(m.cpu().numpy().view(np.uint16), mo.view(np.uint16))
    assert np.array_equal(q.cpu().numpy(), qo)


def test_unaligned_views(mods, oracle):
    pack, pl = mods
    base = torch.randn(65 * 96 + 1, device="cuda")
    w = base[1:].view(65, 96)                       # 4-byte offset: scalar paths
    q, mu = pack.quantize_int8_device(w)
    qo, muo = oracle.int8_quantize(w.cpu().numpy())
    assert np.array_equal(q.cpu().numpy(), qo)
    qb = torch.zeros(q.numel() + 1, dtype=torch.int8, device="cuda")
    qb[1:] = q.reshape(-1)
    w16 = pl.int8_dequant(qb[1:].view(65, 96), mu)
    assert np.array_equal(w16.cpu().numpy().view(np.uint16), oracle.int8_dequant(qo, muo).view(np.uint16))


def test_errors(mods):
    pack, pl = mods
    with pytest.raises(TypeError):
        pl.int8_dequant(torch.zeros(2, 4, dtype=torch.uint8, device="cuda"),
                        torch.ones(2, dtype=torch.float16, device="cuda"))
    with pytest.raises(TypeError):
        pl.int8_dequant(torch.zeros(2, 4, dtype=torch.int8, device="cuda"),
                        torch.ones(2, dtype=torch.float32, device="cuda"))
    with pytest.raises(RuntimeError):
        pl.int8_dequant(torch.zeros(2, 4, dtype=torch.int8, device="cuda"),
                        torch.ones(3, dtype=torch.float16, device="cuda"))
