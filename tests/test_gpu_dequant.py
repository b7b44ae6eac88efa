"""LUT dequant on the GPU (PackedH24Linear.materialize, pollux.py:485-504):
bit-exact against the reference's golden outputs and the oracle."""
from __future__ import annotations

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def PL(lib):
    from pollux_b200 import packed_linear
    return packed_linear


def test_golden_materialize(PL, golden):
    m = golden("materialize.npz")
    for t in "abcd":
        rows, in_f = (int(v) for v in m[t + "_shape"])
        w = PL.dequant(torch.from_numpy(m[t + "_packed"]).cuda(),
                       torch.from_numpy(m[t + "_sigma16"]).cuda(), rows, in_f)
        assert np.array_equal(w.cpu().numpy().view(np.uint16), m[t + "_weight16"].view(np.uint16)), t


def test_module_materialize(PL, golden):
    m = golden("materialize.npz")
    layer = PL.PackedH24Linear(192, 48).cuda()
    layer.packed_weights.copy_(torch.from_numpy(m["a_packed"]))
    layer.sigma_rows.copy_(torch.from_numpy(m["a_sigma16"]))
    layer.materialize()
    assert not hasattr(layer, "packed_weights") and layer._materialized
    assert layer.weight.dtype == torch.float16 and not layer.weight.requires_grad
    assert np.array_equal(layer.weight.detach().cpu().numpy().view(np.uint16),
                          m["a_weight16"].view(np.uint16))
    y = layer(torch.randn(3, 192, device="cuda", dtype=torch.float16))
    assert y.shape == (3, 48)


def test_config5_layer_against_oracle(PL, oracle):
    from pollux_b200 import synth, castor
    idx, sigma = synth.config5_layer(seed=5, device="cuda")
    packed = castor.pack_indices(idx)
    w = PL.dequant(packed, sigma, 7680, 1920)
    ref = oracle.dequant(packed.cpu().numpy(), sigma.cpu().numpy(), 7680, 1920)
    assert np.array_equal(w.cpu().numpy().view(np.uint16), ref.view(np.uint16))


def test_batched_equals_single(PL):
    from pollux_b200 import castor
    torch.manual_seed(0)
    shapes = [(3, 24), (17, 72), (128, 1920), (5, 4608)]
    mods, singles = [], []
    for (o, i) in shapes:
        n = o * i // 24
        idx = torch.randint(0, 196561, (n,), device="cuda")
        sig = (torch.rand(o, device="cuda") * 0.1 + 0.001).half()
        m = PL.PackedH24Linear(i, o).cuda()
        m.packed_weights.copy_(castor.pack_indices(idx))
        m.sigma_rows.copy_(sig)
        singles.append(PL.dequant(m.packed_weights, m.sigma_rows, o, i))
        mods.append(m)
    model = torch.nn.ModuleList(mods)
    assert PL.materialize_all(model) == len(shapes)
    for m, w in zip(mods, singles):
        assert torch.equal(m.weight.data, w)


def test_out_of_range_index_raises(PL, oracle):
    packed = torch.from_numpy(oracle.pack_indices(np.array([5, 196561, 7, 9]))).cuda()
    with pytest.raises(IndexError):
        PL.dequant(packed, torch.ones(1, dtype=torch.float16, device="cuda"), 1, 96)


@pytest.mark.parametrize("in_f", [24, 48, 72, 96, 120, 4608])
def test_rows_per_tile_regimes(PL, oracle, in_f):
    # 128-atom warp tiles span >34 rows for in_features < 96 (values computed
    # per element) and at most 33 rows otherwise (per-warp row table).
    from pollux_b200 import castor
    rows = 517
    gen = torch.Generator(device="cuda").manual_seed(in_f)
    idx = torch.randint(0, 196561, (rows * in_f // 24,), generator=gen, device="cuda")
    sig = (torch.rand(rows, generator=gen, device="cuda") * 0.2 + 1e-4).half()
    packed = castor.pack_indices(idx)
    w = PL.dequant(packed, sig, rows, in_f)
    ref = oracle.dequant(packed.cpu().numpy(), sig.cpu().numpy(), rows, in_f)
    assert np.array_equal(w.cpu().numpy().view(np.uint16), ref.view(np.uint16))


@pytest.mark.parametrize("shift", [1, 7, 9, 15])
def test_unaligned_packed_view(PL, oracle, shift):
    # A packed stream that starts at any byte offset (e.g. inside a .plx
    # buffer) dequantises to the same weights as an aligned copy.
    from pollux_b200 import castor
    rows, in_f = 333, 288
    gen = torch.Generator(device="cuda").manual_seed(100 + shift)
    idx = torch.randint(0, 196561, (rows * in_f // 24,), generator=gen, device="cuda")
    sig = (torch.rand(rows, generator=gen, device="cuda") * 0.2 + 1e-4).half()
    packed = castor.pack_indices(idx)
    buf = torch.zeros(packed.numel() + 64, dtype=torch.uint8, device="cuda")
    buf[shift:shift + packed.numel()] = packed
    w = PL.dequant(buf[shift:shift + packed.numel()], sig, rows, in_f)
    ref = oracle.dequant(packed.cpu().numpy(), sig.cpu().numpy(), rows, in_f)
    assert np.array_equal(w.cpu().numpy().view(np.uint16), ref.view(np.uint16))
