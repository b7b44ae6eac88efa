"""Matrix-free LUT GEMV over packed H24 layers (the README's "future native
kernel", README.md:88, 155-156): y = x @ W.T with W the fp16 weight that
PackedH24Linear.materialize produces, checked against the oracle's W in fp64
(fp32 accumulation tolerance stated below)."""
from __future__ import annotations

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

# |y - y_exact| <= 2^-14 * sum_i |x_i W_oi|: fp32 products of fp16 weights are
# exact; each lane sums at most 24 * ceil(in/768) terms, then a 32-lane tree.
RTOL = 2.0 ** -14


@pytest.fixture(scope="module")
def PL(lib):
    from pollux_b200 import packed_linear
    return packed_linear


def _layer(out_f, in_f, seed):
    from pollux_b200 import castor
    gen = torch.Generator(device="cuda").manual_seed(seed)
    idx = torch.randint(0, 196561, (out_f * in_f // 24,), generator=gen, device="cuda")
    sig = (torch.rand(out_f, generator=gen, device="cuda") * 0.1 + 1e-3).half()
    return castor.pack_indices(idx), sig


def _check(oracle, packed, sig, out_f, in_f, x, y):
    w = oracle.dequant(packed.cpu().numpy(), sig.cpu().numpy(), out_f, in_f).astype(np.float64)
    xd = x.reshape(-1, in_f).cpu().double().numpy()
    ref = xd @ w.T
    bound = RTOL * (np.abs(xd) @ np.abs(w).T) + 1e-30
    err = np.abs(y.reshape(-1, out_f).cpu().double().numpy() - ref)
    assert (err <= bound).all(), float((err / bound).max())


@pytest.mark.parametrize("out_f,in_f", [(7680, 1920), (1152, 4608), (37, 72), (5, 24)])
@pytest.mark.parametrize("batch", [1, 3, 8, 9])
def test_against_oracle_weight(PL, oracle, out_f, in_f, batch):
    packed, sig = _layer(out_f, in_f, out_f + in_f)
    gen = torch.Generator(device="cuda").manual_seed(batch)
    x = torch.randn(batch, in_f, generator=gen, device="cuda")
    y = PL.lut_linear(x, packed, sig, out_f, in_f)
    assert y.shape == (batch, out_f) and y.dtype == torch.float32
    _check(oracle, packed, sig, out_f, in_f, x, y)


@pytest.mark.parametrize("offset", [1, 7, 15])
def test_unaligned_packed_view(PL, offset):
    """Packed bytes at any address: the kernel reads them in aligned 16-byte
    blocks and never touches bytes outside the buffer; the result equals the
    aligned call's bit for bit."""
    out_f, in_f = 37, 72
    packed, sig = _layer(out_f, in_f, 11)
    store = torch.zeros(packed.numel() + offset, dtype=torch.uint8, device="cuda")
    store[offset:] = packed
    x = torch.randn(3, in_f, device="cuda")
    y0 = PL.lut_linear(x, packed, sig, out_f, in_f)
    y1 = PL.lut_linear(x, store[offset:], sig, out_f, in_f)
    assert torch.equal(y0, y1)


def test_module_forward_before_and_after_materialize(PL, oracle):
    packed, sig = _layer(96, 192, 5)
    m = PL.PackedH24Linear(192, 96, bias=True).cuda()
    m.packed_weights.copy_(packed)
    m.sigma_rows.copy_(sig)
    with torch.no_grad():
        m.bias.copy_(torch.randn(96))
    x = torch.randn(2, 4, 192, device="cuda")
    y_lut = m(x)
    assert y_lut.shape == (2, 4, 96)
    m.materialize()
    y_dense = m(x)
    torch.testing.assert_close(y_lut, y_dense, rtol=1e-4, atol=1e-5)


def test_large_batch_uses_dense_path_with_same_result(PL):
    packed, sig = _layer(64, 96, 6)
    x = torch.randn(40, 96, device="cuda")
    y = PL.lut_linear(x, packed, sig, 64, 96)
    y8 = torch.cat([PL.lut_linear(x[i:i + 8], packed, sig, 64, 96) for i in range(0, 40, 8)])
    torch.testing.assert_close(y, y8, rtol=1e-4, atol=1e-5)


def test_enable_lut_forward_and_bad_index(PL, oracle):
    from pollux_b200 import castor
    mods = torch.nn.ModuleList([PL.PackedH24Linear(96, 48).cuda() for _ in range(2)])
    assert PL.enable_lut_forward(mods) == 2
    bad = torch.from_numpy(oracle.pack_indices(np.array([5, 196561, 7, 9]))).cuda()
    with pytest.raises(IndexError):
        PL.lut_linear(torch.randn(1, 96, device="cuda"), bad, torch.ones(1, dtype=torch.float16, device="cuda"), 1, 96)
