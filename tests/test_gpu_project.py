"""Fused H24 projection of pollux_step (pollux.py:874-884) on the GPU:
p.data = (nearest codeword of latent/sigma/s_lattice) * sigma * s_lattice,
batched over parameters.  Everything after sigma is bit-exact (checked from
the kernel's own sigma with the oracle's exact search); sigma itself is the
correctly rounded fp32 row RMS, within 2 ulp of torch's fp32 reduction."""
from __future__ import annotations

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def C(lib):
    from pollux_b200 import castor
    return castor


def _expected(C, oracle, latent, sigma):
    """Reference formula (pollux.py:876-883) evaluated from a given sigma."""
    s_lat = float(C.s_lattice)
    x = (latent / sigma.reshape(-1, 1).clamp_min(1e-8)) / s_lat
    idx = oracle.nearest_exact(x.reshape(-1, 24).cpu().numpy(), 0)
    cb = torch.from_numpy(np.array(oracle.codebook_f32())).to(latent.device)
    center_abs = cb[torch.from_numpy(idx).to(latent.device).long()].reshape(latent.shape)
    return idx, (center_abs * sigma.reshape(-1, 1)) * s_lat


@pytest.mark.parametrize("shapes", [[(96, 1152)], [(48, 192), (3, 96), (200, 4608)]])
def test_projection_bit_exact_from_sigma(C, oracle, shapes):
    gen = torch.Generator(device="cuda").manual_seed(len(shapes))
    lats = [torch.randn(*s, generator=gen, device="cuda") * 0.02 for s in shapes]
    ps = [torch.empty_like(l) for l in lats]
    ex = C.project_h24_many(list(zip(ps, lats)), sigma_out=True, idx_out=True)
    for lat, p, e in zip(lats, ps, ex):
        idx, want = _expected(C, oracle, lat, e["sigma"])
        assert np.array_equal(e["idx"].cpu().numpy(), idx)
        assert torch.equal(p, want)
        ref_sigma = C.row_rms_from_matrix(lat)
        ulp = torch.abs(e["sigma"] - ref_sigma) / torch.finfo(torch.float32).eps / ref_sigma
        assert float(ulp.max()) <= 2.0


def test_matches_reference_block_where_sigma_agrees(C):
    """Against the reference block built from the mirror's own functions
    (normalize_matrix_by_row_rms, castor_quantize_leech, scale_matrix_by_row_rms)."""
    gen = torch.Generator(device="cuda").manual_seed(9)
    lat = torch.randn(256, 1152, generator=gen, device="cuda") * 0.02
    p = torch.empty_like(lat)
    ex = C.project_h24_many([(p, lat)], sigma_out=True)[0]
    normed, sig = C.normalize_matrix_by_row_rms(lat)
    cb = C.get_h24_codebook("cuda", torch.float32)
    center_abs = C.castor_quantize_leech(normed / float(C.s_lattice), cb)
    ref = C.scale_matrix_by_row_rms(center_abs, sig) * float(C.s_lattice)
    same = ex["sigma"] == sig
    assert float(same.float().mean()) > 0.5
    assert torch.equal(p[same], ref[same])
    torch.testing.assert_close(p, ref, rtol=1e-5, atol=1e-6)


def test_single_and_errors(C):
    lat = torch.randn(4, 96, device="cuda")
    p = torch.empty_like(lat)
    assert C.project_h24_(p, lat) is p
    assert torch.isfinite(p).all()
    with pytest.raises(ValueError):
        C.project_h24_(torch.empty(4, 96, device="cuda", dtype=torch.float16), lat)
    with pytest.raises(ValueError):
        C.project_h24_(torch.empty(4, 100, device="cuda"), torch.randn(4, 100, device="cuda"))
