"""Nearest-codeword search on the GPU (tcgen05 screening + fp64 rescore)
against the exact fp64 oracle (bit-exact) and the reference's own outputs
(within the stated near-tie tolerance): castor.py:386-560, pack.py:139-180."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import tie_ok

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def C(lib):
    from pollux_b200 import castor
    return castor


def q(C, x, rule):
    idx = C.quantize_indices(torch.as_tensor(x).cuda(), rule)
    C.device_check()
    return idx.cpu().numpy().astype(np.int64)


def test_config1_pack_rule_equals_reference(C, oracle, golden):
    from pollux_b200 import synth, pack
    c1 = golden("config1.npz")
    w = synth.config1_weight("cpu")
    ref = oracle.unpack_indices(c1["pack_packed"], w.numel() // 24)
    ours = q(C, w.reshape(-1, 24), 1)
    assert np.array_equal(ours, ref)
    packed, sigma = pack._quantize_h24_layer(w, C.get_h24_codebook("cpu", torch.float32))
    assert packed.device.type == "cpu" and sigma.dtype == torch.float16
    assert np.array_equal(packed.numpy(), c1["pack_packed"])
    assert np.array_equal(sigma.numpy().view(np.uint16), c1["pack_sigma16"].view(np.uint16))


def test_config1_training_rule(C, oracle, golden):
    from pollux_b200 import synth
    c1 = golden("config1.npz")
    w = synth.config1_weight("cuda")
    normed, _ = C.normalize_matrix_by_row_rms(w)
    x = (normed / float(C.s_lattice)).cpu().numpy().reshape(-1, 24)
    ours = q(C, x, 0)
    exact = oracle.nearest_exact(x, oracle.RULE_TRAIN)
    assert np.array_equal(ours, exact)
    ref_bf16 = oracle.unpack_indices(c1["train_bf16_packed"], x.shape[0])
    assert not tie_ok(oracle, x, ours, ref_bf16, rel=1e-5).any()
    assert (ours == 0).sum() == 0


def test_stress_subset(C, oracle, golden):
    s = golden("stress.npz")
    x = s["atoms"]
    for rule, ref in ((1, s["pack_rule_idx"]), (0, s["train_bf16_idx"])):
        ours = q(C, x, rule)
        assert np.array_equal(ours, oracle.nearest_exact(x, rule))
        assert not tie_ok(oracle, x, ours, ref).any()


def test_every_codeword_maps_to_itself(C, oracle):
    kp = torch.from_numpy(oracle.kissing_points_f32().copy())
    for rule in (0, 1):
        ours = q(C, kp, rule)
        assert np.array_equal(ours, np.arange(1, 196561))
    # Scaled below the snap radius -> origin (training rule), kept (pack rule).
    small = kp[::97] * 0.3
    assert (q(C, small, 0) == 0).all()
    assert np.array_equal(q(C, small, 1), np.arange(1, 196561)[::97])
    assert np.array_equal(q(C, kp[::97] * 0.6, 0), np.arange(1, 196561)[::97])


def test_edge_atoms(C, oracle):
    eye = np.eye(24, dtype=np.float32)
    atoms = np.concatenate([
        np.zeros((3, 24), np.float32),                     # exact zeros
        eye, -eye, 5 * eye,                                  # massive exact ties
        np.full((2, 24), 1e-9, np.float32),                  # below the pack-rule norm
        np.full((2, 24), 1e-3, np.float32),
        np.ones((2, 24), np.float32), -np.ones((2, 24), np.float32),
        np.array([[1e30] + [0] * 23, [-7e-39] * 24], np.float32),
    ])
    for rule in (0, 1):
        ours = q(C, atoms, rule)
        assert np.array_equal(ours, oracle.nearest_exact(atoms, rule)), rule


def test_octad_pattern_ties(C, oracle):
    # Atoms dominated by one octad with an odd number of negative coordinates
    # whose two smallest |x_i| are equal (two best sign patterns tie exactly:
    # the rescore scores every pattern) or one ulp apart (one best pattern,
    # listed alone).
    rng = np.random.default_rng(7)
    raw = oracle.raw_kissing_points()
    type2 = np.where((raw != 0).sum(1) == 8)[0]
    atoms = []
    for j in rng.choice(type2, 96, replace=False):
        supp = np.where(raw[j] != 0)[0]
        x = rng.normal(0, 0.05, 24).astype(np.float32)
        x[supp] = np.sign(raw[j][supp]) * rng.uniform(1.0, 2.0, 8).astype(np.float32)
        a, b = rng.choice(supp, 2, replace=False)
        x[a] = -np.float32(0.5) * np.sign(x[a])
        x[b] = np.float32(0.5) * np.sign(x[b])
        y = x.copy()
        y[b] = np.nextafter(np.float32(0.5), np.float32(1.0)) * np.sign(y[b])
        atoms += [x, y]
    atoms = np.stack(atoms)
    for rule in (0, 1):
        assert np.array_equal(q(C, atoms, rule), oracle.nearest_exact(atoms, rule)), rule


def test_non_finite_atoms(C):
    atoms = np.zeros((4, 24), np.float32)
    atoms[0, 3] = np.nan
    atoms[1, 0] = np.inf
    atoms[2] = 1.0
    atoms[3, 5] = -np.inf
    assert q(C, atoms, 0).tolist()[0:2] == [0, 0]
    assert q(C, atoms, 1).tolist()[0:2] == [1, 1]


@pytest.mark.parametrize("n", [1, 5, 255, 256, 257, 1000])
def test_ragged_sizes(C, oracle, n):
    gen = torch.Generator().manual_seed(n)
    x = torch.randn(n, 24, generator=gen) * 1.4
    for rule in (0, 1):
        assert np.array_equal(q(C, x, rule), oracle.nearest_exact(x.numpy(), rule))


def test_config4_scale_sample(C, oracle):
    """2^20 stress atoms in one call: a seeded sample is bit-exact against the
    oracle, and the exhaustive path and the exact rescoring stay rare."""
    from pollux_b200 import synth
    cb = C.get_h24_codebook("cuda", torch.float32)
    x = synth.stress_atoms(1 << 20, cb, seed=3, device="cuda")
    C.quantize_stats()
    ours = C.quantize_indices(x, 1)
    C.device_check()
    stats = C.quantize_stats()
    exhaustive, exact_scores, units = stats  # units: 32 Golay columns behind a flag
    assert exhaustive < 0.01 * (1 << 20), stats
    assert exact_scores < 64 * (1 << 20), stats
    assert units < 48 * (1 << 20), stats
    sel = torch.randperm(1 << 20, generator=torch.Generator().manual_seed(0))[:3000]
    xs = x[sel.cuda()].cpu().numpy()
    assert np.array_equal(ours[sel.cuda()].cpu().numpy(), oracle.nearest_exact(xs, 1))


def test_castor_quantize_leech_dropin(C, oracle):
    gen = torch.Generator().manual_seed(11)
    lat = torch.randn(6, 5, 48, generator=gen)
    for dt in (torch.float32, torch.bfloat16, torch.float16):
        cb = C.get_h24_codebook("cuda", torch.float32)
        x = lat.to(dt).cuda()
        out = C.castor_quantize_leech(x, cb)
        assert out.shape == x.shape and out.dtype == dt
        idx = oracle.nearest_exact(x.float().cpu().numpy().reshape(-1, 24), 0)
        expect = torch.from_numpy(oracle.codebook_f32()[idx]).to(dt).reshape(x.shape)
        assert torch.equal(out.cpu(), expect)
    assert C.castor_quantize_leech(torch.zeros(0, 24, device="cuda"), cb).numel() == 0
    with pytest.raises(ValueError):
        C.castor_quantize_leech(lat.cuda(), cb[:100])
    g = torch.randn(4, 24, device="cuda", requires_grad=True)
    y = C.CastorQuantizeLeech.apply(g, cb)
    y.sum().backward()
    assert torch.equal(g.grad, torch.ones_like(g))


def test_no_timeouts_recorded(C):
    C.device_check()


def test_segments_equal_single_calls(C, oracle):
    gen = torch.Generator().manual_seed(5)
    xs = [torch.randn(n, 24, generator=gen) * 1.3 for n in (1, 300, 4096, 77)]
    many = C.quantize_indices_many([x.cuda() for x in xs], 1)
    for x, idx in zip(xs, many):
        assert np.array_equal(idx.cpu().numpy(), oracle.nearest_exact(x.numpy(), 1))


def test_quantize_layers_batched(C, golden):
    from pollux_b200 import synth, pack
    c1 = golden("config1.npz")
    w1 = synth.config1_weight("cuda")
    ws = [w1[:96], w1, torch.randn(48, 36, device="cuda") * 0.02]
    res = pack.quantize_layers(ws)
    for w, (p, s) in zip(ws, res):
        p1, s1 = pack._quantize_h24_layer(w, C.get_h24_codebook("cuda", torch.float32))
        assert torch.equal(p.cpu(), p1) and torch.equal(s.cpu(), s1)
    assert np.array_equal(res[1][0].cpu().numpy(), c1["pack_packed"])
