"""The CPU oracle is pinned against fixtures produced by the reference's own
code (tests/golden/make_golden.py).  No GPU needed."""
from __future__ import annotations

import hashlib
import json
import os

import numpy as np
import pytest

from conftest import GOLDEN, tie_ok


def _sha(a):
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


@pytest.fixture(scope="module")
def cbmeta():
    with open(os.path.join(GOLDEN, "codebook.json")) as f:
        return json.load(f)


def test_codebook_bytes_match_reference(oracle, cbmeta):
    cb = oracle.codebook_f32()
    assert cb.shape == (196561, 24)
    assert _sha(cb) == cbmeta["sha256_f32"]
    assert _sha(cb.astype(np.float16)) == cbmeta["sha256_f16"]
    raw = np.rint(cb * np.sqrt(8.0)).astype(np.int8)
    assert _sha(raw) == cbmeta["sha256_raw_int8"]
    for k, row in cbmeta["rows_sample"].items():
        assert raw[int(k)].tolist() == row


def test_codebook_invariants(oracle):
    raw = oracle.raw_kissing_points().astype(np.int32)
    assert (np.sum(raw * raw, axis=1) == 32).all()
    assert len(np.unique(raw, axis=0)) == 196560
    # Not closed under negation: no +3 coordinate exists (type 3 uses -3 only).
    assert raw.max() == 4 and (raw == 3).sum() == 0


def test_fingerprint_and_threshold(oracle, cbmeta):
    assert list(oracle.fingerprint()) == cbmeta["fingerprint"]
    assert oracle.C_SQ_NORM == cbmeta["c_sq_norm"]


def test_pack_unpack_vectors(oracle, golden):
    g = golden("pack_vectors.npz")
    for k in g.files:
        if not k.startswith("idx_"):
            continue
        tag = k[4:]
        v = g[k]
        assert np.array_equal(oracle.pack_indices(v), g["packed_" + tag]), tag
        assert np.array_equal(oracle.pack_indices_c(v), g["packed_" + tag]), tag
        if tag != "odd":
            assert np.array_equal(oracle.unpack_indices(g["packed_" + tag], len(v)), g["unpacked_" + tag])
            assert np.array_equal(oracle.unpack_indices_c(g["packed_" + tag], len(v)), g["unpacked_" + tag])
    for n in (0, 1, 100, 148, 200):
        assert np.array_equal(oracle.unpack_indices_c(g["rand_bytes"], n), g[f"rand_unpacked_{n}"])


def test_dequant_matches_materialize(oracle, golden):
    m = golden("materialize.npz")
    for t in "abcd":
        rows, in_f = m[t + "_shape"]
        for fn in (oracle.dequant, oracle.dequant_numpy):
            w = fn(m[t + "_packed"], m[t + "_sigma16"], int(rows), int(in_f))
            assert np.array_equal(w.view(np.uint16), m[t + "_weight16"].view(np.uint16)), (t, fn)


def test_dequant_rejects_out_of_range(oracle):
    packed = oracle.pack_indices(np.array([196561, 0, 0, 0]))
    with pytest.raises(ValueError):
        oracle.dequant(packed, np.ones(1, np.float16), 1, 96)


def test_config1_pack_rule_exact(oracle, golden):
    """The fp64 oracle reproduces pack._quantize_h24_layer on all 55,296 atoms."""
    from pollux_b200 import synth
    c1 = golden("config1.npz")
    w = synth.config1_weight("cpu").numpy()
    assert _sha(w) == str(c1["weight_sha256"])
    ref = oracle.unpack_indices(c1["pack_packed"], w.size // 24)
    ours = oracle.nearest_exact(w.reshape(-1, 24), oracle.RULE_PACK)
    assert np.array_equal(ours, ref)
    assert np.array_equal(oracle.pack_indices(ours), c1["pack_packed"])
    s16 = oracle.sigma16_pack_rule(w)
    assert np.array_equal(s16.view(np.uint16), c1["pack_sigma16"].view(np.uint16))


def test_stress_subset_tie_tolerance(oracle, golden):
    s = golden("stress.npz")
    x = s["atoms"]
    ex = oracle.nearest_exact(x, oracle.RULE_PACK)
    assert not tie_ok(oracle, x, ex, s["pack_rule_idx"]).any()
    # Ties exist (midpoints of codeword pairs) and resolve within 1e-5.
    assert (ex != s["pack_rule_idx"]).sum() < 0.1 * len(x)
    ext = oracle.nearest_exact(x, oracle.RULE_TRAIN)
    # Against the reference's bf16-score CPU path only a one-sided bound holds.
    assert not tie_ok(oracle, x, ext, s["train_bf16_idx"]).any()


def test_bf16_fallback_differs_from_exact(oracle, golden):
    """The reference's autocast fallback is not exact (it disagrees with the
    exact argmax on about 4.2 % of config-1 atoms); the training-rule golden is
    kept as a one-sided check only."""
    from pollux_b200 import synth
    import torch
    c1 = golden("config1.npz")
    w = synth.config1_weight("cpu")
    normed = w / torch.sqrt(w.pow(2).mean(dim=-1) + 1e-8).reshape(-1, 1).clamp_min(1e-8)
    x = (normed / float(1 / np.sqrt(2.0))).numpy().reshape(-1, 24)
    assert _sha(x) == str(c1["train_x_sha256"])
    ref = oracle.unpack_indices(c1["train_bf16_packed"], x.shape[0])
    sample = np.arange(0, x.shape[0], 7)
    ex = oracle.nearest_exact(x[sample], oracle.RULE_TRAIN)
    frac = (ex != ref[sample]).mean()
    assert 0.01 < frac < 0.1
    # Our exact choice is never farther than the reference's.
    d_ex = oracle.dist2_fp64(x[sample], ex)
    d_ref = oracle.dist2_fp64(x[sample], ref[sample])
    assert (d_ex <= d_ref * (1 + 1e-6)).all()


def _same_f16(a, b):
    """Equal fp16 arrays, NaN positions included (NaN payloads not compared)."""
    a, b = np.asarray(a, np.float16), np.asarray(b, np.float16)
    return (np.array_equal(np.isnan(a), np.isnan(b)) and
            np.array_equal(np.where(np.isnan(a), 0, a).view(np.uint16),
                           np.where(np.isnan(b), 0, b).view(np.uint16)))


def test_int8_oracle_matches_reference(oracle, golden):
    g = golden("int8.npz")
    for k in ("normal", "odd", "ties", "edge"):
        q, mu = oracle.int8_quantize(g[k + "_w"])
        assert np.array_equal(q, g[k + "_q"]), k
        assert _same_f16(mu, g[k + "_mu"]), k
        w16 = oracle.int8_dequant(g[k + "_q"], g[k + "_mu"])
        assert _same_f16(w16, g[k + "_emb"]) and _same_f16(w16, g[k + "_head"]), k
