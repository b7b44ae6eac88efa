"""Host-side logic that needs no GPU: the .plx container (pack.py:77-104,
187-247; generate.py:76-136), the install() hook, shape helpers."""
from __future__ import annotations

import json
import os
import types

import numpy as np
import pytest
import torch

from conftest import GOLDEN


def _state_from_fixture():
    z = np.load(os.path.join(GOLDEN, "plx_state.npz"))
    state = {k.replace("__", "."): torch.from_numpy(z[k]) for k in z.files if k != "config"}
    return state, json.loads(str(z["config"]))


def test_reader_parses_reference_written_file():
    from pollux_b200 import plx
    from oracle import oracle as O
    state, cfg = _state_from_fixture()
    payload = plx.read_plx(os.path.join(GOLDEN, "tiny.plx"))
    assert payload["format"] == "pollux_packed_v4"
    assert payload["config"] == cfg
    assert tuple(payload["codebook_fingerprint"]) == tuple(np.float32(v) for v in O.fingerprint())
    assert list(payload["state_dict"]) == list(state)
    for k, v in state.items():
        got = payload["state_dict"][k]
        assert got.dtype == v.dtype and torch.equal(got, v), k


def test_writer_reproduces_reference_bytes(tmp_path):
    from pollux_b200 import plx
    from oracle import oracle as O
    state, cfg = _state_from_fixture()
    out = tmp_path / "ours.plx"
    plx.write_plx(str(out), cfg, state, fingerprint=O.fingerprint())
    assert out.read_bytes() == open(os.path.join(GOLDEN, "tiny.plx"), "rb").read()


def test_reader_rejects_bad_files(tmp_path):
    from pollux_b200 import plx
    bad = tmp_path / "bad.plx"
    bad.write_bytes(b"NOTPLX!!" + bytes(64))
    with pytest.raises(ValueError, match="magic"):
        plx.read_plx(str(bad))
    raw = open(os.path.join(GOLDEN, "tiny.plx"), "rb").read()
    v5 = tmp_path / "v5.plx"
    v5.write_bytes(raw[:8] + bytes([5]) + raw[9:])
    with pytest.raises(ValueError, match="version"):
        plx.read_plx(str(v5))
    cut = tmp_path / "cut.plx"
    cut.write_bytes(raw[:-10])
    with pytest.raises(ValueError, match="truncated"):
        plx.read_plx(str(cut))


def test_install_rebinds_reference_names():
    import pollux_b200
    from pollux_b200 import castor, pack, packed_linear
    ref_castor = types.SimpleNamespace(castor_quantize_leech=None, pack_indices=None,
                                       unpack_indices=None, centers_to_indices=None,
                                       CastorQuantizeLeech=None, get_h24_codebook=object())
    class RefPacked:  # stands in for pollux.PackedH24Linear
        def materialize(self):
            raise AssertionError("reference path must not run")
    class RefEmb:  # stands in for pollux.PackedInt8Embedding
        def materialize(self):
            raise AssertionError("reference path must not run")
    class RefHead(RefEmb):  # pollux.PackedInt8Linear
        pass
    ref_pollux = types.SimpleNamespace(castor_quantize_leech=None, unpack_indices=None,
                                       PackedH24Linear=RefPacked, PackedInt8Embedding=RefEmb,
                                       PackedInt8Linear=RefHead)
    ref_pack = types.SimpleNamespace(pack_indices=None, _quantize_h24_layer=None, _quantize_int8=None)
    done = pollux_b200.install({"castor": ref_castor, "pollux": ref_pollux, "pack": ref_pack})
    assert ref_castor.castor_quantize_leech is castor.castor_quantize_leech
    assert ref_castor.unpack_indices is castor.unpack_indices
    assert ref_pollux.castor_quantize_leech is castor.castor_quantize_leech
    assert ref_pack._quantize_h24_layer is pack._quantize_h24_layer
    assert RefPacked.materialize is packed_linear.materialize
    assert "pollux.PackedH24Linear.materialize" in done
    assert ref_pack._quantize_int8 is pack._quantize_int8
    assert RefEmb.materialize is packed_linear.materialize_int8
    assert RefHead.materialize is packed_linear.materialize_int8
    assert not isinstance(ref_castor.get_h24_codebook, type(castor.get_h24_codebook))


def test_shape_helpers_match_reference_rules():
    from pollux_b200 import castor
    assert castor.h24_linear_atom_count(1152, 1152) == 55296
    with pytest.raises(ValueError):
        castor.h24_linear_atom_count(5, 5)
    with pytest.raises(ValueError):
        castor.assert_row_aligned_in_features(100)
    assert castor.scale_bits_per_param(1920) == 16.0 / 1920
    assert castor.h24_linear_scale_row_count(7) == 7
    w = torch.randn(48, 96)
    normed, sig = castor.normalize_matrix_by_row_rms(w)
    assert torch.allclose(castor.scale_matrix_by_row_rms(normed, sig), w, rtol=1e-5, atol=1e-6)
    with pytest.raises(ValueError):
        castor.row_rms_from_matrix(torch.zeros(2, 2, 24))


def test_packed_linear_buffers_match_reference_layout():
    from pollux_b200 import packed_linear
    m = packed_linear.PackedH24Linear(1920, 7680)
    assert m.packed_weights.dtype == torch.uint8 and m.packed_weights.numel() == 614400 // 4 * 9
    assert m.sigma_rows.dtype == torch.float16 and m.sigma_rows.numel() == 7680
    assert set(dict(m.named_buffers())) == {"packed_weights", "sigma_rows"}


def test_row_division_by_multiply_high_is_exact():
    # The dequant kernel divides in-row positions x < d + 128 by the row
    # length d (atoms per row) as floor(x * ceil(2^32 / d) / 2^32) for
    # d <= 65,000 (h24_dequant.cu, RowDiv).  Exhaustive for short rows, and at
    # the largest d the kernel uses it for, where the error term is largest.
    rng = np.random.default_rng(0)
    ds = list(range(1, 1025)) + [int(v) for v in rng.integers(1025, 65001, 200)] + list(range(64900, 65001))
    for d in ds:
        m = np.uint64(((1 << 32) + d - 1) // d)
        x = np.arange(0, d + 128, dtype=np.uint64)
        assert np.array_equal((x * m) >> np.uint64(32), x // np.uint64(d)), d
