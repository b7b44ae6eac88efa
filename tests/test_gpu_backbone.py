"""The pack-rule quantiser at the benchmark's full sizes (pack._quantize_h24_layer,
pack.py:139-180, over pack_checkpoint's loop, pack.py:268-283):

* config 2 (48 fp32 matrices, 7.96M atoms) and config 3 (72 bf16 matrices,
  33.2M atoms) are quantised whole on the GPU; a seeded sample of whole rows of
  every matrix is checked bit-exact against the oracle (exact fp64 argmax,
  lowest index on ties, the pack rule's origin test), and those rows' packed
  bytes against the oracle's 18-bit pack;
* bf16 weights are read natively and give the indices of their fp32 widening;
* row shards (the unit of multi-GPU sharding) concatenate into the whole
  matrix's bytes and scales, for every shard count up to 8 and ragged shards;
* size-independent properties on the whole backbone: unpack(pack) round trip
  and every index within the codebook."""
from __future__ import annotations

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

SAMPLE_ATOMS_PER_MATRIX = 1536


@pytest.fixture(scope="module")
def mods(lib):
    from pollux_b200 import castor, pack, shard, synth
    return castor, pack, shard, synth


@pytest.mark.parametrize("config", [2, 3])
def test_backbone_sample_parity(mods, oracle, config):
    C, P, _, S = mods
    ws = S.backbone_weights(config, device="cuda")
    res = P.quantize_layers(ws)
    C.device_check()
    rng = np.random.default_rng(100 + config)
    xs, ours, packed_rows, rows_meta = [], [], [], []
    for w, (packed, sigma) in zip(ws, res):
        rows, in_f = w.shape
        apr = in_f // 24
        assert apr % 4 == 0
        k = max(1, SAMPLE_ATOMS_PER_MATRIX // apr)
        sel = np.sort(rng.choice(rows, k, replace=False))
        wf = w[torch.from_numpy(sel).cuda()].float().cpu().numpy()
        pk = packed.cpu().numpy().reshape(rows, apr // 4 * 9)[sel]
        xs.append(wf.reshape(-1, 24))
        ours.append(oracle.unpack_indices(pk.reshape(-1), k * apr))
        packed_rows.append(pk)
        rows_meta.append((tuple(w.shape), k))
        # Whole-matrix properties: in range, and unpack(pack) is the identity.
        n = rows * apr
        idx_all = C.unpack_indices(packed, n)
        assert int(idx_all.max()) <= 196560 and int(idx_all.min()) >= 0
        assert torch.equal(C.pack_indices(idx_all), packed)
    x = np.concatenate(xs)
    got = np.concatenate(ours)
    exact = oracle.nearest_exact(x, oracle.RULE_PACK)
    bad = np.nonzero(got != exact)[0]
    assert bad.size == 0, f"{bad.size} of {x.shape[0]} sampled atoms differ from the oracle"
    off = 0
    for pk, ((rows, in_f), k) in zip(packed_rows, rows_meta):
        m = k * in_f // 24
        assert np.array_equal(oracle.pack_indices(exact[off:off + m]), pk.reshape(-1))
        off += m
    print(f"config {config}: {x.shape[0]} sampled atoms of {len(ws)} matrices equal the oracle")


def test_bf16_equals_fp32_widening(mods, oracle):
    C, P, _, _ = mods
    g = torch.Generator(device="cuda").manual_seed(21)
    xb = (torch.randn(100_000, 24, generator=g, device="cuda") * 0.02).to(torch.bfloat16)
    for rule in (0, 1):
        a = C.quantize_indices(xb, rule)
        b = C.quantize_indices(xb.float(), rule)
        assert torch.equal(a, b)
    sub = xb[:2000].float().cpu().numpy()
    assert np.array_equal(C.quantize_indices(xb[:2000], 1).cpu().numpy(), oracle.nearest_exact(sub, 1))
    w = (torch.randn(96, 1920, generator=g, device="cuda") * 0.02).to(torch.bfloat16)
    (pb, sb), (pf, sf) = P.quantize_layers([w, w.float()])
    assert torch.equal(pb, pf) and torch.equal(sb, sf)
    # The host bf16 path of the drop-in returns the same bytes.
    cb = C.get_h24_codebook("cpu", torch.float32)
    ph, sh = P._quantize_h24_layer(w.cpu(), cb)
    assert torch.equal(ph, pb.cpu()) and torch.equal(sh, sb.cpu())


@pytest.mark.parametrize("shape", [(5760, 1920), (1920, 7680), (1152, 1152), (100, 1920), (13, 192)])
def test_row_shards_concatenate(mods, shape):
    C, P, SH, _ = mods
    g = torch.Generator(device="cuda").manual_seed(shape[0])
    w = (torch.randn(*shape, generator=g, device="cuda") * 0.02).to(torch.bfloat16)
    whole_p, whole_s = P.quantize_layers([w])[0]
    rows, in_f = shape
    for world in (2, 3, 4, 8):
        parts = [(w, *SH.shard_rows(rows, in_f, world, r)) for r in range(world)]
        res = P.quantize_layer_rows(parts)
        assert torch.equal(torch.cat([p for p, _ in res]), whole_p)
        assert torch.equal(torch.cat([s for _, s in res]), whole_s)
    # A shard of a host weight through the chunked host path.
    r0, r1 = SH.shard_rows(rows, in_f, 4, 1)
    ph, sh = P.quantize_layer_rows_host(w.cpu().contiguous(), r0, r1)
    b0, b1 = SH.packed_range(r0, r1, in_f)
    assert torch.equal(ph, whole_p[b0:b1].cpu()) and torch.equal(sh, whole_s[r0:r1].cpu())


def test_host_pipeline_many_small_matrices(mods):
    """More row ranges than one batch holds (the host pipeline closes a batch
    at 64 pieces), of assorted widths and row starts, through one call: every
    range's bytes and scales equal the device path's for those rows."""
    C, P, SH, _ = mods
    g = torch.Generator().manual_seed(17)
    shapes = [(8 + (k % 5) * 4, (1 + k % 7) * 24) for k in range(80)]
    ws = [(torch.randn(o, i, generator=g) * 0.02).to(torch.bfloat16).pin_memory() for o, i in shapes]
    parts = []
    for k, w in enumerate(ws):
        rows, in_f = w.shape
        world = 1 + k % 3
        parts.append((w, *SH.shard_rows(rows, in_f, world, world - 1)))
    res = P.quantize_layers_host(parts)
    assert len(res) == len(parts)
    for (w, r0, r1), (p, s) in zip(parts, res):
        wp, wsig = P.quantize_layers([w.cuda()])[0]
        b0, b1 = SH.packed_range(r0, r1, w.shape[1])
        assert torch.equal(p, wp[b0:b1].cpu()) and torch.equal(s, wsig[r0:r1].cpu())


def test_row_range_validation(mods):
    C, P, _, _ = mods
    w = torch.randn(16, 72, device="cuda")  # 3 atoms per row: groups end every 4 rows
    with pytest.raises(ValueError):
        P.quantize_layer_rows([(w, 1, 8)])  # starts inside a 4-atom group
    with pytest.raises(ValueError):
        P.quantize_layer_rows([(w, 0, 5)])  # ends inside a group before the last row
    with pytest.raises(ValueError):
        P.quantize_layer_rows([(w, 8, 20)])  # beyond the matrix
    (p, s), = P.quantize_layer_rows([(w, 4, 16)])
    whole_p, whole_s = P.quantize_layers([w])[0]
    assert torch.equal(p, whole_p[27:]) and torch.equal(s, whole_s[4:])


def test_state_dict_loop_equals_per_matrix_calls(mods):
    """pack_checkpoint's tensor loop (pack.py:268-287) through
    quantize_state_dict: every H24 matrix of the (host) state_dict in one
    pipelined call, INT8 for tok_emb / head, pass-through for the rest; each
    output equals the per-matrix drop-in call."""
    C, P, SH, _ = mods
    g = torch.Generator().manual_seed(5)
    state = {
        "tok_emb.weight": torch.randn(300, 192, generator=g) * 0.02,
        "pos_emb.weight": torch.randn(64, 192, generator=g) * 0.02,
        "layers.0.qkv.weight": (torch.randn(576, 192, generator=g) * 0.02).to(torch.bfloat16).pin_memory(),
        "layers.0.o.weight": (torch.randn(192, 192, generator=g) * 0.02).to(torch.bfloat16).pin_memory(),
        "layers.0.norm.gain": torch.ones(192),
        "layers.0.up.weight": torch.randn(768, 192, generator=g) * 0.02,        # fp32, pageable
        "layers.0.down.weight": (torch.randn(192, 768, generator=g) * 0.02).cuda(),  # on the GPU
        "layers.1.big.weight": (torch.randn(7000, 1920, generator=g) * 0.02).to(torch.bfloat16),
        "head.weight": torch.randn(300, 192, generator=g) * 0.02,
    }
    cb = C.get_h24_codebook("cpu", torch.float32)
    out = P.quantize_state_dict(state, cb)
    assert list(out) == ["tok_emb.weight_int8", "tok_emb.mu_rows", "pos_emb.weight",
                         "layers.0.qkv.packed_weights", "layers.0.qkv.sigma_rows",
                         "layers.0.o.packed_weights", "layers.0.o.sigma_rows", "layers.0.norm.gain",
                         "layers.0.up.packed_weights", "layers.0.up.sigma_rows",
                         "layers.0.down.packed_weights", "layers.0.down.sigma_rows",
                         "layers.1.big.packed_weights", "layers.1.big.sigma_rows",
                         "head.weight_int8", "head.mu_rows"]
    for n, t in state.items():
        base = n[:-len(".weight")]
        if n in ("tok_emb.weight", "head.weight"):
            q, mu = P._quantize_int8(t)
            assert torch.equal(out[base + ".weight_int8"], q) and torch.equal(out[base + ".mu_rows"], mu)
        elif n.endswith(".weight") and n != "pos_emb.weight":
            p, s = P._quantize_h24_layer(t, cb)
            assert torch.equal(out[base + ".packed_weights"], p.cpu())
            assert torch.equal(out[base + ".sigma_rows"], s.cpu())
            assert out[base + ".packed_weights"].device.type == "cpu"
        else:
            assert torch.equal(out[n], t)
    # Row ranges of several host matrices in one pipeline.
    ws = [state["layers.1.big.weight"], state["layers.0.qkv.weight"]]
    parts = [(ws[0], *SH.shard_rows(7000, 1920, 3, 1)), (ws[1], *SH.shard_rows(576, 192, 3, 2))]
    for (w, r0, r1), (p, s) in zip(parts, P.quantize_layers_host(parts)):
        wp, wsig = P.quantize_layers([w.cuda()])[0]
        b0, b1 = SH.packed_range(r0, r1, w.shape[1])
        assert torch.equal(p, wp[b0:b1].cpu()) and torch.equal(s, wsig[r0:r1].cpu())
