#!/usr/bin/env python3
"""Generate the golden fixtures in tests/golden/ by running the REFERENCE's own
Python code (alavicka/pollux: castor.py, pack.py, pollux.py) on seeded inputs.

The reference is imported read-only from the path given by --reference (its
checkout is not available on the GPU machines, which is why its outputs are
frozen here).  Run from the repository root:

    PYTHONDONTWRITEBYTECODE=1 python tests/golden/make_golden.py --reference <path>

Fixtures written (all small):
  codebook.json          SHA-256 of the fp32 / fp16 / raw-int8 codebook, the
                         fingerprint (castor.py:263) and c_sq_norm (castor.py:522)
  pack_vectors.npz       pack_indices / unpack_indices in/out pairs, including
                         ragged lengths and out-of-range values (castor.py:226-260)
  config1.npz            config 1 (1152x1152, seed 0): pack._quantize_h24_layer
                         packed bytes + sigma16 (pack.py:139-180) and the
                         training-rule indices of castor_quantize_leech's CPU
                         path (castor.py:487-560, bf16 autocast scores)
  stress.npz             4096 config-4 atoms (seed 3) with the reference's
                         pack-rule and training-rule indices
  materialize.npz        PackedH24Linear.materialize outputs (pollux.py:485-504)
  tiny.plx, plx_state.npz  (with --plx) a .plx written by pack._write_plx and
                         the tensors that went into it
  int8.npz               (with --int8) pack._quantize_int8 and
                         PackedInt8Embedding/Linear.materialize on seeded and
                         edge-case matrices (pack.py:124-136, pollux.py:510-563)
"""
from __future__ import annotations

import argparse
import hashlib
import json
import os
import sys
import time

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))


def sha(a: np.ndarray) -> str:
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def vectors_to_indices(vec: torch.Tensor, raw_table: np.ndarray) -> np.ndarray:
    """Map codeword vectors (exact rows of the fp32 codebook) back to indices."""
    raw = np.rint(vec.float().numpy().reshape(-1, 24) * np.sqrt(8.0)).astype(np.int8)
    lut = {raw_table[k].tobytes(): k for k in range(raw_table.shape[0])}
    return np.array([lut[r.tobytes()] for r in raw], dtype=np.int32)


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True, help="path of the reference checkout")
    ap.add_argument("--plx", action="store_true", help="only write the .plx fixture")
    ap.add_argument("--int8", action="store_true", help="only write the INT8 fixture")
    args = ap.parse_args()
    if args.plx:
        make_plx(args.reference)
        return
    if args.int8:
        make_int8(args.reference)
        return
    sys.path.insert(0, args.reference)
    sys.path.insert(0, REPO)
    import castor  # noqa: E402  (reference)
    import pack as ref_pack  # noqa: E402  (reference)
    import pollux as ref_pollux  # noqa: E402  (reference)
    from pollux_b200 import synth  # noqa: E402

    torch.manual_seed(1234)
    cb = castor.get_h24_codebook("cpu", torch.float32)
    cb_np = cb.numpy()
    raw = np.rint(cb_np * np.sqrt(8.0)).astype(np.int8)
    meta = {
        "count": int(cb.shape[0]),
        "sha256_f32": sha(cb_np),
        "sha256_f16": sha(cb.to(torch.float16).numpy()),
        "sha256_raw_int8": sha(raw),
        "fingerprint": list(castor.codebook_fingerprint()),
        "c_sq_norm": float(cb[1:][0].pow(2).sum().item()),
        "values_f32": sorted(set(float(v) for v in np.unique(cb_np))),
        "values_f16": sorted(set(float(v) for v in np.unique(cb.to(torch.float16).numpy()))),
        "rows_sample": {str(k): raw[k].tolist() for k in (0, 1, 2, 3, 1104, 98256, 196559, 196560)},
    }
    with open(os.path.join(HERE, "codebook.json"), "w") as f:
        json.dump(meta, f, indent=1)
    print("codebook.json written")

    # ---- pack / unpack vectors -------------------------------------------
    rng = np.random.default_rng(7)
    pv = {}
    lengths = [0, 1, 2, 3, 4, 5, 7, 8, 9, 13, 64, 1000, 4099]
    for n in lengths:
        v = rng.integers(0, 196561, size=n, dtype=np.int64)
        if n >= 4:
            v[0], v[1], v[2], v[3] = 0, 196560, (1 << 18) - 1, 1
        p = castor.pack_indices(torch.from_numpy(v)).numpy()
        pv[f"idx_{n}"] = v
        pv[f"packed_{n}"] = p
        u = castor.unpack_indices(torch.from_numpy(p), n).numpy()
        pv[f"unpacked_{n}"] = u
    # Out-of-range and negative inputs: the reference truncates silently.
    odd = np.array([1 << 18, (1 << 20) + 5, -1, -123456, (1 << 33) + 7, 2**31 - 1, -(2**31), 5],
                   dtype=np.int64)
    pv["idx_odd"] = odd
    pv["packed_odd"] = castor.pack_indices(torch.from_numpy(odd)).numpy()
    # Unpack of random bytes with num_indices below / at / above capacity.
    rb = rng.integers(0, 256, size=9 * 37, dtype=np.uint8)
    pv["rand_bytes"] = rb
    for k in (0, 1, 100, 148, 200):
        pv[f"rand_unpacked_{k}"] = castor.unpack_indices(torch.from_numpy(rb.copy()), k).numpy()
    np.savez_compressed(os.path.join(HERE, "pack_vectors.npz"), **pv)
    print("pack_vectors.npz written")

    # ---- config 1 ---------------------------------------------------------
    w = synth.config1_weight("cpu")
    t = time.time()
    packed, sigma16 = ref_pack._quantize_h24_layer(w, cb)
    t_pack = time.time() - t
    normed, _sig = castor.normalize_matrix_by_row_rms(w)
    x = normed / float(castor.s_lattice)
    t = time.time()
    centers = castor.castor_quantize_leech(x, cb)
    t_train = time.time() - t
    train_idx = vectors_to_indices(centers, raw)
    np.savez_compressed(
        os.path.join(HERE, "config1.npz"),
        weight_sha256=np.array(sha(w.numpy())),
        pack_packed=packed.numpy(),
        pack_sigma16=sigma16.numpy(),
        train_x_sha256=np.array(sha(x.numpy())),
        train_bf16_packed=castor.pack_indices(torch.from_numpy(train_idx.astype(np.int64))).numpy(),
        seconds=np.array([t_pack, t_train]),
    )
    print(f"config1.npz written (pack rule {t_pack:.1f}s, training rule {t_train:.1f}s)")

    # ---- stress subset (config 4 distribution) ---------------------------
    xs = synth.stress_atoms(4096, cb, seed=3, device="cpu")
    p_s, _ = ref_pack._quantize_h24_layer(xs, cb)
    pack_rule_idx = castor.unpack_indices(p_s, xs.shape[0]).numpy().astype(np.int32)
    train_rule_idx = vectors_to_indices(castor.castor_quantize_leech(xs, cb), raw)
    np.savez_compressed(os.path.join(HERE, "stress.npz"), atoms=xs.numpy(),
                        pack_rule_idx=pack_rule_idx, train_bf16_idx=train_rule_idx)
    print("stress.npz written")

    # ---- materialize -------------------------------------------------------
    mat = {}
    for tag, (rows, in_f, seed) in {"a": (48, 192, 11), "b": (3, 24, 12), "c": (5, 72, 13)}.items():
        g = torch.Generator().manual_seed(seed)
        n_atoms = rows * in_f // 24
        idx = torch.randint(0, 196561, (n_atoms,), generator=g)
        idx[: min(4, n_atoms)] = torch.tensor([0, 196560, 1, 98256])[: min(4, n_atoms)]
        sig = (torch.rand(rows, generator=g) * 0.09 + 0.01).to(torch.float16)
        layer = ref_pollux.PackedH24Linear(in_f, rows)
        layer.packed_weights.copy_(castor.pack_indices(idx))
        layer.sigma_rows.copy_(sig)
        layer.materialize()
        mat[f"{tag}_shape"] = np.array([rows, in_f])
        mat[f"{tag}_packed"] = castor.pack_indices(idx).numpy()
        mat[f"{tag}_sigma16"] = sig.numpy()
        mat[f"{tag}_weight16"] = layer.weight.detach().numpy()
    # Extreme scales: tiny (fp16 subnormal) and large sigma.
    rows, in_f = 4, 48
    idx = torch.tensor([1, 196560, 1104, 98256, 50000, 7, 150000, 0])
    sig = torch.tensor([6.0e-8, 1.0e-3, 7.5, 6.0e4], dtype=torch.float16)
    layer = ref_pollux.PackedH24Linear(in_f, rows)
    layer.packed_weights.copy_(castor.pack_indices(idx))
    layer.sigma_rows.copy_(sig)
    layer.materialize()
    mat["d_shape"] = np.array([rows, in_f])
    mat["d_packed"] = castor.pack_indices(idx).numpy()
    mat["d_sigma16"] = sig.numpy()
    mat["d_weight16"] = layer.weight.detach().numpy()
    np.savez_compressed(os.path.join(HERE, "materialize.npz"), **mat)
    print("materialize.npz written")



def make_plx(reference: str) -> None:
    """tiny.plx written by the reference's own pack._write_plx (pack.py:187-247)
    plus the tensors that went in (plx_state.npz)."""
    sys.path.insert(0, reference)
    sys.path.insert(0, REPO)
    import castor  # noqa: E402
    import pack as ref_pack  # noqa: E402
    g = torch.Generator().manual_seed(21)
    idx = torch.randint(0, 196561, (96 * 4,), generator=g)
    state = {
        "blocks.0.attn.q.packed_weights": castor.pack_indices(idx),
        "blocks.0.attn.q.sigma_rows": (torch.rand(96, generator=g) * 0.1).to(torch.float16),
        "tok_emb.weight_int8": torch.randint(-128, 128, (7, 24), generator=g, dtype=torch.int8),
        "ln_f.weight": torch.randn(24, generator=g),
        "head.mu_rows": (torch.rand(7, generator=g) + 0.5).to(torch.float16),
    }
    cfg = {"n_embd": 24, "n_layers": 1, "scales_per_row": 1, "note": "tiny fixture"}
    path = os.path.join(HERE, "tiny.plx")
    ref_pack._write_plx(path, cfg, state)
    np.savez_compressed(os.path.join(HERE, "plx_state.npz"),
                        **{k.replace(".", "__"): (v.float().numpy() if v.dtype == torch.bfloat16
                                                  else v.numpy()) for k, v in state.items()},
                        config=np.array(json.dumps(cfg)))
    print("tiny.plx written")



def make_int8(reference: str) -> None:
    """int8.npz: the reference's pack._quantize_int8 and the INT8 modules'
    materialize() on seeded and edge-case matrices."""
    sys.path.insert(0, reference)
    import pack as ref_pack  # noqa: E402
    import pollux as ref_pollux  # noqa: E402
    g = torch.Generator().manual_seed(31)
    cases = {
        "normal": torch.randn(64, 1152, generator=g) * 0.02,
        "odd": torch.randn(5, 37, generator=g),
    }
    # Exact ties at .5: a row with max 1.0 and values i/256 (127 i / 256 is exact).
    cases["ties"] = torch.arange(-256, 257, dtype=torch.float32).reshape(1, -1) / 256.0
    e = torch.randn(8, 48, generator=g)
    e[0] = 0.0                      # zero row: mu clamps to 1e-8
    e[1, 3] = float("nan")          # NaN row
    e[2, 5] = float("inf")          # inf row
    e[3] *= 1e5                     # mu above the fp16 range -> inf
    e[4] *= 1e-6                    # fp16-subnormal mu
    e[5, :] = 1e-9                  # below the clamp
    cases["edge"] = e
    out = {}
    for k, w in cases.items():
        q, mu = ref_pack._quantize_int8(w)
        out[f"{k}_w"] = w.numpy()
        out[f"{k}_q"] = q.numpy()
        out[f"{k}_mu"] = mu.numpy()
        rows, cols = w.shape
        emb = ref_pollux.PackedInt8Embedding(rows, cols)
        emb.weight_int8.copy_(q)
        emb.mu_rows.copy_(mu)
        emb.materialize()
        out[f"{k}_emb"] = emb.weight.detach().numpy()
        head = ref_pollux.PackedInt8Linear(cols, rows)
        head.weight_int8.copy_(q)
        head.mu_rows.copy_(mu)
        head.materialize()
        out[f"{k}_head"] = head.weight.detach().numpy()
    np.savez_compressed(os.path.join(HERE, "int8.npz"), **out)
    print("int8.npz written")


if __name__ == "__main__":
    main()
