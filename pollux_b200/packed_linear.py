"""Drop-in mirror of ``PackedH24Linear`` and its ``materialize`` (pollux.py:461-507),
the inference-time LUT dequantisation, on libh24.

``materialize`` rebuilds the dense fp16 weight from the packed 18-bit indices
and the per-row fp16 scales,
    weight = fp16( fp32( fp16(cb16[idx] * sigma16[row]) ) * fp32(s_lattice) ),
bit-identical to the reference's two torch multiplications (pollux.py:497-499),
then drops the packed buffers exactly as the reference does (pollux.py:500-504).
``materialize_all`` dequantises every packed layer of a model with one launch
per 64 layers (the loop of from_packed_checkpoint, pollux.py:748-750).

``lut_linear`` computes ``x @ W.T`` straight from the packed indices (the
README's "future native kernel", README.md:88, 155-156) with W never
materialised; ``PackedH24Linear.forward`` uses it until the layer is
materialised, and ``enable_lut_forward`` switches the packed layers of any
model (the reference's included) to it.

``PackedInt8Embedding`` / ``PackedInt8Linear`` (pollux.py:510-563) and
``materialize_int8`` rebuild the INT8 token embedding and output head,
weight = fp16(q * fp16(mu / 127)), with one launch per tensor.
"""
from __future__ import annotations

import ctypes

import torch
import torch.nn as nn
import torch.nn.functional as F

from . import _native as N
from .castor import (BYTES_PER_CHUNK, H24_DIM, _aligned, _call, _stream, _work_device,
                     assert_row_aligned_in_features, h24_linear_atom_count,
                     h24_linear_scale_row_count)


def _raise_bad(bad: torch.Tensor) -> None:
    n = int(bad.item())
    if n:
        raise IndexError(f"index out of range in self ({n} packed indices exceed 196560)")


def dequant(packed: torch.Tensor, sigma_rows: torch.Tensor, out_features: int,
            in_features: int) -> torch.Tensor:
    """fp16 [out_features, in_features] weight from packed indices and fp16 row scales."""
    if sigma_rows.dtype != torch.float16:
        raise TypeError(f"sigma_rows must be float16, got {sigma_rows.dtype}")
    atoms = h24_linear_atom_count(out_features, in_features)
    if in_features % H24_DIM != 0:
        raise ValueError(f"in_features must be a multiple of {H24_DIM}, got {in_features}")
    need = ((atoms + 3) // 4) * BYTES_PER_CHUNK
    flat = packed.reshape(-1)
    if flat.dtype != torch.uint8 or flat.numel() < need:
        raise ValueError(f"packed_weights must be uint8 with at least {need} bytes")
    if sigma_rows.numel() < out_features:
        raise ValueError(f"sigma_rows must hold {out_features} scales")
    dev = _work_device(flat)
    p = flat.to(dev).contiguous()
    s = sigma_rows.reshape(-1).to(dev).contiguous()
    out = torch.empty(out_features, in_features, dtype=torch.float16, device=dev)
    bad = torch.zeros(1, dtype=torch.int32, device=dev)
    _call(dev, "h24_dequant", p.data_ptr(), s.data_ptr(), out_features, in_features,
          out.data_ptr(), bad.data_ptr(), _stream(dev))
    _raise_bad(bad)
    return out


def materialize(self) -> None:
    """PackedH24Linear.materialize (pollux.py:485-504) on libh24."""
    if self._materialized:
        return
    weight = dequant(self.packed_weights, self.sigma_rows, self.out_features, self.in_features)
    self.weight = nn.Parameter(weight.to(self.packed_weights.device), requires_grad=False)
    del self.packed_weights
    del self.sigma_rows
    self._materialized = True


LUT_GEMV_MAX_BATCH = 32  # larger batches: dequantise once and use a dense GEMM


def lut_linear(x: torch.Tensor, packed: torch.Tensor, sigma_rows: torch.Tensor, out_features: int,
               in_features: int, bias: torch.Tensor | None = None) -> torch.Tensor:
    """F.linear(x, W, bias) for the packed H24 weight W ([out_features,
    in_features], the fp16 values materialize() produces), computed in fp32
    without materialising W for up to LUT_GEMV_MAX_BATCH input rows; the result
    has x's dtype."""
    if x.shape[-1] != in_features:
        raise RuntimeError(f"mat1 and mat2 shapes cannot be multiplied "
                           f"({x.numel() // max(1, x.shape[-1])}x{x.shape[-1]} and {in_features}x{out_features})")
    if sigma_rows.dtype != torch.float16:
        raise TypeError(f"sigma_rows must be float16, got {sigma_rows.dtype}")
    lead = x.shape[:-1]
    batch = x.numel() // in_features if in_features else 0
    dev = _work_device(x)
    if batch > LUT_GEMV_MAX_BATCH:
        w = dequant(packed, sigma_rows, out_features, in_features).float()
        y = torch.matmul(x.to(device=dev, dtype=torch.float32).reshape(batch, in_features), w.t())
    else:
        atoms = h24_linear_atom_count(out_features, in_features)
        need = ((atoms + 3) // 4) * BYTES_PER_CHUNK
        flat = packed.reshape(-1)
        if flat.dtype != torch.uint8 or flat.numel() < need:
            raise ValueError(f"packed_weights must be uint8 with at least {need} bytes")
        p = flat.to(dev).contiguous()
        s = sigma_rows.reshape(-1).to(dev).contiguous()
        xf = _aligned(x.to(device=dev, dtype=torch.float32).reshape(batch, in_features))
        y = torch.empty(batch, out_features, dtype=torch.float32, device=dev)
        bad = torch.zeros(1, dtype=torch.int32, device=dev)
        if batch:
            _call(dev, "h24_lut_gemv", p.data_ptr(), s.data_ptr(), out_features, in_features,
                  xf.data_ptr(), batch, y.data_ptr(), bad.data_ptr(), _stream(dev))
            _raise_bad(bad)
    y = y.reshape(*lead, out_features)
    if bias is not None:
        y = y + bias.to(y)
    return y.to(x.dtype)


def _lut_forward(self, x: torch.Tensor) -> torch.Tensor:
    if getattr(self, "_materialized", False):
        return F.linear(x, self.weight.to(dtype=x.dtype), self.bias)
    return lut_linear(x, self.packed_weights, self.sigma_rows, self.out_features, self.in_features,
                      self.bias)


def enable_lut_forward(model: nn.Module) -> int:
    """Make every not-yet-materialised packed H24 layer of ``model`` run its
    forward through the LUT GEMV (instance attribute, so the reference's
    PackedH24Linear is covered too); returns the number of layers."""
    n = 0
    for m in model.modules():
        if hasattr(m, "packed_weights") and hasattr(m, "sigma_rows") and not getattr(m, "_materialized", False):
            m.forward = _lut_forward.__get__(m, type(m))
            n += 1
    return n


class PackedH24Linear(nn.Module):
    """H24 linear layer with packed uint8 indices + fp16 per-row sigma
    (same buffers, shapes and forward as pollux.py:461-507)."""

    def __init__(self, in_features: int, out_features: int, bias: bool = False) -> None:
        super().__init__()
        assert_row_aligned_in_features(in_features)
        self.in_features = int(in_features)
        self.out_features = int(out_features)
        self.num_atoms = h24_linear_atom_count(self.out_features, self.in_features)
        self.num_sigma_rows = h24_linear_scale_row_count(self.out_features)
        packed_len = ((self.num_atoms + 3) // 4) * BYTES_PER_CHUNK
        self.register_buffer("packed_weights", torch.zeros(packed_len, dtype=torch.uint8))
        self.register_buffer("sigma_rows", torch.ones(self.num_sigma_rows, dtype=torch.float16))
        self._materialized = False
        if bias:
            self.bias = nn.Parameter(torch.zeros(self.out_features))
        else:
            self.register_parameter("bias", None)

    materialize = materialize

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        """F.linear with the materialised weight, as the reference; before
        materialize(), the LUT GEMV over the packed indices."""
        return _lut_forward(self, x)


def materialize_all(model: nn.Module) -> int:
    """Materialise every not-yet-materialised packed H24 layer of ``model`` with
    batched launches; returns the number of layers.  Layers must already be on
    one CUDA device (as after model.to(device))."""
    mods = [m for m in model.modules()
            if hasattr(m, "packed_weights") and hasattr(m, "sigma_rows")
            and not getattr(m, "_materialized", False)]
    if not mods:
        return 0
    dev = mods[0].packed_weights.device
    if dev.type != "cuda":
        for m in mods:
            materialize(m)
        return len(mods)
    layers = (N.DequantLayer * len(mods))()
    outs, keep = [], []
    for i, m in enumerate(mods):
        if m.sigma_rows.dtype != torch.float16:
            raise TypeError(f"sigma_rows must be float16, got {m.sigma_rows.dtype}")
        p = m.packed_weights.contiguous()
        s = m.sigma_rows.contiguous()
        o = torch.empty(m.out_features, m.in_features, dtype=torch.float16, device=dev)
        keep += [p, s]
        outs.append(o)
        layers[i] = N.DequantLayer(p.data_ptr(), s.data_ptr(), o.data_ptr(),
                                   m.out_features, m.in_features)
    bad = torch.zeros(1, dtype=torch.int32, device=dev)
    _call(dev, "h24_dequant_batched", ctypes.cast(layers, ctypes.c_void_p), len(mods),
          bad.data_ptr(), _stream(dev))
    _raise_bad(bad)
    for m, o in zip(mods, outs):
        m.weight = nn.Parameter(o, requires_grad=False)
        del m.packed_weights
        del m.sigma_rows
        m._materialized = True
    return len(mods)


def int8_dequant(weight_int8: torch.Tensor, mu_rows: torch.Tensor) -> torch.Tensor:
    """fp16 weight = q * (mu / 127) per row, both fp16 roundings of the
    reference (pollux.py:519-523)."""
    if weight_int8.dtype != torch.int8:
        raise TypeError(f"weight_int8 must be int8, got {weight_int8.dtype}")
    if mu_rows.dtype != torch.float16:
        raise TypeError(f"mu_rows must be float16, got {mu_rows.dtype}")
    dev = _work_device(weight_int8)
    cols = weight_int8.shape[-1]
    rows = weight_int8.numel() // cols if cols else 0
    if mu_rows.numel() != rows:
        raise RuntimeError(f"mu_rows has {mu_rows.numel()} scales for {rows} rows")
    q = _aligned(weight_int8.to(dev).reshape(rows, cols))
    mu = mu_rows.reshape(-1).to(dev).contiguous()
    out = torch.empty(rows, cols, dtype=torch.float16, device=dev)
    if rows and cols:
        _call(dev, "h24_int8_dequant", q.data_ptr(), mu.data_ptr(), rows, cols, out.data_ptr(),
              _stream(dev))
    return out.reshape(weight_int8.shape)


def materialize_int8(self) -> None:
    """PackedInt8Embedding.materialize / PackedInt8Linear.materialize
    (pollux.py:519-528, 545-554) on libh24."""
    if self._materialized:
        return
    weight = int8_dequant(self.weight_int8, self.mu_rows)
    self.weight = nn.Parameter(weight.to(self.weight_int8.device), requires_grad=False)
    del self.weight_int8
    del self.mu_rows
    self._materialized = True


class PackedInt8Embedding(nn.Module):
    """Token embedding with INT8 weights and per-row FP16 scales mu (same
    buffers and forward as pollux.py:510-532)."""

    def __init__(self, num_embeddings: int, embedding_dim: int) -> None:
        super().__init__()
        self.num_embeddings = int(num_embeddings)
        self.embedding_dim = int(embedding_dim)
        self.register_buffer("weight_int8", torch.zeros(num_embeddings, embedding_dim, dtype=torch.int8))
        self.register_buffer("mu_rows", torch.ones(num_embeddings, dtype=torch.float16))
        self._materialized = False

    materialize = materialize_int8

    def forward(self, idx: torch.Tensor) -> torch.Tensor:
        return F.embedding(idx, self.weight.to(dtype=torch.float32))


class PackedInt8Linear(nn.Module):
    """Output projection with INT8 weights and per-row FP16 scales mu (same
    buffers and forward as pollux.py:535-558)."""

    def __init__(self, in_features: int, out_features: int, bias: bool = False) -> None:
        super().__init__()
        self.in_features = int(in_features)
        self.out_features = int(out_features)
        self.register_buffer("weight_int8", torch.zeros(out_features, in_features, dtype=torch.int8))
        self.register_buffer("mu_rows", torch.ones(out_features, dtype=torch.float16))
        self._materialized = False
        if bias:
            self.bias = nn.Parameter(torch.zeros(out_features))
        else:
            self.register_parameter("bias", None)

    materialize = materialize_int8

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        return F.linear(x, self.weight.to(dtype=x.dtype), self.bias)
