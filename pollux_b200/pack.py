"""Drop-in mirror of the reference's ``pack._quantize_h24_layer``
(pack.py:139-180) and ``pack._quantize_int8`` (pack.py:124-136), the
checkpoint -> .plx quantisers, on libh24.

``_quantize_h24_layer(weight, codebook) -> (packed_u8_cpu, sigma_f16_cpu)``:
  * sigma_rows = fp16(clamp_min(sqrt(mean(w^2)+1e-8) * sqrt(12), 1e-8)) per row
    (pack.py:164);
  * atoms = w.reshape(-1, 24); index = argmax(atom . kp) + 1, 0 only when
    ||atom||_2 < 1e-8 (pack.py:166-177) -- computed as the exact fp64 argmax
    with the lowest index on ties;
  * packed with the 18-bit format (pack.py:179, castor.py:226-246).
Quantisation, scale and packing run in one pass on the GPU
(h24_quantize_layer); only the results are copied back to the host, as the
reference returns them.
"""
from __future__ import annotations

import ctypes

import torch

from . import _native as N
from .castor import (BYTES_PER_CHUNK, H24_DIM, _aligned, _call, _check_codebook, _stream,
                     _work_device, device_check)


_LAYER_DTYPES = {torch.float32: N.DTYPE_F32, torch.bfloat16: N.DTYPE_BF16}


def _layer_input(w: torch.Tensor, dev: torch.device) -> tuple[torch.Tensor, int]:
    """The weight on ``dev`` in a dtype the kernels read directly (fp32 or
    bf16, widened exactly in registers); other dtypes go through weight.float()
    as the reference does (pack.py:159)."""
    code = _LAYER_DTYPES.get(w.dtype)
    if code is None:
        return _aligned(w.to(device=dev, dtype=torch.float32)), N.DTYPE_F32
    return _aligned(w.to(device=dev)), code


def _quantize_h24_layer(weight: torch.Tensor, codebook: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """Map an H24 weight matrix to packed 18-bit indices + per-row FP16 sigma."""
    w = weight.detach()
    if w.dim() != 2:
        raise ValueError(f"row_rms_from_matrix expects a 2D weight matrix, got {w.dim()}D.")
    if w.numel() % H24_DIM != 0:
        raise RuntimeError(f"shape '[-1, {H24_DIM}]' is invalid for input of size {w.numel()}")
    _check_codebook(codebook)
    rows, in_f = w.shape
    atoms = w.numel() // H24_DIM
    dev = _work_device(w)
    if w.device.type == "cpu" and w.dtype in _LAYER_DTYPES and w.is_contiguous():
        # Host weight: the chunked host entry overlaps the copy of one chunk
        # with the search of the previous one and fills host outputs (bf16
        # crosses PCIe at two bytes per parameter).
        pin = w.is_pinned()
        packed = torch.empty(((atoms + 3) // 4) * BYTES_PER_CHUNK, dtype=torch.uint8, pin_memory=pin)
        sigma = torch.empty(rows, dtype=torch.float16, pin_memory=pin)
        if rows:
            L = N.LayerRows(w.data_ptr(), rows, in_f, 0, rows, sigma.data_ptr(), packed.data_ptr())
            _call(dev, "h24_quantize_layer_rows_host", ctypes.byref(L), _LAYER_DTYPES[w.dtype], _stream(dev))
        return packed, sigma
    packed, sigma = quantize_layer_device(w)
    packed, sigma = packed.cpu(), sigma.cpu()
    device_check(dev)
    return packed, sigma


def quantize_layer_device(weight: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """Device-resident variant: (packed u8, sigma16) left on the weight's CUDA
    device (the staging device for a host weight)."""
    return quantize_layers([weight])[0]


def quantize_layers(weights: list[torch.Tensor]) -> list[tuple[torch.Tensor, torch.Tensor]]:
    """Pack-rule quantisation of many 2-D weights (on one CUDA device) with one
    shared search pipeline; returns device-resident (packed u8, sigma16) pairs.
    fp32 and bf16 weights are read as they are (one pipeline per dtype)."""
    return quantize_layer_rows([(w, 0, w.shape[0] if w.dim() == 2 else 0) for w in weights])


def quantize_layer_rows(parts: list[tuple[torch.Tensor, int, int]],
                        outs: list[tuple[torch.Tensor, torch.Tensor]] | None = None
                        ) -> list[tuple[torch.Tensor, torch.Tensor]]:
    """Pack-rule quantisation of rows [begin, end) of each 2-D weight (the row
    shard of one rank), all on one CUDA device, in one shared search pipeline
    per dtype.  Returns per part the device-resident (packed u8, sigma16) of
    those rows: the bytes and scales the whole-matrix call writes for them
    (row scales included, bit for bit).  A range must start on a 4-atom group
    and end on one or at the last row (pollux_b200.shard.shard_rows).
    ``outs`` optionally gives the (packed, sigma16) device tensors to write,
    e.g. views of one buffer that a collective then gathers."""
    if not parts:
        return []
    dev = _work_device(parts[0][0])
    given = outs
    outs = []
    by_dtype: dict[int, list] = {}
    keep = []
    for (w, r0, r1) in parts:
        if w.dim() != 2 or w.numel() % H24_DIM != 0:
            raise ValueError(f"weights must be 2-D with a multiple of {H24_DIM} elements, got {tuple(w.shape)}")
        wd, code = _layer_input(w.detach(), dev)
        keep.append(wd)
        rows, in_f = wd.shape
        atoms = (r1 - r0) * in_f // H24_DIM
        nbytes = ((atoms + 3) // 4) * BYTES_PER_CHUNK
        if given is not None:
            packed, sigma = given[len(outs)]
            if (packed.numel() != nbytes or packed.dtype != torch.uint8 or sigma.numel() != max(r1 - r0, 0)
                    or sigma.dtype != torch.float16 or packed.device != dev or sigma.device != dev):
                raise ValueError("outs must hold uint8 packed bytes and fp16 scales of each part's size")
        else:
            packed = torch.empty(nbytes, dtype=torch.uint8, device=dev)
            sigma = torch.empty(max(r1 - r0, 0), dtype=torch.float16, device=dev)
        by_dtype.setdefault(code, []).append(
            N.LayerRows(wd.data_ptr(), rows, in_f, r0, r1, sigma.data_ptr(), packed.data_ptr()))
        outs.append((packed, sigma))
    for code, lst in by_dtype.items():
        layers = (N.LayerRows * len(lst))(*lst)
        _call(dev, "h24_quantize_layer_rows", ctypes.cast(layers, ctypes.c_void_p), len(lst), code,
              _stream(dev))
    return outs


def quantize_layer_rows_host(weight: torch.Tensor, row_begin: int, row_end: int
                             ) -> tuple[torch.Tensor, torch.Tensor]:
    """Rows [row_begin, row_end) of a HOST weight (fp32 or bf16, contiguous)
    to host (packed u8, sigma16): only those rows cross PCIe, in chunks that
    overlap the search (page-locked outputs when the weight is pinned)."""
    w = weight.detach()
    if w.device.type != "cpu" or w.dtype not in _LAYER_DTYPES or not w.is_contiguous() or w.dim() != 2:
        raise ValueError("quantize_layer_rows_host wants a contiguous 2-D fp32 or bf16 host tensor")
    rows, in_f = w.shape
    atoms = (row_end - row_begin) * in_f // H24_DIM
    pin = w.is_pinned()
    packed = torch.empty(((atoms + 3) // 4) * BYTES_PER_CHUNK, dtype=torch.uint8, pin_memory=pin)
    sigma = torch.empty(max(row_end - row_begin, 0), dtype=torch.float16, pin_memory=pin)
    dev = _work_device(w)
    L = N.LayerRows(w.data_ptr(), rows, in_f, row_begin, row_end, sigma.data_ptr(), packed.data_ptr())
    _call(dev, "h24_quantize_layer_rows_host", ctypes.byref(L), _LAYER_DTYPES[w.dtype], _stream(dev))
    return packed, sigma


def quantize_int8_device(weight: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """Per-row INT8 quantisation on the GPU: (q int8 with weight's shape, mu
    fp16 with weight.shape[:-1]) on the weight's CUDA device (the staging
    device for host tensors)."""
    w = weight.detach()
    if w.dim() == 0:
        raise IndexError("Dimension specified as -1 but tensor has no dimensions")
    dev = _work_device(w)
    cols = w.shape[-1]
    rows = w.numel() // cols if cols else 0
    wd = _aligned(w.to(device=dev, dtype=torch.float32).reshape(rows, cols))
    q = torch.empty(rows, cols, dtype=torch.int8, device=dev)
    mu = torch.empty(rows, dtype=torch.float16, device=dev)
    if rows and cols:
        _call(dev, "h24_int8_quantize", wd.data_ptr(), rows, cols, q.data_ptr(), mu.data_ptr(),
              _stream(dev))
    return q.reshape(w.shape), mu.reshape(w.shape[:-1])


def _quantize_int8(weight: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """Per-row INT8 quantization with FP16 per-row operational scales mu
    (pack._quantize_int8): weight ~ (q / 127) * mu_rows[:, None].  Returns
    host tensors, as the reference does."""
    q, mu = quantize_int8_device(weight)
    return q.cpu(), mu.cpu()
