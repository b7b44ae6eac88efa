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
                     _work_device)


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
    if w.device.type == "cpu" and w.dtype == torch.float32 and w.is_contiguous():
        # Host fp32 weight: the chunked host entry overlaps the copy of one
        # chunk with the search of the previous one and fills host outputs.
        pin = w.is_pinned()
        packed = torch.empty(((atoms + 3) // 4) * BYTES_PER_CHUNK, dtype=torch.uint8, pin_memory=pin)
        sigma = torch.empty(rows, dtype=torch.float16, pin_memory=pin)
        if rows:
            _call(dev, "h24_quantize_layer_host", w.data_ptr(), rows, in_f, sigma.data_ptr(),
                  packed.data_ptr(), _stream(dev))
        return packed, sigma
    wd = _aligned(w.to(device=dev, dtype=torch.float32))
    packed = torch.empty(((atoms + 3) // 4) * BYTES_PER_CHUNK, dtype=torch.uint8, device=dev)
    sigma = torch.empty(rows, dtype=torch.float16, device=dev)
    if rows:
        _call(dev, "h24_quantize_layer", wd.data_ptr(), rows, in_f, sigma.data_ptr(),
              packed.data_ptr(), _stream(dev))
    return packed.cpu(), sigma.cpu()


def quantize_layer_device(weight: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """Device-resident variant: (packed u8, sigma16) left on the weight's CUDA device."""
    w = weight.detach()
    rows, in_f = w.shape
    atoms = w.numel() // H24_DIM
    dev = _work_device(w)
    wd = _aligned(w.to(device=dev, dtype=torch.float32))
    packed = torch.empty(((atoms + 3) // 4) * BYTES_PER_CHUNK, dtype=torch.uint8, device=dev)
    sigma = torch.empty(rows, dtype=torch.float16, device=dev)
    if rows:
        _call(dev, "h24_quantize_layer", wd.data_ptr(), rows, in_f, sigma.data_ptr(),
              packed.data_ptr(), _stream(dev))
    return packed, sigma


def quantize_layers(weights: list[torch.Tensor]) -> list[tuple[torch.Tensor, torch.Tensor]]:
    """Pack-rule quantisation of many 2-D weights (on one CUDA device) with one
    shared search pipeline; returns device-resident (packed u8, sigma16) pairs."""
    if not weights:
        return []
    dev = _work_device(weights[0])
    ws = []
    for w in weights:
        if w.dim() != 2 or w.numel() % H24_DIM != 0:
            raise ValueError(f"weights must be 2-D with a multiple of {H24_DIM} elements, got {tuple(w.shape)}")
        ws.append(_aligned(w.detach().to(device=dev, dtype=torch.float32)))
    outs = []
    layers = (N.Layer * len(ws))()
    for i, w in enumerate(ws):
        rows, in_f = w.shape
        atoms = w.numel() // H24_DIM
        packed = torch.empty(((atoms + 3) // 4) * BYTES_PER_CHUNK, dtype=torch.uint8, device=dev)
        sigma = torch.empty(rows, dtype=torch.float16, device=dev)
        layers[i] = N.Layer(w.data_ptr(), rows, in_f, sigma.data_ptr(), packed.data_ptr())
        outs.append((packed, sigma))
    _call(dev, "h24_quantize_layers", ctypes.cast(layers, ctypes.c_void_p), len(ws), _stream(dev))
    return outs


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
