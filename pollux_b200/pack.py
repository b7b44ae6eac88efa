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
            _call(dev, "h24_quantize_layer_rows_host", ctypes.byref(L), 1, _LAYER_DTYPES[w.dtype],
                  _stream(dev))
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
    return quantize_layers_host([(weight, row_begin, row_end)])[0]


def quantize_layers_host(parts: list[tuple[torch.Tensor, int, int]]) -> list[tuple[torch.Tensor, torch.Tensor]]:
    """Rows [begin, end) of each HOST weight (contiguous 2-D fp32 or bf16, all
    of one dtype) to host (packed u8, sigma16), in one pipeline: rows of
    several matrices are gathered into batches of up to 2^20 atoms, and the
    copy of each batch overlaps the search of the previous one (page-locked
    weights give the overlap).  The outputs are the
    bytes and scales _quantize_h24_layer returns for those rows."""
    if not parts:
        return []
    dtypes = {w.dtype for w, _, _ in parts}
    if len(dtypes) != 1 or next(iter(dtypes)) not in _LAYER_DTYPES:
        raise ValueError("quantize_layers_host wants fp32 or bf16 host weights of one dtype")
    code = _LAYER_DTYPES[next(iter(dtypes))]
    dev = _work_device(parts[0][0])
    layers, outs = [], []
    for (w, r0, r1) in parts:
        w = w.detach()
        if w.device.type != "cpu" or not w.is_contiguous() or w.dim() != 2:
            raise ValueError("quantize_layers_host wants contiguous 2-D host tensors")
        rows, in_f = w.shape
        atoms = max(r1 - r0, 0) * in_f // H24_DIM
        pin = w.is_pinned()
        packed = torch.empty(((atoms + 3) // 4) * BYTES_PER_CHUNK, dtype=torch.uint8, pin_memory=pin)
        sigma = torch.empty(max(r1 - r0, 0), dtype=torch.float16, pin_memory=pin)
        layers.append(N.LayerRows(w.data_ptr(), rows, in_f, r0, r1, sigma.data_ptr(), packed.data_ptr()))
        outs.append((packed, sigma))
    arr = (N.LayerRows * len(layers))(*layers)
    _call(dev, "h24_quantize_layer_rows_host", ctypes.cast(arr, ctypes.c_void_p), len(layers), code,
          _stream(dev))
    return outs


def _is_packable_h24(name: str, tensor: torch.Tensor) -> bool:
    """pack._is_packable_h24 (pack.py:111-117): hidden H24 weight matrices
    (``*.weight``, >= 2-D, a multiple of 24 elements), not tok_emb, pos_emb or
    head."""
    if not name.endswith(".weight"):
        return False
    if name.startswith(("tok_emb.", "pos_emb.", "head.")):
        return False
    return tensor.dim() >= 2 and tensor.numel() > 0 and tensor.numel() % H24_DIM == 0


def quantize_state_dict(state_in: dict, codebook: torch.Tensor | None = None) -> dict:
    """The tensor loop of pack_checkpoint (pack.py:268-287) on a model
    state_dict: tok_emb / head to INT8 + fp16 mu (``.weight_int8``,
    ``.mu_rows``), every packable H24 matrix to packed 18-bit indices + fp16
    row scales (``.packed_weights``, ``.sigma_rows``), everything else passed
    through on the host; the entries keep the reference's names and order.
    All H24 matrices of one dtype go through one pipelined call
    (host-resident ones overlap their transfer with the search); the result
    equals _quantize_h24_layer per matrix."""
    if codebook is not None:
        _check_codebook(codebook)
    out: dict = {}
    h24_names = [n for n, t in state_in.items()
                 if n not in ("tok_emb.weight", "head.weight") and _is_packable_h24(n, t)]
    mats = {n: state_in[n].detach() for n in h24_names}
    for n, m in mats.items():
        if m.dim() != 2:  # row_rms_from_matrix raises the same (castor.py:311)
            raise ValueError(f"row_rms_from_matrix expects a 2D weight matrix, got {m.dim()}D.")
    results: dict = {}
    host_groups: dict = {}
    device_list = []
    for n in h24_names:
        m = mats[n]
        if m.device.type == "cpu" and m.dtype in _LAYER_DTYPES and m.is_contiguous():
            host_groups.setdefault(m.dtype, []).append(n)
        else:
            device_list.append(n)
    for names in host_groups.values():
        for n, r in zip(names, quantize_layers_host([(mats[n], 0, mats[n].shape[0]) for n in names])):
            results[n] = r
    if device_list:
        res = quantize_layers([mats[n] for n in device_list])
        for n, (p, s) in zip(device_list, res):
            results[n] = (p.cpu(), s.cpu())
        device_check(res[0][0].device)
    for name, tensor in state_in.items():
        if name in ("tok_emb.weight", "head.weight"):
            q, mu = _quantize_int8(tensor)
            out[name.replace(".weight", ".weight_int8")] = q
            out[name.replace(".weight", ".mu_rows")] = mu
        elif name in results:
            p, s = results[name]
            out[name.replace(".weight", ".packed_weights")] = p
            out[name.replace(".weight", ".sigma_rows")] = s
        else:
            out[name] = tensor.detach().cpu()
    return out


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
