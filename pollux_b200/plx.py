"""The .plx container that carries packed H24 layers (the input of the LUT
dequant path): writer of pack._write_plx (pack.py:77-104, 187-247) and reader
of generate._read_plx / evaluate._read_plx (generate.py:64-136).

Layout (little endian):
  HEADER        16 B   b"POLLUXH2", version 0x04, 7 zero bytes
  CONFIG        u32 length + compact UTF-8 JSON, zero-padded so that the block
                ends on a 64-byte boundary from the start of the file
  FINGERPRINT   16 x f32 (codebook_fingerprint, castor.py:263-266)
  TENSOR_COUNT  u32
  TENSORS       u16 name length, name, u8 dtype id, u8 ndim, ndim x u32 shape,
                u64 byte length, raw bytes
dtype ids: 0 uint8, 1 int8, 2 float16, 3 float32 (other dtypes are written as
float32).

``read_plx(path, device=...)`` memory-maps the file and moves the tensors to
``device`` through pinned host memory, so packed layers reach the GPU without
an intermediate Python copy.
"""
from __future__ import annotations

import json
import mmap
import struct
from typing import Any

import numpy as np
import torch

PLX_MAGIC = b"POLLUXH2"
PLX_VERSION = 0x04
_TORCH_TO_ID = {torch.uint8: 0, torch.int8: 1, torch.float16: 2, torch.float32: 3}
_ID_TO_NUMPY = {0: np.dtype("uint8"), 1: np.dtype("int8"), 2: np.dtype("float16"),
                3: np.dtype("float32")}


def write_plx(path: str, cfg_dict: dict, state: dict[str, torch.Tensor],
              fingerprint: tuple[float, ...] | None = None) -> None:
    """Serialise config + tensors in the reference's .plx layout."""
    if fingerprint is None:
        from .castor import codebook_fingerprint
        fingerprint = codebook_fingerprint()
    fp = list(fingerprint)[:16] + [0.0] * max(0, 16 - len(fingerprint))
    config_json = json.dumps(cfg_dict, separators=(",", ":")).encode("utf-8")
    pad = (64 - (16 + 4 + len(config_json)) % 64) % 64
    with open(path, "wb") as f:
        f.write(PLX_MAGIC)
        f.write(struct.pack("B7x", PLX_VERSION))
        f.write(struct.pack("<I", len(config_json)))
        f.write(config_json)
        f.write(b"\x00" * pad)
        f.write(struct.pack("<16f", *fp))
        f.write(struct.pack("<I", len(state)))
        for name, tensor in state.items():
            t = tensor.detach().contiguous().cpu()
            dtype_id = _TORCH_TO_ID.get(t.dtype, 3)
            arr = t.numpy() if t.dtype != torch.bfloat16 else t.float().numpy()
            arr = arr.astype(_ID_TO_NUMPY[dtype_id], copy=False)
            name_enc = name.encode("utf-8")
            shape = list(t.shape)
            raw = arr.tobytes()
            f.write(struct.pack("<H", len(name_enc)))
            f.write(name_enc)
            f.write(struct.pack("BB", dtype_id, len(shape)))
            f.write(struct.pack(f"<{len(shape)}I", *shape))
            f.write(struct.pack("<Q", len(raw)))
            f.write(raw)


def read_plx(path: str, device: torch.device | str | None = None) -> dict[str, Any]:
    """Payload dict accepted by PolluxModel.from_packed_checkpoint
    ({"format", "config", "codebook_fingerprint", "state_dict"}).  With
    ``device`` set, every tensor is copied there through pinned memory."""
    with open(path, "rb") as fh:
        mm = mmap.mmap(fh.fileno(), 0, access=mmap.ACCESS_READ)
    try:
        return _parse(path, mm, device)
    finally:
        mm.close()


def _parse(path: str, mm: mmap.mmap, device) -> dict[str, Any]:
    # Every view of the mapping lives in this frame, so all of them are gone
    # (also after an exception) before the caller closes the mapping.
    with memoryview(mm) as buf:
        if bytes(buf[:8]) != PLX_MAGIC:
            raise ValueError(f"{path!r} is not a .plx file (bad magic {bytes(buf[:8])!r}).")
        (version,) = struct.unpack_from("B7x", buf, 8)
        if version != PLX_VERSION:
            raise ValueError(f"Unsupported .plx version {version} (expected {PLX_VERSION}).")
        (config_len,) = struct.unpack_from("<I", buf, 16)
        pos = 20
        config = json.loads(bytes(buf[pos:pos + config_len]).decode("utf-8"))
        pos += config_len
        pos += (64 - pos % 64) % 64
        fingerprint = struct.unpack_from("<16f", buf, pos)
        pos += 64
        (count,) = struct.unpack_from("<I", buf, pos)
        pos += 4
        state: dict[str, torch.Tensor] = {}
        for _ in range(count):
            (name_len,) = struct.unpack_from("<H", buf, pos)
            pos += 2
            name = bytes(buf[pos:pos + name_len]).decode("utf-8")
            pos += name_len
            dtype_id, ndim = struct.unpack_from("BB", buf, pos)
            pos += 2
            shape = list(struct.unpack_from(f"<{ndim}I", buf, pos))
            pos += 4 * ndim
            (nbytes,) = struct.unpack_from("<Q", buf, pos)
            pos += 8
            if pos + nbytes > len(buf):
                raise ValueError(f"{path!r} is truncated inside tensor {name!r}")
            np_dtype = _ID_TO_NUMPY.get(dtype_id, np.dtype("float32"))
            with buf[pos:pos + nbytes] as view:
                arr = np.frombuffer(view, dtype=np_dtype).reshape(shape)
                state[name] = (torch.from_numpy(arr.copy()) if device is None
                               else _to_device(arr, device))
                del arr
            pos += nbytes
    return {"format": "pollux_packed_v4", "config": config,
            "codebook_fingerprint": fingerprint, "state_dict": state}


def _to_device(arr: np.ndarray, device) -> torch.Tensor:
    host = torch.empty(arr.shape, dtype=torch.from_numpy(arr[:0].copy()).dtype, pin_memory=True)
    host.numpy()[...] = arr
    return host.to(device, non_blocking=True)
