"""Row sharding of the hot path across GPUs (one process per GPU).

The work is independent per weight row: the fp16 row scale is per row and the
atoms of a row never mix with another row's.  Rank r of W takes a contiguous
range of rows; when every row holds a multiple of 4 atoms (in_features a
multiple of 96, true for every Pollux layer) each range maps to a contiguous
slice of the packed byte stream, so shards concatenate into exactly the bytes
the single-GPU path writes.  No collective is needed on the data path; the
optional gather of the packed shards is one all_gather of equal-size padded
byte buffers (NCCL over NVLink on GPUs, gloo on CPU).
"""
from __future__ import annotations

import math
from typing import Callable

import torch

H24_DIM = 24
BYTES_PER_CHUNK = 9


def row_granularity(in_features: int) -> int:
    """Smallest row count whose atoms fill whole 4-index groups."""
    if in_features % H24_DIM != 0:
        raise ValueError(f"in_features must be a multiple of {H24_DIM}, got {in_features}")
    apr = in_features // H24_DIM
    return 4 // math.gcd(4, apr)


def shard_rows(rows: int, in_features: int, world: int, rank: int) -> tuple[int, int]:
    """[start, end) rows of `rank`, contiguous, in units of row_granularity."""
    if not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside world of {world}")
    g = row_granularity(in_features)
    units = (rows + g - 1) // g
    per, extra = divmod(units, world)
    u0 = rank * per + min(rank, extra)
    u1 = u0 + per + (1 if rank < extra else 0)
    return min(rows, u0 * g), min(rows, u1 * g)


def packed_range(start: int, end: int, in_features: int) -> tuple[int, int]:
    """Byte range of rows [start, end) in the packed stream of the whole matrix
    (empty for an empty shard, placed at the end of the rows before it)."""
    apr = in_features // H24_DIM
    a0, a1 = start * apr, end * apr
    if end <= start:
        b = (a1 + 3) // 4 * BYTES_PER_CHUNK
        return b, b
    if a0 % 4 != 0:
        raise ValueError("shard does not start on a 4-index group")
    return a0 // 4 * BYTES_PER_CHUNK, (a1 + 3) // 4 * BYTES_PER_CHUNK


def quantize_layer_sharded(weight: torch.Tensor, world: int = 1, rank: int = 0, group=None,
                           gather: bool = False,
                           quantize: Callable | None = None):
    """Pack-rule quantisation of this rank's row shard of ``weight``.

    Returns (packed_shard, sigma_shard, (start, end)) or, with gather=True, the
    whole matrix's (packed, sigma) assembled on every rank.  ``quantize`` maps
    a 2-D block of rows to (packed u8, sigma16); the default is the libh24
    row-range pipeline (pollux_b200.pack.quantize_layer_rows), which reads the
    rows in place and computes their scales with the whole matrix's reduction
    order, so the shards carry exactly the single-GPU bytes."""
    rows, in_f = weight.shape
    start, end = shard_rows(rows, in_f, world, rank)
    if end > start and quantize is None:
        from .pack import quantize_layer_rows
        packed, sigma = quantize_layer_rows([(weight, start, end)])[0]
    elif end > start:
        packed, sigma = quantize(weight[start:end])
    else:
        packed = torch.zeros(0, dtype=torch.uint8, device=weight.device)
        sigma = torch.zeros(0, dtype=torch.float16, device=weight.device)
    if not gather or world == 1:
        return packed, sigma, (start, end)
    import torch.distributed as dist
    # Equal-size buffers: the largest shard's packed bytes and row count.
    max_rows = max(e - s for s, e in (shard_rows(rows, in_f, world, r) for r in range(world)))
    max_bytes = max(packed_range(*shard_rows(rows, in_f, world, r), in_f)[1]
                    - packed_range(*shard_rows(rows, in_f, world, r), in_f)[0] for r in range(world))
    pbuf = torch.zeros(max_bytes, dtype=torch.uint8, device=packed.device)
    pbuf[:packed.numel()] = packed
    sbuf = torch.zeros(max_rows, dtype=torch.float16, device=sigma.device)
    sbuf[:sigma.numel()] = sigma
    pall = torch.empty(world * max_bytes, dtype=torch.uint8, device=packed.device)
    sall = torch.empty(world * max_rows, dtype=torch.float16, device=sigma.device)
    dist.all_gather_into_tensor(pall, pbuf, group=group)
    dist.all_gather_into_tensor(sall, sbuf, group=group)
    out_p, out_s = [], []
    for r in range(world):
        s0, e0 = shard_rows(rows, in_f, world, r)
        b0, b1 = packed_range(s0, e0, in_f)
        out_p.append(pall[r * max_bytes: r * max_bytes + (b1 - b0)])
        out_s.append(sall[r * max_rows: r * max_rows + (e0 - s0)])
    return torch.cat(out_p), torch.cat(out_s)
