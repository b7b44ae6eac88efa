"""Row sharding and the packed-shard all_gather, with world_size 2 gloo ranks on
CPU.  The per-shard quantiser is the CPU oracle here (the host logic under test
is the partition and the gather); on GPUs it is libh24."""
from __future__ import annotations

import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

from conftest import REPO


def test_partition_covers_rows_and_bytes():
    from pollux_b200.shard import packed_range, row_granularity, shard_rows
    for rows, in_f in [(1152, 1152), (7680, 1920), (3, 24), (10, 48), (5, 72)]:
        g = row_granularity(in_f)
        for world in (1, 2, 3, 4, 8):
            spans = [shard_rows(rows, in_f, world, r) for r in range(world)]
            assert spans[0][0] == 0 and spans[-1][1] == rows
            prev = 0
            for s, e in spans:
                assert s == prev and e >= s and (s % g == 0 or s == rows)
                prev = e
            if rows % g == 0:
                bytes_ = [packed_range(s, e, in_f) for s, e in spans]
                assert bytes_[-1][1] == ((rows * in_f // 24 + 3) // 4) * 9
                for (a0, a1), (b0, b1) in zip(bytes_, bytes_[1:]):
                    assert a1 == b0


def _oracle_quantize(w):
    import sys
    sys.path.insert(0, REPO)
    from oracle import oracle as O
    x = w.numpy().reshape(-1, 24)
    idx = O.nearest_exact(x, O.RULE_PACK, nthreads=2)
    return torch.from_numpy(O.pack_indices(idx)), torch.from_numpy(O.sigma16_pack_rule(w.numpy()))


def _worker(rank, world, port, w, q):
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from pollux_b200.shard import quantize_layer_sharded
        p, s = quantize_layer_sharded(w, world, rank, gather=True, quantize=_oracle_quantize)
        q.put((rank, p.numpy().tobytes(), s.numpy().tobytes()))
    finally:
        dist.destroy_process_group()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.parametrize("rows,in_f", [(40, 96), (7, 48)])
def test_gather_reassembles_single_device_bytes(rows, in_f):
    gen = torch.Generator().manual_seed(rows)
    w = torch.randn(rows, in_f, generator=gen) * 0.02
    p_ref, s_ref = _oracle_quantize(w)
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, w, q)) for r in range(2)]
    for p in procs:
        p.start()
    got = [q.get(timeout=300) for _ in procs]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank, pb, sb in got:
        assert pb == p_ref.numpy().tobytes(), rank
        assert sb == s_ref.numpy().tobytes(), rank
