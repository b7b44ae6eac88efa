"""Row sharding on two GPUs (one process per GPU, NCCL): each rank quantises
its rows of config-3 matrices in place (pack.quantize_layer_rows via
shard.quantize_layer_sharded) and one all_gather of the padded packed shards
and fp16 scales reassembles the matrix on every rank; the bytes must equal the
single-GPU call's.  Skipped with fewer than two GPUs."""
from __future__ import annotations

import multiprocessing as mp
import os
import socket
from datetime import timedelta

import pytest
import torch

pytestmark = pytest.mark.gpu

WORLD = 2


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank: int, port: int, q) -> None:
    import sys
    sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    import torch.distributed as dist
    from pollux_b200 import pack, shard, synth
    try:
        dev = torch.device("cuda", rank)
        torch.cuda.set_device(dev)
        dist.init_process_group("nccl", rank=rank, world_size=WORLD, timeout=timedelta(seconds=120),
                                device_id=dev)
        ws = synth.backbone_weights(3, device=dev, shapes=[(5760, 1920), (1920, 7680), (100, 1920)])
        ok = []
        for w in ws:
            p, s = shard.quantize_layer_sharded(w, WORLD, rank, gather=True)
            wp, wsig = pack.quantize_layers([w])[0]
            ok.append(bool(torch.equal(p, wp) and torch.equal(s, wsig)))
        dist.barrier(device_ids=[rank])
        dist.destroy_process_group()
        q.put((rank, ok, ""))
    except Exception as e:  # reported to the parent, which fails the test
        q.put((rank, [], repr(e)))


@pytest.mark.skipif(torch.cuda.device_count() < WORLD, reason="needs two GPUs")
def test_sharded_quantize_gathers_single_gpu_bytes():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, port, q)) for r in range(WORLD)]
    for p in procs:
        p.start()
    results = [q.get(timeout=600) for _ in range(WORLD)]
    for p in procs:
        p.join(timeout=120)
    for rank, ok, err in results:
        assert not err, f"rank {rank}: {err}"
        assert ok and all(ok), f"rank {rank}: shard bytes differ {ok}"
