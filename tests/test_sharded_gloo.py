"""Host logic of the row-sharded layer (ctorch_b200/sharded.py) on CPU: the row partition, and
the partial -> all-gather -> rank-order combine of a whole-tensor sum, run as two gloo ranks.
The per-shard partial and the combine are injected as CPU functions here; on GPUs they are
ctb_sum_partial / ctb_sum_combine (tests/test_gpu_sharded.py)."""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from ctorch_b200.sharded import ShardedSum, row_shard


def test_row_shard_partition():
    for total in (0, 1, 7, 262144, 262147):
        for world in (1, 2, 3, 4, 8):
            shards = [row_shard(total, r, world) for r in range(world)]
            assert shards[0].start == 0 and shards[-1].stop == total
            for a, b in zip(shards, shards[1:]):
                assert a.stop == b.start
            sizes = [s.rows for s in shards]
            assert max(sizes) - min(sizes) <= 1
    assert row_shard(262144, 3, 8).start == 3 * 32768
    with pytest.raises(ValueError):
        row_shard(10, 2, 2)


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _partial_cpu(local, out):
    out.copy_(local.double().sum().reshape(1))


def _combine_cpu(parts, out):
    acc = torch.zeros((), dtype=torch.float64)
    for p in parts:  # rank order
        acc = acc + p
    out.copy_(acc.to(out.dtype))


def _worker(rank, world, port, total, cols, results):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        g = torch.Generator().manual_seed(0)
        full = torch.randn(total, cols, generator=g)
        sh = row_shard(total, rank, world)
        summer = ShardedSum(torch.device("cpu"), world, partial_fn=_partial_cpu, combine_fn=_combine_cpu)
        s = summer(full[sh.start:sh.stop])
        gathered = [torch.zeros(()) for _ in range(world)]
        dist.all_gather(gathered, s.clone())
        results[rank] = (float(s), [float(x) for x in gathered], float(full.double().sum()))
    finally:
        dist.destroy_process_group()


def test_sharded_sum_two_gloo_ranks():
    world, total, cols = 2, 1001, 37
    mgr = mp.get_context("spawn").Manager()
    results = mgr.dict()
    mp.start_processes(_worker, args=(world, _free_port(), total, cols, results), nprocs=world,
                       start_method="spawn", join=True)
    s0, g0, ref = results[0]
    s1, g1, _ = results[1]
    assert s0 == s1 == g0[0] == g0[1]  # every rank holds the same value
    assert abs(s0 - ref) <= 1e-5 * max(1.0, abs(ref))
