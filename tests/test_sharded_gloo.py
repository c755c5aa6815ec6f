"""Host logic of the row-sharded layer (ctorch_b200/sharded.py) on CPU: the row partition, and
the partial -> all-gather -> rank-order combine of a whole-tensor sum, run as two gloo ranks.
The per-shard partial and the combine are injected as CPU functions here; on GPUs they are
ctb_sum_partial / ctb_sum_combine and ctb_reduce_index / ctb_minmax_combine (tests/test_gpu_sharded.py)."""
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


def _local_minmax_oracle(op):
    from oracle.oracle import oracle

    O = oracle()

    def fn(local, values, indices):
        v, i = O.reduce_idx(op, local.numpy(), 0, False)
        values.copy_(torch.from_numpy(v))
        indices.copy_(torch.from_numpy(i))

    return fn


def _better(op, v, i, bv, bi):
    """ctorch's max/min-with-index rule (src/ops/reduction_ops_cpu.cpp:236-297), restated."""
    import math

    if bv is None:
        return True
    if isinstance(v, float) and math.isnan(v):
        return not (isinstance(bv, float) and math.isnan(bv)) or i < bi
    if isinstance(bv, float) and math.isnan(bv):
        return False
    if (v > bv) if op == "max" else (v < bv):
        return True
    return v == bv and i < bi


def _minmax_combine_cpu(op):
    def fn(all_values, all_indices, offsets, out_values, out_indices):
        for n in range(all_values.shape[1]):
            bv = bi = None
            for g in range(all_values.shape[0]):  # rank order
                v = all_values[g, n].item()
                i = int(offsets[g]) + int(all_indices[g, n])
                if _better(op, v, i, bv, bi):
                    bv, bi = v, i
            out_values[n] = bv
            out_indices[n] = bi

    return fn


def _minmax_worker(rank, world, port, total, cols, results):
    import numpy as np

    from ctorch_b200.sharded import ShardedColumnMinMax

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        rng = np.random.default_rng(5)
        full = np.round(rng.standard_normal((total, cols)) * 2).astype(np.float32)  # many ties
        full[::17, 3] = np.nan
        full[:, 5] = 7.0  # a column that is one tie all the way down, across the shard boundary
        sh = row_shard(total, rank, world)
        out = {}
        for op in ("max", "min"):
            mm = ShardedColumnMinMax(op, total, cols, torch.float32, torch.device("cpu"), world,
                                     local_fn=_local_minmax_oracle(op), combine_fn=_minmax_combine_cpu(op))
            v, i = mm(torch.from_numpy(full[sh.start:sh.stop]).contiguous())
            out[op] = (v.numpy().copy(), i.numpy().copy())
        results[rank] = (out, full)
    finally:
        dist.destroy_process_group()


def test_sharded_column_minmax_two_gloo_ranks():
    """Per-shard max/min with local indices, all-gathered and combined in rank order with the
    shard offsets, equals the oracle's reduction of the whole tensor on every rank."""
    import numpy as np

    from oracle.oracle import oracle

    world, total, cols = 2, 301, 9
    mgr = mp.get_context("spawn").Manager()
    results = mgr.dict()
    mp.start_processes(_minmax_worker, args=(world, _free_port(), total, cols, results), nprocs=world,
                       start_method="spawn", join=True)
    full = results[0][1]
    O = oracle()
    for op in ("max", "min"):
        rv, ri = O.reduce_idx(op, full, 0, False)
        for rank in range(world):
            v, i = results[rank][0][op]
            assert np.array_equal(i, ri), (op, rank, i, ri)
            assert np.array_equal(np.isnan(v), np.isnan(rv))
            assert np.array_equal(v[~np.isnan(v)], rv[~np.isnan(rv)])
    assert results[0][0]["max"][1][5] == 0  # the all-tie column: first row


def test_sharded_index_select_covers_all_rows():
    from ctorch_b200.sharded import sharded_index_select

    table = torch.arange(40, dtype=torch.float32).reshape(10, 4)
    idx = torch.tensor([3, 1, 4, 1, 5, 9, 2, 6, 5])
    parts = [sharded_index_select(table, idx, len(idx), r, 4, select=torch.index_select) for r in range(4)]
    assert torch.equal(torch.cat(parts), table[idx])


def test_peer_trace_summary():
    """PeerStep.trace_summary on hand-made timestamps (ns): per call (CTA 0 start, first CTA done,
    last CTA done, exchange complete); medians in microseconds, the launch gap between calls."""
    import numpy as np

    from ctorch_b200.sharded import PeerStep

    tr = np.array([[0, 9_000, 10_000, 10_500],
                   [12_500, 20_000, 22_500, 23_000],
                   [25_000, 33_000, 35_000, 36_000]], dtype=np.int64)
    s = PeerStep.trace_summary(tr)
    assert s["calls"] == 3
    assert s["rows_us"] == 10.0          # median of 10, 10, 10
    assert s["tail_us"] == 2.0           # median of 1, 2.5, 2
    assert s["exchange_us"] == 0.5       # median of 0.5, 0.5, 1
    assert s["gap_us"] == 2.0            # median of 2, 2
    assert PeerStep.trace_summary(np.zeros((0, 4), np.int64)) == {}
