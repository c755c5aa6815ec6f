"""The row-sharded layer (ctorch_b200/sharded.py) on GPUs.

- ctb_minmax_combine on one GPU, fed with the per-shard results of G emulated shards (each the
  backend's own max/min over its rows), against the oracle's reduction of the whole tensor:
  bit-exact, for every dtype, with NaNs and ties that straddle shard boundaries.
- The one-launch step with the sum exchanged over NVLink (PeerStep / ctb_chain_rows_allsum): a
  world of one against the unfused step, and a world of two with one rank missing, whose bounded
  wait must run out, be counted and recorded, and leave NaN as the sum.
- Two NCCL ranks on two GPUs (skipped with fewer): the sharded sum, the sharded column max/min,
  the one-pass sharded step and the one-launch step, each against the same computation on one GPU
  or on the NCCL path; and 1000 one-launch steps with the ranks skewed on the host, every sum
  against the NCCL path's.
"""
import os
import socket
from datetime import timedelta

import numpy as np
import pytest

from helpers import assert_bitexact

pytestmark = pytest.mark.gpu


def _shard_inputs(dt, total, cols, seed):
    rng = np.random.default_rng(seed)
    dt = np.dtype(dt)
    if dt.kind == "f":
        x = (np.round(rng.standard_normal((total, cols)) * 2)).astype(dt)  # ties
        x[::37, 1] = np.nan
        x[5::41, 2] = -0.0
    elif dt == np.bool_:
        x = rng.integers(0, 2, (total, cols)).astype(np.bool_)
    else:
        x = rng.integers(-3, 4, (total, cols)).astype(dt)
    x[:, 0] = x[0, 0] if dt != np.bool_ else True  # one tie down the whole column
    return x


@pytest.mark.parametrize("dt", [np.float32, np.float64, np.int32, np.int64, np.bool_])
@pytest.mark.parametrize("world", [2, 3, 8])
def test_minmax_combine_of_emulated_shards(cuda_ok, oracle, dt, world):
    import torch

    import ctorch_b200 as cb
    from ctorch_b200 import _capi as C
    from ctorch_b200.sharded import row_shard

    total, cols = 1003, 700
    x = _shard_inputs(dt, total, cols, world)
    tx = torch.from_numpy(x).cuda()
    offs = torch.tensor([row_shard(total, r, world).start for r in range(world)], dtype=torch.int64, device="cuda")
    for op, code in (("max", C.MAX), ("min", C.MIN)):
        vals, idxs = [], []
        for r in range(world):
            sh = row_shard(total, r, world)
            v, i = getattr(cb, op)(tx[sh.start:sh.stop], 0, False)
            vals.append(v)
            idxs.append(i)
        av, ai = torch.stack(vals), torch.stack(idxs)
        ov = torch.empty(cols, dtype=tx.dtype, device="cuda")
        oi = torch.empty(cols, dtype=torch.int64, device="cuda")
        rc = C.lib.ctb_minmax_combine(code, C.view(av), C.view(ai), offs.data_ptr(), C.view(ov), C.view(oi),
                                      C.stream_handle())
        assert rc == C.OK, C.last_error()
        rv, ri = oracle.reduce_idx(op, x, 0, False)
        assert_bitexact(ov.cpu().numpy(), rv, f"{op} values, {world} shards")
        assert_bitexact(oi.cpu().numpy(), ri, f"{op} indices, {world} shards")
        # indices only
        oi2 = torch.empty(cols, dtype=torch.int64, device="cuda")
        rc = C.lib.ctb_minmax_combine(code, C.view(av), C.view(ai), offs.data_ptr(), None, C.view(oi2),
                                      C.stream_handle())
        assert rc == C.OK, C.last_error()
        assert torch.equal(oi2, oi)


def test_minmax_combine_rejects_bad_arguments(cuda_ok):
    import torch

    from ctorch_b200 import _capi as C

    av = torch.zeros(2, 5, device="cuda")
    ai = torch.zeros(2, 5, dtype=torch.int64, device="cuda")
    offs = torch.zeros(2, dtype=torch.int64, device="cuda")
    oi = torch.empty(5, dtype=torch.int64, device="cuda")
    assert C.lib.ctb_minmax_combine(C.SUM, C.view(av), C.view(ai), offs.data_ptr(), None, C.view(oi),
                                    C.stream_handle()) == C.ERR_ARGUMENT
    bad = torch.empty(4, dtype=torch.int64, device="cuda")
    assert C.lib.ctb_minmax_combine(C.MAX, C.view(av), C.view(ai), offs.data_ptr(), None, C.view(bad),
                                    C.stream_handle()) == C.ERR_SHAPE
    ai32 = torch.zeros(2, 5, dtype=torch.int32, device="cuda")
    assert C.lib.ctb_minmax_combine(C.MAX, C.view(av), C.view(ai32), offs.data_ptr(), None, C.view(oi),
                                    C.stream_handle()) == C.ERR_DTYPE


def test_peer_step_on_one_gpu_matches_the_unfused_step(cuda_ok):
    """World of one: the single launch gives Y and k bit-identical to chain_rows and the same sum
    bits as the partial -> combine path; repeated calls (epochs 1, 2, 3) stay consistent, which
    also checks that the last CTA resets the completion ticket."""
    import torch

    import ctorch_b200 as cb
    from ctorch_b200 import _capi as C
    from ctorch_b200.sharded import PeerStep, ShardedSum, sharded_step_fused
    from ctorch_b200.synth import NORMAL, UNIFORM, device_fill

    dev = torch.device("cuda", 0)
    before = C.wait_timeouts()
    x = device_fill(torch.empty(3001, 1024, device=dev), NORMAL, 11, 0, 0.0, 1.0)
    r = device_fill(torch.empty(1, 1024, device=dev), UNIFORM, 11, 1, -1.0, 1.0)
    y0, s0, k0 = sharded_step_fused(x, r, ShardedSum(dev, 1))
    peer = PeerStep(dev, 0, 1)
    try:
        for _ in range(3):
            y, s, k = peer(x, r)
            assert torch.equal(y, y0) and torch.equal(k, k0)
            assert s.item() == s0.item() and s.dtype == s0.dtype
        empty = torch.empty(0, 1024, device=dev)
        _, s_empty, _ = peer(empty, r)
        assert s_empty.item() == 0.0
        peer.check()
        assert peer.status() == (4, 0)
        tr = peer.trace()
        assert tr.shape == (4, 4)
        assert (tr[:, 0] > 0).all() and (tr[:, 0] <= tr[:, 1]).all() and (tr[:, 1] <= tr[:, 2]).all()
        assert (tr[:, 2] <= tr[:, 3]).all() and (tr[1:, 0] >= tr[:-1, 3]).all()
        summary = PeerStep.trace_summary(tr)
        assert summary["calls"] == 4 and summary["rows_us"] >= 0 and summary["gap_us"] >= 0
    finally:
        peer.close()
    assert C.wait_timeouts() == before


def test_peer_step_with_a_missing_rank_times_out(cuda_ok):
    """A world of two with only one rank: the wait for rank 1's partial (a slot nothing writes)
    gives up after its 5 ms limit, is counted and recorded in the workspace, leaves NaN as the sum
    and as rank 1's partial, and the device keeps working."""
    import ctypes

    import torch

    import ctorch_b200 as cb
    from ctorch_b200 import _capi as C

    dev = torch.device("cuda", 0)
    ws, other = ctypes.c_void_p(), ctypes.c_void_p()
    h = ctypes.create_string_buffer(64)
    assert C.lib.ctb_peer_alloc(ctypes.byref(ws), h) == C.OK, C.last_error()
    assert C.lib.ctb_peer_alloc(ctypes.byref(other), h) == C.OK, C.last_error()
    try:
        peers = torch.tensor([ws.value, other.value], dtype=torch.int64, device=dev)
        x = torch.randn(64, 256, device=dev)
        r = torch.randn(1, 256, device=dev)
        y = torch.empty_like(x)
        k = torch.empty(64, dtype=torch.int64, device=dev)
        out = torch.full((), -7.0, device=dev)
        parts = torch.full((2,), -7.0, dtype=torch.float64, device=dev)
        before = C.wait_timeouts()
        rc = C.lib.ctb_chain_rows_allsum(C.SUB, C.MUL, C.view(x), C.view(r), C.view(r), C.view(y), C.MIN,
                                         C.view(k), peers.data_ptr(), ws.value, 0, 2, 1, C.view(out),
                                         parts.data_ptr(), 5_000_000, C.stream_handle())
        assert rc == C.OK, C.last_error()
        torch.cuda.synchronize()
        assert C.wait_timeouts() == before + 1
        assert torch.isnan(out).item()
        assert not torch.isnan(parts[0]).item() and torch.isnan(parts[1]).item()
        done, failed = ctypes.c_uint64(7), ctypes.c_uint64(7)
        assert C.lib.ctb_peer_status(ws.value, ctypes.byref(done), ctypes.byref(failed)) == C.OK
        assert (done.value, failed.value) == (0, 1)
        assert torch.equal(y, cb.binary_chain("sub", "mul", x, r, r))  # the step itself still ran
    finally:
        C.lib.ctb_peer_free(ws)
        C.lib.ctb_peer_free(other)
    assert cb.sum(torch.ones(5, device=dev)).item() == 5.0


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _nccl_worker(rank, world, port, results):
    import torch
    import torch.distributed as dist

    import ctorch_b200 as cb
    from ctorch_b200.sharded import PeerStep, ShardedColumnMinMax, ShardedSum, row_shard, sharded_step_fused
    from ctorch_b200.synth import NORMAL, UNIFORM, device_fill

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=120),
                            device_id=dev)
    try:
        total, cols = 4099, 2048
        full = device_fill(torch.empty(total, cols, device=dev), NORMAL, 9, 0, 0.0, 1.0)
        r = device_fill(torch.empty(1, cols, device=dev), UNIFORM, 9, 1, -1.0, 1.0)
        sh = row_shard(total, rank, world)
        local = full[sh.start:sh.stop]
        summer = ShardedSum(dev, world)
        y, s, k = sharded_step_fused(local, r, summer)
        mx = ShardedColumnMinMax("max", total, cols, torch.float32, dev, world)
        mv, mi = mx(local)
        mn = ShardedColumnMinMax("min", total, cols, torch.float32, dev, world)
        nv, ni = mn(local)
        peer = PeerStep(dev, rank, world)
        try:
            for _ in range(3):
                py, ps, pk = peer(local, r)
            torch.cuda.synchronize()
            peer_ok = torch.equal(py, y) and torch.equal(pk, k) and ps.item() == s.item()
            peer_parts = peer.parts.cpu()
        finally:
            peer.close()
        torch.cuda.synchronize()
        out = {"s": float(s), "k": k.cpu(), "y_sum": float(y.double().sum()), "mv": mv.cpu(), "mi": mi.cpu(),
               "nv": nv.cpu(), "ni": ni.cpu(), "peer_ok": peer_ok, "peer_parts": peer_parts,
               "timeouts": cb._capi.wait_timeouts()}
        if rank == 0:  # the whole tensor on one GPU
            y1 = cb.binary_chain("sub", "mul", full, r, r)
            out["ref"] = {"s": float(cb.sum(y1)), "k": cb.argmin(y1, 1).cpu(), "max": cb.max(full, 0, False),
                          "min": cb.min(full, 0, False)}
            out["ref"]["max"] = (out["ref"]["max"].values.cpu(), out["ref"]["max"].indices.cpu())
            out["ref"]["min"] = (out["ref"]["min"].values.cpu(), out["ref"]["min"].indices.cpu())
        results[rank] = out
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.timeout(600)
def test_sharded_layer_on_two_gpus(cuda_ok):
    import torch
    import torch.multiprocessing as mp

    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    world = 2
    mgr = mp.get_context("spawn").Manager()
    results = mgr.dict()
    mp.start_processes(_nccl_worker, args=(world, _free_port(), results), nprocs=world, start_method="spawn",
                       join=True)
    ref = results[0]["ref"]
    ks = torch.cat([results[r]["k"] for r in range(world)])
    assert torch.equal(ks, ref["k"])
    for r in range(world):
        o = results[r]
        assert o["s"] == results[0]["s"]  # every rank holds the same sum
        assert abs(o["s"] - ref["s"]) <= 1e-5 * max(1.0, abs(ref["s"]))
        assert torch.equal(o["mv"], ref["max"][0]) and torch.equal(o["mi"], ref["max"][1])
        assert torch.equal(o["nv"], ref["min"][0]) and torch.equal(o["ni"], ref["min"][1])
        assert o["peer_ok"], f"rank {r}: the one-launch step differs from the NCCL step"
        assert torch.equal(o["peer_parts"], results[0]["peer_parts"])
        assert o["timeouts"] == 0


def _stress_worker(rank, world, port, n_calls, results):
    """n_calls back-to-back one-launch steps on small shards whose inputs change from call to call
    (a pool of 5), with host delays between launches on both ranks at different calls, so that
    each rank in turn runs a call ahead of the other. Every call's sum is kept on the device and
    compared afterwards with the NCCL path's sum of the same inputs, bit for bit."""
    import time

    import torch
    import torch.distributed as dist

    from ctorch_b200.sharded import PeerStep, ShardedSum, row_shard, sharded_step_fused
    from ctorch_b200.synth import NORMAL, UNIFORM, device_fill

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=120),
                            device_id=dev)
    try:
        total, cols, pool = 200, 512, 5
        r = device_fill(torch.empty(1, cols, device=dev), UNIFORM, 21, 1, -1.0, 1.0)
        sh = row_shard(total, rank, world)
        xs = [device_fill(torch.empty(total, cols, device=dev), NORMAL, 30 + i, 0, 0.0, 1.0)[sh.start:sh.stop]
              for i in range(pool)]
        summer = ShardedSum(dev, world)
        expect = torch.stack([sharded_step_fused(x, r, summer)[1].clone() for x in xs])
        peer = PeerStep(dev, rank, world)
        sums = torch.empty(n_calls, dtype=torch.float32, device=dev)
        y = torch.empty_like(xs[0])
        k = torch.empty(xs[0].shape[0], dtype=torch.int64, device=dev)
        dist.barrier()
        try:
            for i in range(n_calls):
                if (rank == 1 and i % 10 == 3) or (rank == 0 and i % 13 == 7):
                    torch.cuda.synchronize()
                    time.sleep(((i * 7919) % 300) * 1e-6)
                _, s, _ = peer(xs[i % pool], r, y, k)
                sums[i].copy_(s)
            torch.cuda.synchronize()
            status = peer.status()
        finally:
            peer.close()
        want = expect[torch.arange(n_calls, device=dev) % pool]
        bad = (sums.view(torch.int32) != want.view(torch.int32)).nonzero().flatten()
        results[rank] = {"bad": bad[:10].cpu().tolist(), "n_bad": int(bad.numel()), "status": status}
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.timeout(600)
def test_peer_step_exchange_under_skew_on_two_gpus(cuda_ok):
    """1000 one-launch steps with the ranks skewed on the host: no call may take another call's
    partial (every sum equals the NCCL path's for that call's inputs, bit for bit) and every
    exchange completes."""
    import torch
    import torch.multiprocessing as mp

    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    world, n_calls = 2, 1000
    mgr = mp.get_context("spawn").Manager()
    results = mgr.dict()
    mp.start_processes(_stress_worker, args=(world, _free_port(), n_calls, results), nprocs=world,
                       start_method="spawn", join=True)
    for r in range(world):
        o = results[r]
        assert o["n_bad"] == 0, f"rank {r}: {o['n_bad']} sums differ from the NCCL path, first calls {o['bad']}"
        assert o["status"] == (n_calls, 0), f"rank {r}: exchange status {o['status']}"
