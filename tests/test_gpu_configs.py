"""Parity at the benchmark configurations' full sizes: each configuration's seeded inputs go to
both the CUDA backend and the oracle (oracle/ctb_oracle.c). Where the oracle would take long at
full size, a seeded slice is checked against it and the full output through size-independent
properties (the gather equals an independent device gather; the fused chain equals the eager
pair bit for bit; the sharded sum equals the float64 sum of the same values)."""
import numpy as np
import pytest

from helpers import TOL_SUM, assert_bitexact, assert_close

pytestmark = pytest.mark.gpu


def _dev(a):
    import torch

    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def _fill(shape, dtype, dist, seed, stream, lo, hi, first=0):
    import torch

    from ctorch_b200.synth import device_fill

    t = torch.empty(shape, dtype=dtype, device="cuda")
    return device_fill(t, dist, seed, stream, lo, hi, first=first)


def test_synthetic_generator_device_matches_host(cuda_ok):
    import torch

    from ctorch_b200.synth import NORMAL, UNIFORM, host_fill

    for dt, npdt, dist, lo, hi in ((torch.float32, np.float32, UNIFORM, -1.0, 1.0),
                                   (torch.float64, np.float64, UNIFORM, 0.5, 2.0),
                                   (torch.int32, np.int32, UNIFORM, -1000, 1000),
                                   (torch.int64, np.int64, UNIFORM, 0, 999_999),
                                   (torch.float32, np.float32, NORMAL, 0.0, 1.0)):
        d = _fill((1000, 37), dt, dist, 7, 3, lo, hi, first=12345).cpu().numpy()
        h = host_fill((1000, 37), npdt, dist, 7, 3, lo, hi, first=12345)
        if dist == NORMAL:
            assert_close(d, h, 1e-6, "normal fill")
        else:
            assert_bitexact(d, h, f"uniform fill {npdt}")


def test_config1_broadcast_add_relu(cuda_ok, oracle):
    import ctorch_b200 as cb
    from ctorch_b200.synth import UNIFORM, host_fill

    a = host_fill((4096, 4096), np.float32, UNIFORM, 0, 0, -1.0, 1.0)
    b = host_fill((1, 4096), np.float32, UNIFORM, 0, 1, -1.0, 1.0)
    c = cb.add(_dev(a), _dev(b))
    r = cb.relu(c)
    rc = oracle.binary("add", a, b)
    assert_bitexact(c.cpu().numpy(), rc, "config 1 add")
    assert_bitexact(r.cpu().numpy(), oracle.unary("relu", rc), "config 1 relu")


def test_config2_axis_reductions(cuda_ok, oracle):
    import torch

    import ctorch_b200 as cb
    from ctorch_b200.synth import NORMAL, UNIFORM

    tx = _fill((8192, 8192), torch.float32, NORMAL, 1, 0, 0.0, 1.0)
    u = _fill((8192, 8192), torch.float32, UNIFORM, 1, 1, -1.0, 1.0)
    tp = cb.add(cb.mul(u, torch.tensor(0.001, device="cuda")), torch.tensor(1.0, device="cuda"))
    x, xp = tx.cpu().numpy(), tp.cpu().numpy()
    assert_close(cb.sum(tx, [1], True).cpu().numpy(), oracle.reduce("sum", x, [1], True), TOL_SUM[x.dtype], "sum dim1")
    assert_close(cb.mean(tx, [1], True).cpu().numpy(), oracle.reduce("mean", x, [1], True), TOL_SUM[x.dtype], "mean dim1")
    v, i = cb.max(tx, 0, False)
    rv, ri = oracle.reduce_idx("max", x, 0, False)
    assert_bitexact(v.cpu().numpy(), rv, "max dim0 values")
    assert_bitexact(i.cpu().numpy(), ri, "max dim0 indices")
    assert_bitexact(cb.argmax(tx, 0, False).cpu().numpy(), ri, "argmax dim0")
    assert_close(cb.prod(tp, [1], False).cpu().numpy(), oracle.reduce("prod", xp, [1], False), TOL_SUM[x.dtype], "prod dim1")


@pytest.mark.parametrize("dt", ["float32", "int32"])
def test_config3_index_select(cuda_ok, oracle, dt):
    import torch

    import ctorch_b200 as cb
    from ctorch_b200.synth import NORMAL, UNIFORM

    if dt == "float32":
        table = _fill((1_000_000, 256), torch.float32, NORMAL, 2, 0, 0.0, 1.0)
    else:
        table = _fill((1_000_000, 256), torch.int32, UNIFORM, 2, 1, -(2**30), 2**30 - 1)
    idx = _fill((4_194_304,), torch.int64, UNIFORM, 2, 2, 0, 999_999)
    out = cb.index_select(table, 0, idx)
    assert out.shape == (4_194_304, 256)
    # the whole output against an independent device gather
    assert torch.equal(out, torch.index_select(table, 0, idx))
    # a seeded slice of the indices against the oracle, bit for bit
    sl = slice(1_000_000, 1_131_072)
    got = out[sl].cpu().numpy()
    ref = oracle.index_select(table.cpu().numpy(), 0, idx[sl].cpu().numpy())
    assert_bitexact(got, ref, f"config 3 {dt} slice")
    del out
    torch.cuda.empty_cache()


def test_config4_strided_mixed_dtypes(cuda_ok, oracle):
    import torch

    import ctorch_b200 as cb
    from ctorch_b200.synth import UNIFORM

    ti = _fill((64, 512, 1024), torch.int32, UNIFORM, 3, 0, -1000, 1000)
    tf = _fill((64, 1024, 512), torch.float32, UNIFORM, 3, 1, -1.0, 1.0)
    td = _fill((1, 512, 1), torch.float64, UNIFORM, 3, 2, 0.5, 2.0)
    tft = tf.permute(0, 2, 1)
    p = cb.mul(ti, tft)
    q = cb.div(p, td)
    assert p.dtype == torch.float32 and q.dtype == torch.float64
    i, f, d = ti.cpu().numpy(), tf.cpu().numpy(), td.cpu().numpy()
    rp = oracle.binary("mul", i, f.transpose(0, 2, 1))
    assert_bitexact(p.cpu().numpy(), rp, "config 4 mul")
    assert_bitexact(q.cpu().numpy(), oracle.binary("div", rp, d), "config 4 div")


def test_config5_rows_against_oracle(cuda_ok, oracle):
    import torch

    import ctorch_b200 as cb
    from ctorch_b200.sharded import ShardedSum, sharded_step
    from ctorch_b200.synth import NORMAL, UNIFORM

    rows = 8192
    tx = _fill((rows, 8192), torch.float32, NORMAL, 4, 0, 0.0, 1.0)
    tr = _fill((1, 8192), torch.float32, UNIFORM, 4, 1, -1.0, 1.0)
    y, s, k = sharded_step(tx, tr, ShardedSum(tx.device, 1))
    x, r = tx.cpu().numpy(), tr.cpu().numpy()
    ry = oracle.binary("mul", oracle.binary("sub", x, r), r)
    assert_bitexact(y.cpu().numpy(), ry, "config 5 fused chain")
    assert_close(s.cpu().numpy(), oracle.reduce("sum", ry), TOL_SUM[np.dtype(np.float32)], "config 5 sum")
    assert_bitexact(k.cpu().numpy(), oracle.reduce_idx("min", ry, 1, values=False), "config 5 argmin")


def test_config5_full_size_properties(cuda_ok):
    import torch

    import ctorch_b200 as cb
    from ctorch_b200.sharded import ShardedSum, sharded_step
    from ctorch_b200.synth import NORMAL, UNIFORM

    tx = _fill((262144, 8192), torch.float32, NORMAL, 4, 0, 0.0, 1.0)
    tr = _fill((1, 8192), torch.float32, UNIFORM, 4, 1, -1.0, 1.0)
    y, s, k = sharded_step(tx, tr, ShardedSum(tx.device, 1))
    # fused chain == eager sub then mul, bit for bit
    assert torch.equal(y, cb.mul(cb.sub(tx, tr), tr))
    # sharded sum == float64 sum of the same values, rounded once
    ref = float(y.double().sum())
    assert abs(float(s) - ref) <= 1e-5 * max(1.0, abs(ref))
    # argmin: every row's winner is a minimum and no earlier element equals it
    mins = torch.gather(y, 1, k.view(-1, 1)).view(-1)
    assert torch.equal(mins, y.min(dim=1).values)
    first = (y == mins.view(-1, 1)).int().argmax(dim=1)
    assert torch.equal(first, k)
    # split into 8 row shards: per-shard partials combined in order give the same rounding
    parts = []
    for sh in range(8):
        ys = y[sh * 32768:(sh + 1) * 32768]
        parts.append(float(ys.double().sum()))
    assert abs(float(s) - sum(parts)) <= 1e-5 * max(1.0, abs(ref))
