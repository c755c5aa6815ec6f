"""dtype casts (ctb_cast, ctorch_b200.cast / contiguous).

CPU: the oracle's restatement (oracle/ctb_oracle.c, orc_cast) against ctorch's own cast
(src/ops/cast_cpu.cpp, compiled from its sources into oracle/_ref), bit for bit, for every dtype
pair on well-defined values. A NaN, infinite or out-of-range float -> integer cast is undefined in
C++ and is left out; the GPU saturates there, which the GPU test states.

GPU: ctb_cast against the oracle for every pair and for strided, sliced and broadcast sources."""
import os
import zlib

import numpy as np
import pytest

from helpers import assert_bitexact

DTYPES = [np.float32, np.float64, np.int32, np.int64, np.bool_]
HERE = os.path.dirname(os.path.abspath(__file__))
REF_SO = os.path.join(HERE, "..", "oracle", "_ref", "libctorch_ref.so")


def _source(dt, n, rng, to_int):
    """Values of dtype dt whose cast is defined: floats with fractions, zeros of both signs and
    large magnitudes (kept inside int32 when the target is an integer), NaN/inf/subnormals only
    for float and bool targets; integers over their whole range."""
    dt = np.dtype(dt)
    if dt.kind == "f":
        x = (rng.standard_normal(n) * np.exp2(rng.integers(0, 30, n))).astype(dt)
        x[::7] = np.round(x[::7])
        x[1::11] = -0.0
        x[2::13] = 0.0
        if to_int:
            x = np.clip(x, -2.0e9, 2.0e9).astype(dt)
        else:
            x[3::17] = np.nan
            x[4::19] = np.inf
            x[5::23] = -np.inf
            x[6::29] = np.finfo(dt).tiny / 8  # subnormal
            x[8::31] = np.finfo(dt).max
        return x
    if dt == np.bool_:
        return rng.integers(0, 2, n).astype(np.bool_)
    info = np.iinfo(dt)
    x = rng.integers(info.min, info.max, n, dtype=dt, endpoint=True)
    x[::9] = rng.integers(-300, 300, x[::9].size)
    x[1::10] = 0
    x[2::10] = 256  # a nonzero whose low byte is zero
    return x


def _to_int(src, dst):
    return np.dtype(src).kind == "f" and np.dtype(dst).kind == "i"


PAIRS = [(a, b) for a in DTYPES for b in DTYPES]
IDS = [f"{np.dtype(a).name}-{np.dtype(b).name}" for a, b in PAIRS]


@pytest.mark.skipif(not os.path.exists(REF_SO), reason="ctorch reference not built")
@pytest.mark.parametrize("src,dst", PAIRS, ids=IDS)
def test_oracle_cast_matches_ctorch(oracle, src, dst):
    from oracle.oracle import ref as get_ref

    R = get_ref()
    rng = np.random.default_rng(zlib.crc32(f"{np.dtype(src).name}-{np.dtype(dst).name}".encode()))
    x = _source(src, 4001, rng, _to_int(src, dst)).reshape(4001)
    got = oracle.cast(x, dst)
    want = R.cast(R.tensor(x), dst).numpy()
    assert_bitexact(got, want, f"cast {np.dtype(src).name} -> {np.dtype(dst).name}")


LAYOUTS = {
    "flat": ((100_003,), None),
    "permuted": ((300, 257), "permute"),
    "sliced": ((400, 300), "slice"),
    "broadcast": ((1, 999), "expand"),
}


@pytest.mark.gpu
@pytest.mark.parametrize("layout", sorted(LAYOUTS))
@pytest.mark.parametrize("src,dst", PAIRS, ids=IDS)
def test_cast_matches_oracle(cuda_ok, oracle, src, dst, layout):
    import torch

    import ctorch_b200 as cb

    shape, how = LAYOUTS[layout]
    rng = np.random.default_rng(7)
    base = _source(src, int(np.prod(shape)), rng, _to_int(src, dst)).reshape(shape)
    t = torch.from_numpy(base).cuda()
    if how == "permute":
        base, t = base.T, t.permute(1, 0)
    elif how == "slice":
        base, t = base[3:391:2, 5:], t[3:391:2, 5:]
    elif how == "expand":
        base, t = np.broadcast_to(base, (64, shape[1])), t.expand(64, shape[1])
    got = cb.cast(t, getattr(torch, np.dtype(dst).name if dst != np.bool_ else "bool"))
    assert got.is_contiguous()
    assert_bitexact(got.cpu().numpy(), oracle.cast(np.ascontiguousarray(base), dst),
                    f"cast {np.dtype(src).name} -> {np.dtype(dst).name} {layout}")


@pytest.mark.gpu
def test_float_to_int_saturates_on_the_gpu(cuda_ok):
    """Undefined in C++ (ctorch's x86 build gives the integer minimum); the device conversion
    saturates and maps NaN to 0. Stated here so a change of behaviour is noticed."""
    import torch

    import ctorch_b200 as cb

    x = torch.tensor([float("nan"), float("inf"), -float("inf"), 3e9, -3e9, 2.9, -2.9], device="cuda")
    assert cb.cast(x, torch.int32).cpu().tolist() == [0, 2**31 - 1, -2**31, 2**31 - 1, -2**31, 2, -2]


@pytest.mark.gpu
def test_contiguous_copies_strided_views(cuda_ok):
    import torch

    import ctorch_b200 as cb

    x = torch.randn(64, 48, 40, device="cuda")
    for v in (x.permute(2, 0, 1), x[:, 5:40:3], x.transpose(0, 1)[7], x[0:1].expand(9, 48, 40)):
        c = cb.contiguous(v)
        assert c.is_contiguous() and torch.equal(c, v)
    assert cb.contiguous(x) is x


@pytest.mark.gpu
def test_cast_errors(cuda_ok):
    import torch

    import ctorch_b200 as cb

    x = torch.ones(4, device="cuda")
    with pytest.raises(cb.DTypeError):
        cb.cast(x, torch.bfloat16)
    with pytest.raises(cb.DeviceError):
        cb.cast(torch.ones(4), torch.int32)
