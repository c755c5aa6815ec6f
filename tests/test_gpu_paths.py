"""Every launch shape of the CUDA backend against the oracle (oracle/ctb_oracle.c) on seeded
inputs large enough to exercise it: the flat / row / short-row / tiled-transpose / general
elementwise kernels, every promoted dtype pair, the fused chain, the inner (CTA, warp, split) /
outer (split) / general reduction kernels with NaN, ties and signed zeros, and the row / general
gathers. Same parity bar as test_gpu_golden.py."""
import zlib

import numpy as np
import pytest

from catalog import apply_numpy, apply_torch
from helpers import TOL_SUM, assert_bitexact, assert_close

pytestmark = pytest.mark.gpu


def _seed(*parts) -> int:
    return zlib.crc32(repr(parts).encode())


def _pair(base: np.ndarray, recipe=()):
    import torch

    t = apply_torch(torch.from_numpy(np.ascontiguousarray(base)).cuda(), list(recipe))
    return apply_numpy(base, list(recipe)), t


def _rand(rng, shape, dt):
    dt = np.dtype(dt)
    if dt.kind == "f":
        return rng.standard_normal(shape).astype(dt)
    if dt == np.bool_:
        return rng.integers(0, 2, shape).astype(np.bool_)
    return rng.integers(-1000, 1000, shape).astype(dt)


BIN_LAYOUTS = {
    # name: (shape_a, recipe_a, shape_b, recipe_b)
    "flat_tail": ((1_000_003,), [], (1_000_003,), []),
    "flat_scalar": ((777_777,), [], (), []),
    "rows_long": ((384, 4096), [], (1, 4096), []),
    "rows_long_col": ((300, 8192), [], (300, 1), []),
    "rows_mid": ((300, 1000), [], (1, 1000), []),
    "rows_mid_col": ((200, 4092), [], (200, 1), []),
    "rows_long_wide": ((40, 8200), [], (1, 8200), []),
    "rows_short": ((20_000, 12), [], (1, 12), []),
    "rows_short_3d": ((50, 40, 8), [], (40, 1), []),
    "tiled": ((6, 200, 300), [], (6, 300, 200), [("permute", [0, 2, 1])]),
    "tiled_lhs": ((4, 130, 70), [("permute", [0, 2, 1])], (4, 70, 130), []),
    "tiled_wide": ((3, 512, 384), [], (3, 384, 512), [("permute", [0, 2, 1])]),
    "tiled_wide_edges": ((2, 300, 520), [("permute", [0, 2, 1])], (2, 520, 300), []),
    "general_offset": ((513, 257), [("slice", 0, 1, 513, 1)], (257,), []),
    "general_step": ((300, 200), [("slice", 1, 0, 200, 3)], (300, 1), []),
    "general_select": ((40, 7, 300), [("select", 1, 3)], (40, 300), [("slice", 1, 0, 300, 1)]),
}


@pytest.mark.parametrize("layout", sorted(BIN_LAYOUTS))
@pytest.mark.parametrize("op", ["add", "sub", "mul", "div"])
def test_binary_layouts_f32(cuda_ok, oracle, op, layout):
    import ctorch_b200 as cb

    rng = np.random.default_rng(_seed(op, layout))
    sa, ra, sb, rb = BIN_LAYOUTS[layout]
    a, ta = _pair(_rand(rng, sa, np.float32), ra)
    b, tb = _pair(_rand(rng, sb, np.float32), rb)
    got = getattr(cb, op)(ta, tb).cpu().numpy()
    assert_bitexact(got, oracle.binary(op, a, b), f"{op} {layout}", nan_payload=False)


DTYPE_PAIRS = [
    (np.int32, np.int32), (np.int64, np.int64), (np.int32, np.int64), (np.int64, np.int32),
    (np.float32, np.float32), (np.int32, np.float32), (np.float32, np.int32), (np.int64, np.float32),
    (np.float32, np.int64), (np.float64, np.float64), (np.float32, np.float64), (np.float64, np.float32),
    (np.int32, np.float64), (np.float64, np.int32), (np.int64, np.float64), (np.float64, np.int64),
]


@pytest.mark.parametrize("da,db", DTYPE_PAIRS, ids=[f"{np.dtype(a).name}-{np.dtype(b).name}" for a, b in DTYPE_PAIRS])
@pytest.mark.parametrize("op", ["add", "sub", "mul", "div"])
def test_binary_promotion(cuda_ok, oracle, op, da, db):
    import ctorch_b200 as cb

    if op == "div" and np.dtype(da).kind == "i" and np.dtype(db).kind == "i":
        pytest.skip("integer division is refused")
    rng = np.random.default_rng(11)
    for layout in ("rows_long", "tiled", "general_offset", "flat_tail"):
        sa, ra, sb, rb = BIN_LAYOUTS[layout]
        a, ta = _pair(_rand(rng, sa, da), ra)
        b, tb = _pair(_rand(rng, sb, db), rb)
        got = getattr(cb, op)(ta, tb).cpu().numpy()
        assert_bitexact(got, oracle.binary(op, a, b), f"{op} {layout}", nan_payload=False)


@pytest.mark.parametrize("op", ["relu", "neg", "abs", "sqrt"])
@pytest.mark.parametrize("dt", [np.float32, np.float64, np.int32, np.int64])
def test_unary_exact(cuda_ok, oracle, op, dt):
    import ctorch_b200 as cb

    if op == "sqrt" and np.dtype(dt).kind == "i":
        pytest.skip("float only")
    rng = np.random.default_rng(5)
    for shape, recipe in (((1_000_001,), []), ((256, 2048), [("permute", [1, 0])]), ((99, 77), [("slice", 1, 1, 77, 2)])):
        base = _rand(rng, shape, dt)
        if np.dtype(dt).kind == "f":
            base.flat[::97] = np.nan
            base.flat[1::89] = -0.0
            if op == "sqrt":
                base = np.abs(base)
        x, tx = _pair(base, recipe)
        got = getattr(cb, op)(tx).cpu().numpy()
        assert_bitexact(got, oracle.unary(op, x), f"{op} {shape}", nan_payload=(op == "relu"))


@pytest.mark.parametrize("op", ["exp", "log", "tanh", "sigmoid"])
@pytest.mark.parametrize("dt", [np.float32, np.float64])
def test_unary_transcendental(cuda_ok, oracle, op, dt):
    import ctorch_b200 as cb
    from helpers import TOL_TRANSCENDENTAL

    rng = np.random.default_rng(9)
    base = (rng.standard_normal(300_001) * 4).astype(dt)
    if op == "log":
        base = np.abs(base) + np.asarray(1e-3, dt)
    x, tx = _pair(base)
    got = getattr(cb, op)(tx).cpu().numpy()
    assert_close(got, oracle.unary(op, x), TOL_TRANSCENDENTAL[np.dtype(dt)], op)


@pytest.mark.parametrize("op1,op2", [("sub", "mul"), ("mul", "add"), ("add", "div"), ("div", "sub")])
@pytest.mark.parametrize("dt", [np.float32, np.float64])
def test_chain_is_bitwise_the_eager_pair(cuda_ok, oracle, op1, op2, dt):
    import ctorch_b200 as cb

    rng = np.random.default_rng(3)
    for sx, sr in (((512, 8192), (1, 8192)), ((1000, 12), (1, 12)), ((77, 33), (33,))):
        x, tx = _pair(_rand(rng, sx, dt))
        r, tr = _pair(_rand(rng, sr, dt))
        got = cb.binary_chain(op1, op2, tx, tr, tr).cpu().numpy()
        ref = oracle.binary(op2, oracle.binary(op1, x, r), r)
        assert_bitexact(got, ref, f"{op1}->{op2} {sx}", nan_payload=False)
        eager = getattr(cb, op2)(getattr(cb, op1)(tx, tr), tr).cpu().numpy()
        assert_bitexact(got, eager, "chain vs eager", nan_payload=False)
        # a third operand of its own (the three-input kernel; the above reads r once per element)
        c, tc = _pair(_rand(rng, sr, dt))
        got3 = cb.binary_chain(op1, op2, tx, tr, tc).cpu().numpy()
        ref3 = oracle.binary(op2, oracle.binary(op1, x, r), c)
        assert_bitexact(got3, ref3, f"{op1}->{op2} {sx} distinct c", nan_payload=False)
        # the same row through a different view is not the same operand, and must still agree
        tr2 = tr.reshape(tr.shape)[..., :]
        got_v = cb.binary_chain(op1, op2, tx, tr, tr2.expand(tr.shape) if tr.dim() == 2 else tr2).cpu().numpy()
        assert_bitexact(got_v, ref, f"{op1}->{op2} {sx} aliased view", nan_payload=False)


@pytest.mark.parametrize("offset", [0, 2, 4, 6])
@pytest.mark.parametrize("op", ["add", "mul", "div"])
def test_wide_output_packs_at_any_alignment(cuda_ok, oracle, op, offset):
    """float64 results of float32 operands move in 32-byte packs; a pack that starts on a 32-byte
    boundary is stored in one piece, any other one as two 16-byte halves. Outputs at element
    offsets 0 and 4 (32-byte aligned) and 2 and 6 (16-byte only), in place, for the flat, row and
    per-row-scalar kernels, must all equal the oracle and leave the bytes around them alone."""
    import torch
    import ctorch_b200 as cb

    rng = np.random.default_rng(31 + offset)
    for shape, bshape in (((300_000,), (300_000,)), ((96, 8192), (1, 8192)), ((64, 512, 1024), (1, 512, 1))):
        n = int(np.prod(shape))
        big = rng.standard_normal(n + 8)
        a = big[offset:offset + n].reshape(shape).copy()
        b = _rand(rng, bshape, np.float32) + np.float32(2.0)
        tbig = torch.from_numpy(big).cuda()
        ta = tbig[offset:offset + n].view(shape)
        getattr(cb, op + "_")(ta, torch.from_numpy(b).cuda())
        got = tbig.cpu().numpy()
        assert_bitexact(got[offset:offset + n].reshape(shape), oracle.binary(op, a, b), f"{op} {shape} +{offset}",
                        nan_payload=False)
        untouched = np.concatenate([big[:offset], big[offset + n:]])
        assert np.array_equal(np.concatenate([got[:offset], got[offset + n:]]), untouched), "wrote outside"
    # a widening cast into a fresh (aligned) output
    x = _rand(rng, (1_000_003,), np.float32)
    got = cb.cast(torch.from_numpy(x).cuda(), torch.float64).cpu().numpy()
    assert_bitexact(got, x.astype(np.float64), "cast f32->f64")


CHAIN_ROW_CASES = [
    # (x shape, b shape, c shape; None: c is b), each last dim replaced by the columns of a
    # 32 KiB row (8192 float32 or 4096 float64)
    ((16384, 1), (1, 1), (1, 1)),        # c distinct
    ((2, 8192, 1), (1,), (1,)),          # 3-D matrix, 1-D rows
    ((16384, 1), (1, 1), "scalar"),      # c a one-element tensor
    ((16400, 1), (1,), None),            # c is b (read once)
]


@pytest.mark.parametrize("case", range(4))
@pytest.mark.parametrize("op1,op2", [("sub", "mul"), ("mul", "add"), ("add", "div"), ("div", "sub")])
@pytest.mark.parametrize("dt", [np.float32, np.float64])
def test_chain_row_kernel(cuda_ok, oracle, case, op1, op2, dt):
    """Chains on at least 16384 rows of 32 KiB or more with broadcast-row operands take the
    warp-per-row kernel (rows staged in shared memory); results stay bit-identical to the oracle's
    eager pair, with special values in both the matrix and the rows. Each op pair runs two of the
    four layouts (the layout index is rotated by the op pair), to bound the test time."""
    import ctorch_b200 as cb

    pairs = [("sub", "mul"), ("mul", "add"), ("add", "div"), ("div", "sub")]
    if (case + pairs.index((op1, op2))) % 2:
        pytest.skip("layout covered by the neighbouring op pair")
    cols = 32 * 1024 // np.dtype(dt).itemsize
    sx, sb, sc = CHAIN_ROW_CASES[case]
    sx = sx[:-1] + (cols,)
    sb = sb[:-1] + (cols,)
    rng = np.random.default_rng(11 + case)
    x = _rand(rng, sx, dt)
    flat = x.reshape(-1)
    flat[:64] = np.array([np.nan, np.inf, -np.inf, 0.0, -0.0, 1e-40, -1e30, 3.0] * 8, dtype=dt)
    b = _rand(rng, sb, dt)
    b.reshape(-1)[:6] = np.array([0.0, -0.0, np.inf, np.nan, 1e-39, -2.0], dtype=dt)
    x_, tx = _pair(x)
    b_, tb = _pair(b)
    if sc is None:
        c_, tc = b_, tb
    else:
        c_, tc = _pair(_rand(rng, (1, 1) if sc == "scalar" else sc[:-1] + (cols,), dt))
    got = cb.binary_chain(op1, op2, tx, tb, tc).cpu().numpy()
    ref = oracle.binary(op2, oracle.binary(op1, x_, b_), c_)
    assert_bitexact(got, ref, f"{op1}->{op2} {sx}", nan_payload=False)


@pytest.mark.parametrize("dt", [np.float32, np.float64])
def test_chain_row_kernel_unaligned_falls_back(cuda_ok, oracle, dt):
    """A matrix whose rows are not 16-byte aligned takes the elementwise kernels, same results."""
    import torch
    import ctorch_b200 as cb

    cols = 32 * 1024 // np.dtype(dt).itemsize
    rng = np.random.default_rng(5)
    x = _rand(rng, (16384, cols + 1), dt)
    b = _rand(rng, (1, cols), dt)
    tx = torch.from_numpy(x).cuda()[:, 1:]
    tb = torch.from_numpy(b).cuda()
    got = cb.binary_chain("sub", "mul", tx, tb, tb).cpu().numpy()
    xs = np.ascontiguousarray(x[:, 1:])
    assert_bitexact(got, oracle.binary("mul", oracle.binary("sub", xs, b), b), "unaligned rows", nan_payload=False)


RED_LAYOUTS = {
    # name: (shape, recipe, dims, keepdim)
    "inner_cta": ((96, 20_000), [], [1], True),
    "inner_split": ((3, 1_000_003), [], [1], False),
    "inner_warp": ((5000, 100), [], [1], False),
    "inner_warp_group": ((3000, 4100), [], [1], False),
    "inner_warp_group_offset": ((2600, 3001), [("slice", 1, 1, 3001, 1)], [1], True),
    "inner_whole": ((2_000_003,), [], None, False),
    "inner_offset_rows": ((300, 999), [("slice", 1, 1, 999, 1)], [1], False),
    "outer": ((3000, 520), [], [0], False),
    "outer_batched": ((3, 2000, 260), [], [1], True),
    "outer_narrow": ((5000, 17), [], [0], False),
    "outer_transposed": ((700, 900), [("permute", [1, 0])], [1], False),
    "general_cta": ((1500, 1200), [("permute", [1, 0]), ("slice", 0, 0, 1200, 2)], None, False),
    "general_thread": ((60, 7, 90), [], [0, 2], False),
    # reduced dims that do not collapse, the innermost contiguous and pack-aligned: red_runs_cta
    "general_runs": ((40, 300, 512), [], [0, 2], False),
    "general_runs_split_keepdim": ((8, 2, 6, 4096), [], [1, 3], True),
    "general_runs_batch_offset": ((3, 20, 50, 1024), [("slice", 0, 1, 3, 1)], [1, 3], False),
    # the same with rows of 513 elements cut to 512: runs no longer start on 16-byte boundaries
    "general_runs_unaligned": ((40, 300, 513), [("slice", 2, 0, 512, 1)], [0, 2], False),
}


def _red_dtypes(op):
    if op == "mean":
        return [np.float32, np.float64]
    return [np.float32, np.float64, np.int32, np.int64, np.bool_]


@pytest.mark.parametrize("layout", sorted(RED_LAYOUTS))
@pytest.mark.parametrize("op", ["sum", "mean", "prod", "max", "min"])
def test_reduction_layouts(cuda_ok, oracle, op, layout):
    import ctorch_b200 as cb

    shape, recipe, dims, kd = RED_LAYOUTS[layout]
    rng = np.random.default_rng(_seed(op, layout))
    for dt in _red_dtypes(op):
        base = _rand(rng, shape, dt)
        if op == "prod" and np.dtype(dt).kind == "f":
            base = (1 + 1e-4 * base).astype(dt)
        if op in ("max", "min") and np.dtype(dt).kind == "f":
            base.flat[::1013] = np.nan
            base.flat[7::501] = -0.0
            base.flat[9::503] = 0.0
        x, tx = _pair(base, recipe)
        got = getattr(cb, op)(tx, dims, kd).cpu().numpy()
        ref = oracle.reduce(op, x, dims, kd)
        what = f"{op} {layout} {np.dtype(dt).name}"
        if op in ("sum", "mean", "prod") and np.dtype(dt).kind == "f":
            assert_close(got, ref, TOL_SUM[np.dtype(dt)], what)
        else:
            assert_bitexact(got, ref, what)


IDX_LAYOUTS = {
    # name: (shape, recipe, dim)
    "outer_cols": ((4000, 1000), [], 0),
    "outer_batched": ((3, 1500, 130), [], 1),
    "outer_narrow": ((3000, 9), [], 0),
    "inner_rows": ((3000, 1000), [], 1),
    "inner_long": ((4, 1_000_000), [], 1),
    "general": ((90, 80, 70), [("permute", [2, 0, 1])], 2),
}


@pytest.mark.parametrize("layout", sorted(IDX_LAYOUTS))
@pytest.mark.parametrize("op", ["max", "min"])
@pytest.mark.parametrize("dt", [np.float32, np.float64, np.int32, np.int64, np.bool_])
def test_reduce_index_layouts(cuda_ok, oracle, op, layout, dt):
    import ctorch_b200 as cb

    shape, recipe, dim = IDX_LAYOUTS[layout]
    rng = np.random.default_rng(_seed(op, layout, np.dtype(dt).name))
    base = _rand(rng, shape, dt)
    if np.dtype(dt).kind == "i":
        base = (base % 7).astype(dt)  # many ties -> first index must win
    if np.dtype(dt).kind == "f":
        base = np.round(base * 4) / 4  # ties
        base = base.astype(dt)
        base.flat[::4099] = np.nan
        base.flat[5::307] = -0.0
    x, tx = _pair(base, recipe)
    v, i = getattr(cb, op)(tx, dim, False)
    rv, ri = oracle.reduce_idx(op, x, dim, False)
    assert_bitexact(v.cpu().numpy(), rv, f"{op} values {layout}")
    assert_bitexact(i.cpu().numpy(), ri, f"{op} indices {layout}")
    a = getattr(cb, "arg" + op)(tx, dim, True).cpu().numpy()
    assert_bitexact(a, oracle.reduce_idx(op, x, dim, True, values=False), f"arg{op} {layout}")


def test_reductions_are_deterministic(cuda_ok):
    import torch

    import ctorch_b200 as cb

    g = torch.Generator(device="cuda").manual_seed(0)
    x = torch.randn(3, 5_000_000, device="cuda", generator=g)
    a = cb.sum(x, [1])
    b = cb.sum(x, [1])
    assert torch.equal(a, b)
    y = torch.randn(4096, 4096, device="cuda", generator=g)
    assert torch.equal(cb.max(y, 0, False).indices, cb.max(y, 0, False).indices)
    assert torch.equal(cb.sum(y), cb.sum(y))


GATHER = {
    # name: (src shape, src recipe, dim, n_idx, idx dtype)
    "rows_1k": ((5000, 256), [], 0, 20000, np.int64),
    "rows_i32": ((5000, 256), [], 0, 7000, np.int32),
    "rows_odd_bytes": ((3000, 3), [], 0, 9000, np.int64),
    "inner_dim": ((40, 300, 16), [], 1, 500, np.int64),
    "last_dim": ((200, 300), [], 1, 1000, np.int64),
    "strided_src": ((300, 400), [("permute", [1, 0])], 0, 2000, np.int64),
    "sliced_src": ((400, 300), [("slice", 1, 10, 300, 1)], 0, 2000, np.int32),
}


@pytest.mark.parametrize("layout", sorted(GATHER))
@pytest.mark.parametrize("dt", [np.float32, np.float64, np.int32, np.bool_])
def test_index_select_layouts(cuda_ok, oracle, layout, dt):
    import torch

    import ctorch_b200 as cb

    shape, recipe, dim, n, idt = GATHER[layout]
    rng = np.random.default_rng(_seed(layout, np.dtype(dt).name))
    x, tx = _pair(_rand(rng, shape, dt), recipe)
    size = x.shape[dim]
    idx = rng.integers(-size, size, n).astype(idt)
    ti = torch.from_numpy(idx).cuda()
    got = cb.index_select(tx, dim, ti).cpu().numpy()
    assert_bitexact(got, oracle.index_select(x, dim, idx), layout)
    # strided index vector
    got2 = cb.index_select(tx, dim, ti[::3]).cpu().numpy()
    assert_bitexact(got2, oracle.index_select(x, dim, idx[::3]), layout + " strided idx")


def test_index_select_error_writes_nothing(cuda_ok):
    import torch

    import ctorch_b200 as cb

    src = torch.randn(100, 64, device="cuda")
    idx = torch.tensor([1, 2, 100, 3], device="cuda")
    out, status = cb.index_select_async(src, 0, idx)
    sentinel = torch.full_like(out, 7.0)
    out.copy_(sentinel)
    out2, status2 = cb.index_select_async(src, 0, idx)
    torch.cuda.synchronize()
    assert int(status2[:4].view(torch.int32)[0].item()) == 1
    assert int(status2[8:16].view(torch.int64)[0].item()) == 100
    with pytest.raises(cb.ShapeError):
        cb.index_select(src, 0, torch.tensor([-101], device="cuda"))
    with pytest.raises(cb.ShapeError):
        cb.index_select(src, 0, torch.tensor([-(2**63)], device="cuda"))
    # a valid call after an error on the same stream still works
    ok = cb.index_select(src, 0, torch.tensor([99, -100], device="cuda"))
    assert torch.equal(ok, src[[99, 0]])


def test_front_door_errors(cuda_ok):
    import torch

    import ctorch_b200 as cb

    a = torch.ones(3, 4, device="cuda")
    with pytest.raises(cb.DTypeError):
        cb.add(a.bool(), a)
    with pytest.raises(cb.DTypeError):
        cb.div(a.int(), a.int())
    with pytest.raises(cb.ShapeError):
        cb.add(a, torch.ones(5, device="cuda"))
    with pytest.raises(cb.DeviceError):
        cb.add(a, torch.ones(3, 4))
    with pytest.raises(cb.DTypeError):
        cb.add_(a.int(), a)  # in-place dtype must already be the promoted dtype
    with pytest.raises(cb.AliasError):
        cb.add_(a[:, 1:], a[:, :3])
    with pytest.raises(cb.ShapeError):
        cb.max(torch.ones(3, 0, device="cuda"), [1])
    with pytest.raises(cb.ShapeError):
        cb.argmax(torch.ones(3, 0, device="cuda"), 1)
    with pytest.raises(cb.ShapeError):
        cb.sum(a, [0, -2])
    with pytest.raises(cb.DTypeError):
        cb.mean(a.int())
    assert cb.sum(torch.ones(3, 0, device="cuda"), [1]).tolist() == [0.0, 0.0, 0.0]
    assert torch.isnan(cb.mean(torch.ones(3, 0, device="cuda"), [1])).all()


@pytest.mark.parametrize("shape,dt", [((16384, 8192), np.float32), ((16384, 4096), np.float64)])
def test_row_broadcast_binaries_on_the_fused_row_kernel(cuda_ok, oracle, shape, dt):
    """a op b with b one broadcast row over at least 16384 rows of 32 KiB or more runs the
    software-pipelined row kernel of the chain (its second op absent): bit-exact against the oracle
    for all four ops, NaN and infinities included, in place too, and with the operands the other
    way round (which the row kernel does not take)."""
    import torch

    import ctorch_b200 as cb

    rng = np.random.default_rng(_seed("rowbin", shape, np.dtype(dt).name))
    a = rng.standard_normal(shape).astype(dt)
    a.flat[::7919] = np.nan
    a.flat[5::104729] = np.inf
    b = rng.uniform(-2.0, 2.0, (1, shape[1])).astype(dt)
    b[0, ::997] = 0.0
    b[0, 3] = np.nan
    ta, tb = torch.from_numpy(a).cuda(), torch.from_numpy(b).cuda()
    for op in ("add", "sub", "mul", "div"):
        got = getattr(cb, op)(ta, tb).cpu().numpy()
        assert_bitexact(got, oracle.binary(op, a, b), f"{op} {shape} {np.dtype(dt).name}", nan_payload=False)
    got = getattr(cb, "sub")(tb, ta).cpu().numpy()  # the broadcast row first: elementwise kernels
    assert_bitexact(got, oracle.binary("sub", b, a), "row - matrix", nan_payload=False)
    tc = ta.clone()
    cb.sub_(tc, tb)
    assert_bitexact(tc.cpu().numpy(), oracle.binary("sub", a, b), "sub_ in place", nan_payload=False)


CHAIN_ROWS = [
    # (rows, cols, dtype, row_op, b scalar?, special values?)
    (4096, 8192, np.float32, "min", False, False),
    (3000, 1001, np.float32, "max", False, True),
    (777, 64, np.float64, "min", False, True),
    (500, 130, np.float32, "min", True, True),
    (1, 5, np.float32, "max", False, True),
    # rows of whole 16-byte packs: the pipelined loop, its batch-wise row extreme, a partial last
    # batch (4100 floats: 1025 packs; 1030 doubles: 515 packs)
    (2048, 2048, np.float32, "max", False, True),
    (1000, 4100, np.float32, "min", False, True),
    (600, 1030, np.float64, "max", False, True),
]


@pytest.mark.parametrize("rows,cols,dt,row_op,scalar,special", CHAIN_ROWS)
@pytest.mark.parametrize("ops", [("sub", "mul"), ("add", "div")])
def test_chain_rows_single_pass(cuda_ok, oracle, rows, cols, dt, row_op, scalar, special, ops):
    import torch

    import ctorch_b200 as cb

    rng = np.random.default_rng(_seed(rows, cols, row_op, ops))
    x = rng.standard_normal((rows, cols)).astype(dt)
    if special:
        x = np.round(x * 2) / 2  # ties
        x = x.astype(dt)
        x.flat[::997] = np.nan
        x[0, :] = np.inf if row_op == "min" else -np.inf  # a row of identities -> index 0
        if rows > 2:
            x[1, 3:] = np.inf
            x[1, 2] = -np.inf
        if rows > 3:  # every element a new extreme: each batch improves on the last
            x[3, :] = np.linspace(1.0, -1.0, cols) if row_op == "min" else np.linspace(-1.0, 1.0, cols)
    r = (rng.uniform(0.5, 2.0, () if scalar else (1, cols))).astype(dt)
    tx, tr = torch.from_numpy(x).cuda(), torch.from_numpy(np.asarray(r)).cuda()
    y, k, s = cb.chain_rows(ops[0], ops[1], tx, tr, tr, row_op=row_op)
    ry = oracle.binary(ops[1], oracle.binary(ops[0], x, np.asarray(r)), np.asarray(r))
    assert_bitexact(y.cpu().numpy(), ry, "chain_rows y", nan_payload=False)
    assert_bitexact(k.cpu().numpy(), oracle.reduce_idx(row_op, ry, 1, values=False), "chain_rows index")
    ref_sum = float(np.sum(ry.astype(np.float64)))
    got = float(s.cpu().numpy()[0])
    if np.isnan(ref_sum):
        assert np.isnan(got)
    elif np.isinf(ref_sum):
        assert got == ref_sum
    else:
        assert abs(got - ref_sum) <= 1e-12 * max(1.0, abs(np.sum(np.abs(ry.astype(np.float64)))))
    # without y / without the sum
    _, k2, _ = cb.chain_rows(ops[0], ops[1], tx, tr, tr, row_op=row_op, write_y=False, want_sum=False)
    assert torch.equal(k2, k)


def test_sharded_step_fused_matches_three_kernel_step(cuda_ok):
    import torch

    from ctorch_b200.sharded import ShardedSum, sharded_step, sharded_step_fused
    from ctorch_b200.synth import NORMAL, UNIFORM, device_fill

    x = device_fill(torch.empty((20000, 8192), device="cuda"), NORMAL, 4, 0, 0.0, 1.0)
    r = device_fill(torch.empty((1, 8192), device="cuda"), UNIFORM, 4, 1, -1.0, 1.0)
    y1, s1, k1 = sharded_step(x, r, ShardedSum(x.device, 1))
    y2, s2, k2 = sharded_step_fused(x, r, ShardedSum(x.device, 1))
    assert torch.equal(y1, y2)
    assert torch.equal(k1, k2)
    assert abs(float(s1) - float(s2)) <= 1e-6 * max(1.0, abs(float(s1)))


@pytest.mark.parametrize("uop", ["relu", "neg", "abs"])
@pytest.mark.parametrize("op", ["add", "sub", "mul", "div"])
@pytest.mark.parametrize("dt", [np.float32, np.float64, np.int32, np.int64])
def test_binary_unary_is_bitwise_the_eager_pair(cuda_ok, oracle, op, uop, dt):
    import ctorch_b200 as cb

    if op == "div" and np.dtype(dt).kind == "i":
        pytest.skip("integer division is refused")
    rng = np.random.default_rng(_seed(op, uop, np.dtype(dt).name))
    for layout in ("rows_long", "flat_tail", "rows_short", "general_offset"):
        sa, ra, sb, rb = BIN_LAYOUTS[layout]
        a, ta = _pair(_rand(rng, sa, dt), ra)
        b, tb = _pair(_rand(rng, sb, dt), rb)
        got = cb.binary_unary(op, uop, ta, tb).cpu().numpy()
        ref = oracle.unary(uop, oracle.binary(op, a, b))
        assert_bitexact(got, ref, f"{uop}({op}) {layout}", nan_payload=False)


def _special_divisors(dt):
    """Per-row divisors that probe the reciprocal path of a division by a per-row scalar: unit and
    power-of-two scales, all-ones significands, the exponents on either side of the range where
    the reciprocal is used, and zeros, infinities, NaN and subnormals (which take the IEEE
    division)."""
    dt = np.dtype(dt)
    if dt == np.float32:
        ui, mant, margin, emax = np.uint32, 23, 32, 254
    else:
        ui, mant, margin, emax = np.uint64, 52, 64, 2046
    ones = (1 << mant) - 1
    pats = []
    for e in (1, margin - 1, margin, margin + 1, emax // 2 - 1, emax // 2, emax // 2 + 1,
              emax - margin - 1, emax - margin, emax - margin + 1, emax):
        for m in (0, ones, 1, ones >> 1, 0x5 << (mant - 3)):
            pats.append((e << mant) | m)
    pats += [0, 1, ones, (emax + 1) << mant, ((emax + 1) << mant) | 1]  # 0, subnormals, inf, NaN
    v = np.array(pats, dtype=ui).view(dt)
    return np.concatenate([v, -v, np.array([3, 7, 0.1, 1 / 3, 10, -5e-3], dtype=dt)])


def _dividends(rng, n, dt):
    """Half uniform over every bit pattern (all exponents, NaN, inf, subnormals), half ordinary
    values."""
    dt = np.dtype(dt)
    ui = np.uint32 if dt.itemsize == 4 else np.uint64
    raw = rng.integers(0, np.iinfo(ui).max, n, dtype=ui, endpoint=True).view(dt)
    ordinary = (rng.standard_normal(n) * np.exp2(rng.integers(-20, 20, n))).astype(dt)
    return np.where(rng.random(n) < 0.5, raw, ordinary)


ROW_DIV = [
    # (x shape, divisor shape, x dtype, divisor dtype): the kernel each one plans to
    ((300, 1024), (300, 1), np.float32, np.float32),    # rows_mid
    ((300, 1024), (300, 1), np.float32, np.float64),    # rows_mid, promoted to float64
    ((128, 1000), (128, 1), np.float64, np.float64),    # rows_mid, last tile of each row partial
    ((300, 8192), (300, 1), np.float32, np.float32),    # rows_long, 2048 packs a row
    ((100, 5000), (100, 1), np.float32, np.float32),    # rows_long, 1250 packs a row
    ((96, 8200), (96, 1), np.float64, np.float64),      # rows_long with a tail
    ((3000, 100), (3000, 1), np.float64, np.float64),   # rows_short, 50 packs a row
    ((2000, 12), (2000, 1), np.float32, np.float32),    # rows_short, 3 packs a row
    ((4, 512, 1024), (1, 512, 1), np.float32, np.float64),  # the float32 / float64[1,512,1] shape
]


@pytest.mark.parametrize("sx,sd,dx,dd", ROW_DIV, ids=[f"{'x'.join(map(str, c[0]))}-{np.dtype(c[2]).name}-{np.dtype(c[3]).name}" for c in ROW_DIV])
def test_division_by_a_per_row_scalar_is_correctly_rounded(cuda_ok, oracle, sx, sd, dx, dd):
    import torch

    import ctorch_b200 as cb

    rng = np.random.default_rng(_seed("rowdiv", sx, sd))
    x = _dividends(rng, int(np.prod(sx)), dx).reshape(sx)
    rows = int(np.prod(sd))
    special = _special_divisors(dd)
    d = _dividends(rng, rows, dd)
    d[: min(rows, special.size)] = special[:rows]
    rng.shuffle(d)
    d = d.reshape(sd)
    # exact quotients: a few rows hold small multiples of their divisor
    flat_x = x.reshape(-1, sx[-1])
    flat_d = np.broadcast_to(d, sx[:-1] + (1,)).reshape(-1, 1)
    k = rng.integers(-64, 64, (4, sx[-1])).astype(dx)
    flat_x[:4] = (flat_d[:4].astype(np.float64) * k).astype(dx)
    got = cb.div(torch.from_numpy(x).cuda(), torch.from_numpy(d).cuda()).cpu().numpy()
    assert_bitexact(got, oracle.binary("div", x, d), f"div {sx} / {sd}", nan_payload=False)


BULK_COLS = [
    # (shape, reduced dim): column reductions the bulk-copy kernel takes (rows of at least 512
    # bytes, a whole number of 16-byte chunks), from one stage to thousands, with tiles shared by
    # CTAs; the narrower dtypes of some shapes go to the register kernel instead
    ((8192, 2048), 0),
    ((100_000, 128), 0),
    ((33, 512), 0),
    ((5, 128), 0),
    ((1, 20_000), 0),
    ((4, 300, 272), 1),
    ((7, 65, 304), 1),
    ((3000, 528), 0),
    ((2000, 1024), 0),
    # contiguous rows narrower than 512 bytes (the narrow-column kernel for 4- and 8-byte types)
    ((100_000, 64), 0),
    ((50_001, 16), 0),
    ((7, 300, 12), 1),
    ((3, 1000, 32), 1),
    ((4000, 100), 0),
]


def _column_ops_against_the_oracle(oracle, rng, shape, dim, recipe=(), kernels=None):
    """max/min with and without positions, sum and prod over `dim` of every dtype, bit-exact (sums,
    means and float products within TOL_SUM). `kernels` maps a dtype to the first kernel its
    max-with-positions must launch."""
    from ctorch_b200 import _capi as C

    import ctorch_b200 as cb

    for dt in (np.float32, np.float64, np.int32, np.int64, np.bool_):
        base = _rand(rng, shape, dt)
        if np.dtype(dt).kind == "i":
            base = (base % 5).astype(dt)  # ties: the first row must win
        if np.dtype(dt).kind == "f":
            base = (np.round(base * 4) / 4).astype(dt)
            base.flat[::997] = np.nan
            base.flat[3::389] = -0.0
        x, tx = _pair(base, recipe)
        name = np.dtype(dt).name
        for op in ("max", "min"):
            v, i = getattr(cb, op)(tx, dim, False)
            if kernels and op == "max" and np.dtype(dt) in kernels:
                assert C.last_reduction_kernel() == kernels[np.dtype(dt)], (shape, name, C.last_reduction_kernel())
            rv, ri = oracle.reduce_idx(op, x, dim, False)
            assert_bitexact(v.cpu().numpy(), rv, f"{op} values {shape} {name}")
            assert_bitexact(i.cpu().numpy(), ri, f"{op} indices {shape} {name}")
            got = getattr(cb, op)(tx, [dim], True).cpu().numpy()
            assert_bitexact(got, oracle.reduce(op, x, [dim], True), f"{op} {shape} {name}")
        if np.dtype(dt).kind == "f":
            fbase = np.nan_to_num(base, nan=0.5)
            fx, tfx = _pair(fbase, recipe)
            got = cb.sum(tfx, [dim], False).cpu().numpy()
            assert_close(got, oracle.reduce("sum", fx, [dim], False), TOL_SUM[np.dtype(dt)], f"sum {shape} {name}")
            got = cb.mean(tfx, [dim], True).cpu().numpy()
            assert_close(got, oracle.reduce("mean", fx, [dim], True), TOL_SUM[np.dtype(dt)], f"mean {shape} {name}")
            px, tpx = _pair((1 + 1e-4 * fbase).astype(dt), recipe)
            got = cb.prod(tpx, [dim], False).cpu().numpy()
            assert_close(got, oracle.reduce("prod", px, [dim], False), TOL_SUM[np.dtype(dt)], f"prod {shape} {name}")
        else:
            got = cb.sum(tx, [dim], False).cpu().numpy()
            assert_bitexact(got, oracle.reduce("sum", x, [dim], False), f"sum {shape} {name}")


@pytest.mark.parametrize("shape,dim", BULK_COLS, ids=["x".join(map(str, s)) + f"-d{d}" for s, d in BULK_COLS])
def test_column_reductions_through_the_bulk_copy_ring(cuda_ok, oracle, shape, dim):
    from ctorch_b200 import _capi as C

    before = C.wait_timeouts()
    _column_ops_against_the_oracle(oracle, np.random.default_rng(_seed("bulk", shape, dim)), shape, dim)
    assert C.wait_timeouts() == before, "a bulk-copy wait timed out"


STRIP_COLS = [
    # (base shape, view recipe, reduced dim, bool's kernel): column reductions the strip kernel
    # takes for 4- and 8-byte types (rows of at least 1024, strips of at least 192 bytes over one
    # CTA per SM); bool goes to the bulk kernel, or to the register kernel where its rows do not
    # start on 16-byte boundaries. Row counts leave a partial last stage.
    ((1024, 8192), [], 0, "red_cols_bulk"),
    ((1030, 16384), [], 0, "red_cols_bulk"),
    ((2, 1100, 8192), [], 1, "red_cols_bulk"),
    ((3, 1024, 7104), [], 1, "red_cols_bulk"),  # 49 strips a batch row, of 36 or 37 packs
    ((1024, 8320), [("slice", 1, 0, 8192, 1)], 0, "red_cols_bulk"),  # rows 8320 apart
    ((1100, 8200), [("slice", 1, 8, 8200, 1)], 0, "red_outer"),  # base 8 elements in
]


@pytest.mark.parametrize("shape,recipe,dim,bool_kernel", STRIP_COLS,
                         ids=["x".join(map(str, s)) + ("-view" if r else "") + f"-d{d}" for s, r, d, _ in STRIP_COLS])
def test_column_reductions_through_the_strip_kernel(cuda_ok, oracle, shape, recipe, dim, bool_kernel):
    from ctorch_b200 import _capi as C

    before = C.wait_timeouts()
    kernels = {np.dtype(t): "red_cols_strip" for t in (np.float32, np.float64, np.int32, np.int64)}
    kernels[np.dtype(np.bool_)] = bool_kernel
    _column_ops_against_the_oracle(oracle, np.random.default_rng(_seed("strip", shape, dim)), shape, dim, recipe,
                                   kernels)
    assert C.wait_timeouts() == before, "a tensor-copy wait timed out"


def test_bounded_wait_times_out_and_the_device_stays_usable(cuda_ok):
    """A wait on a barrier that nothing arrives at must give up after its limit, be counted, and
    leave the context working (no trap, no hang)."""
    import ctypes

    import torch

    from ctorch_b200 import _capi as C

    import ctorch_b200 as cb

    before = C.wait_timeouts()
    done = ctypes.c_int(-1)
    rc = C.lib.ctb_debug_wait_timeout(5_000_000, ctypes.byref(done))  # 5 ms
    assert rc == C.OK, C.last_error()
    assert done.value == 0
    assert C.wait_timeouts() == before + 1
    x = torch.arange(12, dtype=torch.float32, device="cuda").reshape(3, 4)
    assert cb.sum(x).item() == 66.0
