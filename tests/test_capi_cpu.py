"""CPU-only checks of the C ABI library (no kernel is launched): it loads, exports every symbol
include/ctb/*.h declares, its planner picks the intended launch shape for the hot-path layouts,
its invariant-divisor arithmetic is exact, and argument / dtype validation fails with the ctorch
error class before any launch."""
import ctypes
import os
import random
import re

import numpy as np
import pytest

ROOT = os.path.abspath(os.path.join(os.path.dirname(__file__), ".."))


def _lib():
    from ctorch_b200 import _capi

    return _capi


def declared_symbols():
    names = set()
    for h in ("ctb.h", "ctb_debug.h"):
        txt = open(os.path.join(ROOT, "include", "ctb", h)).read()
        names |= set(re.findall(r"CTB_API\s+[\w\s\*]+?\b(ctb_\w+)\s*\(", txt))
    return sorted(names)


def test_library_exports_every_declared_symbol():
    C = _lib()
    names = declared_symbols()
    assert len(names) >= 19
    for n in names:
        assert hasattr(C.lib, n), n
    assert C.lib.ctb_abi_version() == C.ABI_VERSION


def test_library_is_built_for_sm100a_only():
    """The build recipes compile device code for sm_100a and nothing else: every -gencode of the
    kernel library's Makefile (and of the package build) names compute_100a / sm_100a."""
    mk = open(os.path.join(ROOT, "ctorch_b200", "csrc", "Makefile")).read()
    gencodes = re.findall(r"-gencode\s+(\S+)", mk)
    assert gencodes and set(gencodes) == {"arch=compute_100a,code=sm_100a"}, gencodes
    assert not re.search(r"sm_(?!100a)\d+|compute_(?!100a)\d+|-arch[= ]", mk)


def view(C, shape, strides=None, dtype=0, data=4096):
    v = C.View()
    v.data = data
    v.dtype = dtype
    v.ndim = len(shape)
    if strides is None:
        strides, acc = [], 1
        for s in reversed(shape):
            strides.insert(0, acc)
            acc *= s
    for d, (s, st) in enumerate(zip(shape, strides)):
        v.shape[d] = s
        v.strides[d] = st
    return v


def plan_ew(C, out, ins, vec=4):
    arr = (ctypes.POINTER(C.View) * len(ins))(*[ctypes.pointer(v) for v in ins])
    buf = ctypes.create_string_buffer(32)
    rank = ctypes.c_int(0)
    shape = (ctypes.c_int64 * 16)()
    rc = C.lib.ctb_debug_plan_elementwise(ctypes.byref(out), arr, len(ins), vec, buf, 32,
                                          ctypes.byref(rank), shape)
    assert rc == 0, C.last_error()
    return buf.value.decode(), list(shape[: rank.value])


def plan_red(C, inp, out, mask):
    buf = ctypes.create_string_buffer(32)
    rk, rr = ctypes.c_int(0), ctypes.c_int(0)
    rc = C.lib.ctb_debug_plan_reduction(ctypes.byref(inp), ctypes.byref(out), mask, buf, 32,
                                        ctypes.byref(rk), ctypes.byref(rr))
    assert rc == 0, C.last_error()
    return buf.value.decode(), rk.value, rr.value


def test_planner_hot_path_shapes():
    C = _lib()
    # config 1: A[4096,4096] + B[1,4096] -> row broadcast, vectorised rows
    out = view(C, [4096, 4096])
    assert plan_ew(C, out, [view(C, [4096, 4096]), view(C, [1, 4096])]) == ("rows_long", [4096, 4096])
    # relu on the contiguous result -> flat
    assert plan_ew(C, out, [view(C, [4096, 4096])]) == ("flat", [16777216])
    # config 4 mul: I[64,512,1024] * F[64,1024,512].transpose(1,2) -> tiled transpose
    o4 = view(C, [64, 512, 1024])
    ft = view(C, [64, 512, 1024], [524288, 1, 512])
    assert plan_ew(C, o4, [view(C, [64, 512, 1024], dtype=2), ft])[0] == "tiled"
    # config 4 div: P[64,512,1024] / D[1,512,1] -> rows of 256 packs with a per-row scalar, in
    # warp tiles of 128 packs
    o4d = view(C, [64, 512, 1024], dtype=1)
    assert plan_ew(C, o4d, [view(C, [64, 512, 1024]), view(C, [1, 512, 1], dtype=1)]) == \
        ("rows_mid", [64, 512, 1024])
    # rows of 127 packs are short, 128 mid, 1023 mid, 1024 long
    for cols, path in ((508, "rows_short"), (512, "rows_mid"), (4092, "rows_mid"), (4096, "rows_long")):
        assert plan_ew(C, view(C, [64, cols]), [view(C, [64, cols]), view(C, [64, 1])])[0] == path
    # config 5 fused chain: (X - r) * r with r [1, 8192]
    o5 = view(C, [32768, 8192])
    assert plan_ew(C, o5, [view(C, [32768, 8192]), view(C, [1, 8192]), view(C, [1, 8192])])[0] == "rows_long"
    # short rows
    assert plan_ew(C, view(C, [1000, 8]), [view(C, [1000, 8]), view(C, [1, 8])])[0] == "rows_short"
    # misaligned base pointer -> no packs
    assert plan_ew(C, view(C, [1000, 8]), [view(C, [1000, 8], data=4100), view(C, [1, 8])])[0] == "general"
    # in-place into a transposed destination: dims are reordered so the destination's unit stride
    # is inner, which turns the broadcast operand into a per-row scalar
    assert plan_ew(C, view(C, [64, 32], [1, 64]), [view(C, [64, 32], [1, 64]), view(C, [32])]) == \
        ("rows_short", [32, 64])
    # empty
    assert plan_ew(C, view(C, [0, 5]), [view(C, [0, 5]), view(C, [5])])[0] == "empty"


def test_planner_collapses_contiguous_dims():
    C = _lib()
    out = view(C, [2, 3, 4, 5])
    assert plan_ew(C, out, [view(C, [2, 3, 4, 5]), view(C, [2, 3, 4, 5])]) == ("flat", [120])
    # broadcast on dim 1 blocks the merge of dims 0/1 but not 2/3
    assert plan_ew(C, out, [view(C, [2, 3, 4, 5]), view(C, [2, 1, 4, 5])])[1] == [2, 3, 20]


def test_planner_reductions():
    C = _lib()
    x = view(C, [8192, 8192])
    assert plan_red(C, x, view(C, [8192, 1]), 0b10) == ("inner", 1, 1)      # sum dim=1 keepdim
    assert plan_red(C, x, view(C, [8192]), 0b01) == ("outer", 1, 1)         # max dim=0
    assert plan_red(C, x, view(C, []), 0b11) == ("inner", 0, 1)             # whole tensor
    xt = view(C, [8192, 8192], [1, 8192])
    assert plan_red(C, xt, view(C, [8192]), 0b10) == ("outer", 1, 1)        # sum over a transposed dim
    x3 = view(C, [6, 7, 8])
    assert plan_red(C, x3, view(C, [7]), 0b101)[0] == "general"            # dims (0, 2)
    assert plan_red(C, x3, view(C, [6]), 0b110) == ("inner", 1, 1)          # dims (1, 2) collapse
    assert plan_red(C, view(C, [3, 0]), view(C, [3]), 0b10)[0] == "general"  # empty slice: identity


def test_fastdiv_is_exact():
    C = _lib()
    rnd = random.Random(7)
    divisors = [1, 2, 3, 5, 7, 10, 255, 256, 257, 4095, 8192, 1000000, 2**31 - 1, 2**31, 2**32 + 1,
                2**40 + 3, 2**62 + 11]
    divisors += [rnd.randrange(1, 2**63) for _ in range(40)]
    for d in divisors:
        for n in [0, 1, d - 1, d, d + 1, 2 * d - 1, 2**63 - 1, 2**63 - d] + [rnd.randrange(0, 2**63) for _ in range(50)]:
            if n < 0 or n >= 2**63:
                continue
            assert C.lib.ctb_debug_fastdiv(n, d) == n // d, (n, d)


def _as_ptr(v):
    import ctypes as ct

    return ct.byref(v)


def test_validation_errors_before_launch():
    C = _lib()
    null = None
    a = view(C, [4, 5])
    # bool arithmetic (binary_ops_cpu.cpp:202-208)
    assert C.lib.ctb_binary(C.ADD, view(C, [4, 5], dtype=C.BOOL), a, a, null) == C.ERR_DTYPE
    # output dtype must be the promoted dtype
    assert C.lib.ctb_binary(C.ADD, view(C, [4, 5], dtype=C.I32), a, view(C, [4, 5], dtype=C.F64), null) == C.ERR_DTYPE
    # integer division refused (binary_ops_cpu.cpp:106-109)
    ai = view(C, [4, 5], dtype=C.I32)
    assert C.lib.ctb_binary(C.DIV, ai, ai, ai, null) == C.ERR_DTYPE
    assert "integer division" in C.last_error()
    # broadcast failure
    assert C.lib.ctb_binary(C.ADD, view(C, [4, 5]), view(C, [3, 5]), view(C, [4, 5]), null) == C.ERR_SHAPE
    # rank above 16 (src/ops/tensor_iter.cpp:362-369)
    big = view(C, [1] * 16)
    big.ndim = 17
    assert C.lib.ctb_binary(C.ADD, big, a, a, null) == C.ERR_SHAPE
    # transcendental on ints, relu on bool
    assert C.lib.ctb_unary(C.EXP, ai, ai, null) == C.ERR_DTYPE
    ab = view(C, [4, 5], dtype=C.BOOL)
    assert C.lib.ctb_unary(C.RELU, ab, ab, null) == C.ERR_DTYPE
    # mean of ints, sum of int32 into int32
    assert C.lib.ctb_reduce(C.MEAN, ai, view(C, [4], dtype=C.I32), 0b10, None, 0, null) == C.ERR_DTYPE
    assert C.lib.ctb_reduce(C.SUM, ai, view(C, [4], dtype=C.I32), 0b10, None, 0, null) == C.ERR_DTYPE
    # reduction axis out of range, wrong keepdim shape
    assert C.lib.ctb_reduce(C.SUM, a, view(C, [4]), 0b100, None, 0, null) == C.ERR_SHAPE
    assert C.lib.ctb_reduce(C.SUM, a, view(C, [4, 5]), 0b10, None, 0, null) == C.ERR_SHAPE
    # zero-length axis for argmax (reduction_ops_cpu.cpp:433-436)
    z = view(C, [3, 0])
    assert C.lib.ctb_reduce_index(C.MAX, z, None, view(C, [3], dtype=C.I64), 1, None, 0, null) == C.ERR_SHAPE
    # index_select: 2-D indices, float indices, dim out of range
    st = ctypes.c_void_p(8192)
    assert C.lib.ctb_index_select(a, 0, view(C, [2, 2], dtype=C.I64), a, st, null) == C.ERR_SHAPE
    assert C.lib.ctb_index_select(a, 0, view(C, [2]), view(C, [2, 5]), st, null) == C.ERR_DTYPE
    assert C.lib.ctb_index_select(a, 2, view(C, [2], dtype=C.I64), view(C, [4, 2]), st, null) == C.ERR_SHAPE
    # unknown op code
    assert C.lib.ctb_binary(9, a, a, a, null) == C.ERR_ARGUMENT


def test_scratch_sizes_are_deterministic():
    C = _lib()
    x = view(C, [64, 1 << 20])
    out = view(C, [64])
    n1 = C.lib.ctb_reduce_scratch_bytes(C.SUM, x, out, 0b10)
    n2 = C.lib.ctb_reduce_scratch_bytes(C.SUM, x, out, 0b10)
    assert n1 == n2 and n1 > 0  # 64 long rows split across CTAs -> double partials
    assert C.lib.ctb_reduce_scratch_bytes(C.SUM, view(C, [8192, 8192]), view(C, [8192, 1]), 0b10) == 0
    assert C.lib.ctb_reduce_index_scratch_bytes(view(C, [8192, 8192]), 0) > 0


def test_noalloc_size_check_refuses_needs_above_its_array():
    """ctb_reduce_noalloc's size check (ctb_debug_noalloc_fits runs the same function without a
    device): needs up to the fixed 4 MiB pass, anything above is CTB_ERR_SCRATCH with a message
    that names both sizes. The planner's split caps keep every real plan well inside the array, so
    the refusal is only reachable through this check: a sweep of row, column and whole-tensor sums
    and max/min over the hot-path dtypes stays under it."""
    C = _lib()
    cap = 4 << 20
    assert C.lib.ctb_debug_noalloc_fits(0) == C.OK
    assert C.lib.ctb_debug_noalloc_fits(cap) == C.OK
    assert C.lib.ctb_debug_noalloc_fits(cap + 1) == C.ERR_SCRATCH
    msg = C.last_error()
    assert str(cap + 1) in msg and str(cap) in msg and "ctb_reduce" in msg
    worst = 0
    for dt in (C.F32, C.F64, C.I64):
        for rows in (2**k for k in range(1, 31, 3)):
            for cols in (1, 7, 520, 2048, 8192, 65536):
                for mask, out in ((0b01, [cols]), (0b10, [rows]), (0b11, [])):
                    for op in (C.SUM, C.MAX):
                        n = C.lib.ctb_reduce_scratch_bytes(op, view(C, [rows, cols], dtype=dt),
                                                           view(C, out, dtype=dt), mask)
                        worst = max(worst, n)
    assert 0 < worst <= cap, worst


def _strip(C, batch, np_, pk_max=64, slots=148):
    s, w = ctypes.c_int64(-1), ctypes.c_int64(-1)
    ok = C.lib.ctb_debug_strip_geometry(batch, np_, pk_max, slots, ctypes.byref(s), ctypes.byref(w))
    return ok, s.value, w.value


def test_strip_geometry_of_the_column_shapes():
    """The strip column kernel's choice of strips: whole columns per CTA when the strips come out
    at least 12 packs (192 bytes) wide and the units spread within 95% of evenly over the CTAs."""
    C = _lib()
    # argmax over dim 0 of [8192, 8192] float32: 2048 packs a row -> 147 strips of 13-14 packs
    assert _strip(C, 1, 2048) == (1, 147, 14)
    # [*, 32768] float32: 8192 packs -> 147 strips of at most 56 packs
    assert _strip(C, 1, 8192) == (1, 147, 56)
    # [*, 65536]: wider than one box row (64 packs) per CTA -> three rounds of 443 strips of 37
    # packs (111 pack-rows for the busiest CTA, against 112 for two rounds of 293 strips of 56)
    assert _strip(C, 1, 16384) == (1, 443, 37)
    # float64 rows of 8192: 4096 packs, boxes up to 128 packs
    assert _strip(C, 1, 4096, pk_max=128) == (1, 147, 28)
    # two and three batch rows of 2048 packs share the CTAs
    assert _strip(C, 2, 2048) == (1, 74, 28)
    assert _strip(C, 3, 2048) == (1, 49, 42)
    # [*, 4096] float32: 1024 packs cannot give 148 strips of 12 packs -> the bulk kernel
    assert _strip(C, 1, 1024)[0] == 0
    # narrow rows: nothing to split
    assert _strip(C, 1000, 8)[0] == 0
    assert _strip(C, 1, 11)[0] == 0


def test_strip_geometry_invariants():
    C = _lib()
    rng = np.random.default_rng(7)
    taken = 0
    for _ in range(3000):
        batch = int(rng.integers(1, 600))
        np_ = int(rng.integers(1, 40000))
        pk_max = int(rng.choice([64, 128]))
        ok, s, w = _strip(C, batch, np_, pk_max)
        if not ok:
            assert (s, w) == (0, 0)
            continue
        taken += 1
        assert 12 <= w <= pk_max and s * w >= np_ and s * (w - 1) < np_
        units = batch * s
        cost = -(-units // 148) * w
        assert batch * np_ / 148 >= 0.95 * cost
    assert taken > 100
