"""Seeded case catalog for the golden vectors in tests/golden/ctorch_ref_cases.npz.

Each case is an op plus inputs. An input is a contiguous base array and a "view recipe" — a list
of ctorch view ops — so the very same strided view can be rebuilt in numpy (for the oracle), in
torch (for the CUDA backend) and in ctorch itself (oracle/_ref, through Tensor::permute / slice /
select, src/tensor.cpp:206-389). The cases port the semantics the ctorch unit tests pin
(tests/ops/*.cpp): broadcasting, signed wrap, permuted operands, NaN/tie rules, empty slices,
index range errors, strided sources.
"""
from __future__ import annotations

import json

import numpy as np

I32_MIN, I32_MAX = np.iinfo(np.int32).min, np.iinfo(np.int32).max
I64_MIN, I64_MAX = np.iinfo(np.int64).min, np.iinfo(np.int64).max


def apply_numpy(base: np.ndarray, recipe):
    v = base
    for step in recipe:
        kind = step[0]
        if kind == "permute":
            v = v.transpose(step[1])
        elif kind == "slice":
            _, dim, start, end, st = step
            idx = [slice(None)] * v.ndim
            idx[dim] = slice(start, end, st)
            v = v[tuple(idx)]
        elif kind == "select":
            _, dim, i = step
            idx = [slice(None)] * v.ndim
            idx[dim] = i
            v = v[tuple(idx)]
        else:
            raise ValueError(kind)
    return v


def apply_torch(base, recipe):
    v = base
    for step in recipe:
        kind = step[0]
        if kind == "permute":
            v = v.permute(*step[1])
        elif kind == "slice":
            _, dim, start, end, st = step
            idx = [slice(None)] * v.dim()
            idx[dim] = slice(start, end, st)
            v = v[tuple(idx)]
        elif kind == "select":
            _, dim, i = step
            v = v.select(dim, i)
        else:
            raise ValueError(kind)
    return v


def apply_ref(t, recipe):
    for step in recipe:
        kind = step[0]
        if kind == "permute":
            t = t.permute(step[1])
        elif kind == "slice":
            _, dim, start, end, st = step
            t = t.slice(dim, start, end, st)
        elif kind == "select":
            t = t.select(step[1], step[2])
        else:
            raise ValueError(kind)
    return t


class Case:
    def __init__(self, name, kind, op, inputs, **kw):
        self.name = name
        self.kind = kind  # binary | inplace | unary | reduce | reduce_idx | arg | index_select
        self.op = op
        self.inputs = inputs  # list of (base ndarray, recipe)
        self.kw = kw

    def meta(self):
        return json.dumps({"kind": self.kind, "op": self.op, "kw": self.kw,
                           "recipes": [r for _, r in self.inputs]})


def _rng(seed):
    return np.random.default_rng(seed)


def _f(rng, shape, dt=np.float32):
    return rng.standard_normal(shape).astype(dt)


def _i(rng, shape, dt=np.int32, lo=-32, hi=32):
    return rng.integers(lo, hi, size=shape, dtype=dt)


def cases():
    out = []
    rng = _rng(1234)

    # ---- binary: broadcast / dtypes / wrap / views (tests/ops/binary_test.cpp, broadcast_test.cpp)
    for op in ("add", "sub", "mul", "div"):
        out.append(Case(f"{op}_f32_contig", "binary", op, [(_f(rng, (7, 33)), []), (_f(rng, (7, 33)), [])]))
        out.append(Case(f"{op}_f64_bcast", "binary", op,
                        [(_f(rng, (5, 1, 7), np.float64), []), (_f(rng, (1, 4, 7), np.float64), [])]))
        out.append(Case(f"{op}_f32_row_bcast", "binary", op, [(_f(rng, (16, 64)), []), (_f(rng, (1, 64)), [])]))
        out.append(Case(f"{op}_f32_col_bcast", "binary", op, [(_f(rng, (9, 40)), []), (_f(rng, (9, 1)), [])]))
        out.append(Case(f"{op}_f32_scalar", "binary", op, [(_f(rng, ()), []), (_f(rng, (17,)), [])]))
        out.append(Case(f"{op}_f32_permuted_rhs", "binary", op,
                        [(_f(rng, (6, 10)), []), (_f(rng, (10, 6)), [("permute", [1, 0])])]))
        out.append(Case(f"{op}_f32_strided_slices", "binary", op,
                        [(_f(rng, (10, 12)), [("slice", 0, 0, 10, 2), ("slice", 1, 1, 12, 3)]),
                         (_f(rng, (5, 4)), [])]))
        out.append(Case(f"{op}_f32_select", "binary", op,
                        [(_f(rng, (4, 5, 6)), [("select", 1, 2)]), (_f(rng, (6,)), [])]))
        out.append(Case(f"{op}_f32_transposed_3d", "binary", op,
                        [(_f(rng, (3, 24, 40)), []), (_f(rng, (3, 40, 24)), [("permute", [0, 2, 1])])]))
        out.append(Case(f"{op}_f32_high_rank", "binary", op,
                        [(_f(rng, (1, 1, 1, 1, 1, 1, 1, 1, 4)), []), (_f(rng, (1, 4)), [])]))
        out.append(Case(f"{op}_f32_empty", "binary", op, [(_f(rng, (0, 5)), []), (_f(rng, (5,)), [])]))
        # mixed dtypes: promotion in registers (ctorch casts on the host first)
        out.append(Case(f"{op}_i32_f32_mixed", "binary", op,
                        [(_i(rng, (8, 12), lo=-1000, hi=1001), []), (_f(rng, (12, 8)), [("permute", [1, 0])])]))
        out.append(Case(f"{op}_f32_f64_mixed", "binary", op,
                        [(_f(rng, (4, 6, 8)), []), (rng.uniform(0.5, 2, (1, 6, 1)), [])]))
        out.append(Case(f"{op}_i64_f32_mixed", "binary", op,
                        [(_i(rng, (5, 7), np.int64, -10**12, 10**12), []), (_f(rng, (7,)), [])]))
        # special values
        sv = np.array([0.0, -0.0, 1.0, -1.0, np.inf, -np.inf, np.nan, 3e38, -3e38, 1e-45], np.float32)
        out.append(Case(f"{op}_f32_special", "binary", op,
                        [(np.repeat(sv, 10).reshape(10, 10), []), (np.tile(sv, 10).reshape(10, 10), [])]))
    for op in ("add", "sub", "mul"):
        out.append(Case(f"{op}_i32", "binary", op, [(_i(rng, (5, 9)), []), (_i(rng, (9,)), [])]))
        out.append(Case(f"{op}_i64_bcast", "binary", op,
                        [(_i(rng, (2, 3), np.int64), []), (_i(rng, (3,), np.int64), [])]))
        out.append(Case(f"{op}_i32_i64_mixed", "binary", op,
                        [(_i(rng, (4, 5)), []), (_i(rng, (4, 5), np.int64, -10**15, 10**15), [])]))
        wrap = np.array([I32_MAX, I32_MIN, 1 << 30, -(1 << 30), 1, -1, 0, 4], np.int32)
        out.append(Case(f"{op}_i32_wrap", "binary", op,
                        [(np.repeat(wrap, 8).reshape(8, 8), []), (np.tile(wrap, 8).reshape(8, 8), [])]))
        wrap64 = np.array([I64_MAX, I64_MIN, 1 << 62, -(1 << 62), 1, -1, 0, 4], np.int64)
        out.append(Case(f"{op}_i64_wrap", "binary", op,
                        [(np.repeat(wrap64, 8).reshape(8, 8), []), (np.tile(wrap64, 8).reshape(8, 8), [])]))
    # in-place (tests/ops/inplace_test.cpp): out = a
    for op in ("add", "sub", "mul", "div"):
        out.append(Case(f"{op}_inplace_f32_bcast", "inplace", op, [(_f(rng, (6, 20)), []), (_f(rng, (20,)), [])]))
        out.append(Case(f"{op}_inplace_f32_permuted_dst", "inplace", op,
                        [(_f(rng, (20, 6)), [("permute", [1, 0])]), (_f(rng, (6, 20)), [])]))
    out.append(Case("add_inplace_f64_f32", "inplace", "add", [(_f(rng, (5, 5), np.float64), []), (_f(rng, (5,)), [])]))

    # ---- unary (tests/ops/unary_test.cpp)
    special = np.array([0.0, -0.0, 1.5, -1.5, np.inf, -np.inf, np.nan, -np.nan, 1e-40, -1e-40], np.float32)
    for dt in (np.float32, np.float64):
        for op in ("relu", "neg", "abs"):
            out.append(Case(f"{op}_{np.dtype(dt).name}_special", "unary", op, [(special.astype(dt), [])]))
    for op in ("relu", "neg", "abs"):
        out.append(Case(f"{op}_i32_edges", "unary", op, [(np.array([I32_MIN, -1, 0, 1, I32_MAX, -7], np.int32), [])]))
        out.append(Case(f"{op}_i64_edges", "unary", op, [(np.array([I64_MIN, -1, 0, 1, I64_MAX, -7], np.int64), [])]))
        out.append(Case(f"{op}_f32_permuted", "unary", op, [(_f(rng, (12, 9)), [("permute", [1, 0])])]))
    for dt in (np.float32, np.float64):
        x = _f(rng, (64,), dt)
        pos = (np.abs(_f(rng, (64,), dt)) + 0.1).astype(dt)
        out.append(Case(f"exp_{np.dtype(dt).name}", "unary", "exp", [(x, [])]))
        out.append(Case(f"tanh_{np.dtype(dt).name}", "unary", "tanh", [(x, [])]))
        out.append(Case(f"sigmoid_{np.dtype(dt).name}", "unary", "sigmoid", [(x * 8, [])]))
        out.append(Case(f"log_{np.dtype(dt).name}", "unary", "log", [(pos, [])]))
        out.append(Case(f"sqrt_{np.dtype(dt).name}", "unary", "sqrt", [(pos, [])]))

    # ---- reductions (tests/ops/reduction_*_test.cpp)
    x3 = {np.float32: _f(rng, (6, 7, 8)), np.float64: _f(rng, (6, 7, 8), np.float64),
          np.int32: _i(rng, (6, 7, 8)), np.int64: _i(rng, (6, 7, 8), np.int64),
          np.bool_: rng.integers(0, 2, (6, 7, 8)).astype(np.bool_)}
    dim_sets = [None, [0], [1], [2], [-1], [0, 2], [1, 2], [0, 1]]
    for op in ("sum", "prod", "mean", "max", "min"):
        for dt, x in x3.items():
            if op == "mean" and dt not in (np.float32, np.float64):
                continue
            for dims in dim_sets:
                for kd in (False, True):
                    if dims is None and kd:
                        continue
                    xin = x
                    if op == "prod" and dt in (np.float32, np.float64):
                        xin = (1 + 0.01 * x).astype(dt)
                    out.append(Case(f"{op}_{np.dtype(dt).name}_d{dims}_k{int(kd)}", "reduce", op,
                                    [(xin, [])], dims=dims, keepdim=kd))
        out.append(Case(f"{op}_f32_permuted", "reduce", op, [(_f(rng, (9, 33)), [("permute", [1, 0])])],
                        dims=[1], keepdim=False))
        out.append(Case(f"{op}_f32_sliced_whole", "reduce", op, [(_f(rng, (12, 30)), [("slice", 1, 3, 30, 2)])],
                        dims=None, keepdim=False))
        out.append(Case(f"{op}_f32_long_rows", "reduce", op, [(_f(rng, (3, 3000)), [])], dims=[1], keepdim=True))
        out.append(Case(f"{op}_f32_long_cols", "reduce", op, [(_f(rng, (700, 24)), [])], dims=[0], keepdim=False))
    # empty slices (reduction_value_test.cpp:141-166)
    for op in ("sum", "mean", "prod"):
        out.append(Case(f"{op}_empty_slice", "reduce", op, [(np.zeros((3, 0), np.float32), [])], dims=[1], keepdim=False))
    out.append(Case("sum_empty_whole_i32", "reduce", "sum", [(np.zeros((0,), np.int32), [])], dims=None, keepdim=False))
    # NaN, signed zeros, infinities, extremes in max/min
    mm = np.array([[0.0, -0.0, 1.0], [-0.0, 0.0, -1.0], [np.nan, 2.0, np.nan], [-np.inf, -np.inf, -np.inf],
                   [3.0, np.nan, 3.0], [-0.0, -0.0, 0.0]], np.float32)
    for op in ("max", "min"):
        for dims in (None, [0], [1]):
            out.append(Case(f"{op}_f32_special_d{dims}", "reduce", op, [(mm, [])], dims=dims, keepdim=False))
        out.append(Case(f"{op}_i64_extremes", "reduce", op,
                        [(np.array([[I64_MIN, I64_MAX], [0, -1]], np.int64), [])], dims=[0], keepdim=False))
    # single-axis max/min with index, argmax/argmin (ties -> first, NaN -> first NaN)
    tied = np.array([1.0, 3.0, 3.0, 2.0, 3.0], np.float32)
    for op in ("max", "min"):
        for dt, x in x3.items():
            for axis in (0, 1, 2, -1):
                for kd in (False, True):
                    out.append(Case(f"{op}idx_{np.dtype(dt).name}_a{axis}_k{int(kd)}", "reduce_idx", op,
                                    [(x, [])], dim=axis, keepdim=kd))
        out.append(Case(f"{op}idx_f32_special_a0", "reduce_idx", op, [(mm, [])], dim=0, keepdim=False))
        out.append(Case(f"{op}idx_f32_special_a1", "reduce_idx", op, [(mm, [])], dim=1, keepdim=False))
        out.append(Case(f"{op}idx_f32_permuted", "reduce_idx", op,
                        [(_f(rng, (40, 9)), [("permute", [1, 0])])], dim=1, keepdim=False))
        out.append(Case(f"{op}idx_f32_long_cols", "reduce_idx", op, [(_f(rng, (700, 24)), [])], dim=0, keepdim=False))
    for op in ("argmax", "argmin"):
        out.append(Case(f"{op}_tied", "arg", op, [(tied, [])], dim=0, keepdim=False))
        out.append(Case(f"{op}_nan", "arg", op, [(np.array([1.0, np.nan, 5.0, np.nan], np.float32), [])], dim=0, keepdim=False))
        out.append(Case(f"{op}_f32_rows", "arg", op, [(_f(rng, (17, 300)), [])], dim=1, keepdim=True))
        out.append(Case(f"{op}_i32_cols", "arg", op, [(_i(rng, (300, 17), lo=-3, hi=3), [])], dim=0, keepdim=False))
        out.append(Case(f"{op}_bool", "arg", op, [(rng.integers(0, 2, (5, 6)).astype(np.bool_), [])], dim=1, keepdim=False))

    # ---- index_select (tests/ops/index_select_test.cpp, index_select_dtype_test.cpp)
    t = _f(rng, (7, 5, 6))
    for dim in (0, 1, 2, -1):
        for idt in (np.int32, np.int64):
            size = t.shape[dim]
            idx = rng.integers(-size, size, 11).astype(idt)
            out.append(Case(f"index_select_f32_d{dim}_{np.dtype(idt).name}", "index_select", None,
                            [(t, []), (idx, [])], dim=dim))
    for dt in (np.float64, np.int32, np.int64, np.bool_):
        src = x3[dt] if dt in x3 else x3[np.float32]
        out.append(Case(f"index_select_{np.dtype(dt).name}_rows", "index_select", None,
                        [(src, []), (np.array([5, 0, 5, 2, -1], np.int64), [])], dim=0))
    out.append(Case("index_select_strided_src", "index_select", None,
                    [(_f(rng, (8, 10)), [("permute", [1, 0]), ("slice", 1, 1, 8, 2)]),
                     (np.array([3, 0, 9, 9], np.int64), [])], dim=0))
    out.append(Case("index_select_strided_idx", "index_select", None,
                    [(_f(rng, (6, 16)), []), (np.array([5, 9, 1, 9, 0, 9, 2], np.int64), [("slice", 0, 0, 7, 2)])],
                    dim=0))
    out.append(Case("index_select_empty_idx", "index_select", None,
                    [(_f(rng, (4, 3)), []), (np.zeros((0,), np.int64), [])], dim=0))
    out.append(Case("index_select_oor", "index_select", None,
                    [(_f(rng, (4, 3)), []), (np.array([0, 4], np.int64), [])], dim=0))
    out.append(Case("index_select_negative_oor", "index_select", None,
                    [(_f(rng, (4, 3)), []), (np.array([-5], np.int64), [])], dim=0))
    out.append(Case("index_select_int64_min", "index_select", None,
                    [(_f(rng, (4, 3)), []), (np.array([I64_MIN], np.int64), [])], dim=0))
    out.append(Case("index_select_rows_1k", "index_select", None,
                    [(_f(rng, (50, 256)), []), (rng.integers(0, 50, 300).astype(np.int64), [])], dim=0))
    return out
