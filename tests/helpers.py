"""Comparison and golden-vector helpers shared by the CPU and GPU tests."""
from __future__ import annotations

import json
import os

import numpy as np

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")

# Tolerances written into the tests, in the |g - r| <= tol * max(1, |r|) form of ctorch's own
# parity tests (tests/parity/binary_parity_test.cpp:53-69,118-127).
TOL_SUM = {np.dtype(np.float32): 1e-5, np.dtype(np.float64): 1e-12}
# exp/log/tanh/sigmoid: CUDA's accurate math functions vs glibc differ by a few ulp.
TOL_TRANSCENDENTAL = {np.dtype(np.float32): 2e-6, np.dtype(np.float64): 1e-14}


def bits(a: np.ndarray) -> np.ndarray:
    a = np.ascontiguousarray(a)
    if a.dtype == np.bool_:
        return a.view(np.uint8)
    return a.view({1: np.uint8, 2: np.uint16, 4: np.uint32, 8: np.uint64}[a.dtype.itemsize])


def assert_bitexact(got: np.ndarray, ref: np.ndarray, what: str = "", nan_payload: bool = True):
    """Identical bits. With nan_payload=False, NaN results only need to be NaN on both sides (IEEE
    leaves NaN payloads of arithmetic unspecified; x86 and NVIDIA GPUs produce different ones)."""
    assert got.shape == ref.shape, f"{what}: shape {got.shape} != {ref.shape}"
    assert got.dtype == ref.dtype, f"{what}: dtype {got.dtype} != {ref.dtype}"
    if got.size == 0:
        return
    g, r = bits(got), bits(ref)
    diff = g != r
    if not nan_payload and ref.dtype.kind == "f":
        both_nan = np.isnan(got) & np.isnan(ref)
        diff &= ~both_nan
    if diff.any():
        i = np.argwhere(diff)[0]
        raise AssertionError(f"{what}: {int(diff.sum())} of {ref.size} differ; first at {tuple(i)}: "
                             f"got {got[tuple(i)]!r} ref {ref[tuple(i)]!r}")


def assert_close(got: np.ndarray, ref: np.ndarray, tol: float, what: str = ""):
    assert got.shape == ref.shape, f"{what}: shape {got.shape} != {ref.shape}"
    assert got.dtype == ref.dtype, f"{what}: dtype {got.dtype} != {ref.dtype}"
    if got.size == 0:
        return
    g = got.astype(np.float64)
    r = ref.astype(np.float64)
    nan_g, nan_r = np.isnan(g), np.isnan(r)
    assert (nan_g == nan_r).all(), f"{what}: NaN positions differ"
    inf = np.isinf(r)
    assert (g[inf] == r[inf]).all(), f"{what}: infinities differ"
    m = ~(nan_r | inf)
    err = np.abs(g[m] - r[m])
    lim = tol * np.maximum(1.0, np.abs(r[m]))
    if (err > lim).any():
        k = int(np.argmax(err - lim))
        raise AssertionError(f"{what}: max error {err[k]:.3e} > {lim[k]:.3e} (got {g[m][k]!r}, ref {r[m][k]!r})")


class GoldenCase:
    def __init__(self, z, name):
        self.name = name
        meta = json.loads(str(z[f"{name}/meta"]))
        self.kind = meta["kind"]
        self.op = meta["op"]
        self.kw = meta["kw"]
        self.recipes = meta["recipes"]
        self.inputs = []
        k = 0
        while f"{name}/in{k}" in z:
            self.inputs.append(z[f"{name}/in{k}"])
            k += 1
        self.status = int(z[f"{name}/status"])
        self.outputs = []
        k = 0
        while f"{name}/out{k}" in z:
            self.outputs.append(z[f"{name}/out{k}"])
            k += 1


def golden_cases():
    z = np.load(os.path.join(GOLDEN, "ctorch_ref_cases.npz"))
    return [GoldenCase(z, str(n)) for n in z["__names__"]]


def exact_kind(case_kind: str, op: str, dtype) -> bool:
    """Whether ctorch's CPU path and a correct CUDA path must agree bit for bit."""
    dt = np.dtype(dtype)
    if case_kind in ("binary", "inplace"):
        return True
    if case_kind == "unary":
        return op in ("relu", "neg", "abs", "sqrt")
    if case_kind == "reduce":
        return op in ("max", "min") or dt.kind != "f"
    return True  # reduce_idx, arg, index_select


def numpy_inputs(case):
    from catalog import apply_numpy

    return [apply_numpy(base, recipe) for base, recipe in zip(case.inputs, case.recipes)]


def run_oracle(O, case):
    """Runs a golden case through the C restatement (oracle/ctb_oracle.c)."""
    xs = numpy_inputs(case)
    kw = case.kw
    if case.kind == "binary":
        return [O.binary(case.op, xs[0], xs[1])]
    if case.kind == "inplace":
        a = xs[0].copy() if False else np.array(xs[0])  # oracle writes a fresh output
        return [O.binary(case.op, a, xs[1], out_dtype=a.dtype)]
    if case.kind == "unary":
        return [O.unary(case.op, xs[0])]
    if case.kind == "reduce":
        return [O.reduce(case.op, xs[0], kw["dims"], kw["keepdim"])]
    if case.kind == "reduce_idx":
        v, i = O.reduce_idx(case.op, xs[0], kw["dim"], kw["keepdim"])
        return [v, i]
    if case.kind == "arg":
        return [O.reduce_idx("max" if case.op == "argmax" else "min", xs[0], kw["dim"], kw["keepdim"],
                             values=False)]
    if case.kind == "index_select":
        return [O.index_select(xs[0], kw["dim"], xs[1])]
    raise ValueError(case.kind)


def torch_inputs(case, device="cuda"):
    import torch

    from catalog import apply_torch

    return [apply_torch(torch.from_numpy(np.ascontiguousarray(base)).to(device), recipe)
            for base, recipe in zip(case.inputs, case.recipes)]


def run_cuda(case):
    """Runs a golden case through the CUDA backend (ctorch_b200 ops, C ABI underneath)."""
    import ctorch_b200 as cb

    xs = torch_inputs(case)
    kw = case.kw
    if case.kind == "binary":
        return [getattr(cb, case.op)(xs[0], xs[1])]
    if case.kind == "inplace":
        getattr(cb, case.op + "_")(xs[0], xs[1])
        return [xs[0]]
    if case.kind == "unary":
        return [getattr(cb, case.op)(xs[0])]
    if case.kind == "reduce":
        return [getattr(cb, case.op)(xs[0], kw["dims"], kw["keepdim"])]
    if case.kind == "reduce_idx":
        r = getattr(cb, case.op)(xs[0], int(kw["dim"]), kw["keepdim"])
        return [r.values, r.indices]
    if case.kind == "arg":
        return [getattr(cb, case.op)(xs[0], kw["dim"], kw["keepdim"])]
    if case.kind == "index_select":
        return [cb.index_select(xs[0], kw["dim"], xs[1])]
    raise ValueError(case.kind)


def compare_case(case, got_list, ref_list):
    """Applies the parity bar for a case's op/dtype."""
    for k, (g, r) in enumerate(zip(got_list, ref_list)):
        what = f"{case.name} out{k}"
        dt = np.dtype(r.dtype)
        if case.kind == "unary" and case.op in ("exp", "log", "tanh", "sigmoid"):
            assert_close(g, r, TOL_TRANSCENDENTAL[dt], what)
        elif case.kind == "reduce" and case.op in ("sum", "mean", "prod") and dt.kind == "f":
            assert_close(g, r, TOL_SUM[dt], what)
        elif case.kind in ("binary", "inplace") or (case.kind == "unary" and case.op in ("neg", "abs", "sqrt")):
            assert_bitexact(g, r, what, nan_payload=False)
        else:
            assert_bitexact(g, r, what)
