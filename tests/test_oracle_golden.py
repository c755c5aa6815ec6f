"""Pins the C restatement (oracle/ctb_oracle.c) against ctorch:
  * ctorch's own parity fixtures (tests/parity/fixtures in the ctorch tree, NumPy-generated),
    with ctorch's tolerances (tests/parity/binary_parity_test.cpp:118-127);
  * the catalog cases run through ctorch's CPU backend itself (tests/golden/make_golden.py),
    bit for bit, including error outcomes.
"""
import os
import re

import numpy as np
import pytest

from helpers import GOLDEN, assert_bitexact, assert_close, golden_cases, run_oracle
from oracle.oracle import OracleError

FIX = np.load(os.path.join(GOLDEN, "ctorch_parity_fixtures.npz"))
FIX_NAMES = sorted(FIX.files)


def _tol(dt):
    return {np.dtype(np.float32): 1e-5, np.dtype(np.float64): 1e-12}.get(np.dtype(dt), 0.0)


def _check(got, ref, what):
    if np.dtype(ref.dtype).kind == "f":
        assert_close(got, ref.astype(got.dtype) if got.dtype != ref.dtype else ref, _tol(ref.dtype), what)
    else:
        assert got.shape == ref.shape, what
        assert np.array_equal(got, ref.astype(got.dtype)), what


def _dims(tag):
    if tag == "dimsAll":
        return None
    if tag.startswith("dims"):
        return [(-int(t[1:]) if t.startswith("n") else int(t)) for t in tag[4:].split("_")]
    t = tag[3:]
    return -int(t[1:]) if t.startswith("n") else int(t)


def _prefixes(suffix):
    return sorted({n[: -len(suffix)] for n in FIX_NAMES if n.endswith(suffix)})


BIN = [p for p in _prefixes("_ref") if re.match(r"^(add|sub|mul|div)_", p) and p + "_a" in FIX.files]
UN = [p for p in _prefixes("_ref") if re.match(r"^(neg|abs|relu|exp|log|sqrt|sigmoid|tanh)_", p)]
RED = [p for p in _prefixes("_ref") if re.match(r"^(sum|mean|prod|maxval|minval)_", p)]
IDX = [p for p in _prefixes("_ref_idx") if re.match(r"^(maxidx|minidx)_", p)]
ARG = [p for p in _prefixes("_ref") if re.match(r"^(argmax|argmin)_", p)]
SEL = [p for p in _prefixes("_ref") if p.startswith("index_select_")]


def test_fixture_catalog_is_complete():
    # every fixture file belongs to exactly one parsed case
    used = set()
    for p in BIN:
        used |= {p + "_a", p + "_b", p + "_ref"}
    for p in UN + RED + ARG:
        used |= {p + "_in", p + "_ref"}
    for p in IDX:
        used |= {p + "_in", p + "_ref", p + "_ref_idx"}
    for p in SEL:
        used |= {p + "_in", p + "_idx", p + "_ref"}
    assert used == set(FIX_NAMES)
    assert len(BIN) == 13 and len(RED) == 18 and len(IDX) == 3 and len(ARG) == 3 and len(SEL) == 6


@pytest.mark.parametrize("p", BIN)
def test_binary_fixtures(oracle, p):
    op = p.split("_")[0]
    got = oracle.binary(op, FIX[p + "_a"], FIX[p + "_b"])
    _check(got, FIX[p + "_ref"], p)


@pytest.mark.parametrize("p", UN)
def test_unary_fixtures(oracle, p):
    op = p.split("_")[0]
    got = oracle.unary(op, FIX[p + "_in"])
    _check(got, FIX[p + "_ref"], p)


@pytest.mark.parametrize("p", RED)
def test_reduce_fixtures(oracle, p):
    tok = p.split("_")
    op = {"maxval": "max", "minval": "min"}.get(tok[0], tok[0])
    m = re.search(r"_(dimsAll|dims[n0-9_]+|dimn?[0-9]+)_(kd[01])$", p)
    dims, kd = _dims(m.group(1)), m.group(2) == "kd1"
    got = oracle.reduce(op, FIX[p + "_in"], dims, kd)
    _check(got, FIX[p + "_ref"], p)


@pytest.mark.parametrize("p", IDX)
def test_reduce_idx_fixtures(oracle, p):
    tok = p.split("_")
    op = "max" if tok[0] == "maxidx" else "min"
    v, i = oracle.reduce_idx(op, FIX[p + "_in"], _dims(tok[-2]), tok[-1] == "kd1")
    _check(v, FIX[p + "_ref"], p)
    assert np.array_equal(i, FIX[p + "_ref_idx"]), p


@pytest.mark.parametrize("p", ARG)
def test_arg_fixtures(oracle, p):
    tok = p.split("_")
    op = "max" if tok[0] == "argmax" else "min"
    kd_tok = [t for t in tok if t.startswith("kd")][0]
    dim_tok = [t for t in tok if t.startswith("dim")][0]
    got = oracle.reduce_idx(op, FIX[p + "_in"], _dims(dim_tok), kd_tok == "kd1", values=False)
    assert np.array_equal(got, FIX[p + "_ref"]), p


def test_argmax_tied_fixture_is_first_index(oracle):
    # scripts/gen_parity.py:180-184 in ctorch: [1, 3, 3, 2, 3] -> index 1
    p = "argmax_float32_5_dim0_kd0_tied"
    assert int(oracle.reduce_idx("max", FIX[p + "_in"], 0, values=False)) == 1


@pytest.mark.parametrize("p", SEL)
def test_index_select_fixtures(oracle, p):
    dim = int(re.search(r"_dim(\d+)_", p).group(1))
    got = oracle.index_select(FIX[p + "_in"], dim, FIX[p + "_idx"])
    assert_bitexact(got, FIX[p + "_ref"], p)


CASES = golden_cases()


@pytest.mark.parametrize("case", CASES, ids=[c.name for c in CASES])
def test_oracle_matches_ctorch_cpu(oracle, case):
    if case.status != 0:
        with pytest.raises(OracleError):
            run_oracle(oracle, case)
        return
    outs = run_oracle(oracle, case)
    assert len(outs) == len(case.outputs)
    for k, (g, r) in enumerate(zip(outs, case.outputs)):
        assert_bitexact(g, r, f"{case.name} out{k}")
