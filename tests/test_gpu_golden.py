"""The CUDA backend against ctorch itself: every catalog case (tests/golden/catalog.py) run on the
B200 and compared with the outputs ctorch's CPU backend produced for the same inputs and views
(tests/golden/ctorch_ref_cases.npz), and ctorch's own NumPy parity fixtures.

Parity bar: bit-exact for integer ops, elementwise float ops, max/min/argmax/argmin values and
indices, and index_select; |g - r| <= 1e-5 * max(1, |r|) for float32 sum/mean/prod (1e-12 for
float64); a few ulp for exp/log/tanh/sigmoid. NaN results of float arithmetic compare as NaN
without their payload bits (IEEE 754 leaves them unspecified)."""
import os
import re

import numpy as np
import pytest

from helpers import GOLDEN, assert_bitexact, assert_close, compare_case, golden_cases, run_cuda

pytestmark = pytest.mark.gpu

CASES = golden_cases()


@pytest.mark.parametrize("case", CASES, ids=[c.name for c in CASES])
def test_cuda_matches_ctorch_cpu(cuda_ok, case):
    import ctorch_b200 as cb

    if case.status != 0:
        with pytest.raises(cb.ShapeError):
            run_cuda(case)
        return
    got = [t.cpu().numpy() for t in run_cuda(case)]
    assert len(got) == len(case.outputs)
    compare_case(case, got, case.outputs)


FIX = np.load(os.path.join(GOLDEN, "ctorch_parity_fixtures.npz"))


def _t(a):
    import torch

    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def test_cuda_matches_ctorch_parity_fixtures(cuda_ok):
    import ctorch_b200 as cb

    tol = {np.dtype(np.float32): 1e-5, np.dtype(np.float64): 1e-12}
    n = 0
    for name in sorted(FIX.files):
        if name.endswith("_ref") and name[:-4] + "_a" in FIX.files:
            p = name[:-4]
            got = getattr(cb, p.split("_")[0])(_t(FIX[p + "_a"]), _t(FIX[p + "_b"])).cpu().numpy()
        elif name.endswith("_ref") and re.match(r"^(neg|abs|relu|exp|log|sqrt|sigmoid|tanh)_", name):
            p = name[:-4]
            got = getattr(cb, p.split("_")[0])(_t(FIX[p + "_in"])).cpu().numpy()
        elif name.endswith("_ref") and name.startswith("index_select_"):
            p = name[:-4]
            dim = int(re.search(r"_dim(\d+)_", p).group(1))
            got = cb.index_select(_t(FIX[p + "_in"]), dim, _t(FIX[p + "_idx"])).cpu().numpy()
        else:
            continue
        ref = FIX[name]
        if ref.dtype.kind == "f":
            assert_close(got, ref.astype(got.dtype), tol[np.dtype(got.dtype)], name)
        else:
            assert np.array_equal(got, ref), name
        n += 1
    assert n == 13 + 15 + 6
