"""ctb_reduce_noalloc: the reductions of ctb_reduce for callers that cannot allocate device
memory — a plain C or FFI host with no device allocator of its own to hand out scratch, or a
process whose device memory is fixed at start-up and must not call cudaMalloc later. It takes its
scratch from a fixed array in the library's device image instead of from the caller.

Each case goes through the C ABI (ctypes) twice in a row and is compared with ctb_reduce given
caller-provided scratch, within the tolerances of the other reduction tests; the second call
reuses the array the first one left behind. This file is collected last so a run that stops at the
first failure has already run every other test; it also passes alone in a fresh process."""
import ctypes

import numpy as np
import pytest

from helpers import TOL_SUM, assert_bitexact, assert_close

pytestmark = pytest.mark.gpu

# (shape, reduced dims, op, keepdim, dtype): every case but the last needs scratch (split
# reductions); the last needs none.
CASES = [
    ((4096, 8192), None, "sum", False, "float32"),
    ((4, 1_000_003), [1], "mean", True, "float32"),
    ((8192, 2048), [0], "max", False, "float32"),
    ((3000, 520), [0], "min", False, "float64"),
    ((2_000_003,), None, "sum", False, "int32"),
    ((3, 1_500_000), [1], "prod", False, "float32"),
    ((1500, 1200), [0, 1], "max", False, "int64"),
    ((8192, 1024), [1], "sum", False, "float32"),
]


def _mask(ndim, dims):
    if dims is None:
        return (1 << ndim) - 1
    m = 0
    for d in dims:
        m |= 1 << (d % ndim)
    return m


@pytest.mark.parametrize("shape,dims,op,keepdim,dt", CASES, ids=[f"{c[2]}-{c[4]}-{len(c[0])}d-{i}" for i, c in enumerate(CASES)])
def test_reduce_without_allocation_matches_ctb_reduce(cuda_ok, shape, dims, op, keepdim, dt):
    import torch

    from ctorch_b200 import _capi as C

    g = torch.Generator(device="cuda").manual_seed(1234)
    tdt = getattr(torch, dt)
    if tdt.is_floating_point:
        x = torch.randn(shape, generator=g, device="cuda", dtype=tdt)
        if op == "prod":
            x = 1 + 1e-4 * x
    else:
        x = torch.randint(-1000, 1000, shape, generator=g, device="cuda", dtype=tdt)
    code = {"sum": C.SUM, "mean": C.MEAN, "prod": C.PROD, "max": C.MAX, "min": C.MIN}[op]
    mask = _mask(x.dim(), dims)
    out_shape = tuple((1 if keepdim else None) if mask >> d & 1 else s for d, s in enumerate(shape))
    out_shape = tuple(s for s in out_shape if s is not None)
    out_dt = tdt if (op in ("max", "min", "mean") or tdt.is_floating_point) else torch.int64

    ref = torch.empty(out_shape, dtype=out_dt, device="cuda")
    vx, vr = C.view(x), C.view(ref)
    need = C.lib.ctb_reduce_scratch_bytes(code, vx, vr, mask)
    scratch = torch.empty(max(need, 1), dtype=torch.uint8, device="cuda")
    rc = C.lib.ctb_reduce(code, vx, vr, mask, ctypes.c_void_p(scratch.data_ptr()), need, C.stream_handle())
    assert rc == C.OK, C.last_error()
    if shape != (8192, 1024):
        assert need > 0, "case should exercise the scratch array"

    results = []
    for _ in range(2):  # two calls in a row: the second reuses what the first left in the array
        out = torch.full(out_shape, 7, dtype=out_dt, device="cuda")
        rc = C.lib.ctb_reduce_noalloc(code, vx, C.view(out), mask, C.stream_handle())
        assert rc == C.OK, C.last_error()
        results.append(out)
    torch.cuda.synchronize()

    r = ref.cpu().numpy()
    for k, out in enumerate(results):
        got = out.cpu().numpy()
        what = f"{op} {shape} call {k + 1}"
        if op in ("sum", "mean", "prod") and np.dtype(r.dtype).kind == "f":
            assert_close(got, r, TOL_SUM[np.dtype(r.dtype)], what)
        else:
            assert_bitexact(got, r, what)


def test_reduce_without_allocation_validates_like_ctb_reduce(cuda_ok):
    import torch

    from ctorch_b200 import _capi as C

    x = torch.ones(4, 5, dtype=torch.int32, device="cuda")
    bad = torch.empty(4, dtype=torch.int32, device="cuda")  # sum of int32 must be int64
    assert C.lib.ctb_reduce_noalloc(C.SUM, C.view(x), C.view(bad), 0b10, C.stream_handle()) == C.ERR_DTYPE
    assert C.lib.ctb_reduce_noalloc(C.MEAN, C.view(x), C.view(bad), 0b10, C.stream_handle()) == C.ERR_DTYPE
    out = torch.empty(4, dtype=torch.int64, device="cuda")
    assert C.lib.ctb_reduce_noalloc(C.SUM, C.view(x), C.view(out), 0b100, C.stream_handle()) == C.ERR_SHAPE


_FRESH = r"""
import ctypes, sys
sys.path.insert(0, {root!r})
import torch
from ctorch_b200 import _capi as C

def run(x, out, mask):
    rc = C.lib.ctb_reduce_noalloc(C.SUM, C.view(x), C.view(out), mask, C.stream_handle())
    assert rc == C.OK, C.last_error()

def ref(x, out, mask):
    need = C.lib.ctb_reduce_scratch_bytes(C.SUM, C.view(x), C.view(out), mask)
    s = torch.empty(max(need, 1), dtype=torch.uint8, device="cuda")
    rc = C.lib.ctb_reduce(C.SUM, C.view(x), C.view(out), mask, ctypes.c_void_p(s.data_ptr()), need,
                          C.stream_handle())
    assert rc == C.OK, C.last_error()
    return need

g = torch.Generator(device="cuda").manual_seed(99)
rows = torch.randn(8192, 1024, generator=g, device="cuda")   # row sums: one warp per row, no scratch
whole = torch.randn(4096, 8192, generator=g, device="cuda")  # whole sum: split, needs scratch
a, b = torch.empty(8192, device="cuda"), torch.empty(8192, device="cuda")
assert ref(rows, b, 0b10) == 0
run(rows, a, 0b10)                       # the first call of the process needs no scratch
c, d = torch.empty((), device="cuda"), torch.empty((), device="cuda")
assert ref(whole, d, 0b11) > 0
run(whole, c, 0b11)                      # the next one does: its address lookup comes now
torch.cuda.synchronize()
assert torch.equal(a, b), "row sums differ"
assert abs(c.item() - d.item()) <= 1e-5 * max(1.0, abs(d.item())), (c.item(), d.item())
print("fresh ok")
"""


def test_first_call_without_scratch_in_a_fresh_process(cuda_ok):
    """In a new process whose first no-alloc call needs no scratch (so it skips the array's
    address lookup), the next call that does need scratch still finds the array: both agree with
    ctb_reduce."""
    import os
    import subprocess
    import sys

    root = os.path.abspath(os.path.join(os.path.dirname(__file__), ".."))
    proc = subprocess.run([sys.executable, "-c", _FRESH.format(root=root)], capture_output=True, text=True,
                          timeout=300)
    assert proc.returncode == 0 and "fresh ok" in proc.stdout, proc.stdout + proc.stderr
