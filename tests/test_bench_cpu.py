"""CPU checks of bench.py's host-side pieces: the reference arm's process maps ctorch's code and
nothing of this backend, the multi-threaded ctorch CPU step agrees with the one-thread step, and
the roofline traffic model built from the committed ncu capture."""
import os
import subprocess
import sys

import pytest

ROOT = os.path.abspath(os.path.join(os.path.dirname(__file__), ".."))

_PROBE = r"""
import os, sys
sys.path.insert(0, {root!r})
import bench
x, r = bench.host_inputs(64)
assert x.shape == (64, 8192) and r.shape == (1, 8192)
maps = open("/proc/self/maps").read()
print("PKG", "ctorch_b200" in sys.modules)
print("LIB", "libctb_cuda.so" in maps)
"""


def test_reference_arm_host_inputs_do_not_load_the_backend():
    """bench.host_inputs (the reference arm's input generator) loads the numpy generator by path:
    neither the package nor its CUDA kernel library enters the process."""
    out = subprocess.run([sys.executable, "-c", _PROBE.format(root=ROOT)], capture_output=True, text=True,
                         timeout=300)
    assert out.returncode == 0, out.stderr
    assert "PKG False" in out.stdout and "LIB False" in out.stdout, out.stdout


def test_host_inputs_match_the_package_generator():
    import numpy as np

    sys.path.insert(0, ROOT)
    import bench
    from ctorch_b200.synth import NORMAL, UNIFORM, host_fill

    x, r = bench.host_inputs(16)
    assert np.array_equal(x, host_fill((16, 8192), "float32", NORMAL, bench.SEED, 0, 0.0, 1.0))
    assert np.array_equal(r, host_fill((1, 8192), "float32", UNIFORM, bench.SEED, 1, -1.0, 1.0))


def test_threaded_ctorch_cpu_step_runs_on_row_blocks():
    """The reference arm's step split over threads: ctorch's own front-doors on each block."""
    sys.path.insert(0, ROOT)
    from oracle.oracle import ref_available

    if not ref_available():
        pytest.skip("ctorch's CPU backend (oracle/_ref) not built")
    import bench

    v1, t1 = bench.time_ctorch_cpu(64, 1, 0, 1)
    v4, t4 = bench.time_ctorch_cpu(64, 1, 0, 4)
    assert v1 > 0 and v4 > 0 and t1 > 0 and t4 > 0


def test_traffic_model_from_the_committed_capture():
    """Reads scale per row, writes are the algorithmic bytes per row less a constant L2 tail: at the
    captured size the model returns the captured bytes."""
    import json

    sys.path.insert(0, ROOT)
    import bench

    d = json.load(open(os.path.join(ROOT, "profiles", "ncu_traffic.json")))
    captured = d["dram_read"] + d["dram_write"]
    assert abs(bench.ncu_traffic(d["rows"]) - captured) < 1.0
    full = bench.ncu_traffic(262144)
    algorithmic = 262144 * 8192 * 8 + 8192 * 4 + 262144 * 8
    assert 0.99 * algorithmic < full < algorithmic
