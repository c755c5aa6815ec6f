"""ctorch's public API on CUDA tensors with the B200 backend linked into ctorch (the drop-in
path), compared with ctorch's own CPU path on the same inputs by plugin_check.cpp.

The plugin is built only where ctorch's sources are present (its Makefile compiles ctorch's core
in place). Where its build folder exists, plugin_check must exist too and pass: the test fails
rather than skips. Its pass count is reported as a warning, so that it shows in the run's summary.
"""
import os
import re
import subprocess
import warnings

import pytest

pytestmark = pytest.mark.gpu

ROOT = os.path.abspath(os.path.join(os.path.dirname(__file__), ".."))
BUILD = os.path.join(ROOT, "ctorch_b200", "ctorch_plugin", "_build")
CHECK = os.path.join(BUILD, "plugin_check")


@pytest.mark.skipif(not os.path.isdir(BUILD), reason="ctorch plugin not built (no ctorch sources at build time)")
def test_ctorch_api_on_b200_backend(cuda_ok):
    assert os.path.exists(CHECK), f"{BUILD} exists but holds no plugin_check"
    r = subprocess.run([CHECK], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stdout + r.stderr
    m = re.search(r"plugin_check: (\d+) passed, (\d+) failed", r.stdout)
    assert m and int(m.group(2)) == 0 and int(m.group(1)) >= 50, r.stdout
    reg = subprocess.run([CHECK, "--registry"], capture_output=True, text=True, timeout=60)
    assert reg.returncode == 0 and "26 of 26" in reg.stdout, reg.stdout
    warnings.warn(f"ctorch API through the B200 backend: {m.group(0)}; {reg.stdout.strip()}", UserWarning)
