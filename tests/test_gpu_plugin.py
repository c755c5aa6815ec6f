"""ctorch's public API on CUDA tensors with the B200 backend linked into ctorch (the drop-in
path), compared with ctorch's own CPU path on the same inputs by plugin_check.cpp."""
import os
import subprocess

import pytest

pytestmark = pytest.mark.gpu

ROOT = os.path.abspath(os.path.join(os.path.dirname(__file__), ".."))
CHECK = os.path.join(ROOT, "ctorch_b200", "ctorch_plugin", "_build", "plugin_check")


@pytest.mark.skipif(not os.path.exists(CHECK), reason="ctorch plugin not built")
def test_ctorch_api_on_b200_backend(cuda_ok):
    r = subprocess.run([CHECK], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stdout + r.stderr
    assert ", 0 failed" in r.stdout
