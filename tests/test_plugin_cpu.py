"""The ctorch plugin (ctorch_b200/ctorch_plugin): ctorch built from its own sources with the B200
backend in place of src/ops/*_cuda.cu. On CPU: the four registration hooks are exported and every
CUDA dispatch slot is filled."""
import os
import subprocess

import pytest

ROOT = os.path.abspath(os.path.join(os.path.dirname(__file__), ".."))
BUILD = os.path.join(ROOT, "ctorch_b200", "ctorch_plugin", "_build")
LIB = os.path.join(BUILD, "libctorch_b200.so")
CHECK = os.path.join(BUILD, "plugin_check")

needs_build = pytest.mark.skipif(not os.path.exists(CHECK),
                                 reason="ctorch plugin not built (needs the ctorch sources at build time)")


@needs_build
def test_registration_hooks_exported():
    out = subprocess.run(["nm", "-D", "--defined-only", LIB], capture_output=True, text=True).stdout
    for hook in ("ctorch_register_cuda_binary_ops", "ctorch_register_cuda_unary_ops",
                 "ctorch_register_cuda_reduction_ops", "ctorch_register_cuda_indexing_ops"):
        assert hook in out, hook


@needs_build
def test_every_cuda_slot_is_filled():
    r = subprocess.run([CHECK, "--registry"], capture_output=True, text=True, timeout=60)
    assert r.returncode == 0, r.stdout + r.stderr
    assert "26 of 26" in r.stdout
