"""The indexer's key and linear-window bin functions (sgsa_b200/csrc/select_keys.cuh),
compiled for the host and checked for the invariants the exact selection relies on."""
import os
import shutil
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_linear_bin_invariants(tmp_path):
    cxx = shutil.which("g++") or shutil.which("c++")
    if cxx is None:
        pytest.skip("no host C++ compiler")
    exe = str(tmp_path / "select_keys_check")
    subprocess.run([cxx, "-std=c++17", "-O2", "-I", os.path.join(ROOT, "sgsa_b200", "csrc"),
                    os.path.join(ROOT, "tests", "select_keys_check.cpp"), "-o", exe], check=True)
    r = subprocess.run([exe], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stdout + r.stderr
    assert r.stdout.startswith("ok")
