"""The batched-decode KV page pool (inference_b200/csrc/page_pool.hpp, host
C++): reference counts, all-or-nothing allocation, prefix sharing by fork,
release -- compiled with g++ and run on the CPU (tests/page_pool_check.cpp)."""
import os
import shutil
import subprocess

import pytest

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(os.path.dirname(HERE), "inference_b200", "csrc")


def test_page_pool(tmp_path):
    gxx = shutil.which("g++")
    if gxx is None:
        pytest.skip("g++ not available")
    exe = tmp_path / "page_pool_check"
    subprocess.run([gxx, "-std=c++17", "-O1", "-Wall", "-Werror", "-I", CSRC,
                    os.path.join(HERE, "page_pool_check.cpp"), "-o", str(exe)], check=True)
    r = subprocess.run([str(exe)], capture_output=True, text=True, timeout=120)
    assert r.returncode == 0, r.stdout + r.stderr
    assert r.stdout.strip().startswith("ok")
