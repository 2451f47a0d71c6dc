"""Native host-logic tests of the interposer (CPU only).

Compiles tests/cpp/test_host.cpp with g++ against include/ and links it to
libgpu_scheduler.so; no GPU and no worker thread are involved (the test
completes captured ops itself, as the reference's test/test_main.cpp
236-276 does).
"""
import os
import subprocess

import pytest

from kernel_intercept_b200 import LIBSHIM, PKG_DIR

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
CUDA_INC = "/usr/local/cuda/include"


@pytest.fixture(scope="module")
def shim():
    if not os.path.exists(LIBSHIM):
        from kernel_intercept_b200 import build
        build.build_all()
    return LIBSHIM


def test_host_logic(shim, tmp_path):
    exe = tmp_path / "test_host"
    cmd = ["g++", "-std=c++17", "-O1", "-pthread", "-I", os.path.join(ROOT, "include"),
           "-I", CUDA_INC, os.path.join(ROOT, "tests", "cpp", "test_host.cpp"),
           "-L", PKG_DIR, "-lgpu_scheduler", f"-Wl,-rpath,{PKG_DIR}", "-o", str(exe)]
    subprocess.run(cmd, check=True, capture_output=True, text=True)
    env = dict(os.environ, ORION_WAIT_TIMEOUT_MS="200", ORION_LOG_LEVEL="ERROR")
    p = subprocess.run([str(exe), str(tmp_path)], capture_output=True, text=True, timeout=120,
                       env=env)
    assert p.returncode == 0 and "ALL PASSED" in p.stdout, p.stdout + p.stderr
