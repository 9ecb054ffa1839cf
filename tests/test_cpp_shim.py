"""The C++ shim (include/mcv_ops.hpp) compiles against the C ABI, binds to a
tensor type with the reference Tensor's accessors, and reports library
statuses as mcv_ops::Error - checked on the host, without a GPU."""
import os
import shutil
import subprocess

import pytest

from conftest import ROOT

PKG = os.path.join(ROOT, "minicpm-v-4.6-orangepi_b200")
CUDA = os.environ.get("CUDA_HOME", "/usr/local/cuda")


def test_shim_compiles_and_raises(tmp_path):
    if shutil.which("g++") is None or not os.path.exists(os.path.join(CUDA, "include", "cuda_runtime_api.h")):
        pytest.skip("g++ or the CUDA headers are missing")
    exe = str(tmp_path / "shim_check")
    cmd = ["g++", "-std=c++17", "-O1", "-Wall", "-Werror", "-I", os.path.join(ROOT, "include"),
           "-I", os.path.join(CUDA, "include"), os.path.join(ROOT, "tests", "shim_check.cpp"), "-o", exe,
           "-L", PKG, "-lmcv_b200", f"-Wl,-rpath,{PKG}", "-L", os.path.join(CUDA, "lib64"), "-lcudart",
           f"-Wl,-rpath,{os.path.join(CUDA, 'lib64')}"]
    subprocess.run(cmd, check=True, capture_output=True, text=True, timeout=300)
    out = subprocess.run([exe], capture_output=True, text=True, timeout=60)
    assert out.returncode == 0, out.stdout + out.stderr
    assert "shim ok" in out.stdout
