"""The C++ shim (include/mcv_ops.hpp) compiles against the C ABI, binds to a
tensor type with the reference Tensor's accessors, and reports library
statuses as mcv_ops::Error - checked on the host, without a GPU - and, on
a GPU, computes through the reference's op names (tests/shim_gpu.cpp)."""
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


@pytest.mark.gpu
def test_shim_success_path_on_gpu(cuda, tmp_path):
    """The C++ shim computing on the GPU through the reference's op names
    (tests/shim_gpu.cpp), each result checked against the CPU oracle."""
    import numpy as np

    import mcv_b200
    import oracle
    from conftest import assert_f16_close
    from mcv_b200 import synth
    if shutil.which("g++") is None:
        pytest.skip("g++ missing")
    d = str(tmp_path)
    x, q, z, s = synth.w4a16_inputs(1, 1024, 3584, seed=21)
    qw, sc, zw = mcv_b200._alloc_layout_host(1024, 3584, 128)
    st = mcv_b200.lib().mcv_w4a16_pack_host(mcv_b200._ptr(np.ascontiguousarray(q)), mcv_b200._ptr(np.ascontiguousarray(z)),
                                            mcv_b200._ptr(np.ascontiguousarray(s).view(np.uint16)), 1024, 3584, 128,
                                            mcv_b200._ptr(qw), mcv_b200._ptr(sc), mcv_b200._ptr(zw))
    assert st == 0
    r = np.random.default_rng(3)
    a = r.standard_normal((3, 1024)).astype(np.float16)
    b = (r.standard_normal((512, 1024)) * 0.05).astype(np.float16)
    h = (r.standard_normal((1, 1024)) * 3).astype(np.float16)
    g = (r.standard_normal(1024) * 0.1).astype(np.float16)
    _, e = synth.lm_head_inputs(1024, 20000, seed=9)
    gt = (r.standard_normal((1, 3584)) * 2).astype(np.float16)
    up = r.standard_normal((1, 3584)).astype(np.float16)
    x8, w8, ws8 = synth.w8a8_inputs(1, 1024, 1024, seed=4)
    for name, arr in (("w4.qw", qw), ("w4.sc", sc), ("w4.zw", zw), ("w4.x", x), ("mm.a", a), ("mm.b", b),
                      ("lm.h", h), ("lm.g", g), ("lm.e", e), ("silu.g", gt), ("silu.u", up), ("w8.x", x8),
                      ("w8.w", w8), ("w8.ws", ws8)):
        np.ascontiguousarray(arr).tofile(os.path.join(d, name))
    exe = str(tmp_path / "shim_gpu")
    cmd = ["g++", "-std=c++17", "-O1", "-Wall", "-Werror", "-I", os.path.join(ROOT, "include"),
           "-I", os.path.join(CUDA, "include"), os.path.join(ROOT, "tests", "shim_gpu.cpp"), "-o", exe,
           "-L", PKG, "-lmcv_b200", f"-Wl,-rpath,{PKG}", "-L", os.path.join(CUDA, "lib64"), "-lcudart",
           f"-Wl,-rpath,{os.path.join(CUDA, 'lib64')}"]
    subprocess.run(cmd, check=True, capture_output=True, text=True, timeout=300)
    out = subprocess.run([exe, d], capture_output=True, text=True, timeout=120)
    assert out.returncode == 0 and "shim gpu ok" in out.stdout, out.stdout + out.stderr
    rd = lambda n, dt: np.fromfile(os.path.join(d, n), dt)
    assert_f16_close(rd("w4.out", np.float16), oracle.w4a16_gemv(x, oracle.w4a16_fold_zeros(q, z), s).reshape(-1),
                     what="shim matmul_w4a16")
    assert_f16_close(rd("mm.out", np.float16).reshape(3, 512), oracle.gemv_f16(a, b, layout=0),
                     what="shim matmul_b_transposed")
    xn = oracle.rms_norm(h, g, eps=1e-6, variant=0)
    assert np.array_equal(rd("norm.out", np.uint16).reshape(1, 1024), xn)
    ref_idx, _, _ = oracle.lm_head_argmax(xn, e, nthreads=8)
    assert int(open(os.path.join(d, "lm.tok")).read()) == int(ref_idx[0])
    assert_f16_close(rd("silu.out", np.float16), oracle.f16_to_f32(oracle.silu_mul(gt, up)).reshape(-1),
                     what="shim silu_mul")
    acc, o8 = oracle.w8a8_fused(x8, w8, ws8)
    assert np.array_equal(rd("w8.acc", np.int32), np.asarray(acc).reshape(-1))
    assert np.array_equal(rd("w8.out", np.uint16), np.asarray(o8).reshape(-1))
