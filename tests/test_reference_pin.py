"""The oracle pinned to the reference engine's own code, run on this CPU.

oracle/ref/Makefile builds, from the reference sources where they lie, the
reference's CPU-checked test programs and its host library code (tensor,
safetensors reader, W4A16 loader, W8A8 quantizer) against a host-only
stand-in for the CANN runtime, with the CPU oracle standing in for the device
ops (oracle/ref/ops_stub.cpp).  So:
  * each reference test draws its own seeded inputs and applies its own
    checker to the oracle's answers - a pass means the reference accepts the
    oracle on the reference's inputs;
  * the reference's loader and quantizer produce their actual outputs, which
    must equal this repository's loader / packers / oracle bit for bit.
Skipped where neither the reference sources nor a built oracle/_ref exist
(the GPU box); the committed fixtures of tests/golden/make_ref_fixtures.py
carry the quantizer's output there."""
import os
import subprocess

import numpy as np
import pytest

import make_golden as golden
import make_ref_fixtures as reffix
import mcv_b200 as mcv
import oracle
from conftest import ROOT, write_safetensors
from mcv_b200 import synth

REF_SRC = "/root/reference"
OUT = os.path.join(ROOT, "oracle", "_ref")


@pytest.fixture(scope="module")
def ref_bin():
    if os.path.isdir(os.path.join(REF_SRC, "src", "csrc")):
        subprocess.run(["make", "-s", "-C", os.path.join(ROOT, "oracle", "ref"), f"REF={REF_SRC}"], check=True,
                       capture_output=True, text=True, timeout=600)
    if not os.path.exists(os.path.join(OUT, "ref_driver")):
        pytest.skip("reference sources absent and oracle/_ref not built")
    return OUT


def run(ref_bin, name, *args):
    return subprocess.run([os.path.join(ref_bin, name), *args], capture_output=True, text=True, timeout=300)


@pytest.mark.parametrize("test,expect", [
    ("test_matmul_w4a16", "large(>0.1)=0/3584"),          # tests/test_matmul_w4a16.cpp:217-240
    ("test_matmul_w8a8_i32", "W8A8 i32 exact match"),     # tests/test_matmul_w8a8_i32.cpp:39-51
    ("test_w8a8_dequant", "W8A8 dequant max_abs_diff"),   # tests/test_w8a8_dequant.cpp:55-60
    ("test_lm_head_pipeline", "lm_head pipeline ok"),     # tests/test_lm_head_pipeline.cpp:95-120
    ("test_natural_b_matmul", "large_diffs(>0.05)=0/"),
    ("test_rms_norm1024", "rms_norm1024 ok"),             # tests/test_rms_norm1024.cpp:97-119
    ("test_matmul", "errors=0"),
])
def test_reference_tests_accept_the_oracle(ref_bin, test, expect):
    out = run(ref_bin, test)
    assert out.returncode == 0, out.stdout + out.stderr
    assert expect in out.stdout, out.stdout


def test_lm_head_pipeline_tokens_equal_golden(ref_bin):
    """The reference test passes only if the tokens it prints equal its own
    checker's; they must also equal the committed golden fixture."""
    out = run(ref_bin, "test_lm_head_pipeline")
    toks = [int(t) for t in out.stdout.split("tokens=")[1].strip().strip(",").split(",")]
    assert toks == golden.load("lm_head.ref").tolist()


def test_reference_rms_norm_test_disagrees_with_its_implementation(ref_bin):
    """tests/test_rms_norm.cpp checks x/rms*gamma, but the engine's rms_norm
    multiplies by (1 + gamma) (src/csrc/lib/ops.cpp:693-736), and lm_head_greedy
    uses that implementation (language_model.cpp:423).  The oracle follows
    the implementation, so the stale test reports every element off by the
    factor (1 + gamma) / gamma - about 2 for its gamma near 1."""
    out = run(ref_bin, "test_rms_norm")
    assert "errors=0" not in out.stdout.split("H=1024")[-1]
    line = [l for l in (out.stdout + out.stderr).splitlines() if l.startswith("row=0 col=0")][0]
    got = float(line.split("got=")[1].split()[0])
    ref = float(line.split("ref=")[1].split()[0])
    assert abs(got / ref - 2.0) < 0.05


def test_reference_w8a8_quantizer_equals_oracle_and_fixture(ref_bin):
    wq, ws = reffix.w8a8_quant_from_reference()
    owq, ows = oracle.quantize_dense_weight_w8a8(reffix.w8a8_quant_input())
    assert np.array_equal(wq, owq) and np.array_equal(ws, np.asarray(ows).reshape(-1))
    cwq, cws = reffix.load_w8a8_quant()
    assert np.array_equal(wq, cwq) and np.array_equal(ws, cws)


@pytest.mark.parametrize("fmt,K,N", [("gptq", 1024, 3584), ("gptq", 256, 128), ("awq", 1024, 1024),
                                     ("awq", 384, 256)])
def test_reference_loader_equals_ours(ref_bin, tmp_path, fmt, K, N):
    """load_w4a16_quantized_weight (the reference's code) and this library's
    loader read the same synthetic checkpoint to the same (q - zero) and
    scales; the reference's tile layout also unpacks to the oracle's."""
    _, q, z, s = synth.w4a16_inputs(1, K, N, seed=K * 7 + N)
    base = "model.language_model.layers.3.mlp.up_proj"
    if fmt == "gptq":
        z = np.maximum(z, 1)
        qw, qz = synth.gptq_pack(q, z)
        tensors = {base + ".qweight": ("I32", qw), base + ".qzeros": ("I32", qz), base + ".scales": ("F16", s),
                   base + ".g_idx": ("I32", (np.arange(K) // 128).astype(np.int32))}
    else:
        qw, qz = synth.awq_pack(q, z)
        tensors = {base + ".qweight": ("I32", qw), base + ".qzeros": ("I32", qz), base + ".scales": ("F16", s)}
    path = str(tmp_path / "ckpt.safetensors")
    write_safetensors(path, tensors, metadata={"format": "pt"})
    prefix = str(tmp_path / "ref")
    out = run(ref_bin, "ref_driver", "load_w4a16", path, base, prefix)
    assert out.returncode == 0, out.stderr
    k2, n2, tile, rows = (int(v) for v in open(prefix + ".meta").read().split())
    assert (k2, n2) == (K, N) and tile == oracle.w4a16_choose_tile_len(N)
    tiles = np.fromfile(prefix + ".tiles", np.int8).reshape(rows, tile)
    ref_scales = np.fromfile(prefix + ".scales", np.uint16).reshape(K // 128, N)
    ref_w = np.empty((K, N), np.int8)
    lib = oracle.lib()
    import ctypes
    lib.orc_w4a16_unpack_tiles(tiles.ctypes.data_as(ctypes.c_void_p), ctypes.c_int64(K), ctypes.c_int64(N),
                               ctypes.c_int64(tile), ref_w.ctypes.data_as(ctypes.c_void_p))
    assert np.array_equal(ref_w, oracle.w4a16_fold_zeros(q, z))        # the reference means (q - zero)
    with mcv.SafeTensors(path) as st:
        ours = mcv.load_w4a16_quantized_weight_host(st, base)
    w_ours, s_ours = mcv.unpack_w4a16_host(ours[0], ours[1], ours[2], ours[3], K, N)
    assert np.array_equal(w_ours, ref_w)
    assert np.array_equal(s_ours, ref_scales)


def test_reference_safetensors_reader_agrees(ref_bin, tmp_path):
    r = np.random.default_rng(4)
    f32 = r.standard_normal((40, 24)).astype(np.float32)
    bf = (f32.view(np.uint32) >> 16).astype(np.uint16)
    tensors = {"b.emb": ("BF16", bf), "a.w": ("F16", r.standard_normal((3, 5)).astype(np.float16)),
               "c.ids": ("I64", np.arange(6, dtype=np.int64))}
    path = str(tmp_path / "m.safetensors")
    write_safetensors(path, tensors, metadata={"k": "v"})
    names = run(ref_bin, "ref_driver", "names", path).stdout.split()
    with mcv.SafeTensors(path) as st:
        assert names == st.names()
    out = str(tmp_path / "emb.f16")
    assert run(ref_bin, "ref_driver", "load_f16", path, "b.emb", out).returncode == 0
    from test_safetensors_loader import bf16_to_f16_trunc
    assert np.array_equal(np.fromfile(out, np.uint16).reshape(40, 24), bf16_to_f16_trunc(bf))
