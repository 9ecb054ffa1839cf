"""Fixtures produced by the reference engine's own host code, run here.

oracle/ref/Makefile compiles the reference's weights.cpp and
quantized_weight.cpp (with a host-only stand-in for the CANN runtime) into
oracle/_ref/ref_driver.  This script feeds it seeded synthetic inputs and
commits what the reference code produced, so tests on machines without the
reference sources (the GPU box) can compare against the reference's actual
output:

  ref_w8a8_quant.wq.bin / .ws.bin
      quantize_dense_weight_w8a8 (src/csrc/lib/quantized_weight.cpp:231-268) of
      the fp16 weight [K=256, N=512] that ``w8a8_quant_input()`` regenerates.

    python tests/golden/make_ref_fixtures.py --write   # regenerate (needs the reference sources)
    python tests/golden/make_ref_fixtures.py           # check the committed files still match
"""
from __future__ import annotations

import os
import subprocess
import sys
import tempfile

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
REF_DIR = os.path.join(ROOT, "oracle", "ref")
DRIVER = os.path.join(ROOT, "oracle", "_ref", "ref_driver")
W8_K, W8_N = 256, 512


def w8a8_quant_input() -> np.ndarray:
    """fp16 [256, 512]: N(0, 0.05) with a few columns scaled up and one all-zero column."""
    r = np.random.Generator(np.random.PCG64(20261))
    w = r.standard_normal((W8_K, W8_N)) * 0.05
    w[:, 7] *= 40.0
    w[:, 100] = 0.0
    w[3, 200] = 65000.0
    return w.astype(np.float16)


def build_driver() -> str:
    subprocess.run(["make", "-s", "-C", REF_DIR], check=True)
    return DRIVER


def run_driver(*args: str) -> None:
    out = subprocess.run([DRIVER, *args], capture_output=True, text=True, timeout=300)
    if out.returncode != 0:
        raise RuntimeError(f"ref_driver {' '.join(args)}: {out.stderr.strip()}")


def w8a8_quant_from_reference():
    build_driver()
    w = w8a8_quant_input()
    with tempfile.TemporaryDirectory() as d:
        src = os.path.join(d, "w.f16")
        w.view(np.uint16).tofile(src)
        run_driver("quantize_w8a8", src, str(W8_K), str(W8_N), os.path.join(d, "q"))
        wq = np.fromfile(os.path.join(d, "q.wq"), np.int8).reshape(W8_K, W8_N)
        ws = np.fromfile(os.path.join(d, "q.ws"), np.uint16)
    return wq, ws


def load_w8a8_quant():
    wq = np.fromfile(os.path.join(HERE, "ref_w8a8_quant.wq.bin"), np.int8).reshape(W8_K, W8_N)
    ws = np.fromfile(os.path.join(HERE, "ref_w8a8_quant.ws.bin"), np.uint16)
    return wq, ws


def main(write: bool) -> int:
    wq, ws = w8a8_quant_from_reference()
    if write:
        wq.tofile(os.path.join(HERE, "ref_w8a8_quant.wq.bin"))
        ws.tofile(os.path.join(HERE, "ref_w8a8_quant.ws.bin"))
        print("wrote ref_w8a8_quant.{wq,ws}.bin")
        return 0
    cwq, cws = load_w8a8_quant()
    ok = np.array_equal(wq, cwq) and np.array_equal(ws, cws)
    print("fixtures match the reference" if ok else "fixtures differ from the reference")
    return 0 if ok else 1


if __name__ == "__main__":
    sys.exit(main("--write" in sys.argv))
