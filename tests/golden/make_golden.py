"""Builds and runs gen_golden.cpp; writes or checks the committed fixtures.

The reference tests' inputs are large (a 3.6 MB int8 weight) but reproducible,
so the repository commits only the checker OUTPUTS (``*.ref.bin``, small) and
the SHA-256 of every generated array (``manifest.json``).  Tests call
:func:`load` which rebuilds the inputs with g++ (libstdc++'s std::mt19937 and
<random> distributions, exactly as the reference tests draw them), verifies
their hashes, and returns numpy arrays.

    python tests/golden/make_golden.py --write   # regenerate the fixtures
"""
from __future__ import annotations

import hashlib
import json
import os
import subprocess
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
BUILD = os.path.join(HERE, "_build")
GEN_SRC = os.path.join(HERE, "gen_golden.cpp")
GEN_BIN = os.path.join(BUILD, "gen_golden")
OUT = os.path.join(BUILD, "out")
MANIFEST = os.path.join(HERE, "manifest.json")

# dtype and shape of every array gen_golden writes
SPECS = {
    "w4a16.x": (np.uint16, (1, 1024)),
    "w4a16.w": (np.int8, (1024, 3584)),
    "w4a16.s": (np.uint16, (8, 3584)),
    "w4a16.ref": (np.float32, (1, 3584)),
    "w4a16_const.x": (np.uint16, (1, 1024)),
    "w4a16_const.w": (np.int8, (1024, 3584)),
    "w4a16_const.s": (np.uint16, (8, 3584)),
    "w4a16_const.ref": (np.float32, (1, 3584)),
    "w8a8_i32.x": (np.int8, (1, 1024)),
    "w8a8_i32.w": (np.int8, (1024, 3584)),
    "w8a8_i32.ref": (np.int32, (1, 3584)),
    "w8a8_dequant.acc": (np.int32, (1, 3584)),
    "w8a8_dequant.ws": (np.uint16, (3584,)),
    "w8a8_dequant.xs": (np.uint16, (1,)),
    "w8a8_dequant.ref": (np.float32, (1, 3584)),
    "lm_head.x": (np.uint16, (4, 64)),
    "lm_head.w": (np.uint16, (64, 128)),
    "lm_head.ref": (np.int64, (4,)),
    "cube.x": (np.uint16, (1, 1024)),
    "cube.w_nk": (np.uint16, (3584, 1024)),
    "cube.ref": (np.float32, (1, 3584)),
    "matmul_4x128x64.x": (np.uint16, (4, 128)),
    "matmul_4x128x64.w_kn": (np.uint16, (128, 64)),
    "matmul_4x128x64.ref": (np.float32, (4, 64)),
    "matmul_1x1024x4096.x": (np.uint16, (1, 1024)),
    "matmul_1x1024x4096.w_kn": (np.uint16, (1024, 4096)),
    "matmul_1x1024x4096.ref": (np.float32, (1, 4096)),
}

_generated = False


def _build_generator() -> None:
    os.makedirs(BUILD, exist_ok=True)
    if (not os.path.exists(GEN_BIN)) or os.path.getmtime(GEN_BIN) < os.path.getmtime(GEN_SRC):
        subprocess.run(["g++", "-O2", "-std=c++17", "-ffp-contract=off", GEN_SRC, "-o", GEN_BIN],
                       check=True)


def generate() -> str:
    """Compile and run the generator once per process; returns the output dir."""
    global _generated
    if not _generated:
        _build_generator()
        os.makedirs(OUT, exist_ok=True)
        subprocess.run([GEN_BIN, OUT], check=True)
        _generated = True
    return OUT


def _sha(path: str) -> str:
    with open(path, "rb") as f:
        return hashlib.sha256(f.read()).hexdigest()


def load(name: str, check_hash: bool = True) -> np.ndarray:
    """One generated array, hash-checked against the committed manifest.

    ``*.ref`` arrays are read from the committed fixture in tests/golden, so a
    changed generator can never silently move the expected values."""
    dtype, shape = SPECS[name]
    if name.endswith(".ref"):
        path = os.path.join(HERE, name + ".bin")
    else:
        path = os.path.join(generate(), name + ".bin")
    if check_hash:
        with open(MANIFEST) as f:
            man = json.load(f)
        got = _sha(path)
        if man[name] != got:
            raise AssertionError(f"golden array {name} hash {got} != manifest {man[name]}")
    return np.fromfile(path, dtype=dtype).reshape(shape)


def write() -> None:
    out = generate()
    man = {}
    for name in SPECS:
        src = os.path.join(out, name + ".bin")
        man[name] = _sha(src)
        if name.endswith(".ref"):
            with open(src, "rb") as f, open(os.path.join(HERE, name + ".bin"), "wb") as g:
                g.write(f.read())
    with open(MANIFEST, "w") as f:
        json.dump(man, f, indent=1, sort_keys=True)
        f.write("\n")


if __name__ == "__main__":
    if "--write" in sys.argv:
        write()
        print("fixtures written to", HERE)
    else:
        for n in SPECS:
            load(n)
        print("all golden arrays match the manifest")
