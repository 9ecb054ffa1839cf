"""pytest setup: the `gpu` marker, import paths, and shared helpers.

`-m "not gpu"` runs the oracle-vs-golden pins, the host-side repack and ABI
checks, and the multi-rank (gloo) host logic on CPU; `-m gpu` runs the CUDA
parity tests through the C ABI on a B200.
"""
import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(ROOT, "minicpm-v-4.6-orangepi_b200")
for p in (ROOT, PKG, os.path.join(ROOT, "oracle"), os.path.join(ROOT, "tests", "golden")):
    if p not in sys.path:
        sys.path.insert(0, p)

# fp16 output tolerance of the hot path: |got - ref| <= ATOL + RTOL * |ref|
ATOL = 1e-2
RTOL = 1e-3


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


def assert_f16_close(got_f16, ref_f32, atol=ATOL, rtol=RTOL, what=""):
    got = np.asarray(got_f16, dtype=np.float32)
    ref = np.asarray(ref_f32, dtype=np.float32)
    assert got.shape == ref.shape, (got.shape, ref.shape)
    err = np.abs(got - ref)
    bound = atol + rtol * np.abs(ref)
    bad = np.argwhere(err > bound)
    assert bad.size == 0, (f"{what}: {len(bad)} of {err.size} outside |d| <= {atol} + {rtol}|ref|; "
                           f"first {bad[:3].tolist()} max_abs={err.max():.3g}")
    return float(err.max())


@pytest.fixture(scope="session")
def cuda():
    torch = pytest.importorskip("torch")
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import mcv_b200
    mcv_b200.lib()
    return torch


def write_safetensors(path, tensors, metadata=None, header_pad=0):
    """Writes a .safetensors file: 8-byte little-endian header length, the
    JSON header {name: {dtype, shape, data_offsets}} (+ __metadata__), then the
    tensors' bytes in order.  tensors: {name: (dtype string, numpy array)}."""
    import json
    import struct
    header, blobs, off = {}, [], 0
    if metadata is not None:
        header["__metadata__"] = metadata
    for name, (dt, arr) in tensors.items():
        b = np.ascontiguousarray(arr).tobytes()
        header[name] = {"dtype": dt, "shape": list(arr.shape), "data_offsets": [off, off + len(b)]}
        blobs.append(b)
        off += len(b)
    h = json.dumps(header).encode() + b" " * header_pad
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(h)))
        f.write(h)
        for b in blobs:
            f.write(b)
