"""CPU-side checks of libmcv_b200.so: it loads, exports every entry point the
header declares, validates arguments without touching a device, and its
load-time repackers produce the mcv-int4 layout the kernels expect."""
import ctypes
import os
import re

import numpy as np
import pytest

import mcv_b200
import oracle
from conftest import ROOT
from mcv_b200 import synth

SLOT = (0, 4, 1, 5, 2, 6, 3, 7)


def header_symbols():
    with open(os.path.join(ROOT, "include", "mcv_matmul.h")) as f:
        text = f.read()
    return sorted(set(re.findall(r"^\s*(?:const\s+)?[a-z_0-9]+\*?\s+\*?(mcv_[a-z0-9_]+)\(", text, re.M)))


FRAG_SLOT = (0, 4, 1, 5, 2, 6, 3, 7)
FRAG_ROW = (0, 0, 8, 8, 0, 0, 8, 8)
FRAG_K = (0, 1, 0, 1, 2, 3, 2, 3)


def decode_layout(w):
    """mcv-int4 device arrays (numpy) -> (q-zero) int16 [K,N], scales [G,N];
    an independent decoder of the layout documented in include/mcv_matmul.h."""
    qw = w.qweight.cpu().numpy().view(np.uint32)
    sc = w.scales.cpu().numpy().view(np.uint16)
    zw = w.zeros.cpu().numpy().view(np.uint32)
    K, N = w.K, w.N
    Np = (N + 15) // 16 * 16
    G = K // w.group_size
    words = qw.reshape(Np // 16, K // 64, 32, 4)          # [strip, quad, lane, j]
    q = np.zeros((K, Np), np.int16)
    for lane in range(32):
        g, t = lane // 4, lane % 4
        for j in range(4):
            for e in range(8):
                vals = ((words[:, :, lane, j] >> np.uint32(4 * FRAG_SLOT[e])) & np.uint32(0xF)).astype(np.int16)
                n = np.arange(Np // 16) * 16 + g + FRAG_ROW[e]          # [strip]
                k = np.arange(K // 64) * 64 + 16 * t + 4 * j + FRAG_K[e]  # [quad]
                q[np.ix_(k, n)] = vals.T
    z = np.zeros((G, Np), np.int16)
    for gg in range(G):
        z[gg] = ((zw[:, gg // 8] >> np.uint32(4 * (gg % 8))) & np.uint32(0xF)).astype(np.int16) + w.zero_bias
    assert np.all(q[:, N:] == 0) and np.all(sc[N:] == 0) and np.all(sc[:, G:] == 0)
    return (q - np.repeat(z, w.group_size, axis=0))[:, :N], sc[:N, :G].T


def test_library_exports_every_header_symbol():
    L = mcv_b200.lib()
    syms = header_symbols()
    assert len(syms) >= 20
    for s in syms:
        assert hasattr(L, s), s
    assert set(syms) == set(mcv_b200.EXPORTED)
    assert L.mcv_version() >> 16 == 1


def test_status_strings_and_errors_without_device():
    L = mcv_b200.lib()
    assert L.mcv_status_string(0) == b"ok"
    # validation happens before any CUDA call
    st = L.mcv_w4a16_gemv(None, None, None, None, 0, None, 1, 1024, 3584, 128, None)
    assert st == 1 and b"null" in L.mcv_last_error()
    fake = ctypes.c_void_p(16)
    st = L.mcv_w4a16_gemv(fake, fake, fake, fake, 0, fake, 65, 1024, 3584, 128, None)
    assert st == 2
    st = L.mcv_w4a16_gemv(fake, fake, fake, fake, 0, fake, 1, 1000, 3584, 128, None)
    assert st == 2
    st = L.mcv_w4a16_gemv(ctypes.c_void_p(18), fake, fake, fake, 0, fake, 1, 1024, 3584, 128, None)
    assert st == 3
    st = L.mcv_gemv_f16(fake, fake, fake, 1, 1024, 4096, 7, None)
    assert st == 7
    st = L.mcv_lm_head_argmax(fake, fake, None, fake, 1, 1024, 1000, 0, 0, None, 0, None)
    assert st == 6
    st = L.mcv_w8a8_gemm_i32(fake, fake, fake, 1, 1000, 3584, 0, None)
    assert st == 2
    st = L.mcv_w4a16_gemv(fake, fake, fake, fake, 0, fake, 1, 1024, 3584, 64, None)
    assert st == 2 and b"128" in L.mcv_last_error()
    assert L.mcv_lm_head_workspace_size(1) == L.mcv_lm_head_workspace_size(8) == 256


def test_layout_bytes():
    qb, sb, zb = ctypes.c_size_t(), ctypes.c_size_t(), ctypes.c_size_t()
    assert mcv_b200.lib().mcv_w4a16_layout_bytes(1024, 3584, 128, ctypes.byref(qb), ctypes.byref(sb),
                                                  ctypes.byref(zb)) == 0
    assert qb.value == 1024 * 3584 // 2 and sb.value == 8 * 3584 * 2 and zb.value == 3584 * 4


class _FakeT:
    """numpy stand-in with the .cpu().numpy() surface used by decode_layout."""

    def __init__(self, a):
        self.a = a

    def cpu(self):
        return self

    def numpy(self):
        return self.a


@pytest.fixture
def host_pack(monkeypatch):
    monkeypatch.setattr(mcv_b200, "_to_device",
                        lambda qw, sc, zw, zb, K, N, g, dev: mcv_b200.W4A16QuantizedWeight(
                            _FakeT(qw), _FakeT(sc), _FakeT(zw), int(zb), K, N, g))


@pytest.mark.parametrize("K,N", [(1024, 3584), (3584, 1024), (256, 16), (384, 40)])
def test_pack_logical(host_pack, K, N):
    x, q, z, s = synth.w4a16_inputs(1, K, N, seed=K + N)
    w = mcv_b200.pack_w4a16(q, z, s)
    got, sc = decode_layout(w)
    expect = oracle.w4a16_fold_zeros(q, z).astype(np.int16)
    assert np.array_equal(got, expect)
    assert np.array_equal(sc, s.view(np.uint16))


def test_pack_gptq(host_pack):
    K, N = 512, 256
    r = synth.rng(11)
    q = r.integers(0, 16, (K, N), dtype=np.uint8)
    z = r.integers(1, 17, (K // 128, N), dtype=np.uint8)
    s = r.uniform(0.002, 0.02, (K // 128, N)).astype(np.float16)
    qw, qz = synth.gptq_pack(q, z)
    gidx = (np.arange(K) // 128).astype(np.int32)
    w = mcv_b200.pack_w4a16_gptq(qw, qz, gidx, s)
    assert w.zero_bias == 1
    got, _ = decode_layout(w)
    assert np.array_equal(got, oracle.unpack_gptq(qw, qz, gidx, K // 128).astype(np.int16))
    bad = gidx.copy()
    bad[0] = 1
    with pytest.raises(RuntimeError, match="g_idx"):
        mcv_b200.pack_w4a16_gptq(qw, qz, bad, s)


def test_pack_awq(host_pack):
    K, N = 512, 256
    r = synth.rng(12)
    q = r.integers(0, 16, (K, N), dtype=np.uint8)
    z = r.integers(0, 16, (K // 128, N), dtype=np.uint8)
    s = r.uniform(0.002, 0.02, (K // 128, N)).astype(np.float16)
    qw, qz = synth.awq_pack(q, z)
    w = mcv_b200.pack_w4a16_awq(qw, qz, s)
    assert w.zero_bias == 0
    got, _ = decode_layout(w)
    assert np.array_equal(got, oracle.unpack_awq(qw, qz).astype(np.int16))


@pytest.mark.parametrize("lo,hi", [(-8, 7), (-16, -2), (0, 15)])
def test_pack_from_reference_tiles(host_pack, lo, hi):
    K, N = 256, 3584
    r = np.random.default_rng(lo + 100)
    w = r.integers(lo, hi + 1, (K, N), dtype=np.int8)
    s = r.uniform(0.002, 0.02, (K // 128, N)).astype(np.float16)
    packed = oracle.w4a16_pack_tiles(w)
    got, sc = decode_layout(mcv_b200.pack_w4a16_from_tiles(packed, s, K, N))
    assert np.array_equal(got, w.astype(np.int16))
    assert np.array_equal(sc, s.view(np.uint16))


def test_pack_from_tiles_rejects_wide_groups(host_pack):
    K, N = 128, 128
    w = np.zeros((K, N), np.int8)
    w[0, 0], w[1, 0] = -9, 8  # 18 levels in one group
    packed = oracle.w4a16_pack_tiles(w)
    with pytest.raises(RuntimeError, match="16 levels"):
        mcv_b200.pack_w4a16_from_tiles(packed, np.ones((1, N), np.float16), K, N)


def test_tuning_keys_round_trip_and_reject_unknown():
    """Every tuning key the header names is accepted, read back and reset to
    its default (0); keys outside the table are refused with a status."""
    lib = mcv_b200.lib()
    header = open(os.path.join(ROOT, "include", "mcv_matmul.h")).read()
    keys = {name: int(v) for name, v in re.findall(r"(MCV_TUNE_[A-Z0-9_]+) = (\d+)", header)}
    count = keys.pop("MCV_TUNE_COUNT")
    assert {"MCV_TUNE_W4A16_MODE", "MCV_TUNE_ROWS_BLOCKS_PER_SM", "MCV_TUNE_ROWS_PREFETCH",
            "MCV_TUNE_GEMM_SPLIT_K"} <= set(keys)
    for name, key in keys.items():
        assert getattr(mcv_b200, name[len("MCV_"):]) == key
        assert lib.mcv_set_tuning(key, 3) == 0
        assert lib.mcv_get_tuning(key) == 3
        assert lib.mcv_set_tuning(key, 0) == 0
        assert lib.mcv_get_tuning(key) == 0
    assert lib.mcv_set_tuning(count, 1) != 0
    assert lib.mcv_set_tuning(0, 1) != 0


try:
    from hypothesis import HealthCheck, given, settings
    from hypothesis import strategies as st
except ImportError:  # pragma: no cover
    given = None


if given is not None:
    @settings(max_examples=25, deadline=None, suppress_health_check=[HealthCheck.function_scoped_fixture])
    @given(kg=st.integers(1, 8), n8=st.integers(1, 40), seed=st.integers(0, 2**31 - 1))
    def test_packers_round_trip_any_shape(host_pack, kg, n8, seed):
        """Random shapes (K = 128 kg, N = 8 n8: ragged strips included): the
        logical, GPTQ and AWQ packers all decode to the oracle's (q - zero)
        and keep the scales exactly."""
        K, N = 128 * kg, 8 * n8
        r = np.random.default_rng(seed)
        q = r.integers(0, 16, (K, N), dtype=np.uint8)
        z = r.integers(0, 16, (kg, N), dtype=np.uint8)
        s = r.uniform(0.002, 0.02, (kg, N)).astype(np.float16)
        w = mcv_b200.pack_w4a16(q, z, s)
        got, sc = decode_layout(w)
        assert np.array_equal(got, oracle.w4a16_fold_zeros(q, z).astype(np.int16))
        assert np.array_equal(sc, s.view(np.uint16))
        qa, za = synth.awq_pack(q, z)
        got_a, _ = decode_layout(mcv_b200.pack_w4a16_awq(qa, za, s))
        assert np.array_equal(got_a, oracle.unpack_awq(qa, za).astype(np.int16))
        zg = (z + 1).astype(np.uint8)  # GPTQ stores zero - 1
        qg, zgp = synth.gptq_pack(q, np.minimum(zg, 16))
        gidx = (np.arange(K) // 128).astype(np.int32)
        got_g, _ = decode_layout(mcv_b200.pack_w4a16_gptq(qg, zgp, gidx, s))
        assert np.array_equal(got_g, oracle.unpack_gptq(qg, zgp, gidx, kg).astype(np.int16))
