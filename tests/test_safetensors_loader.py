"""The checkpoint side of the W4A16 path on the host: the safetensors reader
(WeightsIndex, src/csrc/lib/weights.cpp:197-333) and the GPTQ / AWQ loader
(load_w4a16_quantized_weight, src/csrc/lib/quantized_weight.cpp:204-229),
on synthetic checkpoint files that the tests write.  The loaded mcv-int4
arrays must equal the packers' output for the same tensors; the oracle's
unpackers (which restate quantized_weight.cpp:75-160) pin what the tensors
mean.  The GPU test feeds a loaded weight to the GEMV."""
import ctypes
import struct

import numpy as np
import pytest

import mcv_b200 as mcv
import oracle
from conftest import write_safetensors
from mcv_b200 import synth


def _ptr(a):
    return a.ctypes.data_as(ctypes.c_void_p)


def host_pack_gptq(qweight, qzeros, g_idx, scales, K, N):
    qw, sc, zw = mcv._alloc_layout_host(K, N, 128)
    zb = ctypes.c_int(-1)
    st = mcv.lib().mcv_w4a16_pack_gptq_host(_ptr(qweight), _ptr(qzeros), _ptr(g_idx), _ptr(scales.view(np.uint16)),
                                            K, N, 128, _ptr(qw), _ptr(sc), _ptr(zw), ctypes.byref(zb))
    assert st == 0
    return qw, sc, zw, zb.value


def host_pack_awq(qweight, qzeros, scales, K, N):
    qw, sc, zw = mcv._alloc_layout_host(K, N, 128)
    zb = ctypes.c_int(-1)
    st = mcv.lib().mcv_w4a16_pack_awq_host(_ptr(qweight), _ptr(qzeros), _ptr(scales.view(np.uint16)), K, N, 128,
                                           _ptr(qw), _ptr(sc), _ptr(zw), ctypes.byref(zb))
    assert st == 0
    return qw, sc, zw, zb.value


def bf16_to_f16_trunc(bits):
    """weights.cpp:25-33, restated in numpy."""
    b = bits.astype(np.uint32) << 16
    sign = ((b >> 16) & 0x8000).astype(np.uint16)
    e = ((b >> 23) & 0xFF).astype(np.int32) - 112
    mant = ((b & 0x7FFFFF) >> 13).astype(np.uint16)
    out = sign | (np.clip(e, 0, 31).astype(np.uint16) << 10) | mant
    out = np.where(e <= 0, sign, out)
    out = np.where(e >= 31, sign | 0x7C00, out)
    return out.astype(np.uint16)


def gptq_checkpoint(K, N, seed):
    _, q, z, s = synth.w4a16_inputs(1, K, N, seed=seed)
    z = np.maximum(z, 1)                      # GPTQ stores zero - 1
    qweight, qzeros = synth.gptq_pack(q, z)
    g_idx = (np.arange(K) // 128).astype(np.int32)
    return q, z, s, qweight, qzeros, g_idx


def test_reader_names_info_and_bytes(tmp_path):
    p = tmp_path / "m.safetensors"
    r = np.random.default_rng(0)
    emb = r.standard_normal((64, 32)).astype(np.float16)
    bf = (r.standard_normal((5, 7)).astype(np.float32).view(np.uint32) >> 16).astype(np.uint16)
    ids = np.arange(10, dtype=np.int64)
    write_safetensors(p, {"model.embed.weight": ("F16", emb), "z.bf": ("BF16", bf), "a.ids": ("I64", ids),
                          "e.empty": ("F32", np.zeros((0, 3), np.float32))},
                      metadata={"format": "pt", "nested": {"x": [1, 2, {"y": "\\u00e9"}]}}, header_pad=7)
    with mcv.SafeTensors(str(p)) as st:
        assert st.names() == sorted(["model.embed.weight", "z.bf", "a.ids", "e.empty"])
        assert st.info("model.embed.weight") == ("F16", (64, 32), 64 * 32 * 2)
        assert st.info("z.bf") == ("BF16", (5, 7), 70)
        assert st.info("e.empty") == ("F32", (0, 3), 0)
        assert np.array_equal(st.numpy("model.embed.weight"), emb)
        assert np.array_equal(st.numpy("a.ids"), ids)
        assert np.array_equal(st.numpy("z.bf"), bf)
        assert "a.ids" in st and "nope" not in st
        with pytest.raises(RuntimeError, match="no tensor"):
            st.info("nope")


@pytest.mark.parametrize("K,N", [(1024, 3584), (256, 64), (2048, 1024)])
def test_gptq_checkpoint_loads_as_packer(tmp_path, K, N):
    q, z, s, qweight, qzeros, g_idx = gptq_checkpoint(K, N, seed=K + N)
    p = tmp_path / "gptq.safetensors"
    base = "model.layers.0.mlp.down_proj"
    write_safetensors(p, {base + ".qweight": ("I32", qweight), base + ".qzeros": ("I32", qzeros),
                          base + ".g_idx": ("I32", g_idx), base + ".scales": ("F16", s),
                          "other.weight": ("F16", np.ones((3, 3), np.float16))})
    with mcv.SafeTensors(str(p)) as st:
        assert mcv.has_w4a16_quantized_weight(st, base) and not mcv.has_w4a16_quantized_weight(st, "other")
        qw, sc, zw, zb, k2, n2 = mcv.load_w4a16_quantized_weight_host(st, base)
    assert (k2, n2) == (K, N)
    want = host_pack_gptq(qweight, qzeros, g_idx, s, K, N)
    for a, b in zip((qw, sc, zw, zb), want):
        assert np.array_equal(a, b)
    # the tensors mean what the reference's unpacker says (q - (stored zero + 1))
    assert np.array_equal(oracle.unpack_gptq(qweight, qzeros, g_idx, K // 128), oracle.w4a16_fold_zeros(q, z))


@pytest.mark.parametrize("K,N", [(1024, 3584), (128, 8)])
def test_awq_checkpoint_loads_as_packer(tmp_path, K, N):
    _, q, z, s = synth.w4a16_inputs(1, K, N, seed=7)
    qweight, qzeros = synth.awq_pack(q, z)
    p = tmp_path / "awq.safetensors"
    write_safetensors(p, {"x.qweight": ("I32", qweight), "x.qzeros": ("I32", qzeros), "x.scales": ("F16", s)})
    with mcv.SafeTensors(str(p)) as st:
        qw, sc, zw, zb, k2, n2 = mcv.load_w4a16_quantized_weight_host(st, "x")
    assert (k2, n2) == (K, N)
    for a, b in zip((qw, sc, zw, zb), host_pack_awq(qweight, qzeros, s, K, N)):
        assert np.array_equal(a, b)
    assert np.array_equal(oracle.unpack_awq(qweight, qzeros), oracle.w4a16_fold_zeros(q, z))


def test_bf16_scales_convert_as_the_reference_loader(tmp_path):
    K, N = 256, 64
    q, z, s, qweight, qzeros, g_idx = gptq_checkpoint(K, N, seed=3)
    s_bf = (s.astype(np.float32).view(np.uint32) >> 16).astype(np.uint16)
    p = tmp_path / "bf.safetensors"
    write_safetensors(p, {"w.qweight": ("I32", qweight), "w.qzeros": ("I32", qzeros), "w.g_idx": ("I32", g_idx),
                          "w.scales": ("BF16", s_bf)})
    with mcv.SafeTensors(str(p)) as st:
        got = mcv.load_w4a16_quantized_weight_host(st, "w")
    want = host_pack_gptq(qweight, qzeros, g_idx, bf16_to_f16_trunc(s_bf).view(np.float16), K, N)
    assert np.array_equal(got[1], want[1])


def _expect_fail(path, code, match=None):
    with pytest.raises(RuntimeError, match=match) as ei:
        mcv.SafeTensors(str(path))
    assert getattr(ei.value, "status", code) == code


def test_malformed_files_are_refused(tmp_path):
    FORMAT = 9
    p = tmp_path / "t.safetensors"
    p.write_bytes(b"\x01\x02")
    _expect_fail(p, FORMAT, "shorter")
    p.write_bytes(struct.pack("<Q", 1000) + b"{}")
    _expect_fail(p, FORMAT, "header length")
    good = {"a": ("F16", np.zeros((4, 4), np.float16))}
    write_safetensors(p, good)
    raw = bytearray(p.read_bytes())
    p.write_bytes(bytes(raw[:-2]))                       # data cut short
    _expect_fail(p, FORMAT, "past the end")
    hdr = b'{"a": {"dtype": "F16", "shape": [4, 4], "data_offsets": [0, 30]}}'
    p.write_bytes(struct.pack("<Q", len(hdr)) + hdr + bytes(32))
    _expect_fail(p, FORMAT, "disagrees")                 # 30 bytes for 16 halves
    hdr = b'{"a": {"dtype": "Q4", "shape": [1], "data_offsets": [0, 1]}}'
    p.write_bytes(struct.pack("<Q", len(hdr)) + hdr + bytes(1))
    _expect_fail(p, FORMAT, "dtype")
    hdr = b'{"a": {"dtype": "F16", "shape": [1]}}'
    p.write_bytes(struct.pack("<Q", len(hdr)) + hdr)
    _expect_fail(p, FORMAT, "lacks")
    hdr = b'{"a": {"dtype": "F16", "shape": [1], "data_offsets": [0, 2]'
    p.write_bytes(struct.pack("<Q", len(hdr)) + hdr + bytes(2))
    _expect_fail(p, FORMAT)
    with pytest.raises(RuntimeError, match="cannot open"):
        mcv.SafeTensors(str(tmp_path / "missing.safetensors"))
    # an empty header is a valid file with no tensors
    p.write_bytes(struct.pack("<Q", 2) + b"{}")
    with mcv.SafeTensors(str(p)) as st:
        assert st.names() == []


def test_quantized_tensor_checks(tmp_path):
    K, N = 256, 64
    q, z, s, qweight, qzeros, g_idx = gptq_checkpoint(K, N, seed=5)
    p = tmp_path / "bad.safetensors"
    cases = [
        ({"w.qweight": ("I32", qweight), "w.scales": ("F16", s)}, "no .qweight"),            # qzeros missing
        ({"w.qweight": ("I64", qweight.astype(np.int64)), "w.qzeros": ("I32", qzeros), "w.scales": ("F16", s),
          "w.g_idx": ("I32", g_idx)}, "dtypes"),
        ({"w.qweight": ("I32", qweight), "w.qzeros": ("I32", qzeros), "w.scales": ("F16", s[:1]),
          "w.g_idx": ("I32", g_idx)}, "shapes"),
        ({"w.qweight": ("I32", qweight), "w.qzeros": ("I32", qzeros), "w.scales": ("F16", s),
          "w.g_idx": ("I32", g_idx[::-1].copy())}, "act-order"),                            # permuted groups
    ]
    for tensors, match in cases:
        write_safetensors(p, tensors)
        with mcv.SafeTensors(str(p)) as st:
            with pytest.raises(RuntimeError, match=match):
                mcv.load_w4a16_quantized_weight_host(st, "w")


@pytest.mark.gpu
def test_loaded_checkpoint_gemv_matches_oracle(cuda, tmp_path):
    torch = cuda
    K, N = 1024, 3584
    q, z, s, qweight, qzeros, g_idx = gptq_checkpoint(K, N, seed=11)
    p = tmp_path / "g.safetensors"
    emb = (np.random.default_rng(1).standard_normal((300, K)) * 0.02).astype(np.float32)
    emb_bf = (emb.view(np.uint32) >> 16).astype(np.uint16)
    write_safetensors(p, {"l.qweight": ("I32", qweight), "l.qzeros": ("I32", qzeros), "l.g_idx": ("I32", g_idx),
                          "l.scales": ("F16", s), "embed": ("BF16", emb_bf)})
    x = synth.w4a16_inputs(1, K, N, seed=12)[0]
    with mcv.SafeTensors(str(p)) as st:
        w = mcv.load_w4a16_quantized_weight(st, "l")
        e = st.to_device_f16("embed")
    out = torch.empty((1, N), dtype=torch.float16, device="cuda")
    mcv.matmul_w4a16(torch.from_numpy(x).cuda(), w, out)
    torch.cuda.synchronize()
    ref = oracle.w4a16_gemv(x, oracle.unpack_gptq(qweight, qzeros, g_idx, K // 128), s, nthreads=8)
    from conftest import assert_f16_close
    assert_f16_close(out.cpu().numpy(), ref, what="checkpoint GEMV")
    assert np.array_equal(e.cpu().numpy().view(np.uint16), bf16_to_f16_trunc(emb_bf).reshape(300, K))
