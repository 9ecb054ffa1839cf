"""ctypes front end of the CPU oracle (liboracle.so).  TEST INFRASTRUCTURE ONLY.

This is the checker for the CUDA decode-matmul path and the timed CPU
baseline.  Only tests/, ``__graft_entry__.smoke()`` and bench.py's CPU legs
import it; the shipped library never does.  Every wrapper returns numpy arrays
and documents the reference file:line its C function restates (see oracle.h).
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "liboracle.so")
_lib = None

_i64 = ctypes.c_int64
_p = ctypes.c_void_p


def build() -> str:
    """Compile liboracle.so with the oracle's Makefile (gcc, no CUDA)."""
    subprocess.run(["make", "-s", "-C", _HERE], check=True)
    return _LIB_PATH


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(_LIB_PATH):
            build()
        _lib = ctypes.CDLL(_LIB_PATH)
        _lib.orc_f16_to_f32.restype = ctypes.c_float
        _lib.orc_f16_to_f32.argtypes = [ctypes.c_uint16]
        _lib.orc_f16_to_f32_ftz.restype = ctypes.c_float
        _lib.orc_f16_to_f32_ftz.argtypes = [ctypes.c_uint16]
        _lib.orc_f32_to_f16_rn.restype = ctypes.c_uint16
        _lib.orc_f32_to_f16_rn.argtypes = [ctypes.c_float]
        _lib.orc_f32_to_f16_trunc.restype = ctypes.c_uint16
        _lib.orc_f32_to_f16_trunc.argtypes = [ctypes.c_float]
        _lib.orc_argmax_key.restype = ctypes.c_uint64
        _lib.orc_argmax_key.argtypes = [ctypes.c_float, ctypes.c_uint32]
        _lib.orc_w4a16_choose_tile_len.restype = _i64
        _lib.orc_w4a16_choose_tile_len.argtypes = [_i64]
        _lib.orc_w4a16_tile_rows.restype = _i64
        _lib.orc_w4a16_tile_rows.argtypes = [_i64, _i64, _i64]
        _lib.orc_unpack_gptq.restype = ctypes.c_int
    return _lib


def _ptr(a: np.ndarray):
    assert a.flags["C_CONTIGUOUS"], "oracle inputs must be C-contiguous"
    return a.ctypes.data_as(_p)


def _u16(a) -> np.ndarray:
    a = np.ascontiguousarray(a)
    if a.dtype == np.float16:
        a = a.view(np.uint16)
    assert a.dtype == np.uint16, a.dtype
    return a


# ---- fp16 helpers ---------------------------------------------------------

def f16_to_f32(bits) -> np.ndarray:
    b = _u16(bits)
    out = np.empty(b.shape, np.float32)
    lib().orc_f16_to_f32_array(_ptr(b), _ptr(out), _i64(b.size))
    return out


def f32_to_f16_rn(vals) -> np.ndarray:
    v = np.ascontiguousarray(vals, dtype=np.float32)
    out = np.empty(v.shape, np.uint16)
    lib().orc_f32_to_f16_rn_array(_ptr(v), _ptr(out), _i64(v.size))
    return out


def f32_to_f16_trunc(v: float) -> int:
    return int(lib().orc_f32_to_f16_trunc(ctypes.c_float(v)))


def argmax_key(logit: float, index: int) -> int:
    return int(lib().orc_argmax_key(ctypes.c_float(logit), ctypes.c_uint32(index)))


# ---- W4A16 ------------------------------------------------------------------

def w4a16_gemv(x, w_kn: np.ndarray, scales, group: int = 128, nthreads: int = 1) -> np.ndarray:
    """fp32 [M,N]; x fp16 [M,K], w (q-z) int8 [K,N], scales fp16 [K/group,N].
    tests/test_matmul_w4a16.cpp:217-227."""
    x = _u16(x)
    if x.ndim == 1:
        x = x[None, :]
    w = np.ascontiguousarray(w_kn, dtype=np.int8)
    s = _u16(scales)
    M, K = x.shape
    N = w.shape[1]
    assert w.shape == (K, N) and s.shape == (K // group, N)
    out = np.empty((M, N), np.float32)
    if nthreads > 1:
        lib().orc_w4a16_gemv_mt(_ptr(x), _ptr(w), _ptr(s), _i64(M), _i64(K), _i64(N),
                                _i64(group), _ptr(out), ctypes.c_int(nthreads))
    else:
        lib().orc_w4a16_gemv(_ptr(x), _ptr(w), _ptr(s), _i64(M), _i64(K), _i64(N),
                             _i64(group), _ptr(out))
    return out


def w4a16_fold_zeros(q_kn: np.ndarray, z_gn: np.ndarray, group: int = 128) -> np.ndarray:
    q = np.ascontiguousarray(q_kn, dtype=np.uint8)
    z = np.ascontiguousarray(z_gn, dtype=np.uint8)
    K, N = q.shape
    out = np.empty((K, N), np.int8)
    lib().orc_w4a16_fold_zeros(_ptr(q), _ptr(z), _i64(K), _i64(N), _i64(group), _ptr(out))
    return out


def unpack_gptq(qweight, qzeros, g_idx, groups: int) -> np.ndarray:
    """src/csrc/lib/quantized_weight.cpp:75-120; raises on bad g_idx like the reference."""
    qw = np.ascontiguousarray(qweight, dtype=np.int32)
    qz = np.ascontiguousarray(qzeros, dtype=np.int32)
    gi = np.ascontiguousarray(g_idx, dtype=np.int32)
    K = qw.shape[0] * 8
    N = qw.shape[1]
    out = np.empty((K, N), np.int8)
    rc = lib().orc_unpack_gptq(_ptr(qw), _ptr(qz), _ptr(gi), _i64(K), _i64(N), _i64(groups),
                               _ptr(out))
    if rc != 0:
        raise ValueError("GPTQ g_idx out of range")
    return out


def unpack_awq(qweight, qzeros, group: int = 128) -> np.ndarray:
    """src/csrc/lib/quantized_weight.cpp:122-160."""
    qw = np.ascontiguousarray(qweight, dtype=np.int32)
    qz = np.ascontiguousarray(qzeros, dtype=np.int32)
    K = qw.shape[0]
    N = qw.shape[1] * 8
    out = np.empty((K, N), np.int8)
    lib().orc_unpack_awq(_ptr(qw), _ptr(qz), _i64(K), _i64(N), _i64(group), _ptr(out))
    return out


def w4a16_choose_tile_len(N: int) -> int:
    return int(lib().orc_w4a16_choose_tile_len(_i64(N)))


def w4a16_pack_tiles(w_kn: np.ndarray, tile_len: int | None = None) -> np.ndarray:
    """The reference's tile-packed int8 layout, quantized_weight.cpp:41-73."""
    w = np.ascontiguousarray(w_kn, dtype=np.int8)
    K, N = w.shape
    if tile_len is None:
        tile_len = w4a16_choose_tile_len(N)
    rows = int(lib().orc_w4a16_tile_rows(_i64(K), _i64(N), _i64(tile_len)))
    out = np.empty((rows, tile_len), np.int8)
    lib().orc_w4a16_pack_tiles(_ptr(w), _i64(K), _i64(N), _i64(tile_len), _ptr(out))
    return out


# ---- dense fp16 / lm_head -----------------------------------------------------

def gemv_f16(x, w, layout: int = 0) -> np.ndarray:
    """fp32 [M,N]; layout 0 = w [N,K], 1 = w [K,N]."""
    x = _u16(x)
    if x.ndim == 1:
        x = x[None, :]
    w = _u16(w)
    M, K = x.shape
    N = w.shape[0] if layout == 0 else w.shape[1]
    out = np.empty((M, N), np.float32)
    lib().orc_gemv_f16(_ptr(x), _ptr(w), _i64(M), _i64(K), _i64(N), ctypes.c_int(layout),
                       _ptr(out))
    return out


def lm_head_argmax(x, w, layout: int = 0, fp16_logits: bool = False, n_offset: int = 0,
                   nthreads: int = 1):
    """(idx int64 [M], best fp32 [M], gap fp32 [M]); tests/test_lm_head_pipeline.cpp:95-107."""
    x = _u16(x)
    if x.ndim == 1:
        x = x[None, :]
    w = _u16(w)
    M, K = x.shape
    N = w.shape[0] if layout == 0 else w.shape[1]
    idx = np.empty(M, np.int64)
    best = np.empty(M, np.float32)
    gap = np.empty(M, np.float32)
    args = [_ptr(x), _ptr(w), _i64(M), _i64(K), _i64(N), ctypes.c_int(layout),
            ctypes.c_int(int(fp16_logits)), _i64(n_offset), _ptr(idx), _ptr(best), _ptr(gap)]
    if nthreads > 1:
        lib().orc_lm_head_argmax_mt(*args, ctypes.c_int(nthreads))
    else:
        lib().orc_lm_head_argmax(*args)
    return idx, best, gap


# ---- W8A8 ---------------------------------------------------------------------

def w8a8_quantize(x):
    """(xq int8 [M,K], x_scale fp16-bits [M]); op_kernel/w8a8_quantize_custom.cpp:25-41."""
    x = _u16(x)
    if x.ndim == 1:
        x = x[None, :]
    M, K = x.shape
    xq = np.empty((M, K), np.int8)
    xs = np.empty(M, np.uint16)
    lib().orc_w8a8_quantize(_ptr(x), _i64(M), _i64(K), _ptr(xq), _ptr(xs))
    return xq, xs


def w8a8_gemm_i32(xq, w_kn) -> np.ndarray:
    xq = np.ascontiguousarray(xq, dtype=np.int8)
    if xq.ndim == 1:
        xq = xq[None, :]
    w = np.ascontiguousarray(w_kn, dtype=np.int8)
    M, K = xq.shape
    N = w.shape[1]
    acc = np.empty((M, N), np.int32)
    lib().orc_w8a8_gemm_i32(_ptr(xq), _ptr(w), _i64(M), _i64(K), _i64(N), _ptr(acc))
    return acc


def w8a8_dequant(acc, x_scale, w_scale) -> np.ndarray:
    acc = np.ascontiguousarray(acc, dtype=np.int32)
    if acc.ndim == 1:
        acc = acc[None, :]
    xs = _u16(x_scale).reshape(-1)
    ws = _u16(w_scale).reshape(-1)
    M, N = acc.shape
    out = np.empty((M, N), np.uint16)
    lib().orc_w8a8_dequant(_ptr(acc), _ptr(xs), _ptr(ws), _i64(M), _i64(N), _ptr(out))
    return out


def w8a8_fused(x, w_kn, w_scale, nthreads: int = 1):
    """(acc int32 [M,N], out fp16-bits [M,N])."""
    x = _u16(x)
    if x.ndim == 1:
        x = x[None, :]
    w = np.ascontiguousarray(w_kn, dtype=np.int8)
    ws = _u16(w_scale).reshape(-1)
    M, K = x.shape
    N = w.shape[1]
    acc = np.empty((M, N), np.int32)
    out = np.empty((M, N), np.uint16)
    if nthreads > 1:
        lib().orc_w8a8_fused_mt(_ptr(x), _ptr(w), _ptr(ws), _i64(M), _i64(K), _i64(N),
                                _ptr(acc), _ptr(out), ctypes.c_int(nthreads))
    else:
        lib().orc_w8a8_fused(_ptr(x), _ptr(w), _ptr(ws), _i64(M), _i64(K), _i64(N),
                             _ptr(acc), _ptr(out))
    return acc, out


def quantize_dense_weight_w8a8(w_kn):
    """(wq int8 [K,N], w_scale fp16-bits [N]); quantized_weight.cpp:231-268."""
    w = _u16(w_kn)
    K, N = w.shape
    wq = np.empty((K, N), np.int8)
    ws = np.empty(N, np.uint16)
    lib().orc_quantize_dense_weight_w8a8(_ptr(w), _i64(K), _i64(N), _ptr(wq), _ptr(ws))
    return wq, ws


# ---- rms_norm / silu_mul --------------------------------------------------------

def rms_norm(x, gamma, eps: float = 1e-6, variant: int = 0) -> np.ndarray:
    """fp16 bits [M,H].  variant 0: the engine's fp16 op chain with (1 + gamma)
    (src/csrc/lib/ops.cpp:564-737); 1: the fp32 rms_norm1024 custom kernel
    with gamma (op_kernel/rms_norm1024_custom.cpp:57-70)."""
    x = _u16(x)
    if x.ndim == 1:
        x = x[None, :]
    g = _u16(gamma).reshape(-1)
    M, H = x.shape
    assert g.size == H
    out = np.empty((M, H), np.uint16)
    fn = lib().orc_rms_norm_chain if variant == 0 else lib().orc_rms_norm_fp32
    fn(_ptr(x), _ptr(g), _i64(M), _i64(H), ctypes.c_float(eps), _ptr(out))
    return out


def silu_mul(gate, up) -> np.ndarray:
    """fp16 bits, shape of gate; op_kernel/silu_mul_custom.cpp:63-72."""
    g = _u16(gate)
    u = _u16(up)
    assert g.shape == u.shape
    out = np.empty(g.shape, np.uint16)
    lib().orc_silu_mul(_ptr(g), _ptr(u), _i64(g.size), _ptr(out))
    return out
