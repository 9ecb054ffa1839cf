"""Python binding of libmcv_b200.so (the C ABI in include/mcv_matmul.h).

The functions mirror the reference engine's op surface for the decode matmul
path (src/csrc/include/minicpmv/ops.h of lvyufeng/minicpm-v-4.6-orangepi):
``matmul_w4a16``, ``matmul_b_transposed``, ``argmax_last_dim``,
``matmul_w8a8_i32``, ``w8a8_quantize``, ``w8a8_dequant``, plus the fused
``lm_head_argmax`` that replaces lm_head_greedy's chunk loop, and the
load-time weight preparation of quantized_weight.h.  As in the reference,
outputs are caller-allocated tensors and a failed check raises RuntimeError.

torch is only the device-memory and stream plumbing here: every computation
is one of the library's CUDA kernels, reached through ctypes with raw device
pointers.  There is no CPU fallback; importing without the built library or
calling without a CUDA device fails loudly.
"""
from __future__ import annotations

import ctypes
import os
from dataclasses import dataclass

import numpy as np

_PKG_DIR = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
LIB_PATH = os.path.join(_PKG_DIR, "libmcv_b200.so")
_lib = None

_i64 = ctypes.c_int64
_int = ctypes.c_int
_vp = ctypes.c_void_p
_sz = ctypes.c_size_t
_f32 = ctypes.c_float

# name -> argtypes (restype int unless listed in _RESTYPE)
_SIGS = {
    "mcv_status_string": [_int],
    "mcv_last_error": [],
    "mcv_version": [],
    "mcv_set_pdl": [_int],
    "mcv_set_tuning": [_int, _int],
    "mcv_get_tuning": [_int],
    "mcv_device_errors": [],
    "mcv_w4a16_layout_bytes": [_i64, _i64, _i64, _vp, _vp, _vp],
    "mcv_w4a16_pack_host": [_vp, _vp, _vp, _i64, _i64, _i64, _vp, _vp, _vp],
    "mcv_w4a16_unpack_host": [_vp, _vp, _vp, _int, _i64, _i64, _i64, _vp, _vp],
    "mcv_w4a16_pack_gptq_host": [_vp, _vp, _vp, _vp, _i64, _i64, _i64, _vp, _vp, _vp, _vp],
    "mcv_w4a16_pack_awq_host": [_vp, _vp, _vp, _i64, _i64, _i64, _vp, _vp, _vp, _vp],
    "mcv_w4a16_pack_from_tiles_host": [_vp, _i64, _vp, _i64, _i64, _vp, _vp, _vp, _vp],
    "mcv_w4a16_gemv": [_vp, _vp, _vp, _vp, _int, _vp, _i64, _i64, _i64, _i64, _vp],
    "mcv_w4a16_gemv_grouped": [_vp, _int, _i64, _vp],
    "mcv_w4a16_gemm": [_vp, _vp, _vp, _vp, _int, _vp, _i64, _i64, _i64, _i64, _vp],
    "mcv_gemm_f16": [_vp, _vp, _vp, _i64, _i64, _i64, _vp],
    "mcv_transpose_f16": [_vp, _vp, _i64, _i64, _vp],
    "mcv_gemv_f16": [_vp, _vp, _vp, _i64, _i64, _i64, _int, _vp],
    "mcv_lm_head_workspace_size": [_i64],
    "mcv_lm_head_argmax": [_vp, _vp, _vp, _vp, _i64, _i64, _i64, _i64, _int, _vp, _sz, _vp],
    "mcv_argmax_last_dim_f16": [_vp, _vp, _i64, _i64, _vp],
    "mcv_argmax_key_to_index": [_vp, _vp, _i64, _vp],
    "mcv_lm_head_noalloc_max_bytes": [],
    "mcv_lm_head_argmax_noalloc": [_vp, _vp, _vp, _vp, _i64, _i64, _i64, _i64, _int, _vp],
    "mcv_nccl_unique_id_bytes": [],
    "mcv_nccl_get_unique_id": [_vp],
    "mcv_nccl_comm_init": [_vp, _int, _vp, _int],
    "mcv_nccl_comm_destroy": [_vp],
    "mcv_lm_head_argmax_allreduce": [_vp, _vp, _vp, _vp, _vp, _i64, _i64, _i64, _i64, _int, _vp, _sz, _vp],
    "mcv_p2p_handle_bytes": [],
    "mcv_p2p_create": [_vp, _int, _int, _vp],
    "mcv_p2p_connect": [_vp, _vp],
    "mcv_p2p_destroy": [_vp],
    "mcv_p2p_errors": [_vp],
    "mcv_lm_head_argmax_p2p": [_vp, _vp, _vp, _vp, _vp, _i64, _i64, _i64, _i64, _int, _vp, _sz, _vp],
    "mcv_lm_head_greedy_host": [_vp, _vp, _vp, _vp, _f32, _vp, _vp, _vp, _i64, _i64, _i64, _i64, _int, _vp, _sz, _vp],
    "mcv_lm_head_argmax_rmsnorm": [_vp, _vp, _vp, _f32, _int, _vp, _vp, _vp, _i64, _i64, _i64, _i64, _int, _vp, _sz,
                                   _vp],
    "mcv_rms_norm": [_vp, _vp, _vp, _i64, _i64, _f32, _int, _vp],
    "mcv_silu_mul": [_vp, _vp, _vp, _i64, _vp],
    "mcv_safetensors_open": [ctypes.c_char_p, _vp],
    "mcv_safetensors_close": [_vp],
    "mcv_safetensors_count": [_vp],
    "mcv_safetensors_name": [_vp, _i64],
    "mcv_safetensors_info": [_vp, ctypes.c_char_p, _vp, _vp, _vp, _vp, _vp],
    "mcv_safetensors_copy_f16": [_vp, ctypes.c_char_p, _vp, ctypes.c_uint64, _vp],
    "mcv_w4a16_safetensors_dims": [_vp, ctypes.c_char_p, _vp, _vp, _vp],
    "mcv_w4a16_load_safetensors": [_vp, ctypes.c_char_p, _vp, _vp, _vp, _vp, _vp],
    "mcv_w4a16_load_safetensors_host": [_vp, ctypes.c_char_p, _vp, _vp, _vp, _vp],
    "mcv_w4a16_gemv_gate_up_silu": [_vp, _vp, _vp, _vp, _i64, _vp],
    "mcv_w8a8_quantize": [_vp, _vp, _vp, _i64, _i64, _vp],
    "mcv_w8a8_gemm_i32": [_vp, _vp, _vp, _i64, _i64, _i64, _int, _vp],
    "mcv_w8a8_dequant": [_vp, _vp, _vp, _vp, _i64, _i64, _vp],
    "mcv_w8a8_gemv_prequant": [_vp, _vp, _vp, _vp, _vp, _vp, _i64, _i64, _i64, _vp],
    "mcv_w8a8_fused_grouped": [_vp, _int, _i64, _i64, _vp],
    "mcv_w8a8_fused": [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _i64, _i64, _i64, _int, _vp],
    "mcv_w8a8_quantize_weight": [_vp, _vp, _vp, _i64, _i64, _int, _vp],
    "mcv_lm_head_argmax_w8a8": [_vp, _vp, _vp, _vp, _vp, _i64, _i64, _i64, _i64, _vp, _sz, _vp],
    "mcv_set_w8a8_decode_mode": [ctypes.c_char_p],
    "mcv_w8a8_decode_enabled": [],
    "mcv_w8a8_decode_gate_enabled": [],
    "mcv_w8a8_policy_allows": [ctypes.c_char_p],
    "mcv_w8a8_policy_allows_mode": [ctypes.c_char_p, ctypes.c_char_p],
    "mcv_matmul_decode_dispatch": [_vp, _vp, _vp, _i64, _i64, _i64, _vp],
}
_RESTYPE = {
    "mcv_status_string": ctypes.c_char_p,
    "mcv_last_error": ctypes.c_char_p,
    "mcv_set_pdl": None,
    "mcv_device_errors": ctypes.c_uint,
    "mcv_lm_head_workspace_size": _sz,
    "mcv_nccl_unique_id_bytes": _sz,
    "mcv_p2p_handle_bytes": _sz,
    "mcv_p2p_errors": ctypes.c_uint,
    "mcv_lm_head_noalloc_max_bytes": _sz,
    "mcv_safetensors_count": _i64,
    "mcv_safetensors_name": ctypes.c_char_p,
}
EXPORTED = tuple(_SIGS)


def lib() -> ctypes.CDLL:
    """The loaded library; raises if it has not been built."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(f"libmcv_b200.so not built ({LIB_PATH}); run __graft_entry__.build()")
        L = ctypes.CDLL(LIB_PATH)
        for name, args in _SIGS.items():
            f = getattr(L, name)
            f.argtypes = args
            f.restype = _RESTYPE.get(name, _int)
        _lib = L
    return _lib


class McvError(RuntimeError):
    def __init__(self, status: int, where: str):
        L = lib()
        msg = L.mcv_last_error().decode(errors="replace")
        super().__init__(f"{where}: {L.mcv_status_string(status).decode()} ({status}): {msg}")
        self.status = status


def _check(status: int, where: str) -> None:
    if status != 0:
        raise McvError(status, where)


def _stream(stream=None):
    import torch
    if stream is None:
        stream = torch.cuda.current_stream()
    return _vp(stream.cuda_stream)


def _ptr(t):
    if t is None:
        return None
    if isinstance(t, np.ndarray):
        return t.ctypes.data_as(_vp)
    if not t.is_cuda:
        raise RuntimeError("mcv_b200: expected a CUDA tensor")
    if not t.is_contiguous():
        raise RuntimeError("mcv_b200: tensors must be contiguous")
    return _vp(t.data_ptr())


def set_pdl(enabled: bool) -> None:
    lib().mcv_set_pdl(1 if enabled else 0)


TUNE_W4A16_MODE = 2
TUNE_ROWS_BLOCKS_PER_SM = 3
TUNE_ROWS_PREFETCH = 4
TUNE_GEMM_SPLIT_K = 5
TUNE_W8A8_KERNEL = 6
TUNE_W4A16_GRID = 7
TUNE_W4A16_MATH = 8
TUNE_ROWS_WALK = 9
TUNE_W4A16_KSPLIT_WARPS = 10


def device_errors() -> int:
    """Device-side error bits since the last call (bit 0: a bounded wait gave up)."""
    return int(lib().mcv_device_errors())


def set_tuning(key: int, value: int) -> None:
    _check(lib().mcv_set_tuning(key, value), "set_tuning")


# ---- W4A16 ------------------------------------------------------------------

@dataclass
class W4A16QuantizedWeight:
    """Device weight in the mcv-int4 layout (counterpart of the reference's
    W4A16QuantizedWeight, src/csrc/include/minicpmv/quantized_weight.h:11-17)."""
    qweight: object   # torch.int32 [Npad*K/8]  (Npad = N rounded up to 16)
    scales: object    # torch.float16 [Npad, Gpad]  (Gpad = G rounded up to 8)
    zeros: object     # torch.int32 [Npad, ceil(G/8)]
    zero_bias: int
    K: int
    N: int
    group_size: int = 128

    @property
    def nbytes(self) -> int:
        return sum(t.numel() * t.element_size() for t in (self.qweight, self.scales, self.zeros))


def _alloc_layout_host(K: int, N: int, group: int):
    G = K // group
    Np = (N + 15) // 16 * 16
    Gp = (G + 7) // 8 * 8
    qw = np.empty(Np * K // 8, np.uint32)
    sc = np.empty((Np, Gp), np.uint16)
    zw = np.empty((Np, (G + 7) // 8), np.uint32)
    return qw, sc, zw


def _to_device(qw, sc, zw, zero_bias, K, N, group, device) -> W4A16QuantizedWeight:
    import torch
    return W4A16QuantizedWeight(
        torch.from_numpy(qw.view(np.int32)).to(device),
        torch.from_numpy(sc.view(np.float16)).to(device),
        torch.from_numpy(zw.view(np.int32)).to(device),
        int(zero_bias), K, N, group)


def pack_w4a16(q_kn: np.ndarray, z_gn: np.ndarray, scales_gn: np.ndarray, group: int = 128,
               device="cuda") -> W4A16QuantizedWeight:
    """Logical q uint8 [K,N] (0..15), z uint8 [G,N], scales fp16 [G,N] -> device layout."""
    q = np.ascontiguousarray(q_kn, np.uint8)
    z = np.ascontiguousarray(z_gn, np.uint8)
    s = np.ascontiguousarray(scales_gn).view(np.uint16)
    K, N = q.shape
    qw, sc, zw = _alloc_layout_host(K, N, group)
    _check(lib().mcv_w4a16_pack_host(_ptr(q), _ptr(z), _ptr(s), K, N, group, _ptr(qw), _ptr(sc), _ptr(zw)),
           "pack_w4a16")
    return _to_device(qw, sc, zw, 0, K, N, group, device)


def pack_w4a16_gptq(qweight, qzeros, g_idx, scales, group: int = 128, device="cuda") -> W4A16QuantizedWeight:
    """GPTQ tensors (qweight int32 [K/8,N], qzeros int32 [G,N/8], g_idx int32 [K] or None,
    scales fp16 [G,N]) -> device layout; load_w4a16_quantized_weight's GPTQ branch."""
    qwt = np.ascontiguousarray(qweight, np.int32)
    qz = np.ascontiguousarray(qzeros, np.int32)
    gi = None if g_idx is None else np.ascontiguousarray(g_idx, np.int32)
    s = np.ascontiguousarray(scales).view(np.uint16)
    K, N = qwt.shape[0] * 8, qwt.shape[1]
    qw, sc, zw = _alloc_layout_host(K, N, group)
    zb = ctypes.c_int(0)
    _check(lib().mcv_w4a16_pack_gptq_host(_ptr(qwt), _ptr(qz), _ptr(gi) if gi is not None else None, _ptr(s),
                                          K, N, group, _ptr(qw), _ptr(sc), _ptr(zw), ctypes.byref(zb)),
           "pack_w4a16_gptq")
    return _to_device(qw, sc, zw, zb.value, K, N, group, device)


def pack_w4a16_awq(qweight, qzeros, scales, group: int = 128, device="cuda") -> W4A16QuantizedWeight:
    """AWQ tensors (qweight int32 [K,N/8], qzeros int32 [G,N/8], scales fp16 [G,N])."""
    qwt = np.ascontiguousarray(qweight, np.int32)
    qz = np.ascontiguousarray(qzeros, np.int32)
    s = np.ascontiguousarray(scales).view(np.uint16)
    K, N = qwt.shape[0], qwt.shape[1] * 8
    qw, sc, zw = _alloc_layout_host(K, N, group)
    zb = ctypes.c_int(0)
    _check(lib().mcv_w4a16_pack_awq_host(_ptr(qwt), _ptr(qz), _ptr(s), K, N, group, _ptr(qw), _ptr(sc),
                                         _ptr(zw), ctypes.byref(zb)), "pack_w4a16_awq")
    return _to_device(qw, sc, zw, zb.value, K, N, group, device)


def pack_w4a16_from_tiles(packed: np.ndarray, scales_gn: np.ndarray, K: int, N: int,
                          device="cuda") -> W4A16QuantizedWeight:
    """The reference's tile-packed int8 (q - zero) [rows, tile_len] + scales [G,N]."""
    p = np.ascontiguousarray(packed, np.int8)
    s = np.ascontiguousarray(scales_gn).view(np.uint16)
    qw, sc, zw = _alloc_layout_host(K, N, 128)
    zb = ctypes.c_int(0)
    _check(lib().mcv_w4a16_pack_from_tiles_host(_ptr(p), p.shape[1], _ptr(s), K, N, _ptr(qw), _ptr(sc),
                                                _ptr(zw), ctypes.byref(zb)), "pack_w4a16_from_tiles")
    return _to_device(qw, sc, zw, zb.value, K, N, 128, device)


# ---- checkpoints (safetensors) ---------------------------------------------------

_NP_DTYPE = {1: np.float16, 2: np.uint16, 3: np.float32, 4: np.float64, 5: np.int8, 6: np.uint8, 7: np.int16,
             8: np.int32, 9: np.int64, 10: np.bool_}
DTYPE_NAMES = {1: "F16", 2: "BF16", 3: "F32", 4: "F64", 5: "I8", 6: "U8", 7: "I16", 8: "I32", 9: "I64", 10: "BOOL"}


class SafeTensors:
    """A memory-mapped .safetensors file (mcv_safetensors_open): the
    counterpart of the reference's WeightsIndex (weights.cpp:197-333)."""

    def __init__(self, path: str):
        self.handle = _vp()
        _check(lib().mcv_safetensors_open(os.fsencode(path), ctypes.byref(self.handle)), "safetensors_open")

    def close(self) -> None:
        if self.handle:
            lib().mcv_safetensors_close(self.handle)
            self.handle = _vp()

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def names(self):
        L = lib()
        return [L.mcv_safetensors_name(self.handle, i).decode() for i in range(L.mcv_safetensors_count(self.handle))]

    def __contains__(self, name: str) -> bool:
        return name in set(self.names())

    def info(self, name: str):
        """(dtype name, shape tuple, nbytes)."""
        dt, rank, nb = ctypes.c_int(0), ctypes.c_int(0), ctypes.c_uint64(0)
        shape = (ctypes.c_int64 * 8)()
        _check(lib().mcv_safetensors_info(self.handle, name.encode(), ctypes.byref(dt), ctypes.byref(rank), shape,
                                          None, ctypes.byref(nb)), "safetensors_info")
        return DTYPE_NAMES[dt.value], tuple(shape[i] for i in range(rank.value)), nb.value

    def numpy(self, name: str) -> np.ndarray:
        """A copy of the tensor's elements (BF16 as raw uint16 bits)."""
        dt, rank, nb = ctypes.c_int(0), ctypes.c_int(0), ctypes.c_uint64(0)
        shape = (ctypes.c_int64 * 8)()
        data = _vp()
        _check(lib().mcv_safetensors_info(self.handle, name.encode(), ctypes.byref(dt), ctypes.byref(rank), shape,
                                          ctypes.byref(data), ctypes.byref(nb)), "safetensors_info")
        raw = ctypes.string_at(data, nb.value) if nb.value else b""
        return np.frombuffer(raw, dtype=_NP_DTYPE[dt.value]).reshape([shape[i] for i in range(rank.value)]).copy()

    def to_device_f16(self, name: str, device="cuda"):
        """An F16 (or BF16, converted as the reference's loader does) tensor on the device."""
        import torch
        _, shape, nb = self.info(name)
        elems = int(np.prod(shape)) if shape else 1
        t = torch.empty(shape, dtype=torch.float16, device=device)
        _check(lib().mcv_safetensors_copy_f16(self.handle, name.encode(), _ptr(t), elems * 2, None),
               "safetensors_copy_f16")
        torch.cuda.synchronize(device)
        return t


def has_w4a16_quantized_weight(st: SafeTensors, base: str) -> bool:
    """quantized_weight.cpp:204-210."""
    names = set(st.names())
    return all(base + sfx in names for sfx in (".qweight", ".qzeros", ".scales"))


def _safetensors_dims(st: SafeTensors, base: str):
    K, N, g = ctypes.c_int64(0), ctypes.c_int64(0), ctypes.c_int(0)
    _check(lib().mcv_w4a16_safetensors_dims(st.handle, base.encode(), ctypes.byref(K), ctypes.byref(N),
                                            ctypes.byref(g)), "w4a16_safetensors_dims")
    return K.value, N.value, bool(g.value)


def unpack_w4a16_host(qw, sc, zw, zero_bias: int, K: int, N: int, group: int = 128):
    """mcv-int4 host arrays -> ((q - zero) int8 [K,N], scales fp16 bits [G,N])."""
    w = np.empty((K, N), np.int8)
    s = np.empty((K // group, N), np.uint16)
    _check(lib().mcv_w4a16_unpack_host(_ptr(qw), _ptr(sc), _ptr(zw), zero_bias, K, N, group, _ptr(w), _ptr(s)),
           "w4a16_unpack_host")
    return w, s


def load_w4a16_quantized_weight_host(st: SafeTensors, base: str):
    """(qweight, scales, zeros, zero_bias, K, N) of the mcv-int4 layout as host arrays."""
    K, N, _ = _safetensors_dims(st, base)
    qw, sc, zw = _alloc_layout_host(K, N, 128)
    zb = ctypes.c_int(0)
    _check(lib().mcv_w4a16_load_safetensors_host(st.handle, base.encode(), _ptr(qw), _ptr(sc), _ptr(zw),
                                                 ctypes.byref(zb)), "w4a16_load_safetensors_host")
    return qw, sc, zw, zb.value, K, N


def load_w4a16_quantized_weight(st: SafeTensors, base: str, device="cuda") -> W4A16QuantizedWeight:
    """load_w4a16_quantized_weight (quantized_weight.cpp:212-229): the
    checkpoint's GPTQ or AWQ projection `base` in the mcv-int4 layout on the
    device (mcv_w4a16_load_safetensors)."""
    import torch
    K, N, _ = _safetensors_dims(st, base)
    G = K // 128
    Np, Gp = (N + 15) // 16 * 16, (G + 7) // 8 * 8
    qw = torch.empty(Np * K // 8, dtype=torch.int32, device=device)
    sc = torch.empty((Np, Gp), dtype=torch.float16, device=device)
    zw = torch.empty((Np, (G + 7) // 8), dtype=torch.int32, device=device)
    zb = ctypes.c_int(0)
    _check(lib().mcv_w4a16_load_safetensors(st.handle, base.encode(), _ptr(qw), _ptr(sc), _ptr(zw), ctypes.byref(zb),
                                            None), "w4a16_load_safetensors")
    return W4A16QuantizedWeight(qw, sc, zw, zb.value, K, N, 128)


def matmul_w4a16(x, w: W4A16QuantizedWeight, out, stream=None) -> None:
    """out fp16 [M,N] = x fp16 [M,K] @ dequant(w); M = 1..64 (ops.h:95-108)."""
    M = x.shape[0] if x.dim() == 2 else 1
    _check(lib().mcv_w4a16_gemv(_ptr(x), _ptr(w.qweight), _ptr(w.scales), _ptr(w.zeros), w.zero_bias, _ptr(out),
                                M, w.K, w.N, w.group_size, _stream(stream)), "matmul_w4a16")


def _problem(w: "W4A16QuantizedWeight"):
    return W4A16Problem(None, _ptr(w.qweight), _ptr(w.scales), _ptr(w.zeros), None, w.K, w.N, w.group_size,
                        w.zero_bias)


def matmul_w4a16_gate_up_silu(x, w_gate: W4A16QuantizedWeight, w_up: W4A16QuantizedWeight, act, stream=None) -> None:
    """act fp16 [M,N] = silu_mul(x @ dequant(w_gate), x @ dequant(w_up)) in one
    launch (mcv_w4a16_gemv_gate_up_silu): the MLP's gate / up / silu_mul."""
    M = x.shape[0] if x.dim() == 2 else 1
    pg, pu = _problem(w_gate), _problem(w_up)
    _check(lib().mcv_w4a16_gemv_gate_up_silu(_ptr(x), ctypes.byref(pg), ctypes.byref(pu), _ptr(act), M,
                                             _stream(stream)), "matmul_w4a16_gate_up_silu")


def matmul_w4a16_gemm(x, w: W4A16QuantizedWeight, out, stream=None) -> None:
    """out fp16 [M,N] = x fp16 [M,K] @ dequant(w) on the tcgen05 tensor cores (M >= 16)."""
    M = x.shape[0]
    _check(lib().mcv_w4a16_gemm(_ptr(x), _ptr(w.qweight), _ptr(w.scales), _ptr(w.zeros), w.zero_bias, _ptr(out),
                                M, w.K, w.N, w.group_size, _stream(stream)), "matmul_w4a16_gemm")


class W4A16Problem(ctypes.Structure):
    """mirror of mcv_w4a16_problem (include/mcv_matmul.h)"""
    _fields_ = [("x", _vp), ("qweight", _vp), ("scales", _vp), ("zeros", _vp), ("out", _vp),
                ("K", ctypes.c_int32), ("N", ctypes.c_int32), ("group", ctypes.c_int32),
                ("zero_bias", ctypes.c_int32)]


def w4a16_problems(items):
    """[(x, W4A16QuantizedWeight, out), ...] -> ctypes array for matmul_w4a16_grouped."""
    arr = (W4A16Problem * len(items))()
    for i, (x, w, out) in enumerate(items):
        arr[i] = W4A16Problem(_ptr(x), _ptr(w.qweight), _ptr(w.scales), _ptr(w.zeros), _ptr(out),
                              w.K, w.N, w.group_size, w.zero_bias)
    return arr


def matmul_w4a16_grouped(items, M: int = 1, stream=None, problems=None) -> None:
    """Independent W4A16 GEMVs in one launch; items = [(x, weight, out), ...]
    (or a prebuilt ``problems`` array from w4a16_problems)."""
    arr = problems if problems is not None else w4a16_problems(items)
    _check(lib().mcv_w4a16_gemv_grouped(ctypes.cast(arr, _vp), len(arr), M, _stream(stream)),
           "matmul_w4a16_grouped")


# ---- dense fp16 ----------------------------------------------------------------

def matmul_b_transposed(a, b, out, stream=None) -> None:
    """out [M,N] = a [M,K] @ B with b stored [N,K] or [K,N], as the reference
    disambiguates them (src/csrc/lib/ops.cpp:165-171): the GEMV for M <= 8,
    the tensor-core GEMM beyond."""
    M, K = a.shape
    if b.shape[1] == K:
        layout, N = 0, b.shape[0]
    elif b.shape[0] == K:
        layout, N = 1, b.shape[1]
    else:
        raise RuntimeError("matmul_b_transposed K dim mismatch")
    if tuple(out.shape) != (M, N):
        raise RuntimeError("matmul_b_transposed out shape mismatch")
    if M > 8:
        # the tensor-core GEMM (mcv_gemm_f16) takes [N,K]; a [K,N] weight must
        # be transposed once at load time (transpose_f16), as the caller owns memory
        if layout != 0:
            raise RuntimeError("matmul_b_transposed: M > 8 needs the weight as [N,K] (see transpose_f16)")
        _check(lib().mcv_gemm_f16(_ptr(a), _ptr(b), _ptr(out), M, K, N, _stream(stream)), "matmul_b_transposed")
        return
    _check(lib().mcv_gemv_f16(_ptr(a), _ptr(b), _ptr(out), M, K, N, layout, _stream(stream)), "matmul_b_transposed")


def gemm_f16(x, w_nk, out, stream=None) -> None:
    """out fp16 [M,N] = x fp16 [M,K] @ w_nk^T on the tcgen05 tensor cores (mcv_gemm_f16)."""
    M, K = x.shape
    N = w_nk.shape[0]
    _check(lib().mcv_gemm_f16(_ptr(x), _ptr(w_nk), _ptr(out), M, K, N, _stream(stream)), "gemm_f16")


def transpose_f16(src, dst, stream=None) -> None:
    """dst [C,R] = src [R,C]^T (fp16), e.g. a [K,N] weight to the GEMM's [N,K]."""
    R, C = src.shape
    _check(lib().mcv_transpose_f16(_ptr(src), _ptr(dst), R, C, _stream(stream)), "transpose_f16")


def lm_head_workspace(M: int = 1, device="cuda"):
    import torch
    n = int(lib().mcv_lm_head_workspace_size(M))
    return torch.zeros(n, dtype=torch.uint8, device=device)


def lm_head_argmax(x, w_nk, workspace, out_index=None, out_key=None, n_offset: int = 0,
                   fp16_logits: bool = False, stream=None) -> None:
    """Fused lm_head GEMV + greedy argmax over rows of w_nk fp16 [N_shard,K]."""
    M, K = x.shape
    N = w_nk.shape[0]
    _check(lib().mcv_lm_head_argmax(_ptr(x), _ptr(w_nk), _ptr(out_key), _ptr(out_index), M, K, N, n_offset,
                                    int(fp16_logits), _ptr(workspace), workspace.numel(), _stream(stream)),
           "lm_head_argmax")


def argmax_last_dim(logits, out, stream=None) -> None:
    """int64 [M] = argmax over the last dim of fp16 [M,V] (ops.h:21)."""
    M, V = logits.shape
    _check(lib().mcv_argmax_last_dim_f16(_ptr(logits), _ptr(out), M, V, _stream(stream)), "argmax_last_dim")


# ---- sharded lm_head ------------------------------------------------------------

class NcclComm:
    """An NCCL communicator owned by the library (one rank per process/GPU)."""

    def __init__(self, nranks: int, rank: int, unique_id: bytes):
        self.handle = _vp()
        _check(lib().mcv_nccl_comm_init(ctypes.byref(self.handle), nranks, unique_id, rank), "nccl_comm_init")

    @staticmethod
    def unique_id() -> bytes:
        n = int(lib().mcv_nccl_unique_id_bytes())
        buf = ctypes.create_string_buffer(n)
        _check(lib().mcv_nccl_get_unique_id(buf), "nccl_get_unique_id")
        return buf.raw

    def destroy(self) -> None:
        if self.handle:
            _check(lib().mcv_nccl_comm_destroy(self.handle), "nccl_comm_destroy")
            self.handle = _vp()


def lm_head_argmax_allreduce(comm: NcclComm, x, w_shard, workspace, out_key, out_index, n_offset: int,
                             fp16_logits: bool = False, stream=None) -> None:
    M, K = x.shape
    _check(lib().mcv_lm_head_argmax_allreduce(comm.handle, _ptr(x), _ptr(w_shard), _ptr(out_key), _ptr(out_index),
                                              M, K, w_shard.shape[0], n_offset, int(fp16_logits),
                                              _ptr(workspace), workspace.numel(), _stream(stream)),
           "lm_head_argmax_allreduce")


class P2PContext:
    """Peer-mailbox context for the fused sharded lm_head (one per rank)."""

    def __init__(self, nranks: int, rank: int):
        self.handle = _vp()
        n = int(lib().mcv_p2p_handle_bytes())
        buf = ctypes.create_string_buffer(n)
        _check(lib().mcv_p2p_create(ctypes.byref(self.handle), nranks, rank, buf), "p2p_create")
        self.ipc_handle = buf.raw

    def connect(self, all_handles) -> None:
        blob = b"".join(all_handles)
        _check(lib().mcv_p2p_connect(self.handle, blob), "p2p_connect")

    def errors(self) -> int:
        return int(lib().mcv_p2p_errors(self.handle))

    def destroy(self) -> None:
        if self.handle:
            _check(lib().mcv_p2p_destroy(self.handle), "p2p_destroy")
            self.handle = _vp()


def lm_head_argmax_p2p(ctx: P2PContext, x, w_shard, workspace, out_key, out_index, n_offset: int,
                       fp16_logits: bool = False, stream=None) -> None:
    M, K = x.shape
    _check(lib().mcv_lm_head_argmax_p2p(ctx.handle, _ptr(x), _ptr(w_shard), _ptr(out_key), _ptr(out_index),
                                        M, K, w_shard.shape[0], n_offset, int(fp16_logits),
                                        _ptr(workspace), workspace.numel(), _stream(stream)),
           "lm_head_argmax_p2p")


# ---- W8A8 -----------------------------------------------------------------------

def lm_head_greedy_host(x_host, x_dev, w_shard, index_dev, index_host, workspace, ctx: "P2PContext" = None,
                        n_offset: int = 0, fp16_logits: bool = False, norm_gamma=None, norm_eps: float = 1e-6,
                        stream=None) -> None:
    """Host x (pinned fp16 [M,K]) -> host int64 [M] global argmax indices in
    one call: copy in, (final rms_norm with `norm_gamma`,) fused lm_head +
    argmax (peer exchange when `ctx`), copy out, stream sync
    (mcv_lm_head_greedy_host)."""
    M, K = x_host.shape
    N = w_shard.shape[0]
    if x_host.is_cuda or index_host.is_cuda:
        raise RuntimeError("lm_head_greedy_host: x_host and index_host live in host memory")
    _check(lib().mcv_lm_head_greedy_host(ctx.handle if ctx is not None else None, _vp(x_host.data_ptr()), _ptr(x_dev),
                                         _ptr(norm_gamma), norm_eps, _ptr(w_shard), _ptr(index_dev),
                                         _vp(index_host.data_ptr()), M, K, N, n_offset, int(fp16_logits),
                                         _ptr(workspace), workspace.numel(), _stream(stream)),
           "lm_head_greedy_host")


def lm_head_argmax_rmsnorm(x, norm_gamma, w_shard, workspace, out_index=None, out_key=None, norm_eps: float = 1e-6,
                           norm_variant: int = 0, ctx: "P2PContext" = None, n_offset: int = 0,
                           fp16_logits: bool = False, stream=None) -> None:
    """lm_head_greedy's device half with its final rms_norm fused in
    (mcv_lm_head_argmax_rmsnorm): x is the raw last hidden state [M,K]."""
    M, K = x.shape
    _check(lib().mcv_lm_head_argmax_rmsnorm(ctx.handle if ctx is not None else None, _ptr(x), _ptr(norm_gamma),
                                            norm_eps, norm_variant, _ptr(w_shard), _ptr(out_key), _ptr(out_index),
                                            M, K, w_shard.shape[0], n_offset, int(fp16_logits), _ptr(workspace),
                                            workspace.numel(), _stream(stream)),
           "lm_head_argmax_rmsnorm")


def rms_norm(x, gamma, out, eps: float = 1e-6, variant: int = 0, stream=None) -> None:
    """out [rows,H] = rms_norm(x); variant 0 = the engine's rms_norm (fp16
    chain, 1 + gamma), 1 = rms_norm1024's fp32 arithmetic (mcv_rms_norm)."""
    H = x.shape[-1]
    rows = x.numel() // H
    _check(lib().mcv_rms_norm(_ptr(x), _ptr(gamma), _ptr(out), rows, H, eps, variant, _stream(stream)), "rms_norm")


def silu_mul(gate, up, out, stream=None) -> None:
    """out = silu(gate) * up (mcv_silu_mul)."""
    _check(lib().mcv_silu_mul(_ptr(gate), _ptr(up), _ptr(out), gate.numel(), _stream(stream)), "silu_mul")


class LmHeadGreedyStep:
    """A prepared mcv_lm_head_greedy_host call for a decode loop: tensors are
    checked, their addresses resolved and every argument converted to its C
    type once, so each token costs one library call with no per-call
    argument conversion (pass `w_shard` to switch weights between calls)."""

    _proto = ctypes.CFUNCTYPE(_int)

    def __init__(self, x_host, x_dev, w_shard, index_dev, index_host, workspace, ctx: "P2PContext" = None,
                 n_offset: int = 0, fp16_logits: bool = False, norm_gamma=None, norm_eps: float = 1e-6, stream=None):
        if x_host.is_cuda or index_host.is_cuda:
            raise RuntimeError("LmHeadGreedyStep: x_host and index_host live in host memory")
        M, K = x_host.shape
        # an unprototyped handle on the same entry point: the arguments below
        # are already ctypes objects of the declared C types
        self._fn = self._proto(ctypes.cast(lib().mcv_lm_head_greedy_host, _vp).value)
        self._shape = (M, K)
        self._rows = w_shard.shape[0]
        vp = lambda p: _vp(p if isinstance(p, int) else (p.value if p is not None else None))
        self._head = (vp(ctx.handle if ctx is not None else None), _vp(x_host.data_ptr()), vp(_ptr(x_dev)),
                      vp(_ptr(norm_gamma)), ctypes.c_float(norm_eps))
        self._w = vp(_ptr(w_shard))
        self._args = list(self._head) + [self._w, vp(_ptr(index_dev)), _vp(index_host.data_ptr()), _i64(M), _i64(K),
                                         _i64(self._rows), _i64(n_offset), _int(int(fp16_logits)), vp(_ptr(workspace)),
                                         _sz(workspace.numel()), vp(_stream(stream))]
        self._keep = (x_host, x_dev, w_shard, index_dev, index_host, workspace, norm_gamma)

    def __call__(self, w_shard=None) -> None:
        args = self._args
        if w_shard is not None:
            if tuple(w_shard.shape) != (self._rows, self._shape[1]):
                raise RuntimeError("LmHeadGreedyStep: weight shape differs from the prepared one")
            args = list(args)
            args[5] = _vp(w_shard.data_ptr())
        st = self._fn(*args)
        if st != 0:
            _check(st, "lm_head_greedy_host")


def w8a8_quantize(x, x_int8, x_scale, stream=None) -> None:
    M, K = x.shape
    _check(lib().mcv_w8a8_quantize(_ptr(x), _ptr(x_int8), _ptr(x_scale), M, K, _stream(stream)), "w8a8_quantize")


def matmul_w8a8_i32(x_int8, w_int8, out, w_layout: int = 1, stream=None) -> None:
    """int32 [M,N] = int8 [M,K] @ int8 weights; layout 1 = [K,N] (reference), 0 = [N,K]."""
    M, K = x_int8.shape
    N = w_int8.shape[1] if w_layout == 1 else w_int8.shape[0]
    _check(lib().mcv_w8a8_gemm_i32(_ptr(x_int8), _ptr(w_int8), _ptr(out), M, K, N, w_layout, _stream(stream)),
           "matmul_w8a8_i32")


def w8a8_dequant(acc, x_scale, w_scale, out, stream=None) -> None:
    M, N = acc.shape
    _check(lib().mcv_w8a8_dequant(_ptr(acc), _ptr(x_scale), _ptr(w_scale), _ptr(out), M, N, _stream(stream)),
           "w8a8_dequant")


def matmul_decode_w8a8_prequant(x_int8, x_scale, w_int8, w_scale, out, acc=None, stream=None) -> None:
    """out fp16 [M,N] from an already-quantized x (w8a8_quantize) and int8
    [N,K] weights: int32 GEMV + dequant in one kernel (mcv_w8a8_gemv_prequant)."""
    M, K = x_int8.shape
    N = w_int8.shape[0]
    _check(lib().mcv_w8a8_gemv_prequant(_ptr(x_int8), _ptr(x_scale), _ptr(w_int8), _ptr(w_scale), _ptr(out), _ptr(acc),
                                        M, K, N, _stream(stream)), "matmul_decode_w8a8_prequant")


class W8A8Problem(ctypes.Structure):
    """One GEMV of mcv_w8a8_fused_grouped."""
    _fields_ = [("x", _vp), ("w_int8", _vp), ("w_scale", _vp), ("out", _vp), ("N", _i64)]


def w8a8_problems(items):
    """[(x fp16 [M,K], w_int8 [N,K], w_scale [N], out [M,N]), ...] -> ctypes array."""
    arr = (W8A8Problem * len(items))()
    for i, (x, w, ws, out) in enumerate(items):
        arr[i] = W8A8Problem(_ptr(x), _ptr(w), _ptr(ws), _ptr(out), w.shape[0])
    return arr


def w8a8_fused_grouped(items=None, M: int = 1, K: int = None, problems=None, stream=None) -> None:
    """Independent fused W8A8 GEMVs ([N,K] int8 weights) in one launch."""
    arr = problems if problems is not None else w8a8_problems(items)
    if K is None:
        K = items[0][0].shape[1]
        M = items[0][0].shape[0]
    _check(lib().mcv_w8a8_fused_grouped(ctypes.cast(arr, _vp), len(arr), M, K, _stream(stream)), "w8a8_fused_grouped")


def w8a8_fused(x, w_int8, w_scale, out, acc=None, x_int8=None, x_scale=None, w_layout: int = 0,
               stream=None) -> None:
    M, K = x.shape
    N = w_int8.shape[0] if w_layout == 0 else w_int8.shape[1]
    _check(lib().mcv_w8a8_fused(_ptr(x), _ptr(w_int8), _ptr(w_scale), _ptr(out), _ptr(acc), _ptr(x_int8),
                                _ptr(x_scale), M, K, N, w_layout, _stream(stream)), "w8a8_fused")


def lm_head_argmax_w8a8(x, w_int8, w_scale, workspace, out_index=None, out_key=None, n_offset: int = 0,
                        stream=None) -> None:
    """W8A8 lm_head + greedy argmax over int8 rows w_int8 [N_shard, K] with
    fp16 per-row scales (mcv_lm_head_argmax_w8a8)."""
    M, K = x.shape
    N = w_int8.shape[0]
    _check(lib().mcv_lm_head_argmax_w8a8(_ptr(x), _ptr(w_int8), _ptr(w_scale), _ptr(out_key), _ptr(out_index), M, K,
                                         N, n_offset, _ptr(workspace), workspace.numel(), _stream(stream)),
           "lm_head_argmax_w8a8")


def quantize_dense_weight_w8a8(w_kn, wq, w_scale, w_layout: int = 0, stream=None) -> None:
    """Per-channel int8 quantization (mcv_w8a8_quantize_weight); w_layout 2
    takes the weight as [N, K] (e.g. the embedding), 0 and 1 as [K, N]."""
    K, N = w_kn.shape if w_layout != 2 else w_kn.shape[::-1]
    _check(lib().mcv_w8a8_quantize_weight(_ptr(w_kn), _ptr(wq), _ptr(w_scale), K, N, w_layout, _stream(stream)),
           "quantize_dense_weight_w8a8")


# ---- decode dispatch (matmul_decode_dispatch, decoder_layer.cpp:212-244) -------

class DecodeWeights(ctypes.Structure):
    """The formats one projection has on the device (mcv_decode_weights);
    leave a format out by passing None."""
    _fields_ = [("dense", _vp), ("dense_layout", _int), ("w4_qweight", _vp), ("w4_scales", _vp),
                ("w4_zeros", _vp), ("w4_zero_bias", _int), ("w8_weight", _vp), ("w8_scale", _vp)]

    @classmethod
    def of(cls, dense=None, dense_layout: int = 0, w4: "W4A16QuantizedWeight" = None, w8=None, w8_scale=None):
        d = cls()
        d.dense = _ptr(dense).value if dense is not None else None
        d.dense_layout = dense_layout
        if w4 is not None:
            d.w4_qweight, d.w4_scales, d.w4_zeros = (_ptr(w4.qweight).value, _ptr(w4.scales).value,
                                                     _ptr(w4.zeros).value)
            d.w4_zero_bias = w4.zero_bias
        if w8 is not None:
            d.w8_weight, d.w8_scale = _ptr(w8).value, _ptr(w8_scale).value
        return d


def set_w8a8_decode_mode(mode) -> None:
    """Replace the MINICPM_W8A8_DECODE mode (None: read the environment again)."""
    _check(lib().mcv_set_w8a8_decode_mode(None if mode is None else mode.encode()), "set_w8a8_decode_mode")


def w8a8_decode_enabled() -> bool:
    return bool(lib().mcv_w8a8_decode_enabled())


def w8a8_decode_gate_enabled() -> bool:
    """The gate matmul_decode_dispatch applies (decoder_layer.cpp:19-25):
    a set-but-empty MINICPM_W8A8_DECODE counts as on."""
    return bool(lib().mcv_w8a8_decode_gate_enabled())


def w8a8_policy_allows(token: str, mode=None) -> bool:
    """w8a8_policy_allows (language_model.cpp:32-41); an explicit `mode`
    bypasses the process-wide one."""
    if mode is None:
        return bool(lib().mcv_w8a8_policy_allows(token.encode()))
    return bool(lib().mcv_w8a8_policy_allows_mode(mode.encode(), token.encode()))


def matmul_decode_dispatch(x, weights: DecodeWeights, out, stream=None) -> None:
    """out [M,N] = x [M,K] . W on the format matmul_decode_dispatch would pick."""
    M, K = x.shape
    N = out.shape[1]
    _check(lib().mcv_matmul_decode_dispatch(_ptr(x), ctypes.byref(weights), _ptr(out), M, K, N, _stream(stream)),
           "matmul_decode_dispatch")
