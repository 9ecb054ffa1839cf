"""Every entry point refuses bad arguments on the host, with its documented
status, before it touches a device - so these run without a GPU.  Status
codes: 1 null, 2 shape, 3 alignment, 6 workspace, 7 value."""
import ctypes

import pytest

import mcv_b200

NULL, SHAPE, ALIGN, WORKSPACE, VALUE = 1, 2, 3, 6, 7
F = ctypes.c_void_p(256)        # 16-byte aligned stand-in for a device pointer
F2 = ctypes.c_void_p(256 + 2)   # 2-byte aligned only
F4 = ctypes.c_void_p(256 + 4)   # 4-byte aligned only


@pytest.fixture(scope="module")
def L():
    return mcv_b200.lib()


def test_w4a16_gemm_arguments(L):
    g = L.mcv_w4a16_gemm
    assert g(None, F, F, F, 0, F, 64, 1024, 4096, 128, None) == NULL
    assert g(F, F, F, F, 0, F, 64, 1024, 4096, 64, None) == SHAPE        # group
    assert g(F, F, F, F, 0, F, 64, 1000, 4096, 128, None) == SHAPE       # K % 128
    assert g(F, F, F, F, 0, F, 0, 1024, 4096, 128, None) == SHAPE        # M
    assert g(F2, F, F, F, 0, F, 64, 1024, 4096, 128, None) == ALIGN      # x
    assert g(F, F, F4, F, 0, F, 64, 1024, 4096, 128, None) == ALIGN      # scales
    assert g(F, F, F, F, 2, F, 64, 1024, 4096, 128, None) == VALUE       # zero_bias


def test_w4a16_grouped_arguments(L):
    P = mcv_b200.W4A16Problem
    good = P(F, F, F, F, F, 1024, 3584, 128, 0)
    arr = (P * 2)(good, good)
    assert L.mcv_w4a16_gemv_grouped(arr, 0, 1, None) == NULL
    assert L.mcv_w4a16_gemv_grouped(arr, 2, 65, None) == SHAPE
    arr[1] = P(F, F, F, None, F, 1024, 3584, 128, 0)
    assert L.mcv_w4a16_gemv_grouped(arr, 2, 1, None) == NULL
    arr[1] = P(F, F, F, F, F, 1000, 3584, 128, 0)
    assert L.mcv_w4a16_gemv_grouped(arr, 2, 1, None) == SHAPE
    arr[1] = P(F, F, F, F4, F, 1024, 3584, 128, 0)   # zeros need 4 bytes only
    arr[0] = P(F2, F, F, F, F, 1024, 3584, 128, 0)
    assert L.mcv_w4a16_gemv_grouped(arr, 2, 1, None) == ALIGN
    arr[0] = P(F, F, F, F, F, 1024, 3584, 128, 3)
    assert L.mcv_w4a16_gemv_grouped(arr, 2, 1, None) == VALUE


def test_lm_head_arguments(L):
    h = L.mcv_lm_head_argmax
    ws_bytes = L.mcv_lm_head_workspace_size(1)
    assert h(F, F, None, None, 1, 1024, 1000, 0, 0, F, ws_bytes, None) == NULL          # no output
    assert h(F, F, None, F, 9, 1024, 1000, 0, 0, F, ws_bytes, None) == SHAPE            # M
    assert h(F, F, None, F, 1, 1020, 1000, 0, 0, F, ws_bytes, None) == SHAPE            # K % 8
    assert h(F, F, None, F, 1, 1024, 1000, (1 << 32) - 10, 0, F, ws_bytes, None) == SHAPE  # index range
    assert h(F, F, None, F, 1, 1024, 1000, 0, 0, F, ws_bytes - 1, None) == WORKSPACE
    assert h(F, F, None, F, 1, 1024, 1000, 0, 0, F4, ws_bytes, None) == ALIGN          # 8-byte workspace
    assert h(F2, F, None, F, 1, 1024, 1000, 0, 0, F, ws_bytes, None) == ALIGN
    # sharded variants need a connected context / communicator
    assert L.mcv_lm_head_argmax_p2p(None, F, F, None, F, 1, 1024, 1000, 0, 0, F, ws_bytes, None) == NULL
    # the no-workspace variant refuses what its fixed array cannot hold
    assert L.mcv_lm_head_argmax_noalloc(F, F, None, F, 9, 1024, 1000, 0, 0, None) == SHAPE
    assert L.mcv_lm_head_argmax_noalloc(F, F, None, None, 1, 1024, 1000, 0, 0, None) == NULL


def test_lm_head_greedy_host_arguments(L):
    g = L.mcv_lm_head_greedy_host
    ws_bytes = L.mcv_lm_head_workspace_size(1)
    assert g(None, None, F, None, 1e-6, F, F, F, 1, 1024, 1000, 0, 0, F, ws_bytes, None) == NULL
    assert g(None, F, F, None, 1e-6, F, F, F, 9, 1024, 1000, 0, 0, F, ws_bytes, None) == SHAPE


def test_neighbour_arguments(L):
    ws_bytes = L.mcv_lm_head_workspace_size(1)
    r = L.mcv_lm_head_argmax_rmsnorm
    assert r(None, F, None, 1e-6, 0, F, None, F, 1, 1024, 1000, 0, 0, F, ws_bytes, None) == NULL   # gamma
    assert r(None, F, F, 1e-6, 2, F, None, F, 1, 1024, 1000, 0, 0, F, ws_bytes, None) == VALUE    # variant
    assert r(None, F, F, 1e-6, 0, F, None, None, 1, 1024, 1000, 0, 0, F, ws_bytes, None) == NULL  # outputs
    assert L.mcv_rms_norm(F, None, F, 1, 1024, 1e-6, 0, None) == NULL
    assert L.mcv_rms_norm(F, F, F, 1, 1024, 1e-6, 3, None) == VALUE
    assert L.mcv_rms_norm(F, F, F, 0, 1024, 1e-6, 0, None) == SHAPE
    assert L.mcv_silu_mul(F, F, None, 8, None) == NULL
    assert L.mcv_silu_mul(F2, F, F, 8, None) == ALIGN
    assert L.mcv_silu_mul(F, F, F, 0, None) == SHAPE
    P = mcv_b200.W4A16Problem
    good = P(None, F, F, F, None, 1024, 3584, 128, 0)
    g = L.mcv_w4a16_gemv_gate_up_silu
    assert g(F, ctypes.byref(good), None, F, 1, None) == NULL
    assert g(F, ctypes.byref(good), ctypes.byref(good), F, 9, None) == SHAPE               # M
    other = P(None, F, F, F, None, 1024, 1024, 128, 0)
    assert g(F, ctypes.byref(good), ctypes.byref(other), F, 1, None) == SHAPE              # N differs
    big = P(None, F, F, F, None, 8192, 3584, 128, 0)
    assert g(F, ctypes.byref(big), ctypes.byref(big), F, 1, None) == SHAPE                 # K above 4096
    assert g(F2, ctypes.byref(good), ctypes.byref(good), F, 1, None) == ALIGN


def test_w8a8_arguments(L):
    assert L.mcv_w8a8_fused(F, F, F, F, None, None, None, 1, 1000, 3584, 0, None) == SHAPE  # K % 16
    assert L.mcv_w8a8_fused(F, F, F, F, None, None, None, 9, 1024, 3584, 0, None) == SHAPE  # M
    assert L.mcv_w8a8_fused(F, F, F, F, None, None, None, 1, 1024, 3584, 2, None) == VALUE  # layout
    assert L.mcv_w8a8_fused(F, F, F, F, None, None, None, 1, 1024, 3584, 1, None) == WORKSPACE  # [K][N] buffers
    assert L.mcv_w8a8_fused(F2, F, F, F, None, None, None, 1, 1024, 3584, 0, None) == ALIGN
    assert L.mcv_w8a8_fused(None, F, F, F, None, None, None, 1, 1024, 3584, 0, None) == NULL
    assert L.mcv_w8a8_quantize(F, F, F, 0, 1024, None) == SHAPE
    P8 = mcv_b200.W8A8Problem
    ok = P8(F, F, F, F, 3584)
    arr = (P8 * 17)(*([ok] * 17))
    assert L.mcv_w8a8_fused_grouped(arr, 0, 1, 1024, None) == NULL
    assert L.mcv_w8a8_fused_grouped(arr, 17, 1, 1024, None) == SHAPE
    assert L.mcv_w8a8_fused_grouped(arr, 2, 9, 1024, None) == SHAPE
    arr[1] = P8(F2, F, F, F, 3584)
    assert L.mcv_w8a8_fused_grouped(arr, 2, 1, 1024, None) == ALIGN
    assert L.mcv_w8a8_gemv_prequant(F, None, F, F, F, None, 1, 1024, 3584, None) == NULL
    assert L.mcv_w8a8_gemv_prequant(F, F, F, F, F, None, 9, 1024, 3584, None) == SHAPE
    assert L.mcv_w8a8_gemv_prequant(F2, F, F, F, F, None, 1, 1024, 3584, None) == ALIGN
    assert L.mcv_w8a8_quantize_weight(F, F, F, 1024, 3584, 3, None) == VALUE


def test_decode_dispatch_arguments(L):
    d = L.mcv_matmul_decode_dispatch
    none = mcv_b200.DecodeWeights()
    assert d(None, ctypes.byref(none), F, 1, 1024, 1024, None) == NULL
    assert d(F, ctypes.byref(none), F, 0, 1024, 1024, None) == SHAPE
    assert d(F, ctypes.byref(none), F, 1, 1024, 1024, None) == NULL        # no usable format
    dense = mcv_b200.DecodeWeights()
    dense.dense = 256
    dense.dense_layout = 1
    assert d(F, ctypes.byref(dense), F, 9, 1024, 1024, None) == SHAPE      # M > 8 on dense needs [N][K]


def test_gemm_f16_arguments(L):
    g = L.mcv_gemm_f16
    assert g(None, F, F, 64, 1024, 4096, None) == NULL
    assert g(F, F, F, 64, 1000, 4096, None) == SHAPE      # K % 64
    assert g(F, F, F, 64, 1024, 4092, None) == SHAPE      # N % 8
    assert g(F, F, F, 0, 1024, 4096, None) == SHAPE       # M
    assert g(F2, F, F, 64, 1024, 4096, None) == ALIGN
    assert L.mcv_transpose_f16(F, None, 4, 4, None) == NULL
    assert L.mcv_transpose_f16(F, F, 0, 4, None) == SHAPE


def test_context_set_up_arguments(L):
    h = ctypes.create_string_buffer(int(L.mcv_p2p_handle_bytes()))
    ctx = ctypes.c_void_p()
    assert L.mcv_p2p_create(ctypes.byref(ctx), 9, 0, h) == VALUE
    assert L.mcv_p2p_create(ctypes.byref(ctx), 2, 2, h) == VALUE
    assert L.mcv_p2p_create(None, 2, 0, h) == NULL
    comm = ctypes.c_void_p()
    uid = ctypes.create_string_buffer(int(L.mcv_nccl_unique_id_bytes()))
    assert L.mcv_nccl_comm_init(ctypes.byref(comm), 2, uid, 5) == VALUE


def test_lm_head_w8a8_arguments(L):
    h = L.mcv_lm_head_argmax_w8a8
    ws_bytes = L.mcv_lm_head_workspace_size(1)
    assert h(F, F, None, None, F, 1, 1024, 1000, 0, F, ws_bytes, None) == NULL       # scales
    assert h(F, F, F, None, None, 1, 1024, 1000, 0, F, ws_bytes, None) == NULL       # no output
    assert h(F, F, F, None, F, 1, 1032, 1000, 0, F, ws_bytes, None) == SHAPE         # K % 16
    assert h(F, F, F, None, F, 1, 8192, 1000, 0, F, ws_bytes, None) == SHAPE         # K <= 4096
    assert h(F, F, F, None, F, 9, 1024, 1000, 0, F, ws_bytes, None) == SHAPE         # M
    assert h(F, F, F, None, F, 1, 1024, 1000, 0, F, ws_bytes - 1, None) == WORKSPACE
    assert h(F2, F, F, None, F, 1, 1024, 1000, 0, F, ws_bytes, None) == ALIGN
