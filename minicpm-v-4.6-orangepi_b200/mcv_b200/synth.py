"""Seeded synthetic inputs with the shapes and distributions of the benchmark
configurations (numpy only; shared by the tests and bench.py).

No checkpoint is available, so weights are random with the stated
distributions; fp16 values are produced by round-to-nearest conversion and
both the CUDA path and the CPU oracle consume the identical bits.
"""
from __future__ import annotations

import numpy as np

GROUP = 128


def rng(seed: int) -> np.random.Generator:
    return np.random.Generator(np.random.PCG64(seed))


def w4a16_inputs(M: int, K: int, N: int, seed: int = 0, group: int = GROUP):
    """Config 0 distributions: x ~ N(0,1) fp16 [M,K]; q ~ U{0..15} [K,N];
    zeros ~ U{0..15} [G,N]; scales ~ U[0.002, 0.02] fp16 [G,N]."""
    r = rng(seed)
    G = K // group
    x = r.standard_normal((M, K), dtype=np.float32).astype(np.float16)
    q = r.integers(0, 16, size=(K, N), dtype=np.uint8)
    z = r.integers(0, 16, size=(G, N), dtype=np.uint8)
    s = r.uniform(0.002, 0.02, size=(G, N)).astype(np.float16)
    return x, q, z, s


def lm_head_inputs(K: int, N: int, seed: int = 1, M: int = 1, chunk_rows: int = 1 << 16):
    """Config 1 distributions: x ~ N(0,1) fp16 [M,K]; W ~ N(0, 0.02) fp16 [N,K]
    (the tied-embedding row layout)."""
    r = rng(seed)
    x = r.standard_normal((M, K), dtype=np.float32).astype(np.float16)
    w = np.empty((N, K), np.float16)
    for a in range(0, N, chunk_rows):
        b = min(N, a + chunk_rows)
        w[a:b] = (r.standard_normal((b - a, K), dtype=np.float32) * np.float32(0.02)).astype(np.float16)
    return x, w


def w8a8_inputs(M: int, K: int, N: int, seed: int = 2):
    """Config 2 distributions: x ~ N(0,1) fp16 [M,K]; w ~ U[-127,127] int8
    [K,N]; w_scale ~ U[0.001, 0.01] fp16 [N]."""
    r = rng(seed)
    x = r.standard_normal((M, K), dtype=np.float32).astype(np.float16)
    w = r.integers(-127, 128, size=(K, N), dtype=np.int8)
    ws = r.uniform(0.001, 0.01, size=N).astype(np.float16)
    return x, w, ws


def gptq_pack(q_kn: np.ndarray, z_gn: np.ndarray):
    """Logical q [K,N], true zeros z [G,N] (1..16) -> GPTQ qweight int32 [K/8,N]
    and qzeros int32 [G,N/8] storing z-1 (the format the reference unpacks in
    src/csrc/lib/quantized_weight.cpp:104-114)."""
    K, N = q_kn.shape
    qw = np.zeros((K // 8, N), np.uint32)
    for i in range(8):
        qw |= q_kn[i::8].astype(np.uint32) << np.uint32(4 * i)
    zs = (z_gn.astype(np.int32) - 1).astype(np.uint32)
    G = z_gn.shape[0]
    qz = np.zeros((G, N // 8), np.uint32)
    for i in range(8):
        qz |= zs[:, i::8] << np.uint32(4 * i)
    return qw.view(np.int32), qz.view(np.int32)


AWQ_ORDER = (0, 2, 4, 6, 1, 3, 5, 7)


def awq_pack(q_kn: np.ndarray, z_gn: np.ndarray):
    """Logical q [K,N], zeros z [G,N] (0..15) -> AWQ qweight int32 [K,N/8] and
    qzeros int32 [G,N/8]; slot s of word j holds column 8j + AWQ_ORDER[s]
    (src/csrc/lib/quantized_weight.cpp:17, 147-156)."""
    K, N = q_kn.shape
    G = z_gn.shape[0]
    qw = np.zeros((K, N // 8), np.uint32)
    qz = np.zeros((G, N // 8), np.uint32)
    for s, col in enumerate(AWQ_ORDER):
        qw |= q_kn[:, col::8].astype(np.uint32) << np.uint32(4 * s)
        qz |= z_gn[:, col::8].astype(np.uint32) << np.uint32(4 * s)
    return qw.view(np.int32), qz.view(np.int32)


# Decode-step matmul set of the 24-layer hybrid LM (config 3): 18
# linear-attention layers and 6 full-attention layers (every 4th), hidden
# 1024, intermediate 3584.  (K, N) per projection, in call order of
# src/csrc/lib/decoder_layer.cpp:1110-1204 and :970-1048.
LINEAR_LAYER = (("linear_qkv", 1024, 6144), ("linear_z", 1024, 2048), ("linear_a", 1024, 16),
                ("linear_b", 1024, 16), ("linear_out", 2048, 1024))
FULL_LAYER = (("full_q", 1024, 4096), ("full_k", 1024, 512), ("full_v", 1024, 512), ("full_o", 2048, 1024))
MLP = (("mlp_gate", 1024, 3584), ("mlp_up", 1024, 3584), ("mlp_down", 3584, 1024))


def decode_step_shapes(num_layers: int = 24):
    """[(layer, name, K, N)] for one token: 186 projections."""
    out = []
    for layer in range(num_layers):
        attn = FULL_LAYER if layer % 4 == 3 else LINEAR_LAYER
        for name, K, N in attn + MLP:
            out.append((layer, name, K, N))
    return out


def w4a16_bytes(M: int, K: int, N: int, group: int = GROUP) -> int:
    """Algorithmic bytes of one W4A16 GEMV: int4 weights, fp16 scales, int4
    zeros, fp16 activations in, fp16 outputs."""
    G = K // group
    return K * N // 2 + G * N * 2 + G * N // 2 + M * K * 2 + M * N * 2
