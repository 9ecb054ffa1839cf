"""rms_norm, silu_mul and their fused forms (rms_norm in the lm_head
prologue, silu_mul in the down projection's activation load) on the GPU
against the CPU oracle.  rms_norm is bit-exact (every float step explicitly
rounded, the mean's sum exact); silu_mul uses CUDA's expf, so its fp16
outputs are held to |d| <= 1e-2 + 1e-3|ref|; argmax indices are exact."""
import numpy as np
import pytest

import oracle
from conftest import assert_f16_close
from mcv_b200 import synth

pytestmark = pytest.mark.gpu


def dev(torch, a):
    a = np.ascontiguousarray(a)
    if a.dtype == np.uint16:
        a = a.view(np.float16)
    return torch.from_numpy(a).cuda()


def modular_fill(N, H):
    """tests/test_rms_norm.cpp:58-69 / test_rms_norm1024.cpp:54-63 inputs."""
    i = np.arange(N * H, dtype=np.int64)
    x = ((((i * 17 + 5) % 41).astype(np.float32) / np.float32(41.0) - np.float32(0.5)) * np.float32(0.5))
    h = np.arange(H)
    g = np.float32(1.0) + np.float32(0.01) * ((h % 7) - 3).astype(np.float32)
    return x.reshape(N, H).astype(np.float16), g.astype(np.float16)


@pytest.mark.parametrize("variant", [0, 1])
@pytest.mark.parametrize("N,H,kind", [(4, 256, "mod"), (4, 128, "mod"), (8, 1024, "mod"), (4, 1024, "mod"),
                                      (3, 1024, "randn"), (2, 3584, "randn"), (1, 2048, "big"), (5, 100, "randn")])
def test_rms_norm_bit_exact(cuda, variant, N, H, kind):
    import mcv_b200 as mcv
    torch = cuda
    if kind == "mod":
        x, g = modular_fill(N, H)
    else:
        r = synth.rng(N * H + variant)
        scale = 40.0 if kind == "big" else 1.0
        x = (r.standard_normal((N, H)) * scale).astype(np.float16)
        g = (r.standard_normal(H) * 0.1).astype(np.float16)
    out = torch.empty((N, H), dtype=torch.float16, device="cuda")
    mcv.rms_norm(dev(torch, x), dev(torch, g), out, eps=1e-6, variant=variant)
    torch.cuda.synchronize()
    ref = oracle.rms_norm(x, g, eps=1e-6, variant=variant)
    got = out.cpu().numpy().view(np.uint16)
    assert np.array_equal(got, ref), f"{np.count_nonzero(got != ref)} of {ref.size} differ"
    if kind == "mod" and variant == 1:
        # the reference test's own criterion (tests/test_rms_norm1024.cpp:97-112): |d| <= 5e-3
        # against a double-precision x / rms * gamma
        xf = x.astype(np.float64)
        rms = np.sqrt((xf * xf).mean(axis=1, keepdims=True) + 1e-6)
        want = xf / rms * g.astype(np.float64)
        assert np.max(np.abs(got.view(np.float16).astype(np.float64) - want)) <= 5e-3


@pytest.mark.parametrize("n", [3584, 8 * 3584, 1000, 7])
def test_silu_mul(cuda, n):
    import mcv_b200 as mcv
    torch = cuda
    r = synth.rng(n)
    g = (r.standard_normal(n) * 3).astype(np.float16)
    u = r.standard_normal(n).astype(np.float16)
    out = torch.empty(n, dtype=torch.float16, device="cuda")
    mcv.silu_mul(dev(torch, g), dev(torch, u), out)
    torch.cuda.synchronize()
    ref = oracle.silu_mul(g, u)
    got = out.cpu().numpy()
    assert_f16_close(got, oracle.f16_to_f32(ref), what="silu_mul")
    # expf differs from the host's by at most an ulp: nearly every fp16 output is identical
    assert np.count_nonzero(got.view(np.uint16) != ref) <= max(2, n // 200)


@pytest.mark.parametrize("M", [1, 3])
def test_lm_head_with_final_norm(cuda, M):
    """mcv_lm_head_argmax_rmsnorm == oracle rms_norm, then the oracle scan."""
    import mcv_b200 as mcv
    torch = cuda
    K, V = 1024, 32768 if M > 1 else 248094
    r = synth.rng(90 + M)
    h = (r.standard_normal((M, K)) * 4).astype(np.float16)       # raw hidden state
    gamma = (r.standard_normal(K) * 0.2).astype(np.float16)
    _, w = synth.lm_head_inputs(K, V, seed=5)
    xn = oracle.rms_norm(h, gamma, eps=1e-6, variant=0)
    ref_idx, _, gap = oracle.lm_head_argmax(xn, w, nthreads=8)
    ws = mcv.lm_head_workspace(M)
    idx = torch.empty(M, dtype=torch.int64, device="cuda")
    wd = dev(torch, w)
    for _ in range(2):
        idx.fill_(-5)
        mcv.lm_head_argmax_rmsnorm(dev(torch, h), dev(torch, gamma), wd, ws, out_index=idx, norm_eps=1e-6)
        torch.cuda.synchronize()
        assert np.array_equal(idx.cpu().numpy(), ref_idx), (idx.cpu().numpy(), ref_idx, gap)
    # the same through the host entry point (x from host memory, token to host memory)
    x_host = torch.from_numpy(h).pin_memory()
    idx_host = torch.full((M,), -1, dtype=torch.int64).pin_memory()
    mcv.lm_head_greedy_host(x_host, torch.empty_like(x_host, device="cuda"), wd, idx, idx_host, ws,
                            norm_gamma=dev(torch, gamma), norm_eps=1e-6)
    assert np.array_equal(idx_host.numpy(), ref_idx)


@pytest.mark.parametrize("M,K,N", [(1, 1024, 3584), (3, 1024, 3584), (8, 1024, 3584), (1, 4096, 512),
                                   (2, 384, 40), (1, 128, 8)])
def test_gate_up_with_swiglu_epilogue(cuda, M, K, N):
    """act = silu_mul(x . Wg, x . Wu) in one launch against the oracle's
    W4A16 GEMVs, fp16 rounding of gate and up, then its silu_mul (fp16
    tolerance), and bit for bit against the separate GPU kernels (the fused
    kernel splits K over its warps exactly as the single-GEMV kernel does)."""
    import mcv_b200 as mcv
    torch = cuda
    x, qg, zg, sg = synth.w4a16_inputs(M, K, N, seed=K + N + M)
    _, qu, zu, su = synth.w4a16_inputs(M, K, N, seed=K + N + M + 1)
    wg, wu = mcv.pack_w4a16(qg, zg, sg), mcv.pack_w4a16(qu, zu, su)
    xd = dev(torch, x)
    act = torch.empty((M, N), dtype=torch.float16, device="cuda")
    mcv.matmul_w4a16_gate_up_silu(xd, wg, wu, act)
    gate = torch.empty((M, N), dtype=torch.float16, device="cuda")
    up = torch.empty((M, N), dtype=torch.float16, device="cuda")
    mcv.matmul_w4a16(xd, wg, gate)
    mcv.matmul_w4a16(xd, wu, up)
    two = torch.empty((M, N), dtype=torch.float16, device="cuda")
    mcv.silu_mul(gate, up, two)
    torch.cuda.synchronize()
    got = act.cpu().numpy()
    g_ref = oracle.f32_to_f16_rn(oracle.w4a16_gemv(x, oracle.w4a16_fold_zeros(qg, zg), sg, nthreads=8))
    u_ref = oracle.f32_to_f16_rn(oracle.w4a16_gemv(x, oracle.w4a16_fold_zeros(qu, zu), su, nthreads=8))
    ref = oracle.f16_to_f32(oracle.silu_mul(g_ref, u_ref))
    assert_f16_close(got, ref, what=f"gate/up swiglu M={M} K={K} N={N}")
    assert np.array_equal(got.view(np.uint16), two.cpu().numpy().view(np.uint16))
