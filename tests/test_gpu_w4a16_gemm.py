"""tcgen05 W4A16 GEMM (config 4 shapes and ragged ones) against the CPU
oracle.  The kernel scales weights in fp16 before the MMA, so the tolerance is
the path's fp16 one: |got - ref| <= 1e-2 + 1e-3 * |ref|."""
import numpy as np
import pytest

import oracle
from conftest import assert_f16_close
from mcv_b200 import synth

pytestmark = pytest.mark.gpu


def run(torch, x, w):
    import mcv_b200
    xd = torch.from_numpy(np.ascontiguousarray(x)).cuda()
    out = torch.full((x.shape[0], w.N), float("nan"), dtype=torch.float16, device="cuda")
    mcv_b200.matmul_w4a16_gemm(xd, w, out)
    torch.cuda.synchronize()
    return out.cpu().numpy()


@pytest.mark.parametrize("M,K,N", [(16, 1024, 3584), (64, 1024, 4096), (256, 1024, 3584), (1024, 1024, 4096),
                                   (100, 2048, 1000), (1, 128, 16), (130, 3584, 1024),
                                   (300, 4096, 520), (70, 1024, 1001)])
def test_gemm_vs_oracle(cuda, M, K, N):
    import mcv_b200
    x, q, z, s = synth.w4a16_inputs(M, K, N, seed=M + K + N)
    w = mcv_b200.pack_w4a16(q, z, s)
    out = run(cuda, x, w)
    ref = oracle.w4a16_gemv(x, oracle.w4a16_fold_zeros(q, z), s, nthreads=8)
    assert_f16_close(out, ref, what=f"gemm M={M} K={K} N={N}")


def test_gemm_matches_gemv_rows(cuda):
    """Rows of the GEMM equal the M<=8 GEMV on the same weights (both within
    tolerance of the oracle, and of each other)."""
    import mcv_b200
    torch = cuda
    x, q, z, s = synth.w4a16_inputs(8, 1024, 3584, seed=77)
    w = mcv_b200.pack_w4a16(q, z, s)
    g = run(torch, x, w)
    xd = torch.from_numpy(x).cuda()
    o = torch.empty((8, 3584), dtype=torch.float16, device="cuda")
    mcv_b200.matmul_w4a16(xd, w, o)
    torch.cuda.synchronize()
    assert_f16_close(g, o.cpu().numpy().astype(np.float32), what="gemm vs gemv")
    assert mcv_b200.device_errors() == 0


@pytest.mark.parametrize("splits", [1, 2, 3, 8])
def test_gemm_split_k_cluster(cuda, splits):
    """k split over a thread-block cluster (partials summed through
    distributed shared memory) gives the oracle's answer for every split
    count, including uneven slices (3) and the largest cluster (8)."""
    import mcv_b200
    M, K, N = 40, 2048, 640
    x, q, z, s = synth.w4a16_inputs(M, K, N, seed=splits)
    w = mcv_b200.pack_w4a16(q, z, s)
    mcv_b200.set_tuning(mcv_b200.TUNE_GEMM_SPLIT_K, splits)
    try:
        out = run(cuda, x, w)
    finally:
        mcv_b200.set_tuning(mcv_b200.TUNE_GEMM_SPLIT_K, 0)
    ref = oracle.w4a16_gemv(x, oracle.w4a16_fold_zeros(q, z), s, nthreads=8)
    assert_f16_close(out, ref, what=f"gemm split_k={splits}")
    assert mcv_b200.device_errors() == 0
